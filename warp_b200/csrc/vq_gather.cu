// vq_gather.cu — the bank-sliced VQ3R gather, the table images it copies,
// and the device tile layout of a resident expert bank (see vq_gather.cuh
// for the table layout).
//
// Work unit: a 16-row "quarter" of one 64-row index block at one chunk of 32
// vector positions.  Lane p owns position 32c + p and reads that position's
// 48 code bytes for the 16 rows; after the 48 lookups (3 per row) the warp
// reduces the 16 per-lane row partials across the 32 positions, leaving the
// chunk partial of row (p & 15) in lanes p and p + 16.
//
// Two code layouts:
//  * plain — the container's [row_block][v][64 rows][3] (warp_vq_apply on a
//    caller's matrix): lane p reads its 48 contiguous bytes, lanes 192 bytes
//    apart;
//  * tiled — the resident bank after bank_tile_kernel: each (row_block,
//    chunk) span is rearranged in place so that piece j (16 bytes) of quarter
//    q of lane p sits at q*npos*48 + j*npos*16 + p*16 — one warp load reads
//    npos*16 contiguous bytes — and row slot i of lane p holds row
//    16q + (i ^ (p & 15)), which lets the cross-lane reduction run without
//    selects.
#include "vq_gather.cuh"

#include <mutex>

namespace warp {

__device__ __forceinline__ void group_mat(const GatherArgs &a, int g, int m,
                                          int &kind, int &route) {
    const int t = g / a.gpt, sub = g % a.gpt;
    if (a.mpg > 1) { kind = sub; route = t * a.K + m; }
    else { kind = a.gpt == 1 ? 0 : 2; route = t * a.K + sub; }
}

// Start the copy of a compact image into the table regions: 6144 pieces of
// 16 bytes, region A's 4096 linear, region B's 2048 into the stage-2 slots.
__device__ __forceinline__ void issue_image(const uint32_t *img) {
    const uint8_t *src = (const uint8_t *)img;
    for (int i = threadIdx.x; i < kImageWords / 4; i += kGatherThreads) {
        uint32_t dst;
        if (i < 4096) {
            dst = kRegA + (uint32_t)i * 16u;
        } else {
            const int j = i - 4096;
            dst = kRegB + (uint32_t)(j >> 3) * 256u + (uint32_t)(j & 7) * 16u;
        }
        cp_async16(dst, src + (size_t)i * 16);
    }
    cp_async_commit();
}

__device__ __forceinline__ const uint8_t *mat_base(const GatherArgs &a, int g, int m) {
    if (a.plan) {
        const int r = g / a.gpt;
        const uint32_t off = a.gpt == 2 ? ((g & 1) ? a.kind_off[1] : a.kind_off[0])
                                        : a.kind_off[2];
        return a.bank + (size_t)a.plan[1 + a.max_routes + r] * a.rec_bytes + off;
    }
    int kind, route;
    group_mat(a, g, m, kind, route);
    const uint32_t off = kind == 0 ? a.kind_off[0] : kind == 1 ? a.kind_off[1] : a.kind_off[2];
    return a.bank ? a.bank + (size_t)a.route_idx[route] * a.rec_bytes + off : a.idx_plain;
}

// Word k (0..11) of the 48 code bytes held as three uint4.
#define WARP_QW(q, k) (((k) & 3) == 0 ? q[(k) >> 2].x : ((k) & 3) == 1 ? q[(k) >> 2].y \
                       : ((k) & 3) == 2 ? q[(k) >> 2].z : q[(k) >> 2].w)

// 16 rows at this lane's position: 48 lookups, then the cross-lane
// reduction.  Lanes p and p + 16 return the chunk partial of row (p & 15).
// Rows are summed in pairs with packed f32x2 adds (each element rounds as a
// scalar add would), so a quarter costs 48 PRMT + 48 LDS + 24 packed adds +
// 16 shuffles.
template <bool PERM>
__device__ __forceinline__ float quarter(const uint4 (&q)[3], uint32_t bA0,
                                         uint32_t bA1, uint32_t bB) {
    const int lane = threadIdx.x & 31;
    if constexpr (PERM) {
        float2 acc[8];
#pragma unroll
        for (int r2 = 0; r2 < 8; r2++) {
            float v[2][3];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int r = 2 * r2 + h;
                const int b0 = 3 * r, b1 = 3 * r + 1, b2 = 3 * r + 2;
                v[h][0] = lds_f32(prmt(WARP_QW(q, b0 >> 2), bA0, 0x7604u | ((b0 & 3) << 4)));
                v[h][1] = lds_f32(prmt(WARP_QW(q, b1 >> 2), bA1, 0x7604u | ((b1 & 3) << 4)));
                v[h][2] = lds_f32(prmt(WARP_QW(q, b2 >> 2), bB, 0x7604u | ((b2 & 3) << 4)));
            }
            acc[r2] = __fadd2_rn(__fadd2_rn(make_float2(v[0][0], v[1][0]),
                                            make_float2(v[0][1], v[1][1])),
                                 make_float2(v[0][2], v[1][2]));
        }
        // transpose-reduce over the row pairs: rows i and i + m meet at
        // lane distance m (the tile layout's row permutation makes every
        // lane's partner hold the matching row)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, acc[j + 4].x, 8),
                                         __shfl_xor_sync(0xffffffffu, acc[j + 4].y, 8));
            acc[j] = __fadd2_rn(acc[j], o);
        }
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, acc[j + 2].x, 4),
                                         __shfl_xor_sync(0xffffffffu, acc[j + 2].y, 4));
            acc[j] = __fadd2_rn(acc[j], o);
        }
        {
            const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, acc[1].x, 2),
                                         __shfl_xor_sync(0xffffffffu, acc[1].y, 2));
            acc[0] = __fadd2_rn(acc[0], o);
        }
        const float s = acc[0].x + __shfl_xor_sync(0xffffffffu, acc[0].y, 1);
        return s + __shfl_xor_sync(0xffffffffu, s, 16);
    } else {
        float acc[16];
#pragma unroll
        for (int r = 0; r < 16; r++) {
            const int b0 = 3 * r, b1 = 3 * r + 1, b2 = 3 * r + 2;
            const uint32_t a0 = prmt(WARP_QW(q, b0 >> 2), bA0, 0x7604u | ((b0 & 3) << 4));
            const uint32_t a1 = prmt(WARP_QW(q, b1 >> 2), bA1, 0x7604u | ((b1 & 3) << 4));
            const uint32_t a2 = prmt(WARP_QW(q, b2 >> 2), bB, 0x7604u | ((b2 & 3) << 4));
            acc[r] = __fadd_rn(__fadd_rn(lds_f32(a0), lds_f32(a1)), lds_f32(a2));
        }
#pragma unroll
        for (int m = 8; m >= 1; m >>= 1) {
            const bool up = (lane & m) != 0;
#pragma unroll
            for (int i = 0; i < m; i++) {
                const float keep = up ? acc[i + m] : acc[i];
                const float send = up ? acc[i] : acc[i + m];
                acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
            }
        }
        return acc[0] + __shfl_xor_sync(0xffffffffu, acc[0], 16);
    }
}

// A warp's position in the quarter sequence of one segment: matrix m,
// quarter qb inside it, and this lane's code pointer (null: nothing to
// load).  A warp steps one quarter per warp of the CTA at a time, which
// inside a matrix is a whole number of row blocks further in both code
// layouts, so the common step is one add.
struct Cursor {
    int m, qb;
    const uint8_t *src;
};

// Lane `lane`'s code bytes of quarter qb of a matrix whose index blocks
// start at mat, in chunk c.
template <bool TILED>
__device__ __forceinline__ const uint8_t *quarter_src(const GatherArgs &a, const uint8_t *mat,
                                                      int qb, int c, int lane, int npos) {
    const int rb = qb >> 2, qq = qb & 3;
    if (TILED)
        return mat + ((size_t)rb * a.nv + c * kChunk) * (kBlk * kSt) + qq * (npos * 48) +
               lane * 16;
    return mat + ((size_t)rb * a.nv + c * kChunk + lane) * (kBlk * kSt) + qq * 48;
}

template <bool TILED>
__device__ __forceinline__ void cursor_set(const GatherArgs &a, int g, int c, int lane,
                                           int npos, bool live, Cursor &k) {
    k.src = (live && k.m < a.mpg) ? quarter_src<TILED>(a, mat_base(a, g, k.m), k.qb, c, lane, npos)
                                  : nullptr;
}

template <bool TILED>
__device__ __forceinline__ void cursor_step(const GatherArgs &a, int g, int c, int lane,
                                            int npos, bool live, size_t step, Cursor &k) {
    k.qb += kGatherThreads / 32;
    if (k.qb < a.qb_per_mat) {
        if (k.src) k.src += step;
    } else {
        do { k.qb -= a.qb_per_mat; k.m++; } while (k.qb >= a.qb_per_mat);
        cursor_set<TILED>(a, g, c, lane, npos, live, k);
    }
}

// This lane's 48 code bytes of a quarter, as three 16-byte loads straight
// into registers (zeros when the lane has no position or no quarter is left).
template <bool TILED>
__device__ __forceinline__ void load_quarter(uint4 (&q)[3], const uint8_t *src, int npos) {
    if (!src) { q[0] = q[1] = q[2] = make_uint4(0u, 0u, 0u, 0u); return; }
#pragma unroll
    for (int j = 0; j < 3; j++) q[j] = ldg_stream(src + (TILED ? j * npos * 16 : j * 16));
}

template <bool TILED>
__global__ void __launch_bounds__(kGatherThreads, 1)
vq_gather_kernel(const GatherArgs a) {
    extern __shared__ __align__(16) uint8_t dyn_smem[];
    const uint32_t base = smem_u32(dyn_smem);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = kGatherThreads / 32;
    static_assert(NW % 4 == 0, "a warp steps NW quarters: NW / 4 whole row blocks");
    // the table regions must lie inside this CTA's shared-memory window
    if (base > kRegA || kRegEnd > base + (uint32_t)kGatherSmem) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
        return;
    }
    // With a.early the routing was written two or more kernels back, so the
    // first quarters' code loads go out before the wait for the previous
    // kernel (whose output, the tables, is read after it).
    bool waited = false;
    if (!a.early) { pdl_wait(); pdl_trigger(); waited = true; }
    const uint32_t bA0 = kRegA | (uint32_t)(lane * 4);
    const uint32_t bA1 = kRegA | (uint32_t)(lane * 4 + 128);
    const uint32_t bB = kRegB | (uint32_t)(lane * 4);
    const long long G = gridDim.x;
    const long long total =
        a.plan ? (long long)a.plan[0] * a.gpt * a.nchunks * a.qb_per_mat : a.total;
    const long long u0 = total * blockIdx.x / G, u1 = total * (blockIdx.x + 1) / G;
    const long long H = (long long)a.mpg * a.qb_per_mat;   // quarters per segment
    const size_t rows_per_chunk = (size_t)a.n_groups * a.mpg * a.M;
    const size_t step = (size_t)(NW / 4) * a.nv * (kBlk * kSt);  // NW / 4 row blocks of codes

    for (long long seg0 = u0; seg0 < u1;) {
        const long long seg = seg0 / H;                   // (group, chunk)
        const long long s_end = (seg + 1) * H < u1 ? (seg + 1) * H : u1;
        const int g = (int)(seg / a.nchunks), c = (int)(seg % a.nchunks);
        const int qs0 = (int)(seg0 - seg * H), qs1 = (int)(s_end - seg * H);
        const int npos = min(kChunk, a.nv - c * kChunk);
        const bool live = lane < npos;
        // the table image first, then this warp's quarters qs0 + warp + NW i,
        // their code bytes loaded into registers two quarters ahead (buffers
        // A and B alternate, each with the (matrix, quarter) it holds).  The
        // first chunk of an early launch issues its code loads before the
        // wait and the image (the previous kernel's output) after it.
        __syncthreads();                                  // previous table done
        const int ig = (a.plan && a.gpt == 2) ? (a.plan[1 + (g >> 1)] / a.K) * 2 + (g & 1) : g;
        const uint32_t *img = a.image + ((size_t)ig * a.nchunks + c) * kImageWords;
        if (waited) issue_image(img);
        const int n = qs1 - qs0 > warp ? (qs1 - qs0 - warp + NW - 1) / NW : 0;  // quarters of this warp
        Cursor k;
        k.m = (qs0 + warp) / a.qb_per_mat;
        k.qb = qs0 + warp - k.m * a.qb_per_mat;
        cursor_set<TILED>(a, g, c, lane, npos, live, k);
        uint4 qa[3], qb[3];
        int ma = k.m, qba = k.qb;
        load_quarter<TILED>(qa, n > 0 ? k.src : nullptr, npos);
        cursor_step<TILED>(a, g, c, lane, npos, live, step, k);
        int mb = k.m, qbb = k.qb;
        load_quarter<TILED>(qb, n > 1 ? k.src : nullptr, npos);
        cursor_step<TILED>(a, g, c, lane, npos, live, step, k);
        if (!waited) {
            pdl_wait();
            pdl_trigger();
            waited = true;
            issue_image(img);
        }
        cp_async_wait<0>();                               // this thread's image pieces
        __syncthreads();                                  // everyone's

        float *part = a.partial + (size_t)c * rows_per_chunk + (size_t)g * a.mpg * a.M;
        const int lrow = lane & 15;
        for (int i = 0; i < n; i += 2) {
            {
                const float sum = quarter<TILED>(qa, bA0, bA1, bB);
                const int row = 16 * qba + lrow;
                if (lane < 16 && row < a.M) part[(size_t)ma * a.M + row] = sum;
                ma = k.m; qba = k.qb;
                load_quarter<TILED>(qa, i + 2 < n ? k.src : nullptr, npos);
                cursor_step<TILED>(a, g, c, lane, npos, live, step, k);
            }
            if (i + 1 < n) {
                const float sum = quarter<TILED>(qb, bA0, bA1, bB);
                const int row = 16 * qbb + lrow;
                if (lane < 16 && row < a.M) part[(size_t)mb * a.M + row] = sum;
                mb = k.m; qbb = k.qb;
                load_quarter<TILED>(qb, i + 3 < n ? k.src : nullptr, npos);
                cursor_step<TILED>(a, g, c, lane, npos, live, step, k);
            }
        }
        cp_async_wait<0>();                               // nothing in flight at a rebuild
        seg0 = s_end;
    }
}
#undef WARP_QW

// plain LUT [nv][3][256] -> per-chunk compact images.
__global__ void lut_slice_kernel(uint32_t *__restrict__ image,
                                 const float *__restrict__ lut, int nv,
                                 int nchunks) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)nchunks * kImageWords) return;
    const int c = (int)(i / kImageWords);
    const int w = (int)(i % kImageWords);
    int s, code, p;
    if (w < 16384) { code = w >> 6; s = (w >> 5) & 1; p = w & 31; }
    else { code = (w - 16384) >> 5; s = 2; p = w & 31; }
    const int v = c * kChunk + p;
    const float val = v < nv ? lut[((size_t)v * kSt + s) * kEnt + code] : 0.0f;
    image[i] = __float_as_uint(val);
}

// Tables of x straight into compact images: `split` CTAs per (group,
// chunk), each writing a 1/split share of the words; group g = 2t + kind reads
// token t's x and codebooks cb0 + 3*kind.  The kind's three
// books (24 KiB) are staged in shared memory; thread p%32 keeps position p's
// eight x values in registers; consecutive threads write consecutive words.
constexpr int kImageThreads = 256;
// CTAs per image: 16 for one token (a decode step: 0.686 / 0.666 / 0.657 ms
// at 4 / 8 / 16), fewer as tokens add images of their own (every CTA stages
// the kind's 24 KiB of books)
constexpr int kImageSplitMax = 16;

__global__ void __launch_bounds__(kImageThreads)
lut_image_kernel(uint32_t *__restrict__ images, const float *__restrict__ x, int nv,
                 int nchunks, const float *__restrict__ books, int cb0, int split) {
    __shared__ __align__(16) float sb[kSt * kEnt * kVec];
    const int seg = blockIdx.x / split, part = blockIdx.x % split;
    const int g = seg / nchunks, c = seg % nchunks;
    const int t = g >> 1, kind = g & 1;
    const float4 *src = (const float4 *)(books + (size_t)(cb0 + kSt * kind) * kEnt * kVec);
    for (int i = threadIdx.x; i < kSt * kEnt * kVec / 4; i += kImageThreads)
        ((float4 *)sb)[i] = src[i];
    const int p = threadIdx.x & 31;
    const int v = c * kChunk + p;
    float xv[kVec];
    if (v < nv) {
        const float4 *xp = (const float4 *)(x + ((size_t)t * nv + v) * kVec);
        const float4 lo = xp[0], hi = xp[1];
        xv[0] = lo.x; xv[1] = lo.y; xv[2] = lo.z; xv[3] = lo.w;
        xv[4] = hi.x; xv[5] = hi.y; xv[6] = hi.z; xv[7] = hi.w;
    } else {
#pragma unroll
        for (int d = 0; d < kVec; d++) xv[d] = 0.0f;
    }
    __syncthreads();
    uint32_t *img = images + (size_t)seg * kImageWords;
    const int w0 = part * (kImageWords / split), w1 = w0 + kImageWords / split;
#pragma unroll 4
    for (int w = w0 + threadIdx.x; w < w1; w += kImageThreads) {
        int s, code;
        if (w < 16384) { code = w >> 6; s = (w >> 5) & 1; }
        else { code = (w - 16384) >> 5; s = 2; }
        img[w] = __float_as_uint(lut_entry(xv, sb + (s * kEnt + code) * kVec));
    }
}

// y[r] = f16(scale[r]) * sum over chunks (in order) of partial[c][r].
__global__ void gather_finish_kernel(float *__restrict__ y,
                                     const float *__restrict__ partial,
                                     const uint16_t *__restrict__ scale, int M,
                                     int nchunks) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= M) return;
    float acc = 0.0f;
    for (int c = 0; c < nchunks; c++) acc += partial[(size_t)c * M + r];
    y[r] = acc * f16_to_f32(scale[r]);
}

// In-place re-tiling of one matrix kind of every expert record (plain ->
// tiled, see the file comment).  One CTA per (expert, row block, chunk)
// span of npos*192 bytes: the span is read whole into shared memory, then
// written back permuted.  Spans are disjoint, so the transform is safe in
// place.
__global__ void bank_tile_kernel(uint8_t *__restrict__ bank, size_t rec_bytes,
                                 uint32_t off, int M, int nv, int n_experts) {
    __shared__ __align__(16) uint8_t span[kChunk * kBlk * kSt];
    const int nb = (M + kBlk - 1) / kBlk, nch = (nv + kChunk - 1) / kChunk;
    const long long t = blockIdx.x;
    const int e = (int)(t / ((long long)nb * nch));
    const int rb = (int)((t / nch) % nb), c = (int)(t % nch);
    if (e >= n_experts) return;
    const int npos = min(kChunk, nv - c * kChunk);
    const int bytes = npos * kBlk * kSt;
    uint8_t *p = bank + (size_t)e * rec_bytes + off + ((size_t)rb * nv + c * kChunk) * (kBlk * kSt);
    for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x)
        ((uint4 *)span)[i] = ((const uint4 *)p)[i];
    __syncthreads();
    // output byte o -> (quarter q, piece j, lane pl, byte-in-piece k); lane
    // byte b = 16j + k = 3i + s holds row 16q + (i ^ (pl & 15)), stage s
    for (int o = threadIdx.x; o < bytes; o += blockDim.x) {
        const int q = o / (npos * 48);
        const int r1 = o % (npos * 48);
        const int j = r1 / (npos * 16);
        const int r2 = r1 % (npos * 16);
        const int pl = r2 / 16, k = r2 % 16;
        const int b = 16 * j + k, i = b / 3, s = b % 3;
        const int row = 16 * q + (i ^ (pl & 15));
        p[o] = span[pl * (kBlk * kSt) + row * kSt + s];
    }
}

static int set_attr(const void *fn) {
    cudaError_t e = cudaFuncSetAttribute(
        fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kGatherSmem);
    if (e != cudaSuccess) return cuda_fail(e, "gather smem attribute");
    return WARP_OK;
}

int gather_setup() {
    // Per device: the attribute is a property of the function in the
    // current context, so set it on every device that launches.
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && done[dev]) return WARP_OK;
    int rc;
    if ((rc = set_attr((const void *)vq_gather_kernel<false>))) return rc;
    if ((rc = set_attr((const void *)vq_gather_kernel<true>))) return rc;
    if (dev >= 0 && dev < 64) done[dev] = true;
    return WARP_OK;
}

int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// Grid for `total` quarters: one CTA per SM, fewer when there is not enough
// work to give each warp a few quarters.
int gather_grid(long long total) {
    const long long sms = sm_count();
    long long g = (total + 63) / 64;
    if (g > sms) g = sms;
    if (g < 1) g = 1;
    return (int)g;
}

int gather_launch(const GatherArgs &a, bool tiled, cudaStream_t st) {
    int rc = gather_setup();
    if (rc) return rc;
    if (a.total <= 0) return WARP_OK;
    const int grid = gather_grid(a.total);
    const cudaError_t e =
        tiled ? launch_pdl(vq_gather_kernel<true>, dim3(grid), dim3(kGatherThreads), kGatherSmem,
                           st, a)
              : launch_pdl(vq_gather_kernel<false>, dim3(grid), dim3(kGatherThreads),
                           kGatherSmem, st, a);
    if (e != cudaSuccess) return cuda_fail(e, "vq_gather_kernel");
    count_launch();
    return WARP_OK;
}

int lut_images(uint32_t *images, const float *x, int T, int nv, const float *books,
               int cb0, cudaStream_t st) {
    const int nchunks = (nv + kChunk - 1) / kChunk;
    int split = kImageSplitMax / T;                   // a power of two dividing kImageWords
    split = split < 1 ? 1 : split;
    while (split & (split - 1)) split &= split - 1;
    lut_image_kernel<<<(unsigned)(T * 2 * nchunks * split), kImageThreads, 0, st>>>(
        images, x, nv, nchunks, books, cb0, split);
    WARP_CHECK_LAUNCH("lut_image_kernel");
    return WARP_OK;
}

int bank_tile(uint8_t *bank, size_t rec_bytes, uint32_t off, int M, int nv, int E,
              cudaStream_t st) {
    const long long n = (long long)E * ((M + kBlk - 1) / kBlk) * ((nv + kChunk - 1) / kChunk);
    if (n <= 0) return WARP_OK;
    bank_tile_kernel<<<(unsigned)n, 256, 0, st>>>(bank, rec_bytes, off, M, nv, E);
    WARP_CHECK_LAUNCH("bank_tile_kernel");
    return WARP_OK;
}

int vq_apply_gather(float *y, const uint8_t *idx, const uint16_t *scale,
                    const float *lut, int M, int nv, cudaStream_t st) {
    int rc = gather_setup();
    if (rc) return rc;
    const int nchunks = (nv + kChunk - 1) / kChunk;
    const size_t image_bytes = (size_t)nchunks * kImageWords * 4;
    const size_t part_bytes = (size_t)nchunks * M * sizeof(float);
    void *scratch = nullptr;
    cudaError_t e = cudaMallocAsync(&scratch, image_bytes + part_bytes + 256, st);
    if (e != cudaSuccess) return cuda_fail(e, "vq_apply scratch");
    uint32_t *image = (uint32_t *)scratch;
    float *partial = (float *)((char *)scratch + image_bytes);
    int *err = (int *)((char *)scratch + image_bytes + part_bytes);
    cudaMemsetAsync(err, 0, sizeof(int), st);

    const size_t nimg = (size_t)nchunks * kImageWords;
    lut_slice_kernel<<<cdiv(nimg, 256), 256, 0, st>>>(image, lut, nv, nchunks);
    e = cudaGetLastError();
    if (e != cudaSuccess) { cudaFreeAsync(scratch, st); return cuda_fail(e, "lut_slice"); }
    count_launch();

    GatherArgs a = {};
    a.nv = nv;
    a.nchunks = nchunks;
    a.M = M;
    a.qb_per_mat = 4 * ((M + kBlk - 1) / kBlk);
    a.mpg = 1;
    a.gpt = 1;
    a.K = 1;
    a.n_groups = 1;
    a.total = (long long)nchunks * a.qb_per_mat;
    a.partial = partial;
    a.idx_plain = idx;
    a.image = image;
    a.err = err;
    rc = gather_launch(a, false, st);
    if (rc) { cudaFreeAsync(scratch, st); return rc; }
    gather_finish_kernel<<<cdiv(M, 256), 256, 0, st>>>(y, partial, scale, M, nchunks);
    e = cudaGetLastError();
    if (e != cudaSuccess) { cudaFreeAsync(scratch, st); return cuda_fail(e, "gather_finish"); }
    count_launch();
    int herr = 0;
    cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, st);
    cudaFreeAsync(scratch, st);
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "vq_apply sync");
    if (herr) {
        set_error("vq_gather: shared-memory window does not hold the table regions");
        return WARP_E_CUDA;
    }
    return WARP_OK;
}

// ---------------------------------------------------------------------------
// The same gather with fixed scratch (warp_vq_apply_noalloc).
//
// Some callers must not touch a device allocator at all: an engine that sizes
// every byte of HBM once at load and must not grow past it mid-step, a
// context whose stream-ordered memory pool is unsupported or disabled, and a
// decode loop that must not take the allocator's lock or grow a pool while a
// step runs.  This path keeps its scratch in module-scope device memory that
// the CUDA runtime sets aside when the library's module loads, and calls no
// allocating routine.
//
// Scratch: the compact images, then the chunk partials (256-byte aligned),
// then the error word; all of it must fit kNoallocScratchBytes.  Only the
// error word must start at zero (cleared every call); images and partials
// are fully written before they are read.  The scratch is one buffer per
// device, so calls that overlap on one device (another stream, another host
// thread) race on it: the caller serialises them.
constexpr size_t kNoallocScratchBytes = 8u << 20;   // 8 MiB per device
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device (with that
// device current) on the first call made on it.
static int noalloc_scratch(unsigned char **out) {
    static std::mutex mu;
    static unsigned char *addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "vq_apply_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) {
        set_error("vq_apply_noalloc: device ordinal %d out of range", dev);
        return WARP_E_ARG;
    }
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "vq_apply_noalloc: cudaGetSymbolAddress");
        addr[dev] = (unsigned char *)p;
    }
    *out = addr[dev];
    return WARP_OK;
}

size_t vq_apply_noalloc_bytes(int M, int nv) {
    const size_t nchunks = ((size_t)nv + kChunk - 1) / kChunk;
    const size_t image_bytes = nchunks * kImageWords * 4;
    const size_t part_bytes = (nchunks * (size_t)M * sizeof(float) + 255) / 256 * 256;
    return image_bytes + part_bytes + 256;
}

int vq_apply_gather_noalloc(float *y, const uint8_t *idx, const uint16_t *scale,
                            const float *lut, int M, int nv, cudaStream_t st) {
    const size_t need = vq_apply_noalloc_bytes(M, nv);
    if (need > kNoallocScratchBytes) {
        set_error("warp_vq_apply_noalloc: M=%d nv=%d needs %zu bytes of scratch, "
                  "above the fixed %zu; use warp_vq_apply",
                  M, nv, need, kNoallocScratchBytes);
        return WARP_E_ARG;
    }
    unsigned char *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    rc = gather_setup();
    if (rc) return rc;
    const int nchunks = (nv + kChunk - 1) / kChunk;
    const size_t image_bytes = (size_t)nchunks * kImageWords * 4;
    const size_t part_bytes = ((size_t)nchunks * M * sizeof(float) + 255) / 256 * 256;
    uint32_t *image = (uint32_t *)scratch;
    float *partial = (float *)(scratch + image_bytes);
    int *err = (int *)(scratch + image_bytes + part_bytes);
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), st);
    if (e != cudaSuccess) return cuda_fail(e, "vq_apply_noalloc: clear error word");

    const size_t nimg = (size_t)nchunks * kImageWords;
    lut_slice_kernel<<<cdiv(nimg, 256), 256, 0, st>>>(image, lut, nv, nchunks);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "lut_slice");
    count_launch();

    GatherArgs a = {};
    a.nv = nv;
    a.nchunks = nchunks;
    a.M = M;
    a.qb_per_mat = 4 * ((M + kBlk - 1) / kBlk);
    a.mpg = 1;
    a.gpt = 1;
    a.K = 1;
    a.n_groups = 1;
    a.total = (long long)nchunks * a.qb_per_mat;
    a.partial = partial;
    a.idx_plain = idx;
    a.image = image;
    a.err = err;
    rc = gather_launch(a, false, st);
    if (rc) return rc;
    gather_finish_kernel<<<cdiv(M, 256), 256, 0, st>>>(y, partial, scale, M, nchunks);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gather_finish");
    count_launch();
    int herr = 0;
    e = cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(e, "vq_apply_noalloc: read error word");
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "vq_apply_noalloc sync");
    if (herr) {
        set_error("vq_gather: shared-memory window does not hold the table regions");
        return WARP_E_CUDA;
    }
    return WARP_OK;
}

}  // namespace warp
