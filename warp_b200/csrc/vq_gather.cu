// vq_gather.cu — the bank-sliced VQ3R gather and the device tile layout of
// a resident expert bank (see vq_gather.cuh for the table layout).
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

// Shared address of the 64-byte block of codebook pair pr (stage*128 +
// code/2) while a table is built: the spare second slot of region B (the
// 128-byte gaps at code*256 + 128), two pairs per gap.
__device__ __forceinline__ uint32_t book_pair(int pr) {
    return kRegB + (uint32_t)(pr >> 1) * 256u + 128u + (uint32_t)(pr & 1) * 64u;
}

// Build the table of group g, chunk c into the shared regions.  The kind's
// three codebooks (24 KiB) are first staged in region B's spare slot with
// code pairs interleaved, [stage][code/2][dim][code&1], so one 128-bit load
// gives two codes' values for two dimensions.  Lane p computes position v = 32c + p; warp w takes
// (stage, code pair) w, w+16, ... and runs the two codes' FMA chains side by
// side in packed fp32x2 FMAs.  Each entry is still the FMA chain of
// lutb_range_avx512 (d = 0..7 from 0, one rounding per step), so the table
// matches the reference build bit for bit.
__device__ __forceinline__ void build_table(const GatherArgs &a, int g, int c,
                                            int kind) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cb = a.cb0 + kind * kSt;
    const float *src = a.books + (size_t)cb * kEnt * kVec;
    for (int i = threadIdx.x; i < kSt * kEnt * kVec / 4; i += kGatherThreads) {
        const float4 v = ((const float4 *)src)[i];          // code, dims d0..d0+3
        const int sc = i >> 1, d0 = (i & 1) * 4;            // (stage, code)
        const int s = sc >> 8, code = sc & 255;
        const uint32_t o = book_pair(s * 128 + (code >> 1)) +
                           ((uint32_t)d0 * 2u + (uint32_t)(code & 1)) * 4u;
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(o), "f"(v.x));
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(o + 8u), "f"(v.y));
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(o + 16u), "f"(v.z));
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(o + 24u), "f"(v.w));
    }
    const int v = c * kChunk + lane;
    float2 xx[kVec];
    if (v < a.nv) {
        const float4 *xp = (const float4 *)(a.x + (size_t)(g / a.x_gdiv) * a.x_stride +
                                            (size_t)v * kVec);
        const float4 lo = xp[0], hi = xp[1];
        xx[0] = make_float2(lo.x, lo.x); xx[1] = make_float2(lo.y, lo.y);
        xx[2] = make_float2(lo.z, lo.z); xx[3] = make_float2(lo.w, lo.w);
        xx[4] = make_float2(hi.x, hi.x); xx[5] = make_float2(hi.y, hi.y);
        xx[6] = make_float2(hi.z, hi.z); xx[7] = make_float2(hi.w, hi.w);
    } else {
#pragma unroll
        for (int d = 0; d < kVec; d++) xx[d] = make_float2(0.0f, 0.0f);
    }
    __syncthreads();
#pragma unroll 2
    for (int pr = warp; pr < kSt * kEnt / 2; pr += kGatherThreads / 32) {
        const int s = pr >> 7, code = (pr & 127) * 2;
        const uint32_t e = book_pair(pr);
        float2 cc[kVec];
#pragma unroll
        for (int h = 0; h < 4; h++) {
            float4 q;
            asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(q.x), "=f"(q.y), "=f"(q.z), "=f"(q.w) : "r"(e + 16u * h));
            cc[2 * h] = make_float2(q.x, q.y);
            cc[2 * h + 1] = make_float2(q.z, q.w);
        }
        float2 t = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int d = 0; d < kVec; d++) t = __ffma2_rn(xx[d], cc[d], t);
        const uint32_t addr = (s == 2 ? kRegB : kRegA) + (uint32_t)code * 256u +
                              (s == 1 ? 128u : 0u) + (uint32_t)lane * 4u;
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(t.x));
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr + 256u), "f"(t.y));
    }
}

// Copy chunk c of a pre-sliced image (region A then region B, 64 KiB each)
// into the regions: a straight, coalesced, conflict-free copy.
__device__ __forceinline__ void copy_image(const GatherArgs &a, int c) {
    const uint4 *src = (const uint4 *)(a.image + (size_t)c * kImageWords);
    for (int i = threadIdx.x; i < kImageWords / 4; i += kGatherThreads) {
        const uint4 v = src[i];
        const uint32_t addr = kRegA + (uint32_t)i * 16u;   // A and B are adjacent
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr),
                     "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
    }
}

__device__ __forceinline__ const uint8_t *mat_base(const GatherArgs &a, int g, int m) {
    int kind, route;
    group_mat(a, g, m, kind, route);
    return a.bank ? a.bank + (size_t)a.route_idx[route] * a.rec_bytes + a.kind_off[kind]
                  : a.idx_plain;
}

// Word k (0..11) of the 48 code bytes held as three uint4.
#define WARP_QW(q, k) (((k) & 3) == 0 ? q[(k) >> 2].x : ((k) & 3) == 1 ? q[(k) >> 2].y \
                       : ((k) & 3) == 2 ? q[(k) >> 2].z : q[(k) >> 2].w)

// 16 rows at this lane's position: 48 lookups, then the cross-lane
// reduction.  Lanes p and p + 16 return the chunk partial of row (p & 15).
template <bool PERM>
__device__ __forceinline__ float quarter(const uint4 (&q)[3], uint32_t bA0,
                                         uint32_t bA1, uint32_t bB) {
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; r++) {
        const int b0 = 3 * r, b1 = 3 * r + 1, b2 = 3 * r + 2;
        const uint32_t a0 = prmt(WARP_QW(q, b0 >> 2), bA0, 0x7604u | ((b0 & 3) << 4));
        const uint32_t a1 = prmt(WARP_QW(q, b1 >> 2), bA1, 0x7604u | ((b1 & 3) << 4));
        const uint32_t a2 = prmt(WARP_QW(q, b2 >> 2), bB, 0x7604u | ((b2 & 3) << 4));
        acc[r] = __fadd_rn(__fadd_rn(lds_f32(a0), lds_f32(a1)), lds_f32(a2));
    }
    const int lane = threadIdx.x & 31;
    if (PERM) {
#pragma unroll
        for (int m = 8; m >= 1; m >>= 1)
#pragma unroll
            for (int i = 0; i < m; i++)
                acc[i] += __shfl_xor_sync(0xffffffffu, acc[i + m], m);
    } else {
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
    }
    return acc[0] + __shfl_xor_sync(0xffffffffu, acc[0], 16);
}

// A position in the quarter sequence of one segment, advanced without
// division: matrix m, quarter qb inside it, and the matrix's index base.
struct Cursor {
    int m, qb;
    const uint8_t *mat;
};

__device__ __forceinline__ Cursor cursor_at(const GatherArgs &a, int g, int qs) {
    Cursor k;
    k.m = qs / a.qb_per_mat;
    k.qb = qs - k.m * a.qb_per_mat;
    k.mat = k.m < a.mpg ? mat_base(a, g, k.m) : nullptr;
    return k;
}

__device__ __forceinline__ void cursor_advance(const GatherArgs &a, int g, Cursor &k, int by) {
    k.qb += by;
    if (k.qb >= a.qb_per_mat) {
        do { k.qb -= a.qb_per_mat; k.m++; } while (k.qb >= a.qb_per_mat);
        k.mat = k.m < a.mpg ? mat_base(a, g, k.m) : nullptr;
    }
}

// Lane `lane`'s code bytes of the quarter at cursor k in chunk c.
template <bool TILED>
__device__ __forceinline__ const uint8_t *quarter_src(const GatherArgs &a, const Cursor &k,
                                                      int c, int lane, int npos) {
    const int rb = k.qb >> 2, qq = k.qb & 3;
    if (TILED)
        return k.mat + ((size_t)rb * a.nv + c * kChunk) * (kBlk * kSt) + qq * (npos * 48) +
               lane * 16;
    return k.mat + ((size_t)rb * a.nv + c * kChunk + lane) * (kBlk * kSt) + qq * 48;
}

// Start the asynchronous copy of this lane's 48 code bytes of a quarter into
// its ring slot (three 16-byte pieces at slot + 512j); always commits a
// group, empty when there is nothing to copy, so the group count per quarter
// stays one.
template <bool TILED>
__device__ __forceinline__ void issue_quarter(uint32_t slot, const uint8_t *src, int npos,
                                              bool copy) {
    if (copy) {
#pragma unroll
        for (int j = 0; j < 3; j++)
            cp_async16(slot + 512u * j, src + (TILED ? j * npos * 16 : j * 16));
    }
    cp_async_commit();
}

// Per-lane code ring: kRing slots of 48 bytes per lane (16-byte pieces 512
// bytes apart, so a warp's 128-bit reads and writes are conflict-free), one
// ring per warp.  Warps 0..kRingWarpsLow-1 keep theirs below region A, the
// rest above region B.
constexpr int kRing = 3;
constexpr uint32_t kRingWarpBytes = kRing * 1536u;
constexpr int kRingWarpsLow = 13;

template <bool TILED, bool BUILD>
__global__ void __launch_bounds__(kGatherThreads, 1)
vq_gather_kernel(const GatherArgs a) {
    extern __shared__ __align__(16) uint8_t dyn_smem[];
    const uint32_t base = smem_u32(dyn_smem);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = kGatherThreads / 32;
    const uint32_t low0 = (base + 127u) & ~127u;
    const uint32_t ring = warp < kRingWarpsLow ? low0 + warp * kRingWarpBytes
                                               : kRegEnd + (warp - kRingWarpsLow) * kRingWarpBytes;
    if (base > kRegA || low0 + kRingWarpsLow * kRingWarpBytes > kRegA ||
        kRegEnd + (NW - kRingWarpsLow) * kRingWarpBytes > base + (uint32_t)kGatherSmem) {
        if (threadIdx.x == 0) atomicExch(a.err, 1);
        return;
    }
    const uint32_t mine = ring + lane * 16u;        // this lane's piece 0 of slot 0
    const uint32_t bA0 = kRegA | (uint32_t)(lane * 4);
    const uint32_t bA1 = kRegA | (uint32_t)(lane * 4 + 128);
    const uint32_t bB = kRegB | (uint32_t)(lane * 4);
    const long long G = gridDim.x;
    const long long u0 = a.total * blockIdx.x / G, u1 = a.total * (blockIdx.x + 1) / G;
    const long long H = (long long)a.mpg * a.qb_per_mat;   // quarters per segment
    const size_t rows_per_chunk = (size_t)a.n_groups * a.mpg * a.M;

    for (long long seg0 = u0; seg0 < u1;) {
        const long long seg = seg0 / H;                   // (group, chunk)
        const long long s_end = (seg + 1) * H < u1 ? (seg + 1) * H : u1;
        const int g = (int)(seg / a.nchunks), c = (int)(seg % a.nchunks);
        const int qs0 = (int)(seg0 - seg * H), qs1 = (int)(s_end - seg * H);
        const int npos = min(kChunk, a.nv - c * kChunk);
        const bool live = lane < npos;
        // this warp's quarters qs0 + warp + NW*i; the first kRing-1 start
        // copying before the table is built
        int qs = qs0 + warp;
        Cursor kc = cursor_at(a, g, qs);                  // next quarter to compute
        Cursor ki = kc;                                   // next quarter to copy
        int qi = qs;
#pragma unroll
        for (int p = 0; p < kRing - 1; p++) {
            issue_quarter<TILED>(mine + (uint32_t)p * 1536u,
                                 qi < qs1 ? quarter_src<TILED>(a, ki, c, lane, npos) : nullptr,
                                 npos, live && qi < qs1);
            if (qi < qs1) cursor_advance(a, g, ki, NW);
            qi += NW;
        }
        int kind0, route0;
        group_mat(a, g, 0, kind0, route0);
        __syncthreads();                                  // previous table done
        if (BUILD) build_table(a, g, c, kind0);
        else copy_image(a, c);
        __syncthreads();

        float *part = a.partial + (size_t)c * rows_per_chunk + (size_t)g * a.mpg * a.M;
        for (int i = 0; qs < qs1; i++, qs += NW) {
            // slot i % kRing holds quarter qs once all but kRing-2 groups landed
            cp_async_wait<kRing - 2>();
            const uint32_t slot = mine + (uint32_t)(i % kRing) * 1536u;
            uint4 q[3];
#pragma unroll
            for (int j = 0; j < 3; j++) q[j] = lds_u4(slot + 512u * j);
            // refill the slot freed last iteration with quarter qs + (kRing-1)*NW
            issue_quarter<TILED>(mine + (uint32_t)((i + kRing - 1) % kRing) * 1536u,
                                 qi < qs1 ? quarter_src<TILED>(a, ki, c, lane, npos) : nullptr,
                                 npos, live && qi < qs1);
            if (qi < qs1) cursor_advance(a, g, ki, NW);
            qi += NW;
            if (!live) q[0] = q[1] = q[2] = make_uint4(0, 0, 0, 0);
            const float sum = quarter<TILED>(q, bA0, bA1, bB);
            const int row = (kc.qb >> 2) * kBlk + (kc.qb & 3) * 16 + (lane & 15);
            if (lane < 16 && row < a.M) part[(size_t)kc.m * a.M + row] = sum;
            cursor_advance(a, g, kc, NW);
        }
        cp_async_wait<0>();                               // nothing in flight at a rebuild
        seg0 = s_end;
    }
}
#undef WARP_QW

// plain LUT [nv][3][256] -> per-chunk images in the bank-sliced layout.
__global__ void lut_slice_kernel(uint32_t *__restrict__ image,
                                 const float *__restrict__ lut, int nv,
                                 int nchunks) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)nchunks * kImageWords) return;
    const int c = (int)(i / kImageWords);
    const uint32_t w = (uint32_t)(i % kImageWords);
    const uint32_t region = w >> 14, off = (w & 16383u) * 4u;   // byte offset
    const int code = (int)(off >> 8), slot = (int)((off >> 7) & 1), p = (int)((off >> 2) & 31);
    const int s = region == 0 ? slot : (slot == 0 ? 2 : -1);
    const int v = c * kChunk + p;
    float val = 0.0f;
    if (s >= 0 && v < nv) val = lut[((size_t)v * kSt + s) * kEnt + code];
    image[i] = __float_as_uint(val);
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
    if ((rc = set_attr((const void *)vq_gather_kernel<false, false>))) return rc;
    if ((rc = set_attr((const void *)vq_gather_kernel<false, true>))) return rc;
    if ((rc = set_attr((const void *)vq_gather_kernel<true, false>))) return rc;
    if ((rc = set_attr((const void *)vq_gather_kernel<true, true>))) return rc;
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

int gather_launch(const GatherArgs &a, bool build, bool tiled, cudaStream_t st) {
    int rc = gather_setup();
    if (rc) return rc;
    if (a.total <= 0) return WARP_OK;
    const int grid = gather_grid(a.total);
    if (build && tiled)
        vq_gather_kernel<true, true><<<grid, kGatherThreads, kGatherSmem, st>>>(a);
    else if (build)
        vq_gather_kernel<false, true><<<grid, kGatherThreads, kGatherSmem, st>>>(a);
    else if (tiled)
        vq_gather_kernel<true, false><<<grid, kGatherThreads, kGatherSmem, st>>>(a);
    else
        vq_gather_kernel<false, false><<<grid, kGatherThreads, kGatherSmem, st>>>(a);
    WARP_CHECK_LAUNCH("vq_gather_kernel");
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
    rc = gather_launch(a, false, false, st);
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

}  // namespace warp
