// mvq.cu — trunk / shared-expert dequant-matvec (Q4G, Q8G).
//
// y[b][o] = sum_k f16(ws[o][k]) * sum_i q(o, k*g+i) * x[b][k*g+i], the
// arithmetic of waste_mvq_rows_f32 (model.c:423-519).  HBM-bound: each warp
// streams one row at a time with 128-bit loads, every lane a 16-byte chunk
// (32 Q4 weights or 16 Q8 weights, inside one group because groups are
// multiples of 32), the activations staged once per CTA in shared memory as
// fp32.  A nibble becomes an exact float through the 2^23 magic
// (0x4B000000 | n is 2^23 + n), so the unpack costs an OR and a subtract.
#include <map>
#include <mutex>

#include "common.cuh"
#include "mvq.cuh"

namespace warp {

constexpr int kMvqThreads = 256;
constexpr int kMvqRowsPerCta = 8;

__device__ __forceinline__ float nib(uint32_t w, int j) {
    return __uint_as_float(0x4B000000u | ((w >> (4 * j)) & 15u)) - 8388616.0f;
}
__device__ __forceinline__ float sbyte(uint32_t w, int j) {
    return (float)(int)(int8_t)(uint8_t)(w >> (8 * j));
}

// Stage X (or, in SwiGLU-input mode, silu(a)*b) as fp32 [batch][in_pad] in
// shared memory, four values per thread step, zero past `in`.

// The staged activations are padded by 16 bytes after every chunk of WPC
// values (xs[b][chunk][WPC + 4]), so the lanes of a warp, which read
// consecutive chunks, start on different bank quads: conflict-free 128-bit
// reads (WPC + 4 = 36 words for Q4, 20 for Q8).
template <int WPC>
__device__ __forceinline__ int xs_index(int in_pad, int b, int k) {
    return b * (in_pad / WPC) * (WPC + 4) + (k / WPC) * (WPC + 4) + (k % WPC);
}

template <int WPC>
__device__ __forceinline__ void stage_x(const MvqArgs &a, float *xs, int in_pad) {
    const int n4 = in_pad / 4;
#pragma unroll 4
    for (int i = threadIdx.x; i < a.batch * n4; i += blockDim.x) {
        const int b = i / n4, k = (i % n4) * 4;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k + 3 < a.in) {
            if (a.act_a) {
                const float4 g = *(const float4 *)(a.act_a + (size_t)b * a.act_stride + k);
                const float4 u = *(const float4 *)(a.act_b + (size_t)b * a.act_stride + k);
                v = make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z),
                                silu_mul(g.w, u.w));
            } else if (a.x_bf16) {
                const uint2 r = *(const uint2 *)((const __nv_bfloat16 *)a.X + (size_t)b * a.in + k);
                v = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u),
                                __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xffff0000u));
            } else {
                v = *(const float4 *)((const float *)a.X + (size_t)b * a.in + k);
            }
        } else {
            float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int j = 0; j < 4 && k + j < a.in; j++) {
                if (a.act_a)
                    t[j] = silu_mul(a.act_a[(size_t)b * a.act_stride + k + j],
                                    a.act_b[(size_t)b * a.act_stride + k + j]);
                else if (a.x_bf16)
                    t[j] = __bfloat162float(((const __nv_bfloat16 *)a.X)[(size_t)b * a.in + k + j]);
                else
                    t[j] = ((const float *)a.X)[(size_t)b * a.in + k + j];
            }
            v = make_float4(t[0], t[1], t[2], t[3]);
        }
        *(float4 *)(xs + xs_index<WPC>(in_pad, b, k)) = v;
    }
}

// One row of one tensor against every batch column: acc[b] =
// sum_k f16(ws[k]) * sum_i q(k*g + i) * x[b][k*g + i], lane-partial.
template <int BITS, int MAXB>
__device__ __forceinline__ void row_dot(const MvqArgs &a, const uint8_t *W,
                                        const uint16_t *ws, const float *xs, int in_pad,
                                        float (&acc)[MAXB]) {
    const int lane = threadIdx.x & 31;
    constexpr int WPC = BITS == 4 ? 32 : 16;          // weights per 16-byte chunk
    const int nchunk = min((int)(a.rowbytes / 16), (a.in + WPC - 1) / WPC);
#pragma unroll
    for (int b = 0; b < MAXB; b++) acc[b] = 0.0f;
#pragma unroll 4
    for (int c = lane; c < nchunk; c += 32) {
        const int k0 = c * WPC;
        const uint4 q = ldg_stream(W + (size_t)c * 16);
        const float s = f16_to_f32(ws[a.group_shift >= 0 ? k0 >> a.group_shift : k0 / a.group]);
        if (BITS == 4 && a.x_smem) {
            // Q4 against staged activations: each nibble becomes the magic
            // float 2^23 + n by one byte permute (even nibbles from w &
            // 0x0F0F0F0F, odd ones from (w >> 4) & 0x0F0F0F0F), pairs drop
            // 2^23 + 8 with one packed subtract (exact), and the dot runs as
            // two interleaved fp32 chains of packed FMAs.
            const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
            float2 wp[16];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const uint32_t lo = w4[t] & 0x0F0F0F0Fu, hi = (w4[t] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                for (int m = 0; m < 4; m++)
                    wp[4 * t + m] = __fadd2_rn(
                        make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650u | m)),
                                    __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650u | m))),
                        make_float2(-8388616.0f, -8388616.0f));
            }
#pragma unroll
            for (int b = 0; b < MAXB; b++) {
                if (b >= a.batch) break;
                const float4 *xp = (const float4 *)(xs + xs_index<WPC>(in_pad, b, k0));
                float2 part2 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int i = 0; i < WPC / 4; i++) {
                    const float4 xv = xp[i];
                    part2 = __ffma2_rn(wp[2 * i], make_float2(xv.x, xv.y), part2);
                    part2 = __ffma2_rn(wp[2 * i + 1], make_float2(xv.z, xv.w), part2);
                }
                acc[b] = __fmaf_rn(s, __fadd_rn(part2.x, part2.y), acc[b]);
            }
            continue;
        }
        const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
        float wf[WPC];
#pragma unroll
        for (int t = 0; t < 4; t++) {
            if (BITS == 4) {
#pragma unroll
                for (int j = 0; j < 8; j++) wf[t * 8 + j] = nib(w4[t], j);
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) wf[t * 4 + j] = sbyte(w4[t], j);
            }
        }
#pragma unroll
        for (int b = 0; b < MAXB; b++) {
            if (b >= a.batch) break;
            float part = 0.0f;
            if (a.x_smem) {
                const float4 *xp = (const float4 *)(xs + xs_index<WPC>(in_pad, b, k0));
#pragma unroll
                for (int i = 0; i < WPC / 4; i++) {
                    const float4 xv = xp[i];
                    part = __fmaf_rn(wf[4 * i + 0], xv.x, part);
                    part = __fmaf_rn(wf[4 * i + 1], xv.y, part);
                    part = __fmaf_rn(wf[4 * i + 2], xv.z, part);
                    part = __fmaf_rn(wf[4 * i + 3], xv.w, part);
                }
            } else {
#pragma unroll
                for (int i = 0; i < WPC; i++) {
                    const int k = k0 + i;
                    float xv = 0.0f;
                    if (k < a.in)
                        xv = a.x_bf16
                            ? __bfloat162float(((const __nv_bfloat16 *)a.X)[(size_t)b * a.in + k])
                            : ((const float *)a.X)[(size_t)b * a.in + k];
                    part = __fmaf_rn(wf[i], xv, part);
                }
            }
            acc[b] = __fmaf_rn(s, part, acc[b]);
        }
    }
#pragma unroll
    for (int b = 0; b < MAXB; b++) {
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], m);
    }
}

template <int BITS, int MAXB>
__global__ void __launch_bounds__(kMvqThreads)
mvq_kernel(const MvqArgs a) {
    extern __shared__ __align__(16) float xs[];      // [batch][in_pad] or unused
    const int in_pad = a.ng * a.group;
    const int nrows = a.pair ? a.seg[0].rows : a.total_rows;
    // stream this CTA's rows into L2 while the activations are staged
    if (threadIdx.x < 32) {
        const int r0 = blockIdx.x * kMvqRowsPerCta;
        const int r1 = min(nrows, r0 + kMvqRowsPerCta);
        for (int sgi = 0; sgi < a.nseg; sgi++) {
            const int lo = (a.pair || sgi == 0) ? 0 : a.seg[0].rows;
            const int hi = lo + a.seg[sgi].rows;
            const int b0 = max(r0, lo), b1 = min(r1, hi);
            if (b0 >= b1) continue;
            const uint8_t *p = a.seg[sgi].W + (size_t)(b0 - lo) * a.rowbytes;
            const size_t bytes = (size_t)(b1 - b0) * a.rowbytes;
            for (size_t off = (size_t)threadIdx.x * 32768; off < bytes; off += 32 * 32768)
                prefetch_l2_bulk(p + off, (uint32_t)min((size_t)32768, bytes - off));
        }
    }
    if (a.x_smem) {
        stage_x<BITS == 4 ? 32 : 16>(a, xs, in_pad);
        __syncthreads();
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r_end = min(nrows, (int)(blockIdx.x + 1) * kMvqRowsPerCta);
    for (int row = blockIdx.x * kMvqRowsPerCta + warp; row < r_end;
         row += kMvqThreads / 32) {
        if (a.pair) {
            // gate row and up row together; y = silu(gate) * up
            float g[MAXB], u[MAXB];
            row_dot<BITS, MAXB>(a, a.seg[0].W + (size_t)row * a.rowbytes,
                                a.seg[0].ws + (size_t)row * a.ng, xs, in_pad, g);
            row_dot<BITS, MAXB>(a, a.seg[1].W + (size_t)row * a.rowbytes,
                                a.seg[1].ws + (size_t)row * a.ng, xs, in_pad, u);
            if (lane == 0)
#pragma unroll
                for (int b = 0; b < MAXB; b++)
                    if (b < a.batch) a.Y[(size_t)b * a.y_stride + row] = silu_mul(g[b], u[b]);
        } else {
            const MvqSeg &sg = row < a.seg[0].rows ? a.seg[0] : a.seg[1];
            const int r = row < a.seg[0].rows ? row : row - a.seg[0].rows;
            float acc[MAXB];
            row_dot<BITS, MAXB>(a, sg.W + (size_t)r * a.rowbytes, sg.ws + (size_t)r * a.ng,
                                xs, in_pad, acc);
            if (lane == 0)
#pragma unroll
                for (int b = 0; b < MAXB; b++)
                    if (b < a.batch) a.Y[(size_t)b * a.y_stride + sg.y_off + r] = acc[b];
        }
    }
}

template <int BITS>
static int launch_bits(const MvqArgs &a, cudaStream_t st) {
    constexpr int WPC = BITS == 4 ? 32 : 16;
    const size_t smem = a.x_smem ? (size_t)a.batch * (a.ng * a.group / WPC) * (WPC + 4) *
                                       sizeof(float)
                                 : 0;
    const unsigned grid = cdiv(a.pair ? a.seg[0].rows : a.total_rows, kMvqRowsPerCta);
#define WARP_MVQ_CASE(B)                                                         \
    if (a.batch <= B) {                                                          \
        auto fn = mvq_kernel<BITS, B>;                                          \
        if (smem > 48 * 1024) {                                                  \
            cudaError_t e = cudaFuncSetAttribute(                                \
                fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);     \
            if (e != cudaSuccess) return cuda_fail(e, "mvq smem attribute");    \
        }                                                                        \
        fn<<<grid, kMvqThreads, smem, st>>>(a);                                 \
        WARP_CHECK_LAUNCH("mvq_kernel");                                         \
        return WARP_OK;                                                          \
    }
    WARP_MVQ_CASE(1)
    WARP_MVQ_CASE(2)
    WARP_MVQ_CASE(4)
    WARP_MVQ_CASE(8)
    WARP_MVQ_CASE(16)
#undef WARP_MVQ_CASE
    set_error("mvq: batch %d above 16", a.batch);
    return WARP_E_ARG;
}

// ------------------------------------------- the block-split down matvec --
//
// The shared expert's down projection in nb fixed column blocks of gpb
// groups.  The partial of (row o, block b) has one definition, whichever
// launch computes it: lane l of an L-lane team (L = gpb rounded up to a power
// of two, at most 32) takes the block's groups l, l + L, ... in order, each
// group a run of 16-byte pieces whose dots (piece_dot) are added in order
// and then scaled into the lane's sum, and the team meets in an xor tree
// (m = 1, 2, ..., L / 2).
//  * split launch (an expert-parallel rank's blocks [b0, b1)): one block per
//    grid row, a warp = 32 / L rows of it; the partials go to P + b * pb +
//    t * pt and the combine adds them in block order;
//  * folded launch (every block on this GPU): a warp per row, its 32 / L
//    teams taking blocks b0 + team, b0 + team + 32 / L, ...; the team
//    leaders park the partials in shared memory and the row's fold
//    0 + p_b0 + p_b0+1 + ... (the combine's order) goes to P + t * pt.  The
//    same bits as the split launches summed by the combine, from a launch
//    shaped like the plain matvec (a warp streaming one row, the CTA's rows
//    prefetched into L2 while the activations are staged).
// Activations: silu(act_a) * act_b of the launch's columns, staged once per
// CTA in the padded chunk layout of row_dot (conflict-free 128-bit reads).

constexpr int kBlkThreads = 256;
constexpr int kBlkWarps = kBlkThreads / 32;
constexpr int kBlkMaxNb = 8;

// One 16-byte piece (32 Q4 or 16 Q8 weights) against staged activations.
template <int BITS>
__device__ __forceinline__ float piece_dot(const uint4 q, const float *xs) {
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
    const float4 *xp = (const float4 *)xs;
    if (BITS == 4) {
        // nibble pairs (2i, 2i + 1) as exact floats, two interleaved chains
        float2 part2 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t lo = w4[t] & 0x0F0F0F0Fu, hi = (w4[t] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int m = 0; m < 4; m += 2) {
                const float2 wa = __fadd2_rn(
                    make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650u | m)),
                                __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650u | m))),
                    make_float2(-8388616.0f, -8388616.0f));
                const float2 wb = __fadd2_rn(
                    make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7651u | m)),
                                __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7651u | m))),
                    make_float2(-8388616.0f, -8388616.0f));
                const float4 xv = xp[2 * t + m / 2];
                part2 = __ffma2_rn(wa, make_float2(xv.x, xv.y), part2);
                part2 = __ffma2_rn(wb, make_float2(xv.z, xv.w), part2);
            }
        }
        return __fadd_rn(part2.x, part2.y);
    } else {
        float part = 0.0f;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const float4 xv = xp[t];
            part = __fmaf_rn(sbyte(w4[t], 0), xv.x, part);
            part = __fmaf_rn(sbyte(w4[t], 1), xv.y, part);
            part = __fmaf_rn(sbyte(w4[t], 2), xv.z, part);
            part = __fmaf_rn(sbyte(w4[t], 3), xv.w, part);
        }
        return part;
    }
}

// Lane l's share of the partial of (row o, block b), every batch column,
// then the team's xor tree.  Every lane of the warp calls it together
// (`live` false: zeros into the tree).
template <int BITS, int MAXB>
__device__ __forceinline__ void block_partial(const MvqBlocks &a, const float *xs, int ncols,
                                              int cs, int o, int b, int l, int L, bool live,
                                              float (&acc)[MAXB]) {
    constexpr int WPC = 128 / BITS;                       // weights per 16-byte piece
    const int cpb = a.in / a.nb, gpb = cpb / a.group, ppg = a.group / WPC;
    const int ng = a.in / a.group;
#pragma unroll
    for (int t = 0; t < MAXB; t++) acc[t] = 0.0f;
    if (live) {
        const uint8_t *wr = a.W + (size_t)o * a.rowbytes;
        const uint16_t *sr = a.ws + (size_t)o * ng;
        for (int k = l; k < gpb; k += L) {
            const int gi = b * gpb + k;
            const float s = f16_to_f32(sr[gi]);
            float gv[MAXB];
            for (int j = 0; j < ppg; j++) {
                const uint4 q = ldg_stream(wr + ((size_t)gi * ppg + j) * 16);
                const int col = gi * a.group + j * WPC - cs;
#pragma unroll
                for (int t = 0; t < MAXB; t++) {
                    if (t >= a.batch) break;
                    const float v = piece_dot<BITS>(q, xs + xs_index<WPC>(ncols, t, col));
                    gv[t] = j == 0 ? v : __fadd_rn(gv[t], v);
                }
            }
#pragma unroll
            for (int t = 0; t < MAXB; t++)
                if (t < a.batch) acc[t] = __fmaf_rn(s, gv[t], acc[t]);
        }
    }
    for (int m = 1; m < L; m <<= 1)
#pragma unroll
        for (int t = 0; t < MAXB; t++) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], m);
}

template <int BITS, int MAXB>
__global__ void __launch_bounds__(kBlkThreads)
mvq_blocks_kernel(const MvqBlocks a, int L) {
    extern __shared__ __align__(16) float xs[];          // [batch][ncols] padded
    __shared__ float park[kBlkWarps][kBlkMaxNb][MAXB];   // folded launch: the partials
    constexpr int WPC = 128 / BITS;
    const int cpb = a.in / a.nb;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int team = lane / L, l = lane - team * L, nteam = 32 / L;
    // the staged columns: the grid row's block, or every block of the launch
    const int cs = a.fold ? a.b0 * cpb : (a.b0 + blockIdx.y) * cpb;
    const int ncols = a.fold ? (a.b1 - a.b0) * cpb : cpb;
    if (a.fold && threadIdx.x < 32) {
        const int r0 = blockIdx.x * kBlkWarps, r1 = min(a.rows, r0 + kBlkWarps);
        const uint8_t *p = a.W + (size_t)r0 * a.rowbytes;
        const size_t bytes = (size_t)max(r1 - r0, 0) * a.rowbytes;
        for (size_t off = (size_t)threadIdx.x * 32768; off < bytes; off += 32 * 32768)
            prefetch_l2_bulk(p + off, (uint32_t)min((size_t)32768, bytes - off));
    }
    const int n4 = ncols / 4;
    for (int i = threadIdx.x; i < a.batch * n4; i += kBlkThreads) {
        const int t = i / n4, k = (i - t * n4) * 4;
        const size_t q = (size_t)t * a.act_stride + cs + k;
        const float4 g = *(const float4 *)(a.act_a + q);
        float4 v = g;
        if (a.act_b) {
            const float4 u = *(const float4 *)(a.act_b + q);
            v = make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z),
                            silu_mul(g.w, u.w));
        }
        *(float4 *)(xs + xs_index<WPC>(ncols, t, k)) = v;
    }
    __syncthreads();
    float acc[MAXB];
    if (!a.fold) {
        const int b = a.b0 + blockIdx.y;
        const int o = (blockIdx.x * kBlkWarps + warp) * nteam + team;
        const bool live = o < a.rows;
        block_partial<BITS, MAXB>(a, xs, ncols, cs, o, b, l, L, live, acc);
        if (live && l == 0)
#pragma unroll
            for (int t = 0; t < MAXB; t++)
                if (t < a.batch)
                    a.P[(size_t)b * a.pb_stride + (size_t)t * a.pt_stride + o] = acc[t];
        return;
    }
    const int o = blockIdx.x * kBlkWarps + warp;
    if (o >= a.rows) return;                              // whole warp: no shuffle partner lost
    const int nown = a.b1 - a.b0;
    for (int p0 = 0; p0 < nown; p0 += nteam) {
        const int bi = p0 + team;
        block_partial<BITS, MAXB>(a, xs, ncols, cs, o, a.b0 + bi, l, L, bi < nown, acc);
        if (l == 0 && bi < nown)
#pragma unroll
            for (int t = 0; t < MAXB; t++)
                if (t < a.batch) park[warp][bi][t] = acc[t];
    }
    __syncwarp();
    if (lane < a.batch) {
        float f = 0.0f;
        for (int bi = 0; bi < nown; bi++) f = __fadd_rn(f, park[warp][bi][lane]);
        a.P[(size_t)lane * a.pt_stride + o] = f;
    }
}

int mvq_blocks_launch(const MvqBlocks &a, cudaStream_t st) {
    WARP_ARG(a.bits == 4 || a.bits == 8, "mvq blocks: bits must be 4 or 8");
    WARP_ARG(a.nb >= 1 && a.nb <= kBlkMaxNb && a.group % 32 == 0 &&
                 a.in % (a.nb * a.group) == 0 && a.b0 >= 0 && a.b0 <= a.b1 && a.b1 <= a.nb &&
                 a.batch >= 1 && a.batch <= 16,
             "mvq blocks: in must be a whole number of groups per block (nb 1..8), batch 1..16");
    WARP_ARG(a.rowbytes % 16 == 0 && ((uintptr_t)a.W & 15) == 0 &&
                 (size_t)a.in * a.bits / 8 <= a.rowbytes,
             "mvq blocks: rows must be 16-byte aligned");
    WARP_ARG(((uintptr_t)a.act_a & 15) == 0 && ((uintptr_t)a.act_b & 15) == 0 &&
                 a.act_stride % 4 == 0,
             "mvq blocks: activations must be 16-byte aligned");
    if (a.b1 == a.b0) return WARP_OK;
    const int cpb = a.in / a.nb;
    const int ncols = a.fold ? (a.b1 - a.b0) * cpb : cpb;
    const int wpc = 128 / a.bits;                        // the padded layout's chunk
    const size_t smem = (size_t)a.batch * (ncols / wpc) * (wpc + 4) * sizeof(float);
    const int gpb = cpb / a.group;
    int L = 1;
    while (L < gpb && L < 32) L <<= 1;
    const dim3 grid = a.fold ? dim3(cdiv(a.rows, kBlkWarps))
                             : dim3(cdiv(a.rows, kBlkWarps * (32 / L)), a.b1 - a.b0);
#define WARP_BLK_CASE(B)                                                               \
    if (a.batch <= B) {                                                                \
        auto fn = a.bits == 4 ? mvq_blocks_kernel<4, B> : mvq_blocks_kernel<8, B>;     \
        if (smem > 40 * 1024) {                                                        \
            cudaError_t e = cudaFuncSetAttribute(                                      \
                fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);           \
            if (e != cudaSuccess) return cuda_fail(e, "mvq blocks smem attribute");    \
        }                                                                              \
        fn<<<grid, kBlkThreads, smem, st>>>(a, L);                                     \
        WARP_CHECK_LAUNCH("mvq_blocks_kernel");                                        \
        return WARP_OK;                                                                \
    }
    WARP_BLK_CASE(1)
    WARP_BLK_CASE(4)
    WARP_BLK_CASE(16)
#undef WARP_BLK_CASE
    return WARP_E_ARG;
}

int mvq_launch(MvqArgs a, cudaStream_t st) {
    WARP_ARG(a.bits == 4 || a.bits == 8, "mvq: bits must be 4 or 8 (got %d)", a.bits);
    WARP_ARG(a.group >= 32 && a.group % 32 == 0, "mvq: group must be a multiple of 32");
    a.total_rows = a.seg[0].rows + (a.nseg > 1 ? a.seg[1].rows : 0);
    WARP_ARG(a.nseg >= 1 && a.nseg <= 2 && a.in > 0 && a.total_rows > 0 && a.batch >= 1,
             "mvq: bad shape (nseg %d, in %d, rows %d, batch %d)", a.nseg, a.in,
             a.total_rows, a.batch);
    WARP_ARG(a.rowbytes % 16 == 0, "mvq: rowbytes must be a multiple of 16");
    a.ng = (a.in + a.group - 1) / a.group;
    a.group_shift = (a.group & (a.group - 1)) == 0 ? __builtin_ctz(a.group) : -1;
    WARP_ARG(a.rowbytes >= (size_t)a.ng * a.group * a.bits / 8,
             "mvq: rowbytes shorter than the padded row");
    for (int i = 0; i < a.nseg; i++)
        WARP_ARG(((uintptr_t)a.seg[i].W & 15) == 0, "mvq: W must be 16-byte aligned");
    WARP_ARG(!a.pair || (a.nseg == 2 && a.seg[0].rows == a.seg[1].rows),
             "mvq: pair mode needs two tensors of equal rows");
    WARP_ARG(!a.act_a || ((uintptr_t)a.act_a % 16 == 0 && (uintptr_t)a.act_b % 16 == 0 &&
                          a.act_stride % 4 == 0),
             "mvq: activation inputs must be 16-byte aligned");
    WARP_ARG(a.x_bf16 || ((uintptr_t)a.X % 16 == 0 && a.in % 4 == 0) || a.act_a,
             "mvq: fp32 activations must be 16-byte aligned with in a multiple of 4");
    WARP_ARG(!a.x_bf16 || ((uintptr_t)a.X % 8 == 0 && a.in % 4 == 0),
             "mvq: bf16 activations must be 8-byte aligned with in a multiple of 4");
    // batch 1: the CUDA-core kernel streams rows with 16-byte loads per lane
    // (7168 x 18432 Q4: 68 us against 98 on the tensor cores); batch >= 2
    // with scratch: the tcgen05 matmul (mvq_umma.cu), which reads the weights
    // once for every token of the launch
    if (a.xf && !a.pair && a.batch >= 2) {
        WARP_ARG(a.batch <= kMvqMaxBatch, "mvq: the tensor-core path takes batch 2..64 (got %d)",
                 a.batch);
        WARP_ARG(((uintptr_t)a.xf & 255) == 0, "mvq: tensor-core scratch must be 256-byte aligned");
        return launch_umma(a, st);
    }
    // The CUDA-core kernel stages the activations in shared memory.  When a
    // batch does not fit, it runs as several launches of the largest batch
    // that does, so every token always takes the staged path and gets the
    // same arithmetic whatever the batch (the expert-parallel shared expert
    // relies on that for bit-identity with one GPU).
    const size_t per_tok = (size_t)a.ng * a.group * sizeof(float) * 5 / 4;
    const int bmax = min(16, (int)((200 * 1024) / per_tok));
    if (bmax >= 1) {
        a.x_smem = 1;
        const size_t xb = a.x_bf16 ? 2 : 4;
        for (int b0 = 0; b0 < a.batch; b0 += bmax) {
            MvqArgs p = a;
            p.batch = min(bmax, a.batch - b0);
            if (p.X) p.X = (const uint8_t *)a.X + (size_t)b0 * a.in * xb;
            if (p.act_a) {
                p.act_a = a.act_a + (size_t)b0 * a.act_stride;
                p.act_b = a.act_b + (size_t)b0 * a.act_stride;
            }
            p.Y = a.Y + (size_t)b0 * a.y_stride;
            const int rc = a.bits == 4 ? launch_bits<4>(p, st) : launch_bits<8>(p, st);
            if (rc) return rc;
        }
        return WARP_OK;
    }
    a.x_smem = 0;
    WARP_ARG(!a.act_a, "mvq: activation input too large to stage");
    WARP_ARG(a.batch <= 16, "mvq: batch %d above 16 for an input this wide", a.batch);
    return a.bits == 4 ? launch_bits<4>(a, st) : launch_bits<8>(a, st);
}

}  // namespace warp

// The tensor-core path's fragment scratch for warp_mvq_matvec: one buffer per
// (device, stream), grown (cudaMalloc, which synchronises the device) only
// when a call needs more than any before it on that stream, never freed per
// call.  Work on one stream is ordered, so reusing its buffer is safe; two
// streams never share one.
namespace {
struct XfCache {
    std::mutex mu;
    std::map<std::pair<int, cudaStream_t>, std::pair<void *, size_t>> bufs;
};
XfCache &xf_cache() {
    static XfCache *c = new XfCache();           // never destroyed: lives past atexit users
    return *c;
}
}  // namespace

static int xf_scratch(cudaStream_t st, size_t bytes, void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return warp::cuda_fail(e, "warp_mvq_matvec: cudaGetDevice");
    XfCache &c = xf_cache();
    std::lock_guard<std::mutex> lk(c.mu);
    auto &slot = c.bufs[{dev, st}];
    if (slot.second < bytes) {
        if (slot.first) cudaFree(slot.first);
        slot = {nullptr, 0};
        void *p = nullptr;
        e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return warp::cuda_fail(e, "warp_mvq_matvec scratch");
        slot = {p, bytes};
    }
    *out = slot.first;
    return WARP_OK;
}

extern "C" int warp_mvq_matvec(const void *W, const uint16_t *ws, const void *X,
                               int x_bf16, float *Y, int batch, int out, int in,
                               int group, int bits, size_t rowbytes,
                               void *stream) {
    WARP_ARG(W && ws && X && Y, "warp_mvq_matvec: NULL pointer");
    warp::MvqArgs a = {};
    a.seg[0] = {(const uint8_t *)W, ws, out, 0};
    a.nseg = 1;
    a.total_rows = out;
    a.in = in;
    a.group = group;
    a.bits = bits;
    a.rowbytes = rowbytes;
    a.batch = batch;
    a.X = X;
    a.x_bf16 = x_bf16;
    a.Y = Y;
    a.y_stride = out;
    WARP_ARG(batch >= 1 && batch <= warp::kMvqMaxBatch, "warp_mvq_matvec: batch %d not in 1..%d",
             batch, warp::kMvqMaxBatch);
    cudaStream_t st = (cudaStream_t)stream;
    if (batch >= 2 && in >= 1) {
        void *xf = nullptr;
        const int rc = xf_scratch(st, warp::mvq_xf_bytes(batch, in, out), &xf);
        if (rc) return rc;
        a.xf = xf;
    }
    return warp::mvq_launch(a, st);
}
