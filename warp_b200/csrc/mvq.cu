// mvq.cu — trunk / shared-expert dequant-matvec (Q4G, Q8G).
//
// y[b][o] = sum_k f16(ws[o][k]) * sum_i q(o, k*g+i) * x[b][k*g+i], the
// arithmetic of waste_mvq_rows_f32 (model.c:423-519).  HBM-bound: each warp
// streams one row at a time with 128-bit loads, every lane a 16-byte chunk
// (32 Q4 weights or 16 Q8 weights, inside one group because groups are
// multiples of 32), the activations staged once per CTA in shared memory as
// fp32.  A nibble becomes an exact float through the 2^23 magic
// (0x4B000000 | n is 2^23 + n), so the unpack costs an OR and a subtract.
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
__device__ __forceinline__ float silu_mul(float g, float u) {
    return (g / (1.0f + expf(-g))) * u;
}

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

int mvq_launch(MvqArgs a, cudaStream_t st) {
    WARP_ARG(a.bits == 4 || a.bits == 8, "mvq: bits must be 4 or 8 (got %d)", a.bits);
    WARP_ARG(a.group >= 32 && a.group % 32 == 0, "mvq: group must be a multiple of 32");
    a.total_rows = a.seg[0].rows + (a.nseg > 1 ? a.seg[1].rows : 0);
    WARP_ARG(a.nseg >= 1 && a.nseg <= 2 && a.in > 0 && a.total_rows > 0 && a.batch >= 1 &&
                 a.batch <= 16,
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
    a.x_smem = (size_t)a.batch * a.ng * a.group * sizeof(float) * 5 / 4 <= 200 * 1024;
    WARP_ARG(a.x_smem || !a.act_a, "mvq: activation input too large to stage");
    return a.bits == 4 ? launch_bits<4>(a, st) : launch_bits<8>(a, st);
}

}  // namespace warp

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
    return warp::mvq_launch(a, (cudaStream_t)stream);
}
