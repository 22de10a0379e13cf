// vq.cu — VQ3R kernels: exact LUT build, ordered apply, dequant, encoder.
//
// The bandwidth gather (the decode hot loop) lives in vq_gather.cuh; this
// file holds the kernels whose results are bit-exact against the reference
// and the C-ABI wrappers for all of them.
#include "common.cuh"
#include "vq_gather.cuh"

namespace warp {

// lutb_range_avx512 (simd_avx512.c:90-127): one FMA chain over d = 0..7
// from 0 per table entry.  Thread per entry; the eight x values of a
// position are uniform across a warp (same v), the codebook column is
// coalesced across c.
__global__ void lut_build_kernel(float *__restrict__ lut,
                                 const float *__restrict__ booksT,
                                 const float *__restrict__ x, int nv,
                                 int cb_base) {
    const int c = threadIdx.x;                 // 256 threads = entries
    const int vs = blockIdx.x;                 // v * 3 + s
    const int v = vs / kSt, s = vs % kSt;
    if (v >= nv) return;
    const float *CT = booksT + (size_t)(cb_base + s) * kEnt * kVec;
    const float *xv = x + (size_t)v * kVec;
    float t = 0.0f;
#pragma unroll
    for (int d = 0; d < kVec; d++) t = __fmaf_rn(xv[d], CT[d * kEnt + c], t);
    lut[(size_t)vs * kEnt + c] = t;
}

// vq_rows (model.c:3909-3977) with the reference's accumulation order: one
// thread per row, v ascending, ((T0 + T1) + T2) then into the running sum,
// times f16(scale) at the end.  The precedent is the Metal vq3r kernel
// (metal.m:143-162), which keeps the CPU order for the same reason.
__global__ void vq_apply_ordered_kernel(float *__restrict__ y,
                                        const uint8_t *__restrict__ idx,
                                        const uint16_t *__restrict__ scale,
                                        const float *__restrict__ lut, int M,
                                        int nv) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= M) return;
    const int rb = r / kBlk, ri = r % kBlk;
    float acc = 0.0f;
    for (int v = 0; v < nv; v++) {
        const float *blk = lut + (size_t)v * kSt * kEnt;
        const uint8_t *ix = idx + (((size_t)rb * nv + v) * kBlk + ri) * kSt;
        const float t = __fadd_rn(__fadd_rn(blk[ix[0]], blk[kEnt + ix[1]]),
                                  blk[2 * kEnt + ix[2]]);
        acc = __fadd_rn(acc, t);
    }
    y[r] = __fmul_rn(acc, f16_to_f32(scale[r]));
}

// Dequantized matrix, kimi_ref.py:262-270 order: ((0 + C0) + C1) + C2, then
// times the row's fp16 scale.  Thread per (row, vector position).
__global__ void vq_dequant_kernel(float *__restrict__ W,
                                  const uint8_t *__restrict__ idx,
                                  const uint16_t *__restrict__ scale,
                                  const float *__restrict__ books, int M,
                                  int N, int cb_base) {
    const int nv = N / kVec;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)M * nv) return;
    const int r = (int)(i / nv), v = (int)(i % nv);
    const int rb = r / kBlk, ri = r % kBlk;
    const uint8_t *ix = idx + (((size_t)rb * nv + v) * kBlk + ri) * kSt;
    const float sc = f16_to_f32(scale[r]);
    const float4 *C0 = (const float4 *)(books + ((size_t)(cb_base + 0) * kEnt + ix[0]) * kVec);
    const float4 *C1 = (const float4 *)(books + ((size_t)(cb_base + 1) * kEnt + ix[1]) * kVec);
    const float4 *C2 = (const float4 *)(books + ((size_t)(cb_base + 2) * kEnt + ix[2]) * kVec);
    float4 *out = (float4 *)(W + (size_t)r * N + (size_t)v * kVec);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const float4 a = C0[h], b = C1[h], c = C2[h];
        float4 o;
        o.x = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, a.x), b.x), c.x), sc);
        o.y = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, a.y), b.y), c.y), sc);
        o.z = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, a.z), b.z), c.z), sc);
        o.w = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, a.w), b.w), c.w), sc);
        out[h] = o;
    }
}

// waste_vq_encode (vq.c:50-105), scalar branch: squared distance summed in d
// order (separate multiply and add), strict `<` so the lowest index wins,
// residual = v - C[best], stages in one pass.  The codebooks sit in shared
// memory; each thread encodes one vector.
__global__ void vq_encode_kernel(const float *__restrict__ X, int64_t n,
                                 const float *__restrict__ books, int stages,
                                 uint8_t *__restrict__ codes) {
    extern __shared__ float sbooks[];          // [stages][256][8]
    for (int i = threadIdx.x; i < stages * kEnt * kVec; i += blockDim.x)
        sbooks[i] = books[i];
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float cur[kVec];
        const float4 *xp = (const float4 *)(X + i * kVec);
        const float4 lo = xp[0], hi = xp[1];
        cur[0] = lo.x; cur[1] = lo.y; cur[2] = lo.z; cur[3] = lo.w;
        cur[4] = hi.x; cur[5] = hi.y; cur[6] = hi.z; cur[7] = hi.w;
        for (int s = 0; s < stages; s++) {
            const float *C = sbooks + s * kEnt * kVec;
            int best = 0;
            float bestd = __int_as_float(0x7f800000);
            for (int c = 0; c < kEnt; c++) {
                const float4 e0 = *(const float4 *)(C + c * kVec);
                const float4 e1 = *(const float4 *)(C + c * kVec + 4);
                const float e[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
                float d = 0.0f;
#pragma unroll
                for (int j = 0; j < kVec; j++) {
                    const float t = __fsub_rn(cur[j], e[j]);
                    d = __fadd_rn(d, __fmul_rn(t, t));
                }
                if (d < bestd) { bestd = d; best = c; }
            }
            codes[i * stages + s] = (uint8_t)best;
#pragma unroll
            for (int j = 0; j < kVec; j++)
                cur[j] = __fsub_rn(cur[j], C[best * kVec + j]);
        }
    }
}

int vq_apply_ordered_launch(float *y, const uint8_t *idx, const uint16_t *scale,
                            const float *lut, int M, int nv, cudaStream_t st) {
    vq_apply_ordered_kernel<<<cdiv(M, 128), 128, 0, st>>>(y, idx, scale, lut, M, nv);
    WARP_CHECK_LAUNCH("vq_apply_ordered_kernel");
    return WARP_OK;
}

}  // namespace warp

using namespace warp;

extern "C" int warp_vq_lut_build(float *lut, const float *booksT,
                                 const float *x, int nv, int cb_base,
                                 void *stream) {
    WARP_ARG(lut && booksT && x && nv > 0 && cb_base >= 0,
             "warp_vq_lut_build: bad arguments");
    lut_build_kernel<<<nv * kSt, kEnt, 0, (cudaStream_t)stream>>>(
        lut, booksT, x, nv, cb_base);
    WARP_CHECK_LAUNCH("lut_build_kernel");
    return WARP_OK;
}

extern "C" int warp_vq_apply(float *y, const uint8_t *idx,
                             const uint16_t *scale, const float *lut, int M,
                             int nv, int ordered, void *stream) {
    WARP_ARG(y && idx && scale && lut && M > 0 && nv > 0,
             "warp_vq_apply: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    if (ordered) {
        return vq_apply_ordered_launch(y, idx, scale, lut, M, nv, st);
    }
    return vq_apply_gather(y, idx, scale, lut, M, nv, st);
}

extern "C" int warp_vq_apply_noalloc(float *y, const uint8_t *idx,
                                     const uint16_t *scale, const float *lut,
                                     int M, int nv, void *stream) {
    WARP_ARG(y && idx && scale && lut && M > 0 && nv > 0,
             "warp_vq_apply_noalloc: bad arguments");
    return vq_apply_gather_noalloc(y, idx, scale, lut, M, nv, (cudaStream_t)stream);
}

extern "C" int warp_vq_dequant(float *W, const uint8_t *idx,
                               const uint16_t *scale, const float *books,
                               int M, int N, int cb_base, void *stream) {
    WARP_ARG(W && idx && scale && books && M > 0 && N > 0 && N % kVec == 0 &&
                 cb_base >= 0,
             "warp_vq_dequant: bad arguments (N must be a multiple of 8)");
    const size_t n = (size_t)M * (N / kVec);
    vq_dequant_kernel<<<cdiv(n, 256), 256, 0, (cudaStream_t)stream>>>(
        W, idx, scale, books, M, N, cb_base);
    WARP_CHECK_LAUNCH("vq_dequant_kernel");
    return WARP_OK;
}

extern "C" int warp_vq_encode(const float *X, int64_t n, const float *books,
                              int stages, uint8_t *codes, void *stream) {
    WARP_ARG(X && books && codes && n >= 0 && stages >= 1 && stages <= 4,
             "warp_vq_encode: bad arguments");
    WARP_ARG(((uintptr_t)X & 15) == 0 && ((uintptr_t)books & 15) == 0,
             "warp_vq_encode: X and books must be 16-byte aligned");
    if (n == 0) return WARP_OK;
    const size_t smem = (size_t)stages * kEnt * kVec * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(
            vq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
            (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "vq_encode smem");
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = (n + 255) / 256;
    const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
    vq_encode_kernel<<<grid, 256, smem, (cudaStream_t)stream>>>(X, n, books,
                                                                stages, codes);
    WARP_CHECK_LAUNCH("vq_encode_kernel");
    return WARP_OK;
}
