// vq4p.cu — the VQ4P format: four residual stages of 64 entries, the four
// 6-bit indices of a (row, vector position) packed into three bytes
// (FORMAT.md "VQ4P record"), applied through an int8 table.
//
//  * vq4p_lut_kernel: the fp32 table of x for every position, stage and
//    entry (the FMA chain of lutb_range, model.c:3815-3852, over 64-entry
//    books), then vq_quant_lut (model.c:3996-4068): per block of 32
//    positions, mx = max |entry|, scale = mx / 127, entries rounded to
//    nearest (even) of entry * (127 / mx) and clamped to [-127, 127].  One
//    CTA of 1024 threads per block, the four books and the block's
//    positions staged in shared memory: the table of the block sits there
//    between the two passes, and the max is exact whatever the order.
//  * vq4p_apply_kernel: waste_vq_rows_p6 (model.c:4076-4113).  Per row and
//    block of 32 positions the integer sum of the four lookups of every
//    position (exact in any order), then acc += scale[blk] * sum in block
//    order (fp32 multiply, then add), y = acc * f16(row scale).  A CTA owns
//    one 64-row index block: eight groups of 64 threads take every eighth
//    position block (a thread per row, reading its row's three bytes, so a
//    warp's reads are 96 contiguous bytes, eight positions' loads in flight
//    at a time), park the integer sums in shared memory, and a thread per
//    row folds them in block order.  Bit-exact
//    against the format's portable kernel.
#include "common.cuh"

namespace warp {

constexpr int kP6En = 64, kP6St = 4, kP6Blk = 32;
constexpr int kP6LutThreads = 1024;

__global__ void __launch_bounds__(kP6LutThreads)
vq4p_lut_kernel(int8_t *__restrict__ q, float *__restrict__ lscale,
                const float *__restrict__ booksT, const float *__restrict__ x, int nv,
                int cb_base) {
    __shared__ float tab[kP6Blk * kP6St * kP6En];             // 32 KiB
    __shared__ float bk[kP6St * kVec * kP6En];                // the four books, 8 KiB
    __shared__ float xs[kP6Blk * kVec];                       // the block's positions
    __shared__ float red[kP6LutThreads / 32];
    const int blk = blockIdx.x;
    const int v0 = blk * kP6Blk;
    const int nvb = min(kP6Blk, nv - v0);
    const int n = nvb * kP6St * kP6En;
    for (int i = threadIdx.x; i < kP6St * kVec * kP6En; i += kP6LutThreads)
        bk[i] = booksT[(size_t)cb_base * kP6En * kVec + i];
    for (int i = threadIdx.x; i < nvb * kVec; i += kP6LutThreads)
        xs[i] = x[(size_t)v0 * kVec + i];
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kP6LutThreads) {
        const int vl = i / (kP6St * kP6En), s = (i / kP6En) % kP6St, c = i % kP6En;
        const float *xv = xs + vl * kVec;
        const float *CT = bk + s * kP6En * kVec;
        float t = 0.0f;
#pragma unroll
        for (int d = 0; d < kVec; d++) t = __fmaf_rn(xv[d], CT[d * kP6En + c], t);
        tab[i] = t;
    }
    __syncthreads();
    float mx = 0.0f;
    for (int i = threadIdx.x; i < n; i += kP6LutThreads) mx = fmaxf(mx, fabsf(tab[i]));
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < kP6LutThreads / 32; w++) mx = fmaxf(mx, red[w]);
    if (threadIdx.x == 0) lscale[blk] = __fdiv_rn(mx, 127.0f);
    const float inv = mx > 0.0f ? __fdiv_rn(127.0f, mx) : 0.0f;
    int8_t *dst = q + (size_t)v0 * kP6St * kP6En;
    for (int i = threadIdx.x; i < n; i += kP6LutThreads) {
        int t = __float2int_rn(__fmul_rn(tab[i], inv));
        t = t > 127 ? 127 : (t < -127 ? -127 : t);
        dst[i] = (int8_t)t;
    }
}

constexpr int kP6Groups = 8;

__global__ void __launch_bounds__(kBlk * kP6Groups)
vq4p_apply_kernel(float *__restrict__ y, const uint8_t *__restrict__ idx,
                  const uint16_t *__restrict__ scale, const int8_t *__restrict__ lut8,
                  const float *__restrict__ lscale, int M, int nv) {
    extern __shared__ int isum[];                              // [kBlk][nblk]
    const int nblk = (nv + kP6Blk - 1) / kP6Blk;
    const int rb = blockIdx.x;
    const int r = threadIdx.x % kBlk, g = threadIdx.x / kBlk;
    for (int blk = g; blk < nblk; blk += kP6Groups) {
        const int v0 = blk * kP6Blk, v1 = min(v0 + kP6Blk, nv);
        int sum = 0;
#pragma unroll 8
        for (int v = v0; v < v1; v++) {
            const uint8_t *ix = idx + (((size_t)rb * nv + v) * kBlk + r) * 3;
            const unsigned b0 = ix[0], b1 = ix[1], b2 = ix[2];
            const int8_t *T = lut8 + (size_t)v * kP6St * kP6En;
            sum += (int)T[b0 & 63] + (int)T[kP6En + (((b0 >> 6) | (b1 << 2)) & 63)] +
                   (int)T[2 * kP6En + (((b1 >> 4) | (b2 << 4)) & 63)] +
                   (int)T[3 * kP6En + ((b2 >> 2) & 63)];
        }
        isum[r * nblk + blk] = sum;
    }
    __syncthreads();
    if (g != 0) return;
    const int row = rb * kBlk + r;
    if (row >= M) return;
    float acc = 0.0f;
    for (int blk = 0; blk < nblk; blk++)
        acc = __fadd_rn(acc, __fmul_rn(lscale[blk], (float)isum[r * nblk + blk]));
    y[row] = __fmul_rn(acc, f16_to_f32(scale[row]));
}

}  // namespace warp

using namespace warp;

extern "C" int warp_vq4p_lut(int8_t *q, float *lscale, const float *booksT, int n_books,
                             const float *x, int nv, int cb_base, void *stream) {
    WARP_ARG(q && lscale && booksT && x && nv >= 1 && cb_base >= 0 && cb_base + 4 <= n_books,
             "warp_vq4p_lut: bad arguments (cb_base + 4 books must exist)");
    const int nblk = (nv + kP6Blk - 1) / kP6Blk;
    vq4p_lut_kernel<<<nblk, kP6LutThreads, 0, (cudaStream_t)stream>>>(q, lscale, booksT, x, nv,
                                                                       cb_base);
    WARP_CHECK_LAUNCH("vq4p_lut_kernel");
    return WARP_OK;
}

extern "C" int warp_vq4p_apply(float *y, const uint8_t *idx, const uint16_t *scale,
                               const int8_t *lut8, const float *lscale, int M, int nv,
                               void *stream) {
    WARP_ARG(y && idx && scale && lut8 && lscale && M >= 1 && nv >= 1 && nv <= 8192,
             "warp_vq4p_apply: bad arguments (nv 1..8192)");
    const int nblk = (nv + kP6Blk - 1) / kP6Blk;
    const size_t smem = (size_t)kBlk * nblk * sizeof(int);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            vq4p_apply_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "vq4p apply smem attribute");
    }
    vq4p_apply_kernel<<<cdiv(M, kBlk), kBlk * kP6Groups, smem, (cudaStream_t)stream>>>(
        y, idx, scale, lut8, lscale, M, nv);
    WARP_CHECK_LAUNCH("vq4p_apply_kernel");
    return WARP_OK;
}
