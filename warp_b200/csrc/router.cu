// router.cu — router logits and the softmax top-k of waste_qwen_moe_route.
#include "common.cuh"
#include "router.cuh"

namespace warp {

// logits[t][e] = Wr[e] . x[t] for e < E, and row E (when wsg is given) the
// shared-expert gate.  kSplit warps share a row (each a contiguous
// 1/kSplit of the hidden size) so a 256-row router still spreads over every
// SM; the partials are summed in split order by the route kernel.
constexpr int kSplit = 16;

__global__ void router_logits_kernel(const float *__restrict__ Wr,
                                     const float *__restrict__ wsg,
                                     const float *__restrict__ x, int T, int E,
                                     int hid, float *__restrict__ part) {
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int rows = E + (wsg ? 1 : 0);
    if (gw >= rows * kSplit) return;
    const int e = gw / kSplit, sp = gw % kSplit;
    const float *w = e < E ? Wr + (size_t)e * hid : wsg;
    const int per = (hid / 4 + kSplit - 1) / kSplit * 4;     // float4 aligned
    const int k0 = sp * per, k1 = min(hid, k0 + per);
    if (lane == 0 && k1 > k0) prefetch_l2_bulk(w + k0, (uint32_t)(k1 - k0) * 4u);
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * hid;
        float acc = 0.0f;
#pragma unroll 4
        for (int k = k0 + lane * 4; k < k1; k += 128) {
            const float4 wv = *(const float4 *)(w + k);
            const float4 xv = *(const float4 *)(xt + k);
            acc = __fmaf_rn(wv.x, xv.x, acc);
            acc = __fmaf_rn(wv.y, xv.y, acc);
            acc = __fmaf_rn(wv.z, xv.z, acc);
            acc = __fmaf_rn(wv.w, xv.w, acc);
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
        if (lane == 0) part[((size_t)t * rows + e) * kSplit + sp] = acc;
    }
}

// Exp of a float, correctly rounded: the double-precision exp rounded once.
// glibc's expf is within 0.502 ulp of this and equal to it almost always.
__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }

// waste_qwen_moe_route (qwen_moe.c:10-44), one warp per token:
//   m = max logit; p[e] = exp(l[e] - m); z = p[0] + p[1] + ... in e order,
//   floored at 1e-20; prob[e] = p[e] / z; K passes each taking the strictly
//   greatest unused prob (lowest id wins ties), w[j] = that prob; with renorm,
//   w[j] /= (w[0] + ... + w[K-1]) when that sum exceeds 1e-20.
// The selection is order-exact (a lane-local ascending scan, then a warp
// reduction that prefers the lower id on equal values).  The sum z is
// sequential in e, as in the reference.  Also writes sigmoid of the shared
// gate logit when there is one.
__global__ void route_kernel(const float *__restrict__ part, int T, int E,
                             int K, int renorm, int has_sg, int nsplit,
                             float *__restrict__ prob_ws, int *__restrict__ idx,
                             float *__restrict__ w, float *__restrict__ sg_out,
                             float *__restrict__ logits_out) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const int rows = E + has_sg;
    float *prob = prob_ws + (size_t)t * E;
    // logits, summed over the splits in order
    float mx = -__int_as_float(0x7f800000);
    for (int e = lane; e < E; e += 32) {
        float l = 0.0f;
        for (int s = 0; s < nsplit; s++) l += part[((size_t)t * rows + e) * nsplit + s];
        prob[e] = l;
        if (logits_out) logits_out[(size_t)t * E + e] = l;
    }
    __syncwarp();
    // max in e order (max is order-free, but keep the reference's start)
    float m = prob[0];
    for (int e = lane; e < E; e += 32) m = fmaxf(m, prob[e]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    (void)mx;
    for (int e = lane; e < E; e += 32) prob[e] = exp_cr(__fsub_rn(prob[e], m));
    __syncwarp();
    float z = 0.0f;
    if (lane == 0) {
        for (int e = 0; e < E; e++) z = __fadd_rn(z, prob[e]);
        if (z < 1e-20f) z = 1e-20f;
    }
    z = __shfl_sync(0xffffffffu, z, 0);
    for (int e = lane; e < E; e += 32) prob[e] = __fdiv_rn(prob[e], z);
    __syncwarp();
    // K selection passes; `used` is a bitmask per lane over its e = lane + 32i
    uint32_t used[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};   // E <= 384
    float wj[64];
    int ij[64];
    for (int j = 0; j < K; j++) {
        float bv = -1.0f;
        int best = -1;
        for (int e = lane, i = 0; e < E; e += 32, i++) {
            if ((used[i >> 5] >> (i & 31)) & 1u) continue;
            const float p = prob[e];
            if (p > bv) { bv = p; best = e; }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int ob = __shfl_xor_sync(0xffffffffu, best, o);
            const bool take = ob >= 0 && (best < 0 || ov > bv || (ov == bv && ob < best));
            if (take) { bv = ov; best = ob; }
        }
        ij[j] = best >= 0 ? best : 0;
        wj[j] = best >= 0 ? bv : 0.0f;
        if (best >= 0 && (best & 31) == lane) {
            const int i = best >> 5;
            used[i >> 5] |= 1u << (i & 31);
        }
    }
    if (lane == 0) {
        if (renorm && K > 1) {
            float s = 0.0f;
            for (int j = 0; j < K; j++) s = __fadd_rn(s, wj[j]);
            if (s > 1e-20f)
                for (int j = 0; j < K; j++) wj[j] = __fdiv_rn(wj[j], s);
        }
        for (int j = 0; j < K; j++) {
            idx[(size_t)t * K + j] = ij[j];
            w[(size_t)t * K + j] = wj[j];
        }
        if (sg_out) {
            float sgl = 0.0f;
            if (has_sg) {
                for (int s = 0; s < nsplit; s++) sgl += part[((size_t)t * rows + E) * nsplit + s];
                sg_out[t] = 1.0f / (1.0f + expf(-sgl));
            } else {
                sg_out[t] = 1.0f;
            }
        }
    }
}

int router_launch(const float *Wr, const float *wsg, const float *x, int T,
                  int E, int hid, int K, int renorm, float *part,
                  float *prob_ws, int *idx, float *w, float *sg_out,
                  float *logits_out, cudaStream_t st) {
    WARP_ARG(E >= 1 && E <= 384 && K >= 1 && K <= 64 && K <= E && hid % 4 == 0,
             "router: E must be 1..384, K 1..64 (<= E), hidden a multiple of 4");
    const int rows = E + (wsg ? 1 : 0);
    const int warps = rows * kSplit;
    router_logits_kernel<<<cdiv(warps, 8), 256, 0, st>>>(Wr, wsg, x, T, E, hid, part);
    WARP_CHECK_LAUNCH("router_logits_kernel");
    route_kernel<<<cdiv(T, 4), 128, 0, st>>>(part, T, E, K, renorm, wsg ? 1 : 0,
                                              kSplit, prob_ws, idx, w, sg_out,
                                              logits_out);
    WARP_CHECK_LAUNCH("route_kernel");
    return WARP_OK;
}

// Route given logits directly (the C-ABI entry point): the logits become a
// one-split partial.
int route_only(const float *logits, int T, int E, int K, int renorm,
               float *prob_ws, int *idx, float *w, cudaStream_t st) {
    WARP_ARG(E >= 1 && E <= 384 && K >= 1 && K <= 64 && K <= E,
             "route: E must be 1..384, K 1..64 (<= E)");
    route_kernel<<<cdiv(T, 4), 128, 0, st>>>(logits, T, E, K, renorm, 0, 1,
                                              prob_ws, idx, w, nullptr, nullptr);
    WARP_CHECK_LAUNCH("route_kernel");
    return WARP_OK;
}

}  // namespace warp

extern "C" int warp_qwen_route(const float *logits, int T, int E, int K,
                               int renorm, int *idx, float *w, void *stream) {
    WARP_ARG(logits && idx && w && T >= 1, "warp_qwen_route: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    float *prob = nullptr;
    cudaError_t e = cudaMallocAsync(&prob, (size_t)T * E * sizeof(float), st);
    if (e != cudaSuccess) return warp::cuda_fail(e, "route scratch");
    const int rc = warp::route_only(logits, T, E, K, renorm, prob, idx, w, st);
    cudaFreeAsync(prob, st);
    return rc;
}

namespace warp {

// waste_rmsnorm (model.c:178-184): s = sum x^2 in order, r = 1/sqrtf(s/n +
// eps), o = x * r * w (w = 1 when NULL).  One CTA per row; the sum is a
// block tree (fp32), not the reference's sequential loop.
__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                               float *__restrict__ o, int n, float eps) {
    const float *xr = x + (size_t)blockIdx.x * n;
    float *orow = o + (size_t)blockIdx.x * n;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = __fmaf_rn(xr[i], xr[i], s);
    __shared__ float red[32];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
        if (threadIdx.x == 0) red[0] = s;
    }
    __syncthreads();
    const float r = 1.0f / sqrtf(red[0] / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        orow[i] = xr[i] * r * (w ? w[i] : 1.0f);
}

}  // namespace warp

extern "C" int warp_rmsnorm(const float *x, const float *w, float *o, int rows, int n,
                            float eps, void *stream) {
    WARP_ARG(x && o && rows >= 1 && n >= 1, "warp_rmsnorm: bad arguments");
    warp::rmsnorm_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(x, w, o, n, eps);
    WARP_CHECK_LAUNCH("rmsnorm_kernel");
    return WARP_OK;
}
