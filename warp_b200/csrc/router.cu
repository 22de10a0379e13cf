// router.cu — router logits and the softmax top-k of waste_qwen_moe_route.
#include "common.cuh"
#include "router.cuh"

namespace warp {

// exp(x) for a float x <= 0, rounded once to float from a double-precision
// evaluation: Cody-Waite reduction x = n*ln2 + r with |r| <= ln2/2, ln2
// split as in fdlibm's e_exp.c (a head with trailing zeros, so n*ln2_hi is
// exact, and a tail), e^r from its Taylor
// series to r^13/13! (relative error below 2^-60 on that interval), then
// scaled by 2^n (exactly: n >= -151 keeps 2^n a normal double).  The double
// result carries far more bits than the float, so the final rounding is the
// correctly rounded exp except when the true value sits within ~2^-30 of a
// float rounding boundary.  glibc's expf is within 0.502 ulp of the same
// value and agrees with it almost always.
__device__ __forceinline__ float exp_cr(float xf) {
    if (xf < -104.0f) return 0.0f;                  // below the float range
    const double x = (double)xf;
    const double ln2_hi = 6.93147180369123816490e-01;   // 0x3FE62E42FEE00000
    const double ln2_lo = 1.90821492927058770002e-10;
    const double n = rint(x * 1.44269504088896338700e+00);
    const double r = (x - n * ln2_hi) - n * ln2_lo;
    double p = 1.0 / 6227020800.0;                      // 1/13!
    p = fma(p, r, 1.0 / 479001600.0);
    p = fma(p, r, 1.0 / 39916800.0);
    p = fma(p, r, 1.0 / 3628800.0);
    p = fma(p, r, 1.0 / 362880.0);
    p = fma(p, r, 1.0 / 40320.0);
    p = fma(p, r, 1.0 / 5040.0);
    p = fma(p, r, 1.0 / 720.0);
    p = fma(p, r, 1.0 / 120.0);
    p = fma(p, r, 1.0 / 24.0);
    p = fma(p, r, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    const double two_n = __longlong_as_double((long long)((int)n + 1023) << 52);
    return (float)(p * two_n);
}

// waste_qwen_moe_route (qwen_moe.c:10-44) for one token, by one warp:
//   m = max logit; p[e] = exp(l[e] - m); z = p[0] + p[1] + ... in e order,
//   floored at 1e-20; prob[e] = p[e] / z; K passes each taking the strictly
//   greatest unused prob (lowest id wins ties), w[j] = that prob; with renorm,
//   w[j] /= (w[0] + ... + w[K-1]) when that sum exceeds 1e-20.
// Lane l keeps e = l + 32i in registers.  A pass takes the warp maximum of
// the lanes' best keys (prob bits + 1, monotone for probs >= 0) and, among
// the lanes holding it, the lowest id, each with one redux; lane j % 32 keeps
// pick j.  z is summed as a tree rather than in e order: prob is p/z for one
// z, so the ranking is z's only use that decides indices, and a different
// last bit of z can reorder only probabilities already within an ulp of each
// other.
constexpr int kRouteMaxPerLane = 12;     // E <= 384
constexpr int kRouteWarps = 4;

__device__ __forceinline__ void route_token(const float *__restrict__ lt, int E, int K,
                                            int renorm, int *__restrict__ idx_out,
                                            float *__restrict__ w_out) {
    const int lane = threadIdx.x & 31;
    float p[kRouteMaxPerLane];
    float m = lt[0];
#pragma unroll
    for (int i = 0; i < kRouteMaxPerLane; i++) {
        const int e = lane + 32 * i;
        p[i] = e < E ? lt[e] : 0.0f;
        if (e < E) m = fmaxf(m, p[i]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float z = 0.0f;
#pragma unroll
    for (int i = 0; i < kRouteMaxPerLane; i++) {
        const int e = lane + 32 * i;
        if (e < E) {
            p[i] = exp_cr(__fsub_rn(p[i], m));
            z += p[i];
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    if (z < 1e-20f) z = 1e-20f;
#pragma unroll
    for (int i = 0; i < kRouteMaxPerLane; i++) p[i] = __fdiv_rn(p[i], z);

    // this lane's best unused candidate: key 0 = none
    uint32_t used = 0;
    auto best_key = [&](int &be) {
        uint32_t key = 0;
        be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++) {
            const int e = lane + 32 * i;
            const uint32_t k = __float_as_uint(p[i]) + 1u;
            if (e < E && !((used >> i) & 1u) && k > key) { key = k; be = e; }
        }
        return key;
    };
    int be;
    uint32_t key = best_key(be);
    int my_idx[2] = {0, 0};
    float my_w[2] = {0.0f, 0.0f};
    for (int j = 0; j < K; j++) {
        const uint32_t mk = __reduce_max_sync(0xffffffffu, key);
        // min() keeps the id a valid expert even if no lane had a candidate
        // (impossible for K <= E, which every entry point checks)
        const uint32_t win = min(__reduce_min_sync(0xffffffffu,
                                                   key == mk ? (uint32_t)be : 0x7fffffffu),
                                 (uint32_t)(E - 1));
        const float prob = __uint_as_float(mk - 1u);
        if (lane == (j & 31)) {
            if (j < 32) { my_idx[0] = (int)win; my_w[0] = prob; }
            else { my_idx[1] = (int)win; my_w[1] = prob; }
        }
        if ((int)(win & 31u) == lane) {
            used |= 1u << (win >> 5);
            key = best_key(be);
        }
    }
    if (renorm && K > 1) {
        float wsum = 0.0f;                               // w[0] + ... + w[K-1] in order
        for (int j = 0; j < K; j++)
            wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, j < 32 ? my_w[0] : my_w[1], j & 31));
        if (wsum > 1e-20f) {
            my_w[0] = __fdiv_rn(my_w[0], wsum);
            my_w[1] = __fdiv_rn(my_w[1], wsum);
        }
    }
    if (lane < K) { idx_out[lane] = my_idx[0]; w_out[lane] = my_w[0]; }
    if (lane + 32 < K) { idx_out[lane + 32] = my_idx[1]; w_out[lane + 32] = my_w[1]; }
}

// moe_layer's router (model.c:5466-5556) for one token, by one warp, in the
// layout of route_token (lane l keeps e = l + 32 i):
//   scores as router_scores (model.c:5466-5486): sigmoid 1 / (1 + exp(-x));
//   softmax exp(l - max) / sum with the sum taken in e order (every lane
//   adds the scores in that order, broadcast one by one); sqrt(softplus),
//   softplus = x above 30, else log1p(exp(x)).  exp is exp_cr (the float
//   expf rounds to), log1p the double log1p rounded once to float;
//   selection value score + bias (the bias moves the ranking only), strict >
//   with the lowest id on ties and nothing at or below -1e30 selectable;
//   w[j] = the unbiased score; renorm w[j] /= (sum_j w + 1e-20) with the sum
//   in j order; then w[j] *= routed_scale.
// The selection key maps a float of either sign to an unsigned integer in
// the same order (sign bit flipped for positives, all bits for negatives).
__device__ __forceinline__ void route_scored(const float *__restrict__ lt, int E, int K,
                                             const RouteCfg &rc, int renorm,
                                             int *__restrict__ idx_out,
                                             float *__restrict__ w_out) {
    const int lane = threadIdx.x & 31;
    float sc[kRouteMaxPerLane];
#pragma unroll
    for (int i = 0; i < kRouteMaxPerLane; i++) {
        const int e = lane + 32 * i;
        sc[i] = e < E ? lt[e] : 0.0f;
    }
    if (rc.func == 1) {
        float mx = -1e30f;
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++)
            if (lane + 32 * i < E && sc[i] > mx) mx = sc[i];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++) sc[i] = exp_cr(__fsub_rn(sc[i], mx));
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++) {
            if (32 * i >= E) break;
            for (int src = 0; src < 32; src++) {
                const float v = __shfl_sync(0xffffffffu, sc[i], src);
                if (32 * i + src < E) sum = __fadd_rn(sum, v);
            }
        }
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++) sc[i] = __fdiv_rn(sc[i], sum);
    } else if (rc.func == 2) {
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++) {
            const float x = sc[i];
            const float sp = x > 30.0f ? x : (float)log1p((double)exp_cr(x));
            sc[i] = __fsqrt_rn(sp);
        }
    } else {
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++)
            sc[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-sc[i])));
    }
    // selection keys (0 = not selectable)
    uint32_t kv[kRouteMaxPerLane];
#pragma unroll
    for (int i = 0; i < kRouteMaxPerLane; i++) {
        const int e = lane + 32 * i;
        const float v = rc.bias ? __fadd_rn(sc[i], e < E ? rc.bias[e] : 0.0f) : sc[i];
        const uint32_t u = __float_as_uint(v);
        const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        kv[i] = (e < E && v > -1e30f) ? k : 0u;            // NaN compares false: 0
    }
    uint32_t used = 0;
    auto best_key = [&](int &be, float &bs) {
        uint32_t key = 0;
        be = 0x7fffffff;
        bs = 0.0f;
#pragma unroll
        for (int i = 0; i < kRouteMaxPerLane; i++) {
            const int e = lane + 32 * i;
            if (e < E && !((used >> i) & 1u) && kv[i] > key) { key = kv[i]; be = e; bs = sc[i]; }
        }
        return key;
    };
    int be;
    float bs;
    uint32_t key = best_key(be, bs);
    int my_idx[2] = {0, 0};
    float my_w[2] = {0.0f, 0.0f};
    for (int j = 0; j < K; j++) {
        const uint32_t mk = __reduce_max_sync(0xffffffffu, key);
        const uint32_t win = min(__reduce_min_sync(0xffffffffu,
                                                   key == mk ? (uint32_t)be : 0x7fffffffu),
                                 (uint32_t)(E - 1));
        const float score = __shfl_sync(0xffffffffu, bs, (int)(win & 31u));
        if (lane == (j & 31)) {
            if (j < 32) { my_idx[0] = (int)win; my_w[0] = score; }
            else { my_idx[1] = (int)win; my_w[1] = score; }
        }
        if ((int)(win & 31u) == lane) {
            used |= 1u << (win >> 5);
            key = best_key(be, bs);
        }
    }
    if (renorm && K > 1) {
        float wsum = 0.0f;                               // w[0] + ... + w[K-1] in order
        for (int j = 0; j < K; j++)
            wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, j < 32 ? my_w[0] : my_w[1], j & 31));
        const float d = __fadd_rn(wsum, 1e-20f);
        my_w[0] = __fdiv_rn(my_w[0], d);
        my_w[1] = __fdiv_rn(my_w[1], d);
    }
    my_w[0] = __fmul_rn(my_w[0], rc.scale);
    my_w[1] = __fmul_rn(my_w[1], rc.scale);
    if (lane < K) { idx_out[lane] = my_idx[0]; w_out[lane] = my_w[0]; }
    if (lane + 32 < K) { idx_out[lane + 32] = my_idx[1]; w_out[lane + 32] = my_w[1]; }
}

// The router of the layer: Qwen's (rc.kind 0) or moe_layer's (rc.kind 1).
__device__ __forceinline__ void route_one(const float *lt, int E, int K, const RouteCfg &rc,
                                          int renorm, int *idx_out, float *w_out) {
    if (rc.kind == 1) route_scored(lt, E, K, rc, renorm, idx_out, w_out);
    else route_token(lt, E, K, renorm, idx_out, w_out);
}

__global__ void route_kernel(const float *__restrict__ logits, int T, int E,
                             int K, int renorm, int rows, RouteCfg rc,
                             int *__restrict__ idx, float *__restrict__ w) {
    const int t = blockIdx.x * kRouteWarps + (threadIdx.x >> 5);
    if (t >= T) return;
    route_one(logits + (size_t)t * rows, E, K, rc, renorm, idx + (size_t)t * K,
              w + (size_t)t * K);
}

// Logits and routing in one launch.  CTA (row e, part q) of rows * kParts
// takes part q of the row's float4s for every token and writes its
// fixed-order tree sum to parts[(t * rows + e) * kParts + q].  The weights do
// not depend on the kernels before this one: a thread's first kRouterPre
// float4s are loaded before the wait for the previous kernel, so their HBM
// time overlaps its tail.  The last CTA to finish (ticket) adds each row's
// parts in order into logits[t][e], then routes every token (one warp each),
// writes the shared-gate sigmoid, and resets the ticket for the next launch.
constexpr int kLogitThreads = 256;
constexpr int kParts = 2;
constexpr int kRouterPre = 4;            // weight float4s a thread loads before the wait

__global__ void __launch_bounds__(kLogitThreads)
router_kernel(const float *__restrict__ Wr, const float *__restrict__ wsg,
              const float *__restrict__ x, int T, int E, int hid, int K, int renorm,
              RouteCfg rc, float *__restrict__ parts, float *__restrict__ logits,
              unsigned *__restrict__ ticket, int *__restrict__ idx,
              float *__restrict__ w, float *__restrict__ sg_out, int route_here) {
    __shared__ float red[kLogitThreads / 32];
    __shared__ bool last;
    const int rows = E + (wsg ? 1 : 0);
    const int e = blockIdx.x / kParts, q = blockIdx.x % kParts;
    const float *wr = e < E ? Wr + (size_t)e * hid : wsg;
    const int n4 = hid / 4;
    const int k0 = n4 * q / kParts, k1 = n4 * (q + 1) / kParts;
    const float4 *w4 = (const float4 *)wr;
    uint4 wpre[kRouterPre];
#pragma unroll
    for (int i = 0; i < kRouterPre; i++) {
        const int k = k0 + threadIdx.x + i * kLogitThreads;
        wpre[i] = k < k1 ? ldg_stream(w4 + k) : make_uint4(0u, 0u, 0u, 0u);
    }
    pdl_wait();
    pdl_trigger();
    for (int t = 0; t < T; t++) {
        const float4 *x4 = (const float4 *)(x + (size_t)t * hid);
        float acc = 0.0f;
        int i = 0;
#pragma unroll 4
        for (int k = k0 + threadIdx.x; k < k1; k += kLogitThreads, i++) {
            const uint4 wu = i < kRouterPre ? wpre[i] : ldg_stream(w4 + k);
            const float4 wv = make_float4(__uint_as_float(wu.x), __uint_as_float(wu.y),
                                          __uint_as_float(wu.z), __uint_as_float(wu.w));
            const float4 xv = x4[k];
            acc = __fmaf_rn(wv.x, xv.x, acc);
            acc = __fmaf_rn(wv.y, xv.y, acc);
            acc = __fmaf_rn(wv.z, xv.z, acc);
            acc = __fmaf_rn(wv.w, xv.w, acc);
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            float s = 0.0f;
            for (int j = 0; j < kLogitThreads / 32; j++) s += red[j];
            parts[((size_t)t * rows + e) * kParts + q] = s;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = threadIdx.x; i < T * rows; i += kLogitThreads) {
        float s = 0.0f;
#pragma unroll
        for (int qq = 0; qq < kParts; qq++) s += __ldcg(parts + (size_t)i * kParts + qq);
        logits[i] = s;
    }
    __syncthreads();
    if (route_here)                 // Qwen's router only (see router_launch)
        for (int t = threadIdx.x >> 5; t < T; t += kLogitThreads / 32)
            route_token(logits + (size_t)t * rows, E, K, renorm, idx + (size_t)t * K,
                        w + (size_t)t * K);
    if (sg_out)
        for (int t = threadIdx.x; t < T; t += kLogitThreads)
            sg_out[t] = wsg ? 1.0f / (1.0f + expf(-logits[(size_t)t * rows + E])) : 1.0f;
    if (threadIdx.x == 0) *ticket = 0u;
}

// Logits of many tokens (T >= 2): warp w of CTA (b, g) owns row e =
// kRmWarps b + w for tokens [kRmTG g, kRmTG (g + 1)).  The tokens'
// activations are staged 256 k at a time in shared memory; lane l streams the row's float4s l, l + 32, ...
// of each chunk (a coalesced 512-byte read per step) against every token,
// each (token, row) an FMA chain over the lane's k in order, and the warp
// meets in an xor tree.  The weights are read once per kRmTG tokens, not
// once per token as the one-token kernel's per-token block reductions would.
constexpr int kRmWarps = 4, kRmTG = 16, kRmKC = 256;   // 512-token prefill: 0.273 vs 0.343 ms a layer at 8 x 32

__global__ void __launch_bounds__(kRmWarps * 32)
router_multi_kernel(const float *__restrict__ Wr, const float *__restrict__ wsg,
                    const float *__restrict__ x, int T, int E, int hid,
                    float *__restrict__ logits, float *__restrict__ sg_out) {
    __shared__ float4 xs[kRmTG][kRmKC / 4];                 // 32 KiB
    const int rows = E + (wsg ? 1 : 0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kRmWarps + warp;
    const int t0 = blockIdx.y * kRmTG, tn = min(kRmTG, T - t0);
    const float *wr = e < E ? Wr + (size_t)e * hid : (e == E ? wsg : nullptr);
    const float4 *w4 = (const float4 *)wr;
    const float4 *x4 = (const float4 *)x;
    const int n4 = hid / 4;
    float acc[kRmTG];
#pragma unroll
    for (int t = 0; t < kRmTG; t++) acc[t] = 0.0f;
    pdl_wait();
    pdl_trigger();
    for (int c0 = 0; c0 < n4; c0 += kRmKC / 4) {
        __syncthreads();                                   // previous chunk consumed
        for (int i = threadIdx.x; i < tn * (kRmKC / 4); i += kRmWarps * 32) {
            const int t = i / (kRmKC / 4), c = i % (kRmKC / 4);
            xs[t][c] = c0 + c < n4 ? x4[(size_t)(t0 + t) * n4 + c0 + c]
                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        __syncthreads();
        if (wr) {
#pragma unroll
            for (int j = 0; j < kRmKC / 4 / 32; j++) {
                const int c = lane + 32 * j;
                if (c0 + c >= n4) break;
                const uint4 wu = ldg_stream(w4 + c0 + c);
                const float4 wv = make_float4(__uint_as_float(wu.x), __uint_as_float(wu.y),
                                              __uint_as_float(wu.z), __uint_as_float(wu.w));
#pragma unroll
                for (int t = 0; t < kRmTG; t++) {
                    if (t >= tn) break;
                    const float4 xv = xs[t][c];
                    float a = acc[t];
                    a = __fmaf_rn(wv.x, xv.x, a);
                    a = __fmaf_rn(wv.y, xv.y, a);
                    a = __fmaf_rn(wv.z, xv.z, a);
                    acc[t] = __fmaf_rn(wv.w, xv.w, a);
                }
            }
        }
    }
    if (!wr) return;                                       // past the last row
#pragma unroll
    for (int t = 0; t < kRmTG; t++) {
        if (t >= tn) break;
        float v = acc[t];
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
        if (lane == 0) {
            logits[(size_t)(t0 + t) * rows + e] = v;
            if (e == E && sg_out) sg_out[t0 + t] = 1.0f / (1.0f + expf(-v));
        }
    }
    // without a shared-expert gate the gate is 1 (row 0's warp writes it)
    if (!wsg && sg_out && e == 0)
        for (int t = lane; t < tn; t += 32) sg_out[t0 + t] = 1.0f;
}

int router_launch(const float *Wr, const float *wsg, const float *x, int T, int E, int hid,
                  int K, int renorm, RouteCfg rc, float *parts, float *logits,
                  unsigned *ticket, int *idx, float *w, float *sg_out, cudaStream_t st) {
    WARP_ARG(E >= 1 && E <= 384 && K >= 1 && K <= 64 && K <= E && hid % 4 == 0,
             "router: E must be 1..384, K 1..64 (<= E), hidden a multiple of 4");
    const int rows = E + (wsg ? 1 : 0);
    // one token: logits and (Qwen's router) the top-k in one launch, the
    // last CTA routing; several tokens, or moe_layer's scored router: the
    // logits, then a launch that routes
    const int route_here = T == 1 && rc.kind == 0;
    cudaError_t e;
    if (T == 1)
        e = launch_pdl(router_kernel, dim3(rows * kParts), dim3(kLogitThreads), 0, st, Wr, wsg,
                       x, T, E, hid, K, renorm, rc, parts, logits, ticket, idx, w, sg_out,
                       route_here);
    else
        e = launch_pdl(router_multi_kernel, dim3(cdiv(rows, kRmWarps), cdiv(T, kRmTG)),
                       dim3(kRmWarps * 32), 0, st, Wr, wsg, x, T, E, hid, logits, sg_out);
    if (e != cudaSuccess) return cuda_fail(e, T == 1 ? "router_kernel" : "router_multi_kernel");
    count_launch();
    if (!route_here) {
        route_kernel<<<cdiv(T, kRouteWarps), 32 * kRouteWarps, 0, st>>>(
            logits, T, E, K, renorm, rows, rc, idx, w);
        WARP_CHECK_LAUNCH("route_kernel");
    }
    return WARP_OK;
}

// Route given logits directly (the C-ABI entry point).
int route_only(const float *logits, int T, int E, int K, int renorm, int *idx, float *w,
               cudaStream_t st) {
    WARP_ARG(E >= 1 && E <= 384 && K >= 1 && K <= 64 && K <= E,
             "route: E must be 1..384, K 1..64 (<= E)");
    route_kernel<<<cdiv(T, kRouteWarps), 32 * kRouteWarps, 0, st>>>(
        logits, T, E, K, renorm, E, RouteCfg{}, idx, w);
    WARP_CHECK_LAUNCH("route_kernel");
    return WARP_OK;
}

int route_scored_only(const float *logits, int T, int E, int K, RouteCfg rc, int renorm,
                      int *idx, float *w, cudaStream_t st) {
    WARP_ARG(E >= 1 && E <= 384 && K >= 1 && K <= 64 && K <= E,
             "route: E must be 1..384, K 1..64 (<= E)");
    WARP_ARG(rc.func >= 0 && rc.func <= 2, "route: score function must be 0, 1 or 2");
    rc.kind = 1;
    route_kernel<<<cdiv(T, kRouteWarps), 32 * kRouteWarps, 0, st>>>(
        logits, T, E, K, renorm, E, rc, idx, w);
    WARP_CHECK_LAUNCH("route_kernel");
    return WARP_OK;
}

}  // namespace warp

extern "C" int warp_qwen_route(const float *logits, int T, int E, int K,
                               int renorm, int *idx, float *w, void *stream) {
    WARP_ARG(logits && idx && w && T >= 1, "warp_qwen_route: bad arguments");
    return warp::route_only(logits, T, E, K, renorm, idx, w, (cudaStream_t)stream);
}

extern "C" int warp_moe_route(const float *logits, int T, int E, int K, int score_func,
                              const float *bias, int renorm, float routed_scale, int *idx,
                              float *w, void *stream) {
    WARP_ARG(logits && idx && w && T >= 1, "warp_moe_route: bad arguments");
    warp::RouteCfg rc;
    rc.kind = 1;
    rc.func = score_func;
    rc.bias = bias;
    rc.scale = routed_scale;
    return warp::route_scored_only(logits, T, E, K, rc, renorm, idx, w, (cudaStream_t)stream);
}

namespace warp {

// waste_rmsnorm (model.c:178-184): s = sum x^2, r = 1/sqrtf(s/n + eps),
// o = x * r * w (w = 1 when NULL).  One CTA of 1024 threads per row, 128-bit
// loads held in registers across the reduction; the sum is a fixed-order
// tree (fp32), not the reference's sequential loop.
constexpr int kNormThreads = 1024;
constexpr int kNormPerThread = 4;       // float4 per thread held in registers

__global__ void __launch_bounds__(kNormThreads)
rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
               float *__restrict__ o, int n, float eps) {
    __shared__ float red[kNormThreads / 32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *orow = o + (size_t)blockIdx.x * n;
    const int n4 = n / 4;
    pdl_wait();
    pdl_trigger();
    float4 v[kNormPerThread];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < kNormPerThread; j++) {
        const int k = threadIdx.x + j * kNormThreads;
        v[j] = k < n4 ? ((const float4 *)xr)[k] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        s = __fmaf_rn(v[j].x, v[j].x, s);
        s = __fmaf_rn(v[j].y, v[j].y, s);
        s = __fmaf_rn(v[j].z, v[j].z, s);
        s = __fmaf_rn(v[j].w, v[j].w, s);
    }
    // the rest beyond the register-held part, and the scalar tail
    for (int k = threadIdx.x + kNormPerThread * kNormThreads; k < n4; k += kNormThreads) {
        const float4 t = ((const float4 *)xr)[k];
        s = __fmaf_rn(t.x, t.x, s); s = __fmaf_rn(t.y, t.y, s);
        s = __fmaf_rn(t.z, t.z, s); s = __fmaf_rn(t.w, t.w, s);
    }
    for (int k = 4 * n4 + threadIdx.x; k < n; k += kNormThreads) s = __fmaf_rn(xr[k], xr[k], s);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = red[threadIdx.x];
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
        if (threadIdx.x == 0) red[0] = s;
    }
    __syncthreads();
    const float r = 1.0f / sqrtf(red[0] / (float)n + eps);
#pragma unroll
    for (int j = 0; j < kNormPerThread; j++) {
        const int k = threadIdx.x + j * kNormThreads;
        if (k < n4) {
            float4 y = v[j];
            if (w) {
                const float4 ww = ((const float4 *)w)[k];
                y = make_float4(y.x * r * ww.x, y.y * r * ww.y, y.z * r * ww.z, y.w * r * ww.w);
            } else {
                y = make_float4(y.x * r, y.y * r, y.z * r, y.w * r);
            }
            ((float4 *)orow)[k] = y;
        }
    }
    for (int k = threadIdx.x + kNormPerThread * kNormThreads; k < n4; k += kNormThreads) {
        const float4 t = ((const float4 *)xr)[k];
        const float4 ww = w ? ((const float4 *)w)[k] : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        ((float4 *)orow)[k] = make_float4(t.x * r * ww.x, t.y * r * ww.y, t.z * r * ww.z,
                                          t.w * r * ww.w);
    }
    for (int k = 4 * n4 + threadIdx.x; k < n; k += kNormThreads)
        orow[k] = xr[k] * r * (w ? w[k] : 1.0f);
}

}  // namespace warp

extern "C" int warp_rmsnorm(const float *x, const float *w, float *o, int rows, int n,
                            float eps, void *stream) {
    WARP_ARG(x && o && rows >= 1 && n >= 1, "warp_rmsnorm: bad arguments");
    WARP_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)o % 16) == 0 && n % 4 == 0 &&
                 (!w || ((uintptr_t)w % 16) == 0),
             "warp_rmsnorm: rows must be 16-byte aligned with n a multiple of 4");
    cudaError_t e = warp::launch_pdl(warp::rmsnorm_kernel, dim3(rows), dim3(warp::kNormThreads), 0,
                                     (cudaStream_t)stream, x, w, o, n, eps);
    if (e != cudaSuccess) return warp::cuda_fail(e, "rmsnorm_kernel");
    warp::count_launch();
    return WARP_OK;
}
