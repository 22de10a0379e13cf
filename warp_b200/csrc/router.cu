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

// waste_qwen_moe_route for one token by a whole block (blockDim.x >= E,
// 32 | blockDim.x): thread e owns expert e.  The max and z are block trees
// in a fixed order (warp xor trees, then the warp results in warp order),
// z floored at 1e-20, prob = p / z; each of the K passes takes the block's
// greatest key (prob bits + 1) and the lowest id holding it (redux within a
// warp, then over the warps' candidates, which every warp reads from shared
// memory after one barrier); renorm by the sequential sum of the K weights.
// `sm` holds 2 * 32 * 2 + 40 words of shared memory.
__device__ __forceinline__ void route_token_block(const float *__restrict__ lt, int E, int K,
                                                  int renorm, int *__restrict__ idx_out,
                                                  float *__restrict__ w_out, uint32_t *sm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nw = blockDim.x >> 5;
    float *fs = (float *)sm;                       // [32] warp partials
    uint32_t *cand = sm + 32;                      // [2][32][2] (key, id) per pass parity
    float *wsel = (float *)(sm + 160);             // [K <= 64] picks' weights (+ sums)
    const bool mine = tid < E;
    const float l = mine ? __ldcg(lt + tid) : -INFINITY;
    float m = l;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) fs[warp] = m;
    __syncthreads();
    m = fs[0];
    for (int w = 1; w < nw; w++) m = fmaxf(m, fs[w]);
    __syncthreads();
    const float p = mine ? exp_cr(__fsub_rn(l, m)) : 0.0f;
    float z = p;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    if (lane == 0) fs[warp] = z;
    __syncthreads();
    z = 0.0f;
    for (int w = 0; w < nw; w++) z += fs[w];
    if (z < 1e-20f) z = 1e-20f;
    const float prob = __fdiv_rn(p, z);
    uint32_t key = mine ? __float_as_uint(prob) + 1u : 0u;
    for (int j = 0; j < K; j++) {
        const uint32_t wk = __reduce_max_sync(0xffffffffu, key);
        const uint32_t wi = __reduce_min_sync(0xffffffffu,
                                              key == wk ? (uint32_t)tid : 0x7fffffffu);
        uint32_t *c = cand + (j & 1) * 64;
        if (lane == 0) { c[2 * warp] = wk; c[2 * warp + 1] = wi; }
        __syncthreads();
        const uint32_t k2 = lane < nw ? c[2 * lane] : 0u;
        const uint32_t i2 = lane < nw ? c[2 * lane + 1] : 0x7fffffffu;
        const uint32_t mk = __reduce_max_sync(0xffffffffu, k2);
        const uint32_t win = min(__reduce_min_sync(0xffffffffu, k2 == mk ? i2 : 0x7fffffffu),
                                 (uint32_t)(E - 1));
        if ((uint32_t)tid == win) key = 0u;
        if (tid == 0) {
            idx_out[j] = (int)win;
            wsel[j] = __uint_as_float(mk - 1u);
        }
    }
    if (tid == 0) {
        if (renorm && K > 1) {
            float wsum = 0.0f;
            for (int j = 0; j < K; j++) wsum = __fadd_rn(wsum, wsel[j]);
            if (wsum > 1e-20f)
                for (int j = 0; j < K; j++) wsel[j] = __fdiv_rn(wsel[j], wsum);
        }
        for (int j = 0; j < K; j++) w_out[j] = wsel[j];
    }
    __syncthreads();
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

// Logits and routing in one launch.  One CTA per SM owns whole rows: row
// e = blockIdx.x + gridDim.x * j.  Before waiting for the previous kernel a
// thread loads its float4s of those rows (k = threadIdx.x + 512 i), which
// do not depend on it, so the router's HBM time overlaps that kernel's tail.
// Per token the CTA then forms x (the input, or RMSNorm of the input when
// pre-normalising: the norm scale from norm_scale_warp, the same value every
// kernel of the layer computes), dots it with its rows and reduces over the
// block in a fixed order.  The last CTA to finish (ticket) routes every token
// (one warp each), writes the shared-gate sigmoid, and resets the ticket.
constexpr int kRouteInKernel = 16;       // tokens the last CTA routes itself
constexpr int kRtThreads = 512;
constexpr int kRtRows = 3;               // rows per CTA held in registers
constexpr int kRtPre = 4;                // float4s per row and thread held in registers

__global__ void __launch_bounds__(kRtThreads)
router_kernel(const float *__restrict__ Wr, const float *__restrict__ wsg,
              const float *__restrict__ x, PreNorm pn, int T, int E, int hid, int K,
              int renorm, RouteCfg rc, float *__restrict__ logits, unsigned *__restrict__ ticket,
              int *__restrict__ idx, float *__restrict__ w, float *__restrict__ sg_out,
              int route_here) {
    __shared__ float red[kRtThreads / 32];
    __shared__ float nred[8];
    __shared__ float rsc;
    __shared__ bool last;
    const int rows = E + (wsg ? 1 : 0);
    const int G = gridDim.x;
    const int n4 = hid / 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto row_ptr = [&](int e) -> const float4 * {
        return (const float4 *)(e < E ? Wr + (size_t)e * hid : wsg);
    };
    uint4 wpre[kRtRows][kRtPre];
#pragma unroll
    for (int j = 0; j < kRtRows; j++) {
        const int e = blockIdx.x + G * j;
#pragma unroll
        for (int i = 0; i < kRtPre; i++) {
            const int k = tid + kRtThreads * i;
            wpre[j][i] = (e < rows && k < n4) ? ldg_stream(row_ptr(e) + k)
                                              : make_uint4(0u, 0u, 0u, 0u);
        }
    }
    pdl_wait();
    pdl_trigger();
    const float4 *nw4 = (const float4 *)pn.w;
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * hid;
        float r = 1.0f;
        if (pn.on) r = norm_scale_block(xt, hid, pn.eps, nred, &rsc);
        // this thread's x float4s, k = tid + 512 i
        auto xload = [&](int k) -> float4 {
            float4 v = ((const float4 *)xt)[k];
            if (pn.on) {
                v = make_float4(v.x * r, v.y * r, v.z * r, v.w * r);
                if (pn.w) {
                    const float4 g = nw4[k];
                    v = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
                }
            }
            return v;
        };
        float4 xv[kRtPre];
#pragma unroll
        for (int i = 0; i < kRtPre; i++) {
            const int k = tid + kRtThreads * i;
            xv[i] = k < n4 ? xload(k) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        // the block's fixed-order sum of the threads' partials -> logit (t, e)
        auto finish = [&](float acc, int e) {
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
            if (lane == 0) red[warp] = acc;
            __syncthreads();
            if (tid == 0) {
                float sum = 0.0f;
                for (int q = 0; q < kRtThreads / 32; q++) sum += red[q];
                logits[(size_t)t * rows + e] = sum;
            }
            __syncthreads();
        };
        auto tail = [&](float acc, int e) {
            for (int k = tid + kRtThreads * kRtPre; k < n4; k += kRtThreads) {
                const uint4 wu = ldg_stream(row_ptr(e) + k);
                const float4 v = xload(k);
                acc = __fmaf_rn(__uint_as_float(wu.x), v.x, acc);
                acc = __fmaf_rn(__uint_as_float(wu.y), v.y, acc);
                acc = __fmaf_rn(__uint_as_float(wu.z), v.z, acc);
                acc = __fmaf_rn(__uint_as_float(wu.w), v.w, acc);
            }
            return acc;
        };
        // rows held in registers (j is a compile-time index here)
#pragma unroll
        for (int j = 0; j < kRtRows; j++) {
            const int e = blockIdx.x + G * j;
            if (e >= rows) break;                          // block-uniform
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < kRtPre; i++) {
                const uint4 wu = wpre[j][i];
                acc = __fmaf_rn(__uint_as_float(wu.x), xv[i].x, acc);
                acc = __fmaf_rn(__uint_as_float(wu.y), xv[i].y, acc);
                acc = __fmaf_rn(__uint_as_float(wu.z), xv[i].z, acc);
                acc = __fmaf_rn(__uint_as_float(wu.w), xv[i].w, acc);
            }
            finish(tail(acc, e), e);
        }
        // further rows (more rows than kRtRows per CTA), loaded here
        for (int j = kRtRows;; j++) {
            const int e = blockIdx.x + G * j;
            if (e >= rows) break;
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < kRtPre; i++) {
                const int k = tid + kRtThreads * i;
                if (k < n4) {
                    const uint4 wu = ldg_stream(row_ptr(e) + k);
                    acc = __fmaf_rn(__uint_as_float(wu.x), xv[i].x, acc);
                    acc = __fmaf_rn(__uint_as_float(wu.y), xv[i].y, acc);
                    acc = __fmaf_rn(__uint_as_float(wu.z), xv[i].z, acc);
                    acc = __fmaf_rn(__uint_as_float(wu.w), xv[i].w, acc);
                }
            }
            finish(tail(acc, e), e);
        }
        __syncthreads();                                  // rsc of the next token
    }
    if (tid == 0) {
        __threadfence();
        last = atomicAdd(ticket, 1u) == (unsigned)G - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (route_here) {
        if (rc.kind == 0 && T <= 2) {
            // one or two tokens: the whole block routes each in turn
            __shared__ uint32_t rsm[160 + 64];
            for (int t = 0; t < T; t++)
                route_token_block(logits + (size_t)t * rows, E, K, renorm, idx + (size_t)t * K,
                                  w + (size_t)t * K, rsm);
        } else {
            for (int t = warp; t < T; t += kRtThreads / 32)
                route_one(logits + (size_t)t * rows, E, K, rc, renorm, idx + (size_t)t * K,
                          w + (size_t)t * K);
        }
    }
    if (sg_out)
        for (int t = tid; t < T; t += kRtThreads)
            sg_out[t] = wsg ? 1.0f / (1.0f + expf(-__ldcg(logits + (size_t)t * rows + E))) : 1.0f;
    if (tid == 0) *ticket = 0u;
}

int router_launch(const float *Wr, const float *wsg, const float *x, PreNorm pn, int T,
                  int E, int hid, int K, int renorm, RouteCfg rc, float *logits,
                  unsigned *ticket, int *idx, float *w, float *sg_out, cudaStream_t st) {
    WARP_ARG(E >= 1 && E <= 384 && K >= 1 && K <= 64 && K <= E && hid % 4 == 0,
             "router: E must be 1..384, K 1..64 (<= E), hidden a multiple of 4");
    const int rows = E + (wsg ? 1 : 0);
    // a few tokens are routed by the last CTA; many by a launch of their own
    const int route_here = T <= kRouteInKernel;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = rows < sms ? rows : sms;
    cudaError_t e = launch_pdl(router_kernel, dim3(grid), dim3(kRtThreads), 0, st, Wr, wsg, x,
                               pn, T, E, hid, K, renorm, rc, logits, ticket, idx, w, sg_out,
                               route_here);
    if (e != cudaSuccess) return cuda_fail(e, "router_kernel");
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
