// router.cuh — launch interface of the router kernels.
#pragma once
#include "common.cuh"

namespace warp {

// Which router a layer has: kind 0, Qwen's softmax top-k
// (waste_qwen_moe_route, qwen_moe.c:10-44); kind 1, moe_layer's
// (model.c:5466-5556) with score function func (0 sigmoid, 1 softmax, 2
// sqrt-softplus, as model.h:179-181 numbers them), a selection-only bias
// (fp32 [E] or NULL) and routed_scale.
struct RouteCfg {
    int kind = 0;
    int func = 0;
    const float *bias = nullptr;
    float scale = 1.0f;
};

// Logits (plus the shared-gate row when wsg != NULL) and the exact top-k in
// one launch.  parts: [T][rows][2] scratch; logits: [T][rows] output, rows =
// E + (wsg ? 1 : 0); ticket: a device counter that is 0 before the launch
// and 0 again after it (one per concurrently running launch).
int router_launch(const float *Wr, const float *wsg, const float *x, int T, int E, int hid,
                  int K, int renorm, RouteCfg rc, float *parts, float *logits,
                  unsigned *ticket, int *idx, float *w, float *sg_out, cudaStream_t st);

int route_only(const float *logits, int T, int E, int K, int renorm, int *idx, float *w,
               cudaStream_t st);
int route_scored_only(const float *logits, int T, int E, int K, RouteCfg rc, int renorm,
                      int *idx, float *w, cudaStream_t st);

}  // namespace warp
