// router.cuh — launch interface of the router kernels.
#pragma once
#include "common.cuh"

namespace warp {

constexpr int kRouterSplit = 16;

// Logits (plus the shared-gate row when wsg != NULL) and the exact top-k.
// part: [T][E+1][kRouterSplit] scratch; prob_ws: [T][E] scratch.
int router_launch(const float *Wr, const float *wsg, const float *x, int T,
                  int E, int hid, int K, int renorm, float *part,
                  float *prob_ws, int *idx, float *w, float *sg_out,
                  float *logits_out, cudaStream_t st);

int route_only(const float *logits, int T, int E, int K, int renorm,
               float *prob_ws, int *idx, float *w, cudaStream_t st);

}  // namespace warp
