// router.cuh — launch interface of the router kernels.
#pragma once
#include "common.cuh"

namespace warp {

// Logits (plus the shared-gate row when wsg != NULL) and the exact top-k in
// one launch.  parts: [T][rows][2] scratch; logits: [T][rows] output, rows =
// E + (wsg ? 1 : 0); ticket: a device counter that is 0 before the launch
// and 0 again after it (one per concurrently running launch).
int router_launch(const float *Wr, const float *wsg, const float *x, int T,
                  int E, int hid, int K, int renorm, float *parts, float *logits,
                  unsigned *ticket, int *idx, float *w, float *sg_out, cudaStream_t st);

int route_only(const float *logits, int T, int E, int K, int renorm, int *idx, float *w,
               cudaStream_t st);

}  // namespace warp
