// moe_prefill.cuh — the MoE layer for many tokens at once (prefill) on the
// tensor cores: the routed experts as grouped GEMMs over the tokens routed
// to each expert, the shared expert as plain GEMMs over all tokens.
#pragma once
#include "common.cuh"

namespace warp {

// One tcgen05 GEMM launch of the prefill path.  A: weight rows (a VQ3R
// matrix of an expert record, or a Q4G/Q8G-style Q4 matrix of the shared
// expert), B: token rows (the layer input in fp16 by token, or the fp16
// SwiGLU output H by slot), D in tensor memory, then an epilogue (SwiGLU
// pair -> fp16 H, or single -> fp32 slots).
struct PfGemm {
    // A
    const uint8_t *bank;       // expert records (VQ3R)
    size_t rec_bytes;
    int tiled;                 // records in the device tile layout
    uint32_t code_off[2];      // index-block offsets of the pair's matrices (or [0])
    uint32_t sc_off[2];        // fp16 row-scale offsets, same
    const float *books[2];     // fp32 [3][256][8] codebooks per matrix
    const uint8_t *qw[2];      // Q4 rows (shared expert)
    const uint16_t *qs[2];     // Q4 group scales
    int q_group;
    size_t q_rowbytes;
    int M, Kd;                 // rows of A, reduction width
    // B: fp16 rows, copied into the stage as they are
    const uint16_t *Xh;        // [T][Kd] the layer input in fp16 (gate/up launches)
    const uint16_t *Hin;       // [slots][Kd] SwiGLU output (down launches)
    const int *slot_route;     // slot -> route (t*K + j); NULL: slot = token
    int K;
    int T;
    // work: routed n-tiles [0] = count, then (expert, first slot, tokens)
    const int *items;
    // outputs
    uint16_t *Hout;            // pair: fp16 [slot][M]
    float *slots;              // single: fp32 [T][K + 1][hid]
    int hid;
    int *err;                  // a bounded wait gave up
};

// Grouping from the routing of T tokens: counts and first slots per expert,
// slot -> route, the n-tiles.  items holds 1 + 3 * max_items ints.
int prefill_group(const int *idx, int R, int E, int *counts, int *offsets, int *slot_route,
                  int *items, int max_items, cudaStream_t st);

// Launch forms: VQ3R gate+up pair (routed, B from X), VQ3R single (routed
// down, B from H), Q4 pair (shared gate+up, B from X), Q4 single (shared
// down, B from H).  grid_items: the grid's item dimension (upper bound for
// routed launches; ceil(T / 128) for the shared ones).
int prefill_gemm(const PfGemm &g, bool q4, bool pair, int grid_items, cudaStream_t st);

// x [n] fp32 -> xh [n] fp16 (round to nearest), n a multiple of 8, both
// 16-byte aligned: the B operand of the gate/up GEMMs, converted once.
int prefill_half(const float *x, uint16_t *xh, size_t n, cudaStream_t st);

// Upper bound of routed n-tiles for R routes over E experts.
inline int prefill_max_items(int R, int E) { return R / 128 + E; }

}  // namespace warp
