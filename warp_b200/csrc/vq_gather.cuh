// vq_gather.cuh — the VQ3R decode gather, y[r] = sum_v T_v[i0]+T_v[i1]+T_v[i2].
//
// This is the arithmetic of vq_rows (model.c:3909-3977) laid out for an SM:
//
//  * A CTA owns one "segment" at a time: one lookup table (one x vector and
//    one codebook triple) restricted to a chunk of 32 vector positions, and
//    a range of 16-row quarters of the matrices that read that table.
//  * The chunk's table (32 positions x 3 stages x 256 entries, fp32) sits in
//    shared memory BANK-SLICED: every entry of position p lives in bank p.
//    Lane p of every warp handles position p, so the 32 lookups of a warp
//    instruction hit 32 different banks whatever the codes are — the random
//    gather is conflict-free.
//  * The two regions holding the table start at 64 KiB-aligned shared
//    addresses, so a lookup address is one PRMT: byte 0 = 4*lane (+128 for
//    the second table of a region), byte 1 = the code, byte 2 = the region.
//        region A (0x10000): stage 0 at code*256 + 4p, stage 1 at +128
//        region B (0x20000): stage 2 at code*256 + 4p (the +128 slot spare)
//  * Tables are built once per (vector, chunk) into global memory in that
//    exact layout ("images", 96 KiB each, compact: region A's 64 KiB, then
//    region B's used 32 KiB) and copied into shared memory by the CTAs that
//    use them.
//  * Each lane streams its position's code bytes for 16 rows at a time
//    straight into registers, two quarters ahead of their use, produces 16
//    per-row partials, and the warp reduces them across lanes with a
//    transpose-reduce (vq_gather.cu).
//  * Partials go to partial[chunk][matrix-row]; the consumer sums the chunks
//    in order and applies the row scale.
#pragma once
#include "common.cuh"

namespace warp {

constexpr int kChunk = 32;
constexpr uint32_t kRegA = 0x10000u;
constexpr uint32_t kRegB = 0x20000u;
constexpr uint32_t kRegEnd = 0x30000u;
#ifndef WARP_GATHER_THREADS
#define WARP_GATHER_THREADS 512
#endif
constexpr int kGatherThreads = WARP_GATHER_THREADS;
constexpr int kGatherSmem = 227 * 1024;        // the whole window: one CTA/SM
constexpr int kImageWords = 24576;             // compact image: A 16384 + B 8192 words

// Word of the compact image holding stage s, code, position p of a chunk.
__host__ __device__ __forceinline__ int image_word(int s, int code, int p) {
    return s < 2 ? code * 64 + s * 32 + p : 16384 + code * 32 + p;
}

// One table entry: the FMA chain of lutb_range_avx512 (simd_avx512.c:90-127),
// sum over d = 0..7 from 0 of x[d] * C[d], one rounding per step.
__device__ __forceinline__ float lut_entry(const float (&x)[kVec], const float *C) {
    float t = 0.0f;
#pragma unroll
    for (int d = 0; d < kVec; d++) t = __fmaf_rn(x[d], C[d], t);
    return t;
}

// Where a quarter's codes and its output rows come from.
struct GatherArgs {
    int nv;                 // vector positions per row
    int nchunks;            // ceil(nv / 32)
    int M;                  // rows per matrix
    int qb_per_mat;         // 16-row quarters per matrix = 4*ceil(M/64)
    int mpg;                // matrices per group (sharing one table)
    int gpt;                // groups per token (2: gate/up, K: down, 1: plain)
    int K;                  // routes per token
    int n_groups;
    long long total;        // n_groups * nchunks * mpg * qb_per_mat
    float *partial;         // [nchunks][n_groups * mpg * M]
    // matrices: either one plain index array, or routed expert records
    const uint8_t *idx_plain;
    const uint8_t *bank;
    size_t rec_bytes;
    uint32_t kind_off[3];   // gate, up, down index offsets in a record
    const int *route_idx;   // [T*K] expert ids
    // tables: compact images, segment (g, c) at image + (g*nchunks + c)*kImageWords
    const uint32_t *image;
    int *err;               // set non-zero when the smem window does not fit
    // Route-list (expert-parallel) mode when plan != NULL: the work is the
    // plan[0] routes this rank owns, one matrix per group (mpg = 1); group g
    // is work route g / gpt, of kind g % 2 (gate/up, gpt = 2, tables of the
    // route's token: image (t*2 + kind)) or down (gpt = 1, image g).
    // plan[1 + r] = route t*K + j, plan[1 + max_routes + r] = record index
    // in the bank.  n_groups = max_routes * gpt fixes the partial layout;
    // total is an upper bound used only to size the grid.
    const int *plan;
    int max_routes;
    // 1: route_idx / plan were written two or more kernels back on the
    // stream, so code loads may start before the wait for the previous
    // kernel (programmatic dependent launch); 0: they come from it.
    int early;
};

int gather_setup();
int gather_grid(long long total);
int sm_count();
// Launch the gather; tiled = the matrices are in the device tile layout
// bank_tile writes.
int gather_launch(const GatherArgs &a, bool tiled, cudaStream_t st);

// Re-tile matrix kind `off` (index-block offset inside each record) of E
// records in place into the tile layout the gather reads fastest.
int bank_tile(uint8_t *bank, size_t rec_bytes, uint32_t off, int M, int nv, int E,
              cudaStream_t st);

// Images of the gate/up tables of T tokens: group g = 2t + kind reads
// x + t*nv*8 and codebooks cb0 + 3*kind; images[(g*nchunks + c)*kImageWords].
int lut_images(uint32_t *images, const float *x, int T, int nv, const float *books,
               int cb0, cudaStream_t st);

// warp_vq_apply, bandwidth path: slice the caller's LUT, gather, finish.
int vq_apply_gather(float *y, const uint8_t *idx, const uint16_t *scale,
                    const float *lut, int M, int nv, cudaStream_t st);

// The same with fixed module-scope scratch and no allocation; returns
// WARP_E_ARG when vq_apply_noalloc_bytes(M, nv) exceeds the fixed size.
size_t vq_apply_noalloc_bytes(int M, int nv);
int vq_apply_gather_noalloc(float *y, const uint8_t *idx, const uint16_t *scale,
                            const float *lut, int M, int nv, cudaStream_t st);

// vq_rows order, bit-exact (vq.cu).
int vq_apply_ordered_launch(float *y, const uint8_t *idx, const uint16_t *scale,
                            const float *lut, int M, int nv, cudaStream_t st);

}  // namespace warp
