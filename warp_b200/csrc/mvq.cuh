// mvq.cuh — launch interface of the Q4G/Q8G dequant-matvec.
#pragma once
#include "common.cuh"

namespace warp {

constexpr int kMvqMaxBatch = 64;    // tokens one matvec takes (WASTE_CHUNK_MAX, model.h:532)

// Up to two weight tensors with the same input (the shared expert's gate and
// up); rows of segment 1 follow segment 0 in the output.
struct MvqSeg {
    const uint8_t *W;
    const uint16_t *ws;
    int rows;
    int y_off;
};

struct MvqArgs {
    MvqSeg seg[2];
    int nseg;
    int total_rows;
    int in, group, ng, bits;
    int group_shift;        // log2(group) when a power of two, else -1 (set by mvq_launch)
    size_t rowbytes;
    int batch;
    const void *X;          // [batch][in], fp32 or bf16
    int x_bf16;
    const float *act_a;     // SwiGLU input mode: x = silu(a) * b, [batch][stride]
    const float *act_b;
    long long act_stride;
    float *Y;               // Y[b * y_stride + y_off + r]
    long long y_stride;
    int pair;               // seg[0]/seg[1] rows computed together, Y = silu(g)*u
    int x_smem;             // set by mvq_launch
    void *xf;               // fragment scratch (mvq_xf_bytes): the tensor-core path
};

// The shared expert's down projection in fixed column blocks: block b of nb
// covers input columns [b*in/nb, (b+1)*in/nb), a whole number of groups.
//   P[b*pb_stride + t*pt_stride + o] = sum over the block's groups k, in
//   order, of f16(ws[o*ng + k]) * sum_i q(o, k*group + i) * x[t][k*group + i]
// with x = act_a (act_b NULL: the SwiGLU already applied) or silu(act_a) *
// act_b (the gate/up outputs): lane l
// of the (row, block)'s lane group sums its groups l, l + L, ... in order,
// and the group meets in a fixed xor tree.  The arithmetic of a block does
// not depend on which other blocks a launch covers, so the partials of a
// rank that owns some blocks equal the one-GPU launch's bit for bit.
struct MvqBlocks {
    const uint8_t *W;
    const uint16_t *ws;
    int rows, in, group, bits;
    size_t rowbytes;
    int nb, b0, b1;             // blocks b0..b1-1 of nb
    int batch;
    const float *act_a, *act_b;
    long long act_stride;
    float *P;
    long long pb_stride, pt_stride;
    int fold;                   // 1: every block here, P + t * pt gets their sum
};

int mvq_blocks_launch(const MvqBlocks &a, cudaStream_t st);

__device__ __forceinline__ float silu_mul(float g, float u) {
    return (g / (1.0f + expf(-g))) * u;
}

// Activation k of token b as the matvec reads it (0 past `in`).
__device__ __forceinline__ float x_at(const MvqArgs &a, int b, int k) {
    if (k >= a.in) return 0.0f;
    if (a.act_a) {
        const float g = a.act_a[(size_t)b * a.act_stride + k];
        const float u = a.act_b[(size_t)b * a.act_stride + k];
        return silu_mul(g, u);
    }
    if (a.x_bf16)
        return __bfloat162float(((const __nv_bfloat16 *)a.X)[(size_t)b * a.in + k]);
    return ((const float *)a.X)[(size_t)b * a.in + k];
}

// The tensor-core matmul for batch 2..64 (mvq_umma.cu): a.xf must hold
// mvq_xf_bytes(batch, in, rows) bytes, 256-byte aligned.
int launch_umma(const MvqArgs &a, cudaStream_t st);

// Scratch the tensor-core path needs for `batch` activations of width `in`.
size_t mvq_xf_bytes(int batch, int in, int rows);

// The dequant-matvec.  With a.xf set, no pair mode and batch >= 2 it runs
// on the tensor cores (mma.sync, exact fp16 weights, activations split into
// fp16 high and low parts, fp32 accumulation rescaled per weight group in
// registers); otherwise on the CUDA cores.
int mvq_launch(MvqArgs a, cudaStream_t st);

}  // namespace warp
