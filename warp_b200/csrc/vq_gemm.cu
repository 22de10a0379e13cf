// vq_gemm.cu — VQ3R dequant GEMM on the tensor cores: the prefill form of
// vq_rows (model.c:3909-3977) for T tokens at once,
//     Y[t][r] = f16(scale[r]) * sum_k W~[r][k] * X[t][k],
//     W~[r][8v + d] = (C0[i0][d] + C1[i1][d]) + C2[i2][d]   (fp32, rounded once to fp16)
// with X rounded to fp16 and fp32 accumulation in tensor memory.  The
// reference builds a table per token and gathers (moe_chunk,
// model.c:7110-7290); with many tokens per matrix the dequantized tile is
// shared by all of them, which is what a GEMM is for.
//
// One CTA (4 warps) owns a 128-row x 128-token tile of Y.  Per 64-wide K
// step every thread dequantizes the 8 code vectors of its weight row and
// converts 64 values of its token row into the stage's operand tiles (the
// layout of umma.cuh); thread 0 then issues four K = 16 MMAs and commits
// them to the stage's mbarrier, and the next step fills the other stage
// while they run.  The epilogue reads the fp32 accumulator from tensor
// memory, applies the row scale in fp32 and writes Y.
#include "umma.cuh"

namespace warp {

constexpr int kGM = 128;                 // weight rows per tile (MMA M)
constexpr int kGN = 128;                 // tokens per tile (MMA N)
constexpr int kGThreads = 128;
constexpr uint32_t kTileBytes = 128 * 64 * 2;                  // 16 KiB per operand tile
constexpr uint32_t kSmBooks = 0;                               // fp32 [3][256][8]
constexpr uint32_t kSmStage = 24576;                           // stage s: A, then B
constexpr uint32_t kSmBar = kSmStage + 2 * 2 * kTileBytes;     // two mbarriers
constexpr uint32_t kSmTmem = kSmBar + 16;                      // tensor-memory base
constexpr int kGSmem = kSmTmem + 16 + 1024;                    // + alignment slack

// Device-side failure of a tensor-core kernel (a bounded wait gave up);
// read and cleared by warp_umma_status.
__device__ int g_umma_err = 0;

// Two floats rounded to fp16 in one register: a in the low half, b in the
// high half (cvt.rn.f16x2.f32 puts its first source in the high half).
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}

__global__ void __launch_bounds__(kGThreads)
vq_matmul_kernel(float *__restrict__ Y, const float *__restrict__ X, int T,
                 const uint8_t *__restrict__ idx, const uint16_t *__restrict__ scale,
                 const float *__restrict__ books, int M, int N) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sp = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * kGM, n0 = blockIdx.y * kGN;
    const int nv = N / kVec, ksteps = (nv + 7) / 8;

    float *sb = (float *)(sp + kSmBooks);
    for (int i = tid; i < kSt * kEnt * kVec / 4; i += kGThreads)
        ((float4 *)sb)[i] = ((const float4 *)books)[i];
    const uint32_t bar0 = base + kSmBar, bar1 = base + kSmBar + 8;
    if (tid == 0) {
        umma::mbar_init(bar0, 1);
        umma::mbar_init(bar1, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) umma::tmem_alloc(base + kSmTmem, kGN);
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tmem = *(volatile uint32_t *)(sp + kSmTmem);
    const uint32_t idesc = umma::idesc_f16(kGM, kGN);

    const int r = m0 + tid, t = n0 + tid;        // this thread's weight row and token
    const bool row_ok = r < M, tok_ok = t < T;
    const uint8_t *rcodes = idx + (size_t)(r >> 6) * nv * (kBlk * kSt) + (r & 63) * kSt;
    const float *xrow = X + (size_t)t * N;
    uint32_t ph0 = 0u, ph1 = 0u;                  // next phase to wait for, per stage
    bool ok = true;
    int issued = 0;                               // steps whose MMAs were issued
    for (int ks = 0; ks < ksteps; ks++) {
        const int s = ks & 1;
        if (ks >= 2) {                            // stage s: step ks-2's MMAs done?
            bool w = umma::mbar_wait(s ? bar1 : bar0, s ? ph1 : ph0, umma::kWaitLimit);
            if (s) ph1 ^= 1u; else ph0 ^= 1u;
            ok = __syncthreads_and(w);
            if (!ok) break;
        }
        uint8_t *Ap = sp + kSmStage + s * 2 * kTileBytes, *Bp = Ap + kTileBytes;
#pragma unroll 2
        for (int j = 0; j < 8; j++) {
            const int v = ks * 8 + j;
            uint4 h = make_uint4(0u, 0u, 0u, 0u);
            if (row_ok && v < nv) {
                const uint8_t *c = rcodes + (size_t)v * (kBlk * kSt);
                const float4 *c0 = (const float4 *)(sb + (0 * kEnt + c[0]) * kVec);
                const float4 *c1 = (const float4 *)(sb + (1 * kEnt + c[1]) * kVec);
                const float4 *c2 = (const float4 *)(sb + (2 * kEnt + c[2]) * kVec);
                const float4 a0 = c0[0], a1 = c0[1], b0 = c1[0], b1 = c1[1], d0 = c2[0], d1 = c2[1];
                h.x = pack_h2((a0.x + b0.x) + d0.x, (a0.y + b0.y) + d0.y);
                h.y = pack_h2((a0.z + b0.z) + d0.z, (a0.w + b0.w) + d0.w);
                h.z = pack_h2((a1.x + b1.x) + d1.x, (a1.y + b1.y) + d1.y);
                h.w = pack_h2((a1.z + b1.z) + d1.z, (a1.w + b1.w) + d1.w);
            }
            *(uint4 *)(Ap + j * (kGM * 16) + tid * 16) = h;
        }
#pragma unroll 2
        for (int j = 0; j < 8; j++) {
            const int k = ks * 64 + j * 8;
            uint4 h = make_uint4(0u, 0u, 0u, 0u);
            if (tok_ok && k < N) {
                const float4 a = *(const float4 *)(xrow + k), b = *(const float4 *)(xrow + k + 4);
                h = make_uint4(pack_h2(a.x, a.y), pack_h2(a.z, a.w), pack_h2(b.x, b.y),
                               pack_h2(b.z, b.w));
            }
            *(uint4 *)(Bp + j * (kGN * 16) + tid * 16) = h;
        }
        umma::fence_smem_async();
        __syncthreads();
        if (tid == 0) {
            umma::fence_after();
            const uint32_t A = base + kSmStage + s * 2 * kTileBytes, B = A + kTileBytes;
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
                umma::mma_f16(tmem, umma::desc(A + 2 * kk * (kGM * 16), kGM * 16, 128),
                              umma::desc(B + 2 * kk * (kGN * 16), kGN * 16, 128), idesc,
                              ks > 0 || kk > 0);
            umma::commit(s ? bar1 : bar0);
        }
        issued = ks + 1;
    }
    // the last issued step's commit covers every MMA before it
    bool done = true;
    if (issued > 0) {
        const int s = (issued - 1) & 1;
        done = umma::mbar_wait(s ? bar1 : bar0, s ? ph1 : ph0, umma::kWaitLimit);
    }
    done = __syncthreads_and(done);
    if (!ok || !done) {
        if (tid == 0) atomicOr(&g_umma_err, 1);
    } else {
        umma::fence_after();
        const int re = m0 + warp * 32 + lane;
        const float sc = re < M ? f16_to_f32(scale[re]) : 0.0f;
        for (int c0 = 0; c0 < kGN; c0 += 16) {
            float v[16];
            umma::tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
            if (re < M) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int n = n0 + c0 + j;
                    if (n < T) Y[(size_t)n * M + re] = v[j] * sc;
                }
            }
        }
    }
    umma::fence_before();
    __syncthreads();
    if (warp == 0) {
        umma::fence_after();
        umma::tmem_free(tmem, kGN);
    }
}

int vq_matmul_launch(float *Y, const float *X, int T, const uint8_t *idx,
                     const uint16_t *scale, const float *books, int M, int N,
                     cudaStream_t st) {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(vq_matmul_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem);
        if (e != cudaSuccess) return cuda_fail(e, "vq_matmul smem attribute");
        attr_done[dev] = true;
    }
    dim3 grid(cdiv(M, kGM), cdiv(T, kGN));
    vq_matmul_kernel<<<grid, kGThreads, kGSmem, st>>>(Y, X, T, idx, scale, books, M, N);
    WARP_CHECK_LAUNCH("vq_matmul_kernel");
    return WARP_OK;
}

}  // namespace warp

using namespace warp;

extern "C" int warp_vq_matmul(float *Y, const float *X, int T, const uint8_t *idx,
                              const uint16_t *scale, const float *books, int M, int N,
                              int cb_base, void *stream) {
    WARP_ARG(Y && X && idx && scale && books && T >= 1 && M >= 1 && N >= 8 && N % 8 == 0 &&
                 cb_base >= 0,
             "warp_vq_matmul: bad arguments (N a multiple of 8)");
    WARP_ARG(((uintptr_t)X & 15) == 0 && ((uintptr_t)books & 15) == 0,
             "warp_vq_matmul: X and books must be 16-byte aligned");
    return vq_matmul_launch(Y, X, T, idx, scale, books + (size_t)cb_base * kEnt * kVec, M, N,
                            (cudaStream_t)stream);
}

extern "C" int warp_umma_status(int clear) {
    int h = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&h, g_umma_err, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "umma status");
    if (clear && h) {
        const int z = 0;
        cudaMemcpyToSymbol(g_umma_err, &z, sizeof(int));
    }
    if (h) {
        set_error("a tensor-core kernel gave up waiting for its MMAs");
        return WARP_E_TIMEOUT;
    }
    return WARP_OK;
}
