// common.cuh — shared helpers for the warp_b200 sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/warp_cuda.h"

namespace warp {

// Thread-local error text behind warp_last_error().
void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);
void count_launch(unsigned n = 1);

#define WARP_CHECK_LAUNCH(what)                                            \
    do {                                                                    \
        cudaError_t e_ = cudaGetLastError();                               \
        if (e_ != cudaSuccess) return ::warp::cuda_fail(e_, what);          \
        ::warp::count_launch();                                            \
    } while (0)

#define WARP_ARG(cond, ...)                                                \
    do {                                                                    \
        if (!(cond)) { ::warp::set_error(__VA_ARGS__); return WARP_E_ARG; } \
    } while (0)

constexpr int kVec = 8;       // vec_dim
constexpr int kEnt = 256;     // entries per stage
constexpr int kSt = 3;        // VQ3R stages
constexpr int kBlk = 64;      // index_block rows

// waste_f16 (simd.h:81-99): fp16 -> fp32 with subnormals kept as
// mantissa * 2^-24, and no special case for exponent 31 (an fp16 inf/NaN
// pattern becomes the finite value its bits spell with a rebased exponent).
__device__ __forceinline__ float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1f, mn = h & 0x3ff;
    if (e == 0) {
        const float f = (float)mn * 5.9604644775390625e-08f;
        return sign ? -f : f;
    }
    return __uint_as_float(sign | ((e + 112u) << 23) | (mn << 13));
}

// The same value through the hardware conversion, which agrees with it for
// every exponent but 31 (infinities and NaNs in IEEE fp16, finite here).
__device__ __forceinline__ float f16_to_f32_fast(uint16_t h) {
    float f = __half2float(__ushort_as_half(h));
    if ((h & 0x7c00u) == 0x7c00u)
        f = __uint_as_float(((uint32_t)(h >> 15) << 31) | (143u << 23) | ((uint32_t)(h & 0x3ffu) << 13));
    return f;
}

// The codebook decode of the loader (model.c:2916-2922): subnormals flushed.
__device__ __forceinline__ float f16_to_f32_ftz(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1f, man = h & 0x3ff;
    const uint32_t bits = e ? (sign | ((e + 112u) << 23) | (man << 13)) : sign;
    return __uint_as_float(bits);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// L1-allocating read-only 128-bit load: two lanes' consecutive 16-byte
// pieces of one 32-byte sector are then fetched from L2 once.
__device__ __forceinline__ uint4 ldg_nc(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Bulk prefetch of [p, p + bytes) into L2: no data returned, issued by one
// thread for its own CTA.  p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes)
                 : "memory");
}

// 16-byte asynchronous global -> shared copy (no L1 allocation), grouped
// and waited on per thread.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint4 lds_u4(uint32_t saddr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
    return v;
}

__device__ __forceinline__ float lds_f32(uint32_t saddr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(saddr));
    return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

inline unsigned cdiv(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while the kernel before it on the stream is still running: everything it
// does before pdl_wait() overlaps that kernel's tail, so it must read only
// data written two or more kernels back (or constant weights).  pdl_wait()
// returns once the previous kernel has finished and its writes are visible;
// pdl_trigger() lets the next kernel start.  Both are no-ops in a kernel
// launched without the attribute.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// WARP_PDL=0 in the environment launches these kernels as plain launches.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace warp
