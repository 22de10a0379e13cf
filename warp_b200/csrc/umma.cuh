// umma.cuh — the sm_100a tensor-core pieces the prefill GEMMs use:
// tcgen05.mma (kind::f16, one CTA, A and B from shared memory, D in tensor
// memory), its shared-memory matrix descriptors, tensor-memory allocation and
// loads, and mbarrier waits with an iteration limit.
//
// Operand tiles are K-major without swizzle, in "core matrices" of 8 rows x
// 16 bytes (8 fp16 along K) stored as 128 contiguous bytes.  A tile of R rows
// x 64 K is kept as 8 k-groups of R rows x 16 bytes:
//     byte (kg, r) = kg * (R * 16) + r * 16
// so one MMA instruction (K = 16: k-groups 2kk and 2kk+1) sees rows 8 apart
// at SBO = 128 bytes and its second k-group at LBO = R * 16 bytes.
#pragma once
#include "common.cuh"

namespace warp {
namespace umma {

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"): start
// address, leading and stride byte offsets in 16-byte units, version 1 at
// bits 46-47, no swizzle (layout type 0 at bits 61-63), base offset 0.
__device__ __forceinline__ uint64_t desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) |
           ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
           ((uint64_t)1 << 46);
}

// Instruction descriptor of kind::f16 with fp16 A and B (both K-major) and
// an fp32 D of M x N: D format at bits 4-5, N >> 3 at bits 17-22, M >> 4 at
// bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A * B^T for one K = 16 slice; issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b,
                                        uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// The mbarrier at `bar` gets one arrive when every MMA this thread issued
// before has completed.
__device__ __forceinline__ void commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}

__device__ __forceinline__ void fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy writes to shared memory become visible to the tensor core.
__device__ __forceinline__ void fence_smem_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Tensor-memory allocation by one whole warp; the base address lands in
// shared memory at `slot`.  ncols is a power of two >= 32.
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(slot), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 ::"r"(taddr), "r"(ncols) : "memory");
}

// 16 consecutive fp32 columns of this thread's tensor-memory lane (warp w of
// a warpgroup reads lanes 32w..32w+31; taddr carries the lane in bits 16-31).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Wait for phase `parity` of the mbarrier to complete; gives up after
// `limit` polls and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done) : "r"(bar), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// Polls before an mbarrier wait gives up (each poll may itself wait a
// while in hardware): far longer than any tile's MMAs take.
constexpr uint32_t kWaitLimit = 1u << 22;

}  // namespace umma
}  // namespace warp
