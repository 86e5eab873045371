// pokit_tc.cuh -- fifth-generation tensor-core (tcgen05) building blocks for
// sm_100a: tensor-memory allocation, MMA issue with shared-memory and
// tensor-memory operands, completion through mbarriers, and tensor-memory
// loads/stores.  Every wait on an mbarrier is bounded (mbar_wait).
//
// Operand layouts used by this library (kind::f16, fp16 A and B, f32 D):
//   A in tensor memory   row m of an M = 128 tile is lane m; K runs along
//                        32-bit columns, two fp16 values per column (the
//                        even K element in the low half).  One MMA (K = 16)
//                        reads 8 columns.
//   A, B in shared       K-major, no swizzle: 8 x 16-byte "core matrices"
//   memory               (8 rows x 8 fp16, 128 contiguous bytes); the core
//                        matrices of consecutive 8-row groups are `sbo` bytes
//                        apart and the two K halves of one MMA (K 0..7 and
//                        8..15) are `lbo` bytes apart.
//   D in tensor memory   row m is lane m, column n is the n-th 32-bit column.
#pragma once

#include <stdint.h>

#include "pokit_mma.cuh"

namespace pokit {

// Shared-memory matrix descriptor (K-major, no swizzle).
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;   // descriptor version for sm_100
    return d;                              // base offset 0, layout type 0 (no swizzle)
}

// Instruction descriptor for kind::f16 with fp16 A and B, f32 accumulation,
// both operands K-major, an M x N tile (M = 64 or 128, N a multiple of 16).
__host__ __device__ constexpr uint32_t tc_idesc_f16(uint32_t m, uint32_t n) {
    return (1u << 4)                 // D format f32
           | (0u << 7) | (0u << 10)  // A, B format f16
           | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Orders this thread's tensor-core operations against a thread
// synchronisation (barrier or mbarrier) that follows / precedes it.
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The mbarrier receives one arrival once every tcgen05 operation this thread
// issued before the commit has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// D (+)= A x B with A in tensor memory.  accumulate = 0 overwrites D.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// D (+)= A x B with both operands in shared memory.
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// Tensor-memory address of lane `lane`, column `col` relative to `base`.
__device__ __forceinline__ uint32_t tmem_at(uint32_t base, uint32_t lane, uint32_t col) {
    return base + (lane << 16) + col;
}

// A warp moves 8 consecutive 32-bit columns of its 32 lanes (thread i <->
// lane base + i); `taddr` holds the warp's first lane (32 * (warp % 4)).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
// 32 consecutive columns per lane in one instruction.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
// Loads and stores above are asynchronous: wait before using loaded
// registers / before handing stored columns to the tensor core.
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Untiled bulk copy global -> shared completing on `bar` (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* m) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(m)) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Waits for phase `parity` of the mbarrier for at most `limit_ns` of wall
// time; false when it gave up.  Each try_wait suspends the thread until the
// phase completes or `kSuspendNs` passes, so waiting warps take no issue
// slots from working ones.
constexpr uint32_t kSuspendNs = 1000000u;
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* m, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
    uint32_t ok = 0;
    uint64_t start = 0;
    for (uint32_t it = 0; !ok; ++it) {
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(smem_addr(m)), "r"(parity), "r"(kSuspendNs)
            : "memory");
        if (ok) break;
        if (it == 0) start = global_ns();
        else if (global_ns() - start > limit_ns) return false;
    }
    return true;
}
// Makes this thread's generic-proxy shared-memory writes visible to the
// async proxy (tensor-core operand reads, bulk copies).
__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace pokit
