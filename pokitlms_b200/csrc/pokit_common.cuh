// pokit_common.cuh -- shared device helpers for the sm_100a MoE expert kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pokit_types.h"

namespace pokit {

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

// 128-bit read-only global load that does not allocate in L1: weight bytes are
// touched exactly once per token.
__device__ __forceinline__ uint4 ldg_stream128(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_stream32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// Asks the TMA unit to stream [p, p + bytes) from HBM into L2 without
// occupying registers or shared memory.  p and bytes must be 16-byte multiples.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch an arbitrary byte range into L2 in <= 1 MiB bulk pieces, rounding
// the range outward to 16-byte boundaries.
__device__ __forceinline__ void prefetch_l2_range(const void* p, uint64_t bytes) {
    if (bytes == 0) return;
    uint64_t begin = reinterpret_cast<uint64_t>(p) & ~uint64_t(15);
    const uint64_t end = (reinterpret_cast<uint64_t>(p) + bytes + 15) & ~uint64_t(15);
    while (begin < end) {
        const uint64_t n = (end - begin) < (1u << 20) ? (end - begin) : (1u << 20);
        prefetch_l2_bulk(reinterpret_cast<const void*>(begin), static_cast<uint32_t>(n));
        begin += n;
    }
}

// Packed FP32x2 arithmetic (sm_100): two IEEE FP32 results per instruction.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(reinterpret_cast<unsigned long long&>(d))
        : "l"(reinterpret_cast<unsigned long long&>(a)),
          "l"(reinterpret_cast<unsigned long long&>(b)),
          "l"(reinterpret_cast<unsigned long long&>(c)));
    return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(reinterpret_cast<unsigned long long&>(d))
        : "l"(reinterpret_cast<unsigned long long&>(a)),
          "l"(reinterpret_cast<unsigned long long&>(b)));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Release/acquire helpers for the cross-CTA "last block" hand-off.
__device__ __forceinline__ uint32_t atomic_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

}  // namespace pokit
