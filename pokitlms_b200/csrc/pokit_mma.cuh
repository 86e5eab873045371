// pokit_mma.cuh -- tensor-core Q4_K dequant-dot for decode batch 1 (sm_100a).
//
// A warp computes 16 rows of y = W x for a Q4_K matrix W with one
// mma.sync.m16n8k16 (f16 inputs, f32 accumulate) per (sub-block, 16 weights):
//
//   A (16 x 16)  = q * s  for 16 rows and 16 weights of one 32-weight sub-block
//                  (q the 4-bit quant, s its 6-bit scale).  q*s <= 945 is an
//                  integer, exact in fp16; it is formed with one fp16x2 FMA from
//                  the nibble OR-ed into the mantissa of 1024 (or 1024 + 16q for
//                  high nibbles): (1024 + q)*s - 1024*s.
//   B (16 x 8)   = column 0: x_hi = fp16(x'), column 1: x_lo = fp16(x' - x_hi),
//                  columns 2..7 zero, with x' = x * 2^-e per superblock so that
//                  |x'| stays inside fp16 range.  x_hi + x_lo carries ~22
//                  significant bits of x'.
//   D (16 x 8)   accumulates all 8 sub-blocks of a superblock; D[r][0] + D[r][1]
//                = sum_j s_j sum_i q_ij x'_i.
//   mins         one more mma with A = m_j (k = j) and B = -sum_{i in j} x'_i.
//   per superblock and row: acc += (d * 2^e) * D1 + (dmin * 2^e) * D2, FP32.
//
// Algebraically this is sum_i (d*s_j*q_i - dmin*m_j) * x_i, the reference's
// decode_q4_k (src/quantized_linear.cpp:166-205) dotted with x; the products
// are exact and the sums are FP32, so results agree with the reference's FP32
// loop to ~1e-6 relative.
//
// Fragment layout (PTX m16n8k16 .f16): thread (g = lane/4, t = lane%4) holds
// A rows g and g+8 at k = {2t, 2t+1, 2t+8, 2t+9} and B column g at the same k.
// The 16 k-positions of a slice map to weight bytes of a 32-byte qs chunk so
// that thread t reads 8 contiguous bytes per row and chunk: slice s of the
// chunk, k = 2t, 2t+1, 2t+8, 2t+9  <->  bytes 8t+4s + {0, 2, 1, 3}.
#pragma once

#include <cuda.h>   // CUtensorMap

#include "pokit_common.cuh"

namespace pokit {

constexpr uint32_t kHalfMagic = 0x64006400u;     // (1024, 1024) in fp16x2
constexpr uint32_t kHalfNeg1024 = 0xE400E400u;   // (-1024, -1024)
constexpr uint32_t kHalfInv16 = 0x2C002C00u;     // (1/16, 1/16)
constexpr uint32_t kHalfNeg64 = 0xD400D400u;     // (-64, -64)

__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// TMA tensor copies with an mbarrier; every wait is bounded.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* m, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(m)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* m, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(m)), "r"(bytes)
                 : "memory");
}
// Waits for phase `parity` of the mbarrier; gives up after ~`limit` polls
// (each try_wait suspends the thread for a short hardware-chosen time).
__device__ __forceinline__ bool mbar_wait(uint64_t* m, uint32_t parity, uint32_t limit = 4000000u) {
    uint32_t ok = 0;
    for (uint32_t it = 0; it < limit && !ok; ++it) {
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(smem_addr(m)), "r"(parity)
            : "memory");
    }
    return ok != 0;
}
// One box of a 3-D tensor map (x = byte column, y = row, z = expert) into
// shared memory, completing on `bar`.  x must be a multiple of 16.
__device__ __forceinline__ void tma_box_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}
// 16-byte asynchronous global -> shared copy through L2 (no L1 allocation);
// completion by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// A superblock box: 16 rows x 144 bytes, rows 144 bytes apart in shared
// memory.  With that pitch the (row g, lane t) 8-byte reads of a fragment
// fall on distinct bank pairs two lanes at a time: two wavefronts, the
// minimum for 256 bytes.
constexpr uint32_t kBoxRows = 16, kBoxBytes = 16u * 144u;

// ---------------------------------------------------------------------------
// Activation fragments.  One record of kFragWords 32-bit words per superblock
// (256 activations):
//   [0, 256)   B fragments: word ((j*2 + s)*8 + t*2 + half)*2 + {0, 1} holds the
//              two fp16x2 pairs thread t needs for sub-block j, slice s, hi
//              (half 0) or lo (half 1) -- the 8 lanes that load B read 8
//              consecutive 8-byte slots, so the loads are bank-conflict free
//   [256, 264) min fragments: word t*2 + half = fp16x2 (-gsum_{2t}, -gsum_{2t+1})
//   264        the superblock's scale 2^e (float bits); x' = x * 2^-e
// ---------------------------------------------------------------------------
constexpr uint32_t kFragWords = 272;

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(a))) |
           (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(b))) << 16);
}
__device__ __forceinline__ float half_round(float a) { return __half2float(__float2half_rn(a)); }

// One warp builds the record of one superblock from v[0..256).  Every input
// is read into registers before the first write, so v may alias rec (the
// values staged in the record's own space) and be in global or shared memory;
// v and rec are 16-byte aligned.
// The eight 32-element group sums come from one reduce-scatter (lane L ends
// with the sum of group (L >> 2) & 7) instead of eight warp reductions.
__device__ __forceinline__ void q4k_frag_superblock(const float* v, uint32_t* rec, int lane) {
    float x[8];
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        x[j] = v[32 * j + lane];
        m = fmaxf(m, fabsf(x[j]));
    }
    // B-fragment items (j, s, t) = lane and lane + 32: elements
    // 32j + 8t + 4s + {0, 2, 1, 3} (chunk c = j/2, nibble half j%2).
    // Item (j, s, t) = lane + 32h covers elements 4 (8j + 2t + s) + {0, 2, 1, 3}:
    // one 16-byte read per item (a permutation of the warp's slots).
    float it[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int item = lane + 32 * h;
        const int t = item & 3, s = (item >> 2) & 1, j = item >> 3;
        const float4 q = *reinterpret_cast<const float4*>(v + 4 * (8 * j + 2 * t + s));
        it[h][0] = q.x;
        it[h][1] = q.z;
        it[h][2] = q.y;
        it[h][3] = q.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // Keep |x'| <= 2^10 so that x' and the 32-element group sums (<= 2^15)
    // stay inside fp16 range.
    int e = 0;
    if (m > 1024.0f) {
        int ex;
        frexpf(m, &ex);
        e = ex - 10;
    }
    const float inv = ldexpf(1.0f, -e);
    // Reduce-scatter of the eight group sums of x' (lane bits 4, 3, 2 pick
    // the group, bits 1, 0 are summed last).
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float keep = (b4 ? x[4 + i] : x[i]) * inv, send = (b4 ? x[i] : x[4 + i]) * inv;
        y[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float z[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float keep = b3 ? y[2 + i] : y[i], send = b3 ? y[i] : y[2 + i];
        z[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float w = (b2 ? z[1] : z[0]) + __shfl_xor_sync(0xffffffffu, b2 ? z[0] : z[1], 4);
    w += __shfl_xor_sync(0xffffffffu, w, 2);
    w += __shfl_xor_sync(0xffffffffu, w, 1);
    // Lanes 0..7 write min word t*2 + half: groups 2t and 2t+1.
    const int tq = (lane >> 1) & 3;
    const float gA = __shfl_sync(0xffffffffu, w, (2 * tq) << 2);
    const float gB = __shfl_sync(0xffffffffu, w, (2 * tq + 1) << 2);
    __syncwarp();                                   // all reads of v are done
    // Item (j, s, t) fills words ((j*2 + s)*8 + t*2)*2 .. +3 = 4 * item: one
    // 16-byte write per item.
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int item = lane + 32 * h;
        const float e0 = it[h][0] * inv, e1 = it[h][1] * inv;
        const float e2 = it[h][2] * inv, e3 = it[h][3] * inv;
        *reinterpret_cast<uint4*>(rec + 4 * item) =
            make_uint4(pack_half2(e0, e1), pack_half2(e2, e3), pack_half2(e0 - half_round(e0), e1 - half_round(e1)),
                       pack_half2(e2 - half_round(e2), e3 - half_round(e3)));
    }
    if (lane < 8) {
        const int half = lane & 1;
        const float g0 = -gA, g1 = -gB;
        rec[256 + lane] = half == 0 ? pack_half2(g0, g1)
                                    : pack_half2(g0 - half_round(g0), g1 - half_round(g1));
    }
    if (lane == 0) rec[264] = __float_as_uint(ldexpf(1.0f, e));
}

// One superblock of 16 rows (rows g and g+8 at `sb0p` / `sb1p`, 144 bytes
// each, in shared memory) dotted with the activation record `rec`.  Adds the
// FP32 results for rows g (acc0) and g+8 (acc1); valid in lanes with t == 0.
__device__ __forceinline__ void q4k_mma_superblock(const uint8_t* __restrict__ b0p, const uint8_t* __restrict__ b1p,
                                                   const uint32_t* __restrict__ rec, float& acc0, float& acc1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const bool bact = g < 2;
    const uint4 h0 = *reinterpret_cast<const uint4*>(b0p);
    const uint4 h1 = *reinterpret_cast<const uint4*>(b1p);
    uint2 q0[4], q1[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        q0[c] = *reinterpret_cast<const uint2*>(b0p + 16 + 32 * c + 8 * t);
        q1[c] = *reinterpret_cast<const uint2*>(b1p + 16 + 32 * c + 8 * t);
    }
    // 6-bit scales s0..7 and mins m0..7 as bytes (decode_q4_k's scale_min).
    const uint32_t sA0 = h0.y & 0x3F3F3F3Fu, sB0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t sA1 = h1.y & 0x3F3F3F3Fu, sB1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    const uint32_t mA0 = h0.z & 0x3F3F3F3Fu, mB0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t mA1 = h1.z & 0x3F3F3F3Fu, mB1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    const uint32_t* xbl = rec + (t * 2 + (g & 1)) * 2;
    // Two accumulators (even and odd chunks) halve the dependent mma chain.
    float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t sw0 = c < 2 ? sA0 : sB0, sw1 = c < 2 ? sA1 : sB1;
        const uint32_t jl = (2 * c) & 3, jh = (2 * c + 1) & 3;
        const uint32_t Sl0 = hsub2u(__byte_perm(sw0, 0x64u, 0x4040u | (jl << 8) | jl), kHalfMagic);
        const uint32_t Sl1 = hsub2u(__byte_perm(sw1, 0x64u, 0x4040u | (jl << 8) | jl), kHalfMagic);
        uint32_t Sh0 = hsub2u(__byte_perm(sw0, 0x64u, 0x4040u | (jh << 8) | jh), kHalfMagic);
        uint32_t Sh1 = hsub2u(__byte_perm(sw1, 0x64u, 0x4040u | (jh << 8) | jh), kHalfMagic);
        const uint32_t Cl0 = hmul2u(Sl0, kHalfNeg1024), Cl1 = hmul2u(Sl1, kHalfNeg1024);
        const uint32_t Ch0 = hmul2u(Sh0, kHalfNeg64), Ch1 = hmul2u(Sh1, kHalfNeg64);
        Sh0 = hmul2u(Sh0, kHalfInv16);
        Sh1 = hmul2u(Sh1, kHalfInv16);
        float* dc = d[c & 1];
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const uint32_t w0 = s ? q0[c].y : q0[c].x, w1 = s ? q1[c].y : q1[c].x;
            const uint32_t w08 = w0 >> 8, w18 = w1 >> 8;
            const uint32_t a0 = hfma2u((w0 & 0x000F000Fu) | kHalfMagic, Sl0, Cl0);
            const uint32_t a1 = hfma2u((w1 & 0x000F000Fu) | kHalfMagic, Sl1, Cl1);
            const uint32_t a2 = hfma2u((w08 & 0x000F000Fu) | kHalfMagic, Sl0, Cl0);
            const uint32_t a3 = hfma2u((w18 & 0x000F000Fu) | kHalfMagic, Sl1, Cl1);
            const uint2 bl = bact ? *reinterpret_cast<const uint2*>(xbl + ((2 * c) * 2 + s) * 16)
                                  : make_uint2(0u, 0u);
            mma16816(dc, a0, a1, a2, a3, bl.x, bl.y);
            const uint32_t e0 = hfma2u((w0 & 0x00F000F0u) | kHalfMagic, Sh0, Ch0);
            const uint32_t e1 = hfma2u((w1 & 0x00F000F0u) | kHalfMagic, Sh1, Ch1);
            const uint32_t e2 = hfma2u((w08 & 0x00F000F0u) | kHalfMagic, Sh0, Ch0);
            const uint32_t e3 = hfma2u((w18 & 0x00F000F0u) | kHalfMagic, Sh1, Ch1);
            const uint2 bh = bact ? *reinterpret_cast<const uint2*>(xbl + ((2 * c + 1) * 2 + s) * 16)
                                  : make_uint2(0u, 0u);
            mma16816(dc, e0, e1, e2, e3, bh.x, bh.y);
        }
    }
    const uint32_t mw0 = t < 2 ? mA0 : mB0, mw1 = t < 2 ? mA1 : mB1;
    const uint32_t ja = (2 * t) & 3;
    const uint32_t M0 = hsub2u(__byte_perm(mw0, 0x64u, 0x4040u | ((ja + 1) << 8) | ja), kHalfMagic);
    const uint32_t M1 = hsub2u(__byte_perm(mw1, 0x64u, 0x4040u | ((ja + 1) << 8) | ja), kHalfMagic);
    const uint32_t bm = bact ? rec[256 + t * 2 + (g & 1)] : 0u;
    float d2[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(d2, M0, M1, 0u, 0u, bm, 0u);
    const float sc = __uint_as_float(rec[264]);
    const float dd0 = half_bits_to_float(h0.x) * sc, dm0 = half_bits_to_float(h0.x >> 16) * sc;
    const float dd1 = half_bits_to_float(h1.x) * sc, dm1 = half_bits_to_float(h1.x >> 16) * sc;
    acc0 = fmaf(dd0, (d[0][0] + d[1][0]) + (d[0][1] + d[1][1]), fmaf(dm0, d2[0] + d2[1], acc0));
    acc1 = fmaf(dd1, (d[0][2] + d[1][2]) + (d[0][3] + d[1][3]), fmaf(dm1, d2[2] + d2[3], acc1));
}

}  // namespace pokit
