// pokit_mma.cuh -- tensor-core Q4_K dequant-dot for decode batch 1 (sm_100a).
//
// A warp computes 16 rows of y = W x for a Q4_K matrix W with integer
// tensor-core MMAs, mma.sync.m16n8k32 (u8 x s8 -> s32), one per 32-weight
// sub-block:
//
//   A (16 x 32)  the sub-block's 4-bit quants as bytes: q (low nibbles, one
//                LOP3 per four weights) or 16 q (high nibbles, masked in place).
//   B (32 x 8)   columns 0..3: x split into four int8 pieces per superblock,
//                x ~ s0 (p0 + p1 / 2^7 + p2 / 2^14 + p3 / 2^21) with s0 = 2^E0
//                the power of two that brings max|x| to <= 127 (|p1..p3| <=
//                64); columns 4..7 zero.  The residual is below 2^-28 of
//                max|x|, so elements next to a large outlier keep their
//                precision.
//   D (16 x 8)   the exact int32 dot of each piece with the sub-block's quants;
//                multiplied by the sub-block's 6-bit scale (IMAD) and summed
//                over the superblock in int32 (at most 2^28).
//   mins         one fp16 mma with A = m_j (k = j) and B = -sum_{i in j} x_i.
//   per superblock and row: acc += d * s0 * (piece sums, high nibbles / 16)
//                + dmin * 2^e * mins, FP32, in the lanes holding each piece
//                column; callers add the four lanes of a row group (quad_sum).
//
// Algebraically this is sum_i (d*s_j*q_i - dmin*m_j) * x_i, the reference's
// decode_q4_k (src/quantized_linear.cpp:166-205) dotted with x; the integer
// products are exact and the scale arithmetic is FP32, so results agree with
// the reference's FP32 loop to ~1e-6 relative.
//
// Fragment layout (PTX m16n8k32 .s8/.u8): thread (g = lane/4, t = lane%4)
// holds A rows g and g+8 at k = 4t..4t+3 and 4t+16..4t+19, B column g at the
// same k, and D rows g, g+8 at columns 2t, 2t+1.  k = 4t + i is weight byte
// 8t + i of a 32-byte qs chunk and k = 4t + 16 + i is byte 8t + 4 + i, so
// thread t reads 8 contiguous bytes per row and chunk.
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
// One box of a 2-D tensor map (x = column in the map's element units, y =
// row) into shared memory, completing on `bar`.  x * element size must be a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_box_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
// Contiguous global -> shared bulk copy (no multicast) completing on `bar`;
// both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
// 16-byte asynchronous global -> shared copy through L2 (no L1 allocation);
// completion by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before its predecessor in the stream ends;
// grid_dep_wait blocks until the predecessor grid has completed and its
// writes are visible, grid_dep_launch lets the successor start launching.
// Both are no-ops for a normal launch.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// A superblock box: 16 rows x 144 bytes, rows 144 bytes apart in shared
// memory.  With that pitch the (row g, lane t) 8-byte reads of a fragment
// fall on distinct bank pairs two lanes at a time: two wavefronts, the
// minimum for 256 bytes.
constexpr uint32_t kBoxRows = 16, kBoxBytes = 16u * 144u;

// ---------------------------------------------------------------------------
// Activation fragments.  One record of kFragWords 32-bit words per superblock
// (256 activations):
//   bytes [0, 1024) B fragments: byte (j*4 + p)*32 + e = piece p of element e
//                   of sub-block j (int8); thread (g, t) loads the 8 bytes at
//                   (j*4 + g)*32 + 8t for piece g < 4
//   words [256, 264) min fragments: word t*2 + half = fp16x2 of
//                   -(sum of sub-blocks 2t, 2t+1) * 2^-e, hi (half 0) or lo
//   word 264        2^e (float bits), the min fragments' scale
//   word 265        s0 = 2^E0 (float bits), the pieces' scale
// 256 floats can be staged in the record's own space before it is built.
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
// 2^k as a float for k in the normal range, from its exponent bits.
__device__ __forceinline__ float pow2f(int k) { return __int_as_float((127 + k) << 23); }

__device__ __forceinline__ void q4k_frag_superblock(const float* v, uint32_t* rec, int lane) {
    float x[8];
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        x[j] = v[32 * j + lane];
        m = fmaxf(m, fabsf(x[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // s0 = 2^E0 >= max|x| / 127 (E0 from the exponent bits of max|x| / 127,
    // rounded up; the lowest exponents are clamped, where every piece is 0).
    const uint32_t mb = __float_as_uint(m * (1.0f / 127.0f));
    int e0 = static_cast<int>(mb >> 23) - 126;           // 2^e0 > m / 127 for normal m / 127
    e0 = max(e0, -100);
    // N = rint(x * 2^(21 - E0)), |N| < 2^28, split into balanced base-128
    // digits: x ~ 2^E0 (p0 + p1 2^-7 + p2 2^-14 + p3 2^-21), |p1..p3| <= 64.
    const float upN = pow2f(21 - e0), unitN = pow2f(e0 - 21);
    // The min fragments' scale keeps the 32-element sums inside fp16.
    const int e = m > 1024.0f ? static_cast<int>(__float_as_uint(m) >> 23) - 127 - 9 : 0;
    const float inv = pow2f(-e) * unitN;
    int8_t q[8][4];
    float xh[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        int n = __float2int_rn(x[j] * upN);
        xh[j] = static_cast<float>(n) * inv;             // the value the pieces carry, scaled
        const int d3 = ((n + 64) & 127) - 64;
        n = (n - d3) >> 7;
        const int d2 = ((n + 64) & 127) - 64;
        n = (n - d2) >> 7;
        const int d1 = ((n + 64) & 127) - 64;
        n = (n - d1) >> 7;
        q[j][0] = static_cast<int8_t>(max(-127, min(127, n)));
        q[j][1] = static_cast<int8_t>(d1);
        q[j][2] = static_cast<int8_t>(d2);
        q[j][3] = static_cast<int8_t>(d3);
    }
    // Reduce-scatter of the eight group sums of the represented values (lane
    // bits 4, 3, 2 pick the group, bits 1, 0 are summed last): lane L ends
    // with the sum of group (L >> 2) & 7.
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float keep = b4 ? xh[4 + i] : xh[i], send = b4 ? xh[i] : xh[4 + i];
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
    int8_t* bytes = reinterpret_cast<int8_t*>(rec);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int p = 0; p < 4; ++p) bytes[(j * 4 + p) * 32 + lane] = q[j][p];
    if (lane < 8) {
        const int half = lane & 1;
        const float g0 = -gA, g1 = -gB;
        rec[256 + lane] = half == 0 ? pack_half2(g0, g1)
                                    : pack_half2(g0 - half_round(g0), g1 - half_round(g1));
    }
    if (lane == 0) {
        rec[264] = __float_as_uint(pow2f(e));
        rec[265] = __float_as_uint(pow2f(e0));
    }
}

// q4k_frag_superblock for N superblocks at once, their steps interleaved
// (the shuffles of one record overlap the other's): each record is built
// exactly as q4k_frag_superblock builds it.
template <int N>
__device__ __forceinline__ void q4k_frag_superblocks(const float* const (&vp)[N], uint32_t* const (&recp)[N], int lane) {
    float x[N][8], m[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        m[n] = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            x[n][j] = vp[n][32 * j + lane];
            m[n] = fmaxf(m[n], fabsf(x[n][j]));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int n = 0; n < N; ++n) m[n] = fmaxf(m[n], __shfl_xor_sync(0xffffffffu, m[n], o));
    int e0[N], e[N];
    int8_t q[N][8][4];
    float xh[N][8];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const uint32_t mb = __float_as_uint(m[n] * (1.0f / 127.0f));
        e0[n] = max(static_cast<int>(mb >> 23) - 126, -100);
        const float upN = pow2f(21 - e0[n]), unitN = pow2f(e0[n] - 21);
        e[n] = m[n] > 1024.0f ? static_cast<int>(__float_as_uint(m[n]) >> 23) - 127 - 9 : 0;
        const float inv = pow2f(-e[n]) * unitN;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int v = __float2int_rn(x[n][j] * upN);
            xh[n][j] = static_cast<float>(v) * inv;
            const int d3 = ((v + 64) & 127) - 64;
            v = (v - d3) >> 7;
            const int d2 = ((v + 64) & 127) - 64;
            v = (v - d2) >> 7;
            const int d1 = ((v + 64) & 127) - 64;
            v = (v - d1) >> 7;
            q[n][j][0] = static_cast<int8_t>(max(-127, min(127, v)));
            q[n][j][1] = static_cast<int8_t>(d1);
            q[n][j][2] = static_cast<int8_t>(d2);
            q[n][j][3] = static_cast<int8_t>(d3);
        }
    }
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
    float y[N][4], z[N][2], w[N], gA[N], gB[N];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const float keep = b4 ? xh[n][4 + i] : xh[n][i], send = b4 ? xh[n][i] : xh[n][4 + i];
            y[n][i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const float keep = b3 ? y[n][2 + i] : y[n][i], send = b3 ? y[n][i] : y[n][2 + i];
            z[n][i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
    for (int n = 0; n < N; ++n) w[n] = (b2 ? z[n][1] : z[n][0]) + __shfl_xor_sync(0xffffffffu, b2 ? z[n][0] : z[n][1], 4);
#pragma unroll
    for (int n = 0; n < N; ++n) w[n] += __shfl_xor_sync(0xffffffffu, w[n], 2);
#pragma unroll
    for (int n = 0; n < N; ++n) w[n] += __shfl_xor_sync(0xffffffffu, w[n], 1);
    const int tq = (lane >> 1) & 3;
#pragma unroll
    for (int n = 0; n < N; ++n) {
        gA[n] = __shfl_sync(0xffffffffu, w[n], (2 * tq) << 2);
        gB[n] = __shfl_sync(0xffffffffu, w[n], (2 * tq + 1) << 2);
    }
    __syncwarp();                                   // all reads of the inputs are done
#pragma unroll
    for (int n = 0; n < N; ++n) {
        int8_t* bytes = reinterpret_cast<int8_t*>(recp[n]);
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int p = 0; p < 4; ++p) bytes[(j * 4 + p) * 32 + lane] = q[n][j][p];
        if (lane < 8) {
            const int half = lane & 1;
            const float g0 = -gA[n], g1 = -gB[n];
            recp[n][256 + lane] = half == 0 ? pack_half2(g0, g1)
                                            : pack_half2(g0 - half_round(g0), g1 - half_round(g1));
        }
        if (lane == 0) {
            recp[n][264] = __float_as_uint(pow2f(e[n]));
            recp[n][265] = __float_as_uint(pow2f(e0[n]));
        }
    }
}

__device__ __forceinline__ void imma16832(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// One superblock of 16 rows (rows g and g+8 at b0p / b1p, 144 bytes each, in
// shared memory) dotted with the activation record `rec`.  Adds this lane's
// share of rows g (acc0) and g+8 (acc1): the row totals are the sums over
// the four lanes t of the row group (quad_sum).
__device__ __forceinline__ void q4k_mma_superblock(const uint8_t* __restrict__ b0p, const uint8_t* __restrict__ b1p,
                                                   const uint32_t* __restrict__ rec, float& acc0, float& acc1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const bool bact = g < 4;
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
    const uint8_t* rb = reinterpret_cast<const uint8_t*>(rec) + g * 32 + 8 * t;
    int lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t sw0 = c < 2 ? sA0 : sB0, sw1 = c < 2 ? sA1 : sB1;
        const uint32_t bl = (2 * c) & 3, bh = (2 * c + 1) & 3;
        const int sl0 = static_cast<int>(__byte_perm(sw0, 0u, 0x4440u | bl));
        const int sl1 = static_cast<int>(__byte_perm(sw1, 0u, 0x4440u | bl));
        const int sh0 = static_cast<int>(__byte_perm(sw0, 0u, 0x4440u | bh));
        const int sh1 = static_cast<int>(__byte_perm(sw1, 0u, 0x4440u | bh));
        const uint2 xl = bact ? *reinterpret_cast<const uint2*>(rb + (2 * c) * 128) : make_uint2(0u, 0u);
        const uint2 xh = bact ? *reinterpret_cast<const uint2*>(rb + (2 * c + 1) * 128) : make_uint2(0u, 0u);
        int dl[4], dh[4];
        imma16832(dl, q0[c].x & 0x0F0F0F0Fu, q1[c].x & 0x0F0F0F0Fu, q0[c].y & 0x0F0F0F0Fu, q1[c].y & 0x0F0F0F0Fu,
                  xl.x, xl.y);
        imma16832(dh, q0[c].x & 0xF0F0F0F0u, q1[c].x & 0xF0F0F0F0u, q0[c].y & 0xF0F0F0F0u, q1[c].y & 0xF0F0F0F0u,
                  xh.x, xh.y);
        lo[0] += dl[0] * sl0;
        lo[1] += dl[1] * sl0;
        lo[2] += dl[2] * sl1;
        lo[3] += dl[3] * sl1;
        hi[0] += dh[0] * sh0;
        hi[1] += dh[1] * sh0;
        hi[2] += dh[2] * sh1;
        hi[3] += dh[3] * sh1;
    }
    const uint32_t mw0 = t < 2 ? mA0 : mB0, mw1 = t < 2 ? mA1 : mB1;
    const uint32_t ja = (2 * t) & 3;
    const uint32_t M0 = hsub2u(__byte_perm(mw0, 0x64u, 0x4040u | ((ja + 1) << 8) | ja), kHalfMagic);
    const uint32_t M1 = hsub2u(__byte_perm(mw1, 0x64u, 0x4040u | ((ja + 1) << 8) | ja), kHalfMagic);
    const uint32_t bm = g < 2 ? rec[256 + t * 2 + (g & 1)] : 0u;
    float d2[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(d2, M0, M1, 0u, 0u, bm, 0u);
    // Columns 2t, 2t+1 hold pieces 2t, 2t+1: scales s0, s0/2^7 (t = 0),
    // s0/2^14, s0/2^21 (t = 1), none for t >= 2.
    const float s0 = __uint_as_float(rec[265]);
    const float ca = t == 0 ? s0 : (t == 1 ? s0 * (1.0f / 16384.0f) : 0.0f);
    const float cb = t == 0 ? s0 * (1.0f / 128.0f) : (t == 1 ? s0 * (1.0f / 2097152.0f) : 0.0f);
    const float y0 = ca * (static_cast<float>(lo[0]) + static_cast<float>(hi[0]) * 0.0625f) +
                     cb * (static_cast<float>(lo[1]) + static_cast<float>(hi[1]) * 0.0625f);
    const float y1 = ca * (static_cast<float>(lo[2]) + static_cast<float>(hi[2]) * 0.0625f) +
                     cb * (static_cast<float>(lo[3]) + static_cast<float>(hi[3]) * 0.0625f);
    const float me = __uint_as_float(rec[264]);
    const float dd0 = half_bits_to_float(h0.x), dm0 = half_bits_to_float(h0.x >> 16) * me;
    const float dd1 = half_bits_to_float(h1.x), dm1 = half_bits_to_float(h1.x >> 16) * me;
    acc0 = fmaf(dd0, y0, fmaf(dm0, d2[0] + d2[1], acc0));
    acc1 = fmaf(dd1, y1, fmaf(dm1, d2[2] + d2[3], acc1));
}

__device__ __forceinline__ void imma16832_ss(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// q4k_mma_superblock for Q5_K superblocks (176 bytes: d, dmin, the twelve
// scale bytes, qh[32], qs[128]).  Element l of sub-block j carries bit j of
// qh[l] as its fifth bit (the reference's Q5_K decoder, quantized_linear.cpp
// :286-328), so each A byte is the nibble with that bit at 16; the scales,
// mins and the min term are Q4_K's.
__device__ __forceinline__ void q5k_mma_superblock(const uint8_t* __restrict__ b0p, const uint8_t* __restrict__ b1p,
                                                   const uint32_t* __restrict__ rec, float& acc0, float& acc1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const bool bact = g < 4;
    const uint4 h0 = *reinterpret_cast<const uint4*>(b0p);
    const uint4 h1 = *reinterpret_cast<const uint4*>(b1p);
    const uint2 e0 = *reinterpret_cast<const uint2*>(b0p + 16 + 8 * t);
    const uint2 e1 = *reinterpret_cast<const uint2*>(b1p + 16 + 8 * t);
    uint2 q0[4], q1[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        q0[c] = *reinterpret_cast<const uint2*>(b0p + 48 + 32 * c + 8 * t);
        q1[c] = *reinterpret_cast<const uint2*>(b1p + 48 + 32 * c + 8 * t);
    }
    const uint32_t sA0 = h0.y & 0x3F3F3F3Fu, sB0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t sA1 = h1.y & 0x3F3F3F3Fu, sB1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    const uint32_t mA0 = h0.z & 0x3F3F3F3Fu, mB0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t mA1 = h1.z & 0x3F3F3F3Fu, mB1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    const uint8_t* rb = reinterpret_cast<const uint8_t*>(rec) + g * 32 + 8 * t;
    const auto fifth = [](uint32_t e, int bit) { return ((e >> bit) & 0x01010101u) << 4; };
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t sw0 = c < 2 ? sA0 : sB0, sw1 = c < 2 ? sA1 : sB1;
        const uint32_t bl = (2 * c) & 3, bh = (2 * c + 1) & 3;
        const int sl0 = static_cast<int>(__byte_perm(sw0, 0u, 0x4440u | bl));
        const int sl1 = static_cast<int>(__byte_perm(sw1, 0u, 0x4440u | bl));
        const int sh0 = static_cast<int>(__byte_perm(sw0, 0u, 0x4440u | bh));
        const int sh1 = static_cast<int>(__byte_perm(sw1, 0u, 0x4440u | bh));
        const uint2 xl = bact ? *reinterpret_cast<const uint2*>(rb + (2 * c) * 128) : make_uint2(0u, 0u);
        const uint2 xh = bact ? *reinterpret_cast<const uint2*>(rb + (2 * c + 1) * 128) : make_uint2(0u, 0u);
        int dl[4], dh[4];
        imma16832(dl, (q0[c].x & 0x0F0F0F0Fu) | fifth(e0.x, 2 * c), (q1[c].x & 0x0F0F0F0Fu) | fifth(e1.x, 2 * c),
                  (q0[c].y & 0x0F0F0F0Fu) | fifth(e0.y, 2 * c), (q1[c].y & 0x0F0F0F0Fu) | fifth(e1.y, 2 * c), xl.x,
                  xl.y);
        imma16832(dh, ((q0[c].x >> 4) & 0x0F0F0F0Fu) | fifth(e0.x, 2 * c + 1),
                  ((q1[c].x >> 4) & 0x0F0F0F0Fu) | fifth(e1.x, 2 * c + 1),
                  ((q0[c].y >> 4) & 0x0F0F0F0Fu) | fifth(e0.y, 2 * c + 1),
                  ((q1[c].y >> 4) & 0x0F0F0F0Fu) | fifth(e1.y, 2 * c + 1), xh.x, xh.y);
        acc[0] += dl[0] * sl0 + dh[0] * sh0;
        acc[1] += dl[1] * sl0 + dh[1] * sh0;
        acc[2] += dl[2] * sl1 + dh[2] * sh1;
        acc[3] += dl[3] * sl1 + dh[3] * sh1;
    }
    const uint32_t mw0 = t < 2 ? mA0 : mB0, mw1 = t < 2 ? mA1 : mB1;
    const uint32_t ja = (2 * t) & 3;
    const uint32_t M0 = hsub2u(__byte_perm(mw0, 0x64u, 0x4040u | ((ja + 1) << 8) | ja), kHalfMagic);
    const uint32_t M1 = hsub2u(__byte_perm(mw1, 0x64u, 0x4040u | ((ja + 1) << 8) | ja), kHalfMagic);
    const uint32_t bm = g < 2 ? rec[256 + t * 2 + (g & 1)] : 0u;
    float d2[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(d2, M0, M1, 0u, 0u, bm, 0u);
    const float s0 = __uint_as_float(rec[265]);
    const float ca = t == 0 ? s0 : (t == 1 ? s0 * (1.0f / 16384.0f) : 0.0f);
    const float cb = t == 0 ? s0 * (1.0f / 128.0f) : (t == 1 ? s0 * (1.0f / 2097152.0f) : 0.0f);
    const float y0 = ca * static_cast<float>(acc[0]) + cb * static_cast<float>(acc[1]);
    const float y1 = ca * static_cast<float>(acc[2]) + cb * static_cast<float>(acc[3]);
    const float me = __uint_as_float(rec[264]);
    const float dd0 = half_bits_to_float(h0.x), dm0 = half_bits_to_float(h0.x >> 16) * me;
    const float dd1 = half_bits_to_float(h1.x), dm1 = half_bits_to_float(h1.x >> 16) * me;
    acc0 = fmaf(dd0, y0, fmaf(dm0, d2[0] + d2[1], acc0));
    acc1 = fmaf(dd1, y1, fmaf(dm1, d2[2] + d2[3], acc1));
}

// Eight bytes at a 2-byte-aligned shared-memory address: `odd` says p sits 2
// bytes past a word boundary (Q6_K superblocks are 210 bytes, so alternate
// superblocks of a row are).  Reads up to 2 bytes past p + 7.
__device__ __forceinline__ uint2 lds_u64_a2(const uint8_t* p, bool odd) {
    if (!odd) return make_uint2(*reinterpret_cast<const uint32_t*>(p), *reinterpret_cast<const uint32_t*>(p + 4));
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p - 2);
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
    return make_uint2(__funnelshift_r(w0, w1, 16), __funnelshift_r(w1, w2, 16));
}

// Four 6-bit quants (bytes 0..63) as the signed bytes q - 32.
__device__ __forceinline__ uint32_t q6_centered(uint32_t v) {
    const uint32_t r = v ^ 0x20202020u;               // q - 32 for q >= 32; q | 32 otherwise
    return r + (r & 0x20202020u) * 6u;                 // where q < 32, bits 6 and 7 too (no carries)
}

// One Q6_K superblock of 16 rows (210 bytes each: ql[128], qh[64], sc[16],
// d; the reference's decoder, quantized_linear.cpp:330-358) dotted with the
// activation record `rec`, as q4k_mma_superblock: sub-block j = 4 * half +
// quarter holds elements 128 half + 32 quarter + l, whose 6-bit value is
// nibble (quarter / 2) of ql[64 half + 32 (quarter % 2) + l] with bits
// 2 quarter of qh[32 half + l] above it, and whose scale is sc[2 j + l / 16].
// The A bytes are q - 32 (signed), so there is no min term; the two scales of
// a sub-block take one MMA each, the activation pieces of lanes t < 2
// (elements 0..15) feeding the first and those of lanes t >= 2 the second.
__device__ __forceinline__ void q6k_mma_superblock(const uint8_t* __restrict__ b0p, const uint8_t* __restrict__ b1p,
                                                   const uint32_t* __restrict__ rec, float& acc0, float& acc1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const bool bact = g < 4, first16 = t < 2;
    const bool odd = (reinterpret_cast<uintptr_t>(b0p) & 2u) != 0;
    const uint2 s0a = lds_u64_a2(b0p + 192, odd), s0b = lds_u64_a2(b0p + 200, odd);
    const uint2 s1a = lds_u64_a2(b1p + 192, odd), s1b = lds_u64_a2(b1p + 200, odd);
    const uint32_t sc0[4] = {s0a.x, s0a.y, s0b.x, s0b.y}, sc1[4] = {s1a.x, s1a.y, s1b.x, s1b.y};
    const uint8_t* rb = reinterpret_cast<const uint8_t*>(rec) + g * 32 + 8 * t;
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint2 la0 = lds_u64_a2(b0p + 64 * h + 8 * t, odd), lb0 = lds_u64_a2(b0p + 64 * h + 32 + 8 * t, odd);
        const uint2 la1 = lds_u64_a2(b1p + 64 * h + 8 * t, odd), lb1 = lds_u64_a2(b1p + 64 * h + 32 + 8 * t, odd);
        const uint2 qh0 = lds_u64_a2(b0p + 128 + 32 * h + 8 * t, odd);
        const uint2 qh1 = lds_u64_a2(b1p + 128 + 32 * h + 8 * t, odd);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
            const int j = 4 * h + qq, sh = 4 * (qq >> 1), hb = 2 * qq;
            const uint2 l0 = (qq & 1) ? lb0 : la0, l1 = (qq & 1) ? lb1 : la1;
            const auto val = [&](uint32_t lo, uint32_t hi) {
                return q6_centered(((lo >> sh) & 0x0F0F0F0Fu) | (((hi >> hb) & 0x03030303u) << 4));
            };
            const uint32_t a0 = val(l0.x, qh0.x), a1 = val(l1.x, qh1.x), a2 = val(l0.y, qh0.y), a3 = val(l1.y, qh1.y);
            const uint2 xb = bact ? *reinterpret_cast<const uint2*>(rb + j * 128) : make_uint2(0u, 0u);
            // The two scale groups through B: lanes t < 2 hold the k positions
            // of elements 0..15 in both operands, lanes t >= 2 those of 16..31.
            const uint32_t bl0 = first16 ? xb.x : 0u, bl1 = first16 ? xb.y : 0u;
            int dA[4], dB[4];
            imma16832_ss(dA, a0, a1, a2, a3, bl0, bl1);
            imma16832_ss(dB, a0, a1, a2, a3, xb.x ^ bl0, xb.y ^ bl1);
            const int bi = 8 * (2 * (j & 1));
            const int sA0 = static_cast<int8_t>(sc0[j >> 1] >> bi), sB0 = static_cast<int8_t>(sc0[j >> 1] >> (bi + 8));
            const int sA1 = static_cast<int8_t>(sc1[j >> 1] >> bi), sB1 = static_cast<int8_t>(sc1[j >> 1] >> (bi + 8));
            acc[0] += dA[0] * sA0 + dB[0] * sB0;
            acc[1] += dA[1] * sA0 + dB[1] * sB0;
            acc[2] += dA[2] * sA1 + dB[2] * sB1;
            acc[3] += dA[3] * sA1 + dB[3] * sB1;
        }
    }
    const float s0 = __uint_as_float(rec[265]);
    const float ca = t == 0 ? s0 : (t == 1 ? s0 * (1.0f / 16384.0f) : 0.0f);
    const float cb = t == 0 ? s0 * (1.0f / 128.0f) : (t == 1 ? s0 * (1.0f / 2097152.0f) : 0.0f);
    const float y0 = ca * static_cast<float>(acc[0]) + cb * static_cast<float>(acc[1]);
    const float y1 = ca * static_cast<float>(acc[2]) + cb * static_cast<float>(acc[3]);
    const float d0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b0p + 208));
    const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b1p + 208));
    acc0 = fmaf(d0, y0, acc0);
    acc1 = fmaf(d1, y1, acc1);
}

// The row total from the four lanes t of a row group (all four lanes get it).
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

}  // namespace pokit
