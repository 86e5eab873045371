// pokit_quant.cuh -- GGUF K-quant / Q8_0 dequant-dot building blocks (sm_100a).
//
// Block layouts (PokitLMs src/quantized_linear.cpp):
//   Q4_K 144 B / 256 w : fp16 d @0, fp16 dmin @2, 12 B packed 6-bit scales+mins @4,
//                        128 B nibbles @16 (decode_q4_k, :166-205)
//   Q5_K 176 B / 256 w : d, dmin, scales @4, qh[32] @16, qs[128] @48 (decode_q5_k, :286-328)
//   Q6_K 210 B / 256 w : ql[128] @0, qh[64] @128, int8 scales[16] @192, fp16 d @208
//                        (decode_q6_k, :330-358)
//   Q8_0  34 B /  32 w : fp16 d @0, int8 q[32] @2 (linear_quantized<false>, :387-423)
//
// Two evaluation schemes live here:
//
//  * Q4_K "fast chunk" (used by the MoE kernels and the Q4_K matvec): one lane
//    owns one 64-weight chunk (32 qs bytes = sub-blocks 2c and 2c+1) of one
//    superblock and reads it with two 128-bit loads plus the 16-byte header.
//    sum_j (ds*q_j - dm) x_j is evaluated as ds * sum q_j x_j - dm * sum x_j with
//    the per-sub-block sums of x precomputed.  Nibbles become floats without a
//    conversion instruction: OR-ing a nibble sitting at bit p (p <= 16) into
//    the mantissa of 2^23 gives exactly 2^23 + q*2^p, and one packed FP32x2 add
//    removes the 2^23.  The matching x was pre-scaled by 2^-p (exact), so each
//    FMA forms the same rounded product q*x.  FP32 accumulation throughout.
//
//  * Generic "group" scheme (every type): one lane decodes a 32-weight group
//    in the reference's own order (d*s*q - dmin*m in FP32) from a row staged in
//    shared memory, and dots it with plain x.
#pragma once

#include "pokit_common.cuh"

namespace pokit {

constexpr uint32_t kMagic23 = 0x4B000000u;  // 2^23 as FP32 bits
constexpr float kTwo23 = 8388608.0f;

// Floats per prepared Q4_K chunk in shared memory: 64 values + 4 pad so the
// four chunks a quarter-warp reads start in different bank groups.
constexpr int kQ4kChunkStride = 68;

// Pre-scale factors for the 8 nibble slots of one 32-bit qs word, in the order
// q4k_chunk_dot consumes them: lo b0..b3, hi b0..b3 (see the bit map there).
__device__ __forceinline__ float q4k_slot_scale(int slot) {
    // lo: b0 p=0, b1 p=8, b2 p=16, b3 p=12 (after >>12); hi: b0 p=4, b1 p=12, b2 p=8, b3 p=16
    constexpr float s[8] = {1.0f, 0x1p-8f, 0x1p-16f, 0x1p-12f, 0x1p-4f, 0x1p-12f, 0x1p-8f, 0x1p-16f};
    return s[slot];
}

// Writes x (length H, a multiple of 256) into the prepared layout used by
// q4k_chunk_dot:  chunk k = sb*4 + c occupies xp[k*68 .. k*68+63]; within it,
// word m (0..7) holds {x_lo[4m..4m+3], x_hi[4m..4m+3]} pre-scaled per slot,
// where x_lo = x[sb*256 + 64c + i], x_hi = x[sb*256 + 64c + 32 + i].
// gsum[g] = sum of the 32 x values of sub-block g (g = sb*8 + j), in FP32.
// Cooperative over the whole CTA; caller synchronises afterwards.
__device__ __forceinline__ void q4k_prepare_x(const float* __restrict__ x, int H,
                                              float* __restrict__ xp, float* __restrict__ gsum) {
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = x[i];
        const int sb = i >> 8, within = i & 255;
        const int c = within >> 6, t = within & 63;
        const int hi = t >> 5, idx = t & 31;   // sub-block 2c+hi, element idx
        const int m = idx >> 2, b = idx & 3;
        const int slot = hi * 4 + b;
        xp[(sb * 4 + c) * kQ4kChunkStride + m * 8 + slot] = v * q4k_slot_scale(slot);
    }
    const int groups = H >> 5;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int g = warp; g < groups; g += nwarps) {
        const float s = warp_sum(x[g * 32 + lane]);
        if (lane == 0) gsum[g] = s;
    }
}

// Unpacks the 6-bit scale and min of sub-blocks 2c and 2c+1 from the packed
// header words (hy = packed[0..3], hz = packed[4..7], hw = packed[8..11]).
// Restates the scale_min lambda of decode_q4_k (src/quantized_linear.cpp:176-188).
__device__ __forceinline__ void q4k_scale_min_pair(uint32_t hy, uint32_t hz, uint32_t hw, int c,
                                                   float& s0, float& m0, float& s1, float& m1) {
    const int k = (2 * c) & 3;                 // byte index of sub-block 2c within a word
    const uint32_t a0 = (hy >> (8 * k)) & 0xffu, a1 = (hy >> (8 * k + 8)) & 0xffu;
    const uint32_t b0 = (hz >> (8 * k)) & 0xffu, b1 = (hz >> (8 * k + 8)) & 0xffu;
    uint32_t sc0, mn0, sc1, mn1;
    if (c < 2) {
        sc0 = a0 & 63u; mn0 = b0 & 63u;
        sc1 = a1 & 63u; mn1 = b1 & 63u;
    } else {
        const uint32_t c0 = (hw >> (8 * k)) & 0xffu, c1 = (hw >> (8 * k + 8)) & 0xffu;
        sc0 = (c0 & 0x0fu) | ((a0 >> 6) << 4); mn0 = (c0 >> 4) | ((b0 >> 6) << 4);
        sc1 = (c1 & 0x0fu) | ((a1 >> 6) << 4); mn1 = (c1 >> 4) | ((b1 >> 6) << 4);
    }
    s0 = static_cast<float>(sc0); m0 = static_cast<float>(mn0);
    s1 = static_cast<float>(sc1); m1 = static_cast<float>(mn1);
}

// sum over the 32 weights of one qs word pair-accumulated into lo/hi float2s.
__device__ __forceinline__ void q4k_word(uint32_t w, const float4 xa, const float4 xb,
                                         float2& acc_lo, float2& acc_hi) {
    const uint32_t w2 = w >> 12;
    const float2 neg = make_float2(-kTwo23, -kTwo23);
    float2 l01 = make_float2(__uint_as_float((w & 0x0000000Fu) | kMagic23),
                             __uint_as_float((w & 0x00000F00u) | kMagic23));
    float2 l23 = make_float2(__uint_as_float((w & 0x000F0000u) | kMagic23),
                             __uint_as_float((w2 & 0x0000F000u) | kMagic23));
    float2 h01 = make_float2(__uint_as_float((w & 0x000000F0u) | kMagic23),
                             __uint_as_float((w & 0x0000F000u) | kMagic23));
    float2 h23 = make_float2(__uint_as_float((w2 & 0x00000F00u) | kMagic23),
                             __uint_as_float((w2 & 0x000F0000u) | kMagic23));
    l01 = add2(l01, neg); l23 = add2(l23, neg);
    h01 = add2(h01, neg); h23 = add2(h23, neg);
    acc_lo = fma2(l01, make_float2(xa.x, xa.y), acc_lo);
    acc_lo = fma2(l23, make_float2(xa.z, xa.w), acc_lo);
    acc_hi = fma2(h01, make_float2(xb.x, xb.y), acc_hi);
    acc_hi = fma2(h23, make_float2(xb.z, xb.w), acc_hi);
}

// Contribution of chunk c (64 weights) of one Q4_K superblock, given its
// 16-byte header `hdr`, its 32 qs bytes (q0 = bytes 0..15, q1 = 16..31), the
// prepared x chunk `xp` (shared memory, 64 floats) and the two sub-block sums.
__device__ __forceinline__ float q4k_chunk_dot(uint4 hdr, uint4 q0, uint4 q1, int c,
                                               const float* __restrict__ xp, float gs0, float gs1) {
    float2 acc_lo = make_float2(0.f, 0.f), acc_hi = make_float2(0.f, 0.f);
    const float4* x4 = reinterpret_cast<const float4*>(xp);
    q4k_word(q0.x, x4[0], x4[1], acc_lo, acc_hi);
    q4k_word(q0.y, x4[2], x4[3], acc_lo, acc_hi);
    q4k_word(q0.z, x4[4], x4[5], acc_lo, acc_hi);
    q4k_word(q0.w, x4[6], x4[7], acc_lo, acc_hi);
    q4k_word(q1.x, x4[8], x4[9], acc_lo, acc_hi);
    q4k_word(q1.y, x4[10], x4[11], acc_lo, acc_hi);
    q4k_word(q1.z, x4[12], x4[13], acc_lo, acc_hi);
    q4k_word(q1.w, x4[14], x4[15], acc_lo, acc_hi);
    const float d = half_bits_to_float(hdr.x);
    const float dmin = half_bits_to_float(hdr.x >> 16);
    float s0, m0, s1, m1;
    q4k_scale_min_pair(hdr.y, hdr.z, hdr.w, c, s0, m0, s1, m1);
    const float sum_lo = acc_lo.x + acc_lo.y;
    const float sum_hi = acc_hi.x + acc_hi.y;
    // (d*s) and (dmin*m) are formed exactly as the reference forms ds0/dm0.
    const float ds0 = d * s0, dm0 = dmin * m0, ds1 = d * s1, dm1 = dmin * m1;
    float r = ds0 * sum_lo;
    r = fmaf(-dm0, gs0, r);
    r = fmaf(ds1, sum_hi, r);
    r = fmaf(-dm1, gs1, r);
    return r;
}

// ---------------------------------------------------------------------------
// Generic scheme: decode one 32-weight group g of a row held in shared memory
// (bytes, any alignment) and dot it with x[g*32 .. g*32+31] (shared memory).
// Arithmetic per weight follows the reference decoders exactly.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sm_u16(const uint8_t* p) {
    return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
}

template <uint32_t T>
__device__ __forceinline__ float group_dot(const uint8_t* __restrict__ row, int g,
                                           const float* __restrict__ x) {
    const float* xg = x + g * 32;
    float acc = 0.0f;
    if constexpr (T == kF32) {
        const float* w = reinterpret_cast<const float*>(row) + g * 32;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) acc = fmaf(w[i], xg[i], acc);
    } else if constexpr (T == kQ8_0) {
        const uint8_t* blk = row + g * 34;
        const float d = half_bits_to_float(sm_u16(blk));
        const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
        float s = 0.0f;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) s = fmaf(static_cast<float>(q[i]), xg[i], s);
        acc = d * s;
    } else if constexpr (T == kQ4_K || T == kQ5_K) {
        const int sb = g >> 3, j = g & 7;
        const uint8_t* blk = row + sb * block_bytes(T);
        const float d = half_bits_to_float(sm_u16(blk));
        const float dmin = half_bits_to_float(sm_u16(blk + 2));
        const uint8_t* packed = blk + 4;
        uint32_t sc, mn;
        if (j < 4) {
            sc = packed[j] & 63u; mn = packed[j + 4] & 63u;
        } else {
            sc = (packed[j + 4] & 0x0fu) | ((packed[j - 4] >> 6) << 4);
            mn = (packed[j + 4] >> 4) | ((packed[j] >> 6) << 4);
        }
        const float ds = d * static_cast<float>(sc), dm = dmin * static_cast<float>(mn);
        const int chunk = j >> 1, part = j & 1;
        const uint8_t* qs = blk + (T == kQ4_K ? 16 : 48) + chunk * 32;
        if constexpr (T == kQ4_K) {
#pragma unroll 8
            for (int i = 0; i < 32; ++i) {
                const uint32_t q = part ? (qs[i] >> 4) : (qs[i] & 0x0fu);
                acc = fmaf(ds * static_cast<float>(q) - dm, xg[i], acc);
            }
        } else {
            const uint8_t* qh = blk + 16;
            const uint32_t bit = 1u << (2 * chunk + part);
#pragma unroll 8
            for (int i = 0; i < 32; ++i) {
                const uint32_t q = (part ? (qs[i] >> 4) : (qs[i] & 0x0fu)) + ((qh[i] & bit) ? 16u : 0u);
                acc = fmaf(ds * static_cast<float>(q) - dm, xg[i], acc);
            }
        }
    } else if constexpr (T == kQ6_K) {
        const int sb = g >> 3, j = g & 7;
        const uint8_t* blk = row + sb * 210;
        const float d = half_bits_to_float(sm_u16(blk + 208));
        const int half = j >> 2, jj = j & 3;
        const uint8_t* ql = blk + half * 64 + (jj & 1) * 32;
        const uint8_t* qh = blk + 128 + half * 32;
        const int8_t* scales = reinterpret_cast<const int8_t*>(blk + 192 + half * 8);
        const int shift_lo = (jj >> 1) * 4, shift_hi = jj * 2;
#pragma unroll 8
        for (int l = 0; l < 32; ++l) {
            const int q = static_cast<int>(((ql[l] >> shift_lo) & 0x0fu) |
                                           (((qh[l] >> shift_hi) & 0x03u) << 4)) - 32;
            const float s = static_cast<float>(scales[l / 16 + 2 * jj]);
            acc = fmaf(d * s * static_cast<float>(q), xg[l], acc);
        }
    }
    return acc;
}

// Warp-cooperative copy of `bytes` of a weight row from global to shared
// memory.  Uses 16-byte loads when source and size allow it, else 4- or
// 2-byte loads (GGUF rows of Q6_K/Q8_0 are only 2-byte aligned in general).
// kBatch 16-byte loads per lane (4 x kBatch for 4-byte rows) go out before
// their stores: one memory latency per batch (a 2-4 KB row is one batch at
// the default); callers short of registers take smaller batches.
template <uint32_t kBatch = 8>
__device__ __forceinline__ void warp_stage_row(const uint8_t* __restrict__ src, uint32_t bytes,
                                               uint8_t* __restrict__ dst, int lane) {
    const uint64_t a = reinterpret_cast<uint64_t>(src);
    if ((a & 15u) == 0 && (bytes & 15u) == 0) {
        for (uint32_t o0 = lane * 16u; o0 < bytes; o0 += 32u * 16u * kBatch) {
            uint4 v[kBatch];
#pragma unroll
            for (uint32_t j = 0; j < kBatch; ++j)
                if (o0 + j * 512u < bytes) v[j] = ldg_stream128(src + o0 + j * 512u);
#pragma unroll
            for (uint32_t j = 0; j < kBatch; ++j)
                if (o0 + j * 512u < bytes) *reinterpret_cast<uint4*>(dst + o0 + j * 512u) = v[j];
        }
    } else if ((a & 3u) == 0 && (bytes & 3u) == 0) {
        constexpr uint32_t kB4 = 2 * kBatch;
        for (uint32_t o0 = lane * 4u; o0 < bytes; o0 += 32u * 4u * kB4) {
            uint32_t v[kB4];
#pragma unroll
            for (uint32_t j = 0; j < kB4; ++j)
                if (o0 + j * 128u < bytes) v[j] = ldg_stream32(src + o0 + j * 128u);
#pragma unroll
            for (uint32_t j = 0; j < kB4; ++j)
                if (o0 + j * 128u < bytes) *reinterpret_cast<uint32_t*>(dst + o0 + j * 128u) = v[j];
        }
    } else {
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
        uint16_t* d16 = reinterpret_cast<uint16_t*>(dst);
        for (uint32_t o = lane; o < bytes / 2u; o += 32u) d16[o] = __ldg(s16 + o);
    }
}

// This lane's share of the dot of a staged row (cols weights) with x: lane l
// takes elements l, l + 32, l + 64, ...  With that mapping a warp reads 32
// consecutive activations and 32 consecutive quant bytes per step (no shared-
// memory bank conflicts) and, inside a 256-weight superblock, element
// 32 i + l belongs to sub-block i (Q4_K/Q5_K: the low nibbles of qs[32 (i/2) + l]
// for even i, the high ones for odd i; Q5_K's fifth bit is bit i of qh[l];
// Q6_K: quarter i % 4 of half i / 4, scale 8 (i / 4) + l / 16 + 2 (i % 4)).
// Weights are formed as the reference's decoders form them (quantized_linear.cpp
// :166-205, :286-328, :330-358, Q8_0 :430-451); callers sum the lanes.
template <uint32_t T>
__device__ __forceinline__ float lane_row_dot(const uint8_t* __restrict__ row, uint32_t cols,
                                              const float* __restrict__ x, int lane) {
    float acc = 0.0f;
    if constexpr (T == kF32) {
        const float* w = reinterpret_cast<const float*>(row);
        for (uint32_t k = lane; k < cols; k += 32) acc = fmaf(w[k], x[k], acc);
    } else if constexpr (T == kQ8_0) {
        for (uint32_t b = 0; b < cols / 32; ++b) {
            const uint8_t* blk = row + b * 34;
            const float d = half_bits_to_float(sm_u16(blk));
            const float q = static_cast<float>(static_cast<int8_t>(blk[2 + lane]));
            acc = fmaf(d * q, x[32 * b + lane], acc);
        }
    } else if constexpr (T == kQ4_K || T == kQ5_K) {
        constexpr uint32_t BB = T == kQ4_K ? 144u : 176u, QS = T == kQ4_K ? 16u : 48u;
        for (uint32_t sb = 0; sb < cols / 256; ++sb) {
            const uint8_t* blk = row + sb * BB;
            const float d = half_bits_to_float(sm_u16(blk)), dmin = half_bits_to_float(sm_u16(blk + 2));
            const uint8_t* packed = blk + 4;
            uint32_t hbits = 0;
            if constexpr (T == kQ5_K) hbits = blk[16 + lane];
            const float* xs = x + sb * 256 + lane;
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
                uint32_t sc, mn;
                if (i < 4) {
                    sc = packed[i] & 63u;
                    mn = packed[i + 4] & 63u;
                } else {
                    sc = (packed[i + 4] & 0x0fu) | ((packed[i - 4] >> 6) << 4);
                    mn = (packed[i + 4] >> 4) | ((packed[i] >> 6) << 4);
                }
                const uint32_t byte = blk[QS + 32 * (i / 2) + lane];
                uint32_t v = (i & 1) ? (byte >> 4) : (byte & 0x0fu);
                if constexpr (T == kQ5_K) v += ((hbits >> i) & 1u) << 4;
                const float w = (d * static_cast<float>(sc)) * static_cast<float>(v) - dmin * static_cast<float>(mn);
                acc = fmaf(w, xs[32 * i], acc);
            }
        }
    } else if constexpr (T == kQ6_K) {
        for (uint32_t sb = 0; sb < cols / 256; ++sb) {
            const uint8_t* blk = row + sb * 210;
            const float d = half_bits_to_float(sm_u16(blk + 208));
            const float* xs = x + sb * 256 + lane;
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
                const uint32_t half = i >> 2, quarter = i & 3;
                const uint32_t lo = blk[half * 64 + lane + 32 * (quarter & 1)];
                const uint32_t hi = blk[128 + half * 32 + lane];
                const int q = static_cast<int>(((lo >> (4 * (quarter >> 1))) & 0x0fu) |
                                               (((hi >> (2 * quarter)) & 3u) << 4)) - 32;
                const int8_t sc = static_cast<int8_t>(blk[192 + half * 8 + lane / 16 + 2 * quarter]);
                const float w = d * static_cast<float>(sc) * static_cast<float>(q);
                acc = fmaf(w, xs[32 * i], acc);
            }
        }
    }
    return acc;
}

// Four bytes at any (shared-memory) address as one word: two aligned loads and a
// funnel shift (Q6_K superblocks are 210 bytes, so odd superblocks start 2 bytes
// off a word boundary).  Reads up to 3 bytes past p + 3 within the same row.
__device__ __forceinline__ uint32_t load_u32_any(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
    return sh ? __funnelshift_r(w[0], w[1], sh) : w[0];
}

// Four bytes of a 32-bit word as floats: byte j -> (2^23 + byte) - bias.
__device__ __forceinline__ float4 bytes_to_float4(uint32_t w, float bias) {
    const float k = 8388608.0f + bias;
    // __byte_perm selector nibbles: result byte 0 = byte j of w (0..3), bytes
    // 1, 2 = byte 4 (0x00 of the constant), byte 3 = byte 7 (0x4B).
    return make_float4(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)) - k,
                       __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)) - k,
                       __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)) - k,
                       __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)) - k);
}

// lane_row_dot with four consecutive elements per lane and step: lane l takes
// elements 128 s + 4 l .. 128 s + 4 l + 3, whose quants share one 32-bit word
// (and one sub-block scale); the four are decoded byte-parallel and the scale
// is applied once per four.  cols must be a multiple of 256 (K-quants) or 128
// (Q8_0).  The sum differs from lane_row_dot's only in rounding.
template <uint32_t T>
__device__ __forceinline__ float lane_row_dot4(const uint8_t* __restrict__ row, uint32_t cols,
                                               const float* __restrict__ x, int lane) {
    float acc = 0.0f;
    if constexpr (T == kQ6_K) {
        const uint32_t quarter = lane >> 3, l0 = 4u * (lane & 7);
        for (uint32_t sb = 0; sb < cols / 256; ++sb) {
            const uint8_t* blk = row + sb * 210;
            const float d = half_bits_to_float(sm_u16(blk + 208));
#pragma unroll
            for (uint32_t half = 0; half < 2; ++half) {
                const uint32_t lo = load_u32_any(blk + half * 64 + 32 * (quarter & 1) + l0);
                const uint32_t hi = load_u32_any(blk + 128 + half * 32 + l0);
                const uint32_t q = ((lo >> (4 * (quarter >> 1))) & 0x0F0F0F0Fu) | (((hi >> (2 * quarter)) & 0x03030303u) << 4);
                const float sc = static_cast<float>(static_cast<int8_t>(blk[192 + half * 8 + (l0 >> 4) + 2 * quarter]));
                const float4 f = bytes_to_float4(q, 32.0f);
                const float4 xv = *reinterpret_cast<const float4*>(x + sb * 256 + half * 128 + 4 * lane);
                const float part = fmaf(f.x, xv.x, fmaf(f.y, xv.y, fmaf(f.z, xv.z, f.w * xv.w)));
                acc = fmaf(d * sc, part, acc);
            }
        }
    } else if constexpr (T == kQ4_K || T == kQ5_K) {
        constexpr uint32_t BB = T == kQ4_K ? 144u : 176u, QS = T == kQ4_K ? 16u : 48u;
        const bool high = (lane & 8) != 0;
        const uint32_t l0 = 4u * (lane & 7);
        for (uint32_t sb = 0; sb < cols / 256; ++sb) {
            const uint8_t* blk = row + sb * BB;
            const float d = half_bits_to_float(sm_u16(blk)), dmin = half_bits_to_float(sm_u16(blk + 2));
            const uint8_t* packed = blk + 4;
            uint32_t qh = 0;
            if constexpr (T == kQ5_K) qh = *reinterpret_cast<const uint32_t*>(blk + 16 + l0);
#pragma unroll
            for (uint32_t st = 0; st < 2; ++st) {
                const uint32_t chunk = 2 * st + (lane >> 4);
                const uint32_t j = 2 * chunk + (high ? 1u : 0u);
                uint32_t sc, mn;
                if (j < 4) {
                    sc = packed[j] & 63u;
                    mn = packed[j + 4] & 63u;
                } else {
                    sc = (packed[j + 4] & 0x0fu) | ((packed[j - 4] >> 6) << 4);
                    mn = (packed[j + 4] >> 4) | ((packed[j] >> 6) << 4);
                }
                const uint32_t w = *reinterpret_cast<const uint32_t*>(blk + QS + 32 * chunk + l0);
                uint32_t q = high ? ((w >> 4) & 0x0F0F0F0Fu) : (w & 0x0F0F0F0Fu);
                if constexpr (T == kQ5_K) q |= ((qh >> j) & 0x01010101u) << 4;
                const float4 f = bytes_to_float4(q, 0.0f);
                const float4 xv = *reinterpret_cast<const float4*>(x + sb * 256 + st * 128 + 4 * lane);
                const float part = fmaf(f.x, xv.x, fmaf(f.y, xv.y, fmaf(f.z, xv.z, f.w * xv.w)));
                const float xsum = (xv.x + xv.y) + (xv.z + xv.w);
                acc = fmaf(d * static_cast<float>(sc), part, fmaf(-(dmin * static_cast<float>(mn)), xsum, acc));
            }
        }
    } else if constexpr (T == kQ8_0) {
        const uint32_t l0 = 4u * (lane & 7);
        for (uint32_t s0 = 0; s0 < cols; s0 += 128) {
            const uint8_t* blk = row + (s0 / 32 + (lane >> 3)) * 34;
            const float d = half_bits_to_float(sm_u16(blk));
            const uint8_t* q = blk + 2 + l0;
            const float4 xv = *reinterpret_cast<const float4*>(x + s0 + 4 * lane);
            const float part = fmaf(static_cast<float>(static_cast<int8_t>(q[0])), xv.x,
                                    fmaf(static_cast<float>(static_cast<int8_t>(q[1])), xv.y,
                                         fmaf(static_cast<float>(static_cast<int8_t>(q[2])), xv.z,
                                              static_cast<float>(static_cast<int8_t>(q[3])) * xv.w)));
            acc = fmaf(d, part, acc);
        }
    } else {
        acc = lane_row_dot<T>(row, cols, x, lane);
    }
    return acc;
}

__device__ __forceinline__ float lane_row_dot_any(uint32_t type, const uint8_t* row, uint32_t cols, const float* x,
                                                  int lane) {
    switch (type) {
        case kQ4_K: return lane_row_dot4<kQ4_K>(row, cols, x, lane);
        case kQ5_K: return lane_row_dot4<kQ5_K>(row, cols, x, lane);
        case kQ6_K: return lane_row_dot4<kQ6_K>(row, cols, x, lane);
        case kQ8_0: return (cols & 127u) ? lane_row_dot<kQ8_0>(row, cols, x, lane)
                                         : lane_row_dot4<kQ8_0>(row, cols, x, lane);
        default: return lane_row_dot<kF32>(row, cols, x, lane);
    }
}

// Stages the contiguous byte span [src, src + bytes) with 16-byte loads from
// the 16-byte boundary at or below src (all of a lane's loads in flight before
// its stores); returns where src landed in dst (0..15).  dst needs bytes + 16.
template <uint32_t kBatch = 8>
__device__ __forceinline__ uint32_t warp_stage_span(const uint8_t* __restrict__ src, uint32_t bytes,
                                                    uint8_t* __restrict__ dst, int lane) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(src);
    const uint32_t delta = static_cast<uint32_t>(a & 15u);
    const uint8_t* base = reinterpret_cast<const uint8_t*>(a - delta);
    const uint32_t units = (delta + bytes + 15u) / 16u;
    for (uint32_t u0 = lane; u0 < units; u0 += 32u * kBatch) {
        uint4 v[kBatch];
#pragma unroll
        for (uint32_t j = 0; j < kBatch; ++j)
            if (u0 + 32u * j < units) v[j] = ldg_stream128(base + (u0 + 32u * j) * 16u);
#pragma unroll
        for (uint32_t j = 0; j < kBatch; ++j)
            if (u0 + 32u * j < units) *reinterpret_cast<uint4*>(dst + (u0 + 32u * j) * 16u) = v[j];
    }
    return delta;
}

// Bit-exact decoders (explicit round-to-nearest operations so the compiler
// cannot contract them into FMAs): same expressions as the reference's
// decode_q4_k / decode_q5_k / decode_q6_k / Q8_0 scale (quantized_linear.cpp).
template <uint32_t T>
__device__ __forceinline__ void group_decode(const uint8_t* __restrict__ row, int g,
                                             float* __restrict__ out) {
    if constexpr (T == kF32) {
        const float* w = reinterpret_cast<const float*>(row) + g * 32;
        for (int i = 0; i < 32; ++i) out[i] = w[i];
    } else if constexpr (T == kQ8_0) {
        const uint8_t* blk = row + g * 34;
        const float d = half_bits_to_float(sm_u16(blk));
        const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
        for (int i = 0; i < 32; ++i) out[i] = __fmul_rn(d, static_cast<float>(q[i]));
    } else if constexpr (T == kQ4_K || T == kQ5_K) {
        const int sb = g >> 3, j = g & 7;
        const uint8_t* blk = row + sb * block_bytes(T);
        const float d = half_bits_to_float(sm_u16(blk));
        const float dmin = half_bits_to_float(sm_u16(blk + 2));
        const uint8_t* packed = blk + 4;
        uint32_t sc, mn;
        if (j < 4) {
            sc = packed[j] & 63u; mn = packed[j + 4] & 63u;
        } else {
            sc = (packed[j + 4] & 0x0fu) | ((packed[j - 4] >> 6) << 4);
            mn = (packed[j + 4] >> 4) | ((packed[j] >> 6) << 4);
        }
        const float ds = __fmul_rn(d, static_cast<float>(sc));
        const float dm = __fmul_rn(dmin, static_cast<float>(mn));
        const int chunk = j >> 1, part = j & 1;
        const uint8_t* qs = blk + (T == kQ4_K ? 16 : 48) + chunk * 32;
        const uint8_t* qh = blk + 16;
        for (int i = 0; i < 32; ++i) {
            uint32_t q = part ? (qs[i] >> 4) : (qs[i] & 0x0fu);
            if constexpr (T == kQ5_K) q += (qh[i] & (1u << (2 * chunk + part))) ? 16u : 0u;
            out[i] = __fsub_rn(__fmul_rn(ds, static_cast<float>(q)), dm);
        }
    } else if constexpr (T == kQ6_K) {
        const int sb = g >> 3, j = g & 7;
        const uint8_t* blk = row + sb * 210;
        const float d = half_bits_to_float(sm_u16(blk + 208));
        const int half = j >> 2, jj = j & 3;
        const uint8_t* ql = blk + half * 64 + (jj & 1) * 32;
        const uint8_t* qh = blk + 128 + half * 32;
        const int8_t* scales = reinterpret_cast<const int8_t*>(blk + 192 + half * 8);
        const int shift_lo = (jj >> 1) * 4, shift_hi = jj * 2;
        for (int l = 0; l < 32; ++l) {
            const int q = static_cast<int>(((ql[l] >> shift_lo) & 0x0fu) |
                                           (((qh[l] >> shift_hi) & 0x03u) << 4)) - 32;
            out[l] = __fmul_rn(__fmul_rn(d, static_cast<float>(scales[l / 16 + 2 * jj])),
                               static_cast<float>(q));
        }
    }
}


}  // namespace pokit
