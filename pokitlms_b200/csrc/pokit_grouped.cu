// pokit_grouped.cu -- the MoE block for a batch of tokens (prefill, batched
// decode): tokens grouped by expert and every expert's Q4_K gate/up/down
// applied to its tokens as a GEMM on the fifth-generation tensor cores.
//
// The reference runs a batch token by token (Qwen3MoeRunner prefill calls
// forward_into per prompt token, src/qwen3_moe_runner.cpp:785-790, each MoE
// block as in 643-692).  Per token this computes the same thing:
//   out[t] = sum_r w_r * down_e(silu(gate_e x_t) * up_e x_t),  e = ids[t][r]
// with routes from route_experts (qwen3_moe_runner.cpp:267-305).
//
// Launches (one stream):
//   1. router logits [T][E] in F32 (skipped when the caller gives logits)
//   2. route: softmax top-k per token (the single-token router, one CTA/row)
//   3. group: stable counting sort of the T*k (token, rank) pairs by expert;
//      each expert's pairs are cut into tiles of <= 64 tokens
//   4. pack x: per tile and 256-wide superblock, the tile's activation rows
//      as fp16 in the GEMM operand layout (below), with a power-of-two scale
//      per (row, superblock) and per-sub-block sums for the Q4_K mins
//   5. gate/up GEMM: a unit is (tile, 64 rows of gate and the same 64 rows
//      of up); writes silu(g) * u in F32
//   6. pack the activations (fp16 hi + lo parts: 22 significant bits)
//   7. down GEMM: a unit is (tile, 128 rows of down); writes w_r * y per pair
//   8. combine: out[t] = sum over ranks in rank order (the reference's order)
//
// GEMM arithmetic.  For a Q4_K superblock (d, dmin, 6-bit scales s_j and
// mins m_j, 4-bit q) the reference weight is d*s_j*q - dmin*m_j
// (src/quantized_linear.cpp:166-205), so a row's dot with x is
//   sum_sb [ d * sum_k (s_j q_k) x_k  -  dmin * sum_j m_j (sum_{k in j} x_k) ].
// s_j q_k <= 945 is an integer, exact in fp16; x is exact in fp16 for BF16
// inputs (scaled by a power of two into fp16 range) and split into fp16 hi +
// lo for F32 inputs and for the down GEMM's activations.  Per superblock one
// tensor-core MMA chain (A = s_j q_k from tensor memory, B = x from shared
// memory, K = 256) gives the first sum and one MMA (A = m_j, B = the sub-block
// sums as hi + lo) the second, both exactly up to F32 accumulation; the
// epilogue applies d, dmin and the activation scale in F32 per superblock.
//
// Operand layout of a tile's packed activations (one superblock, Np = tile
// tokens rounded up to 16): chunks of 8 fp16 (16 bytes) for chunk c (0..31,
// or 0..63 with the lo parts in 32..63) and token row n at
// (c * Np + n) * 16, then two chunks of sub-block sums (hi, lo), then Np
// floats: each row's power-of-two scale.  Within a
// superblock the K order is permuted to match the dequantiser's output: the
// 32-bit tensor-memory column j = 32c + 4w + o (chunk c = 0..3 of the Q4_K
// nibbles, word w = 0..7, nibble pair o = 0..3) holds the weights of
// sub-block 2c + (o >> 1) at positions 4w + (o & 1) and 4w + (o & 1) + 2.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "pokit_common.cuh"
#include "pokit_kernels.h"
#include "pokit_quant.cuh"
#include "pokit_tc.cuh"
#include "pokit_types.h"

namespace pokit {
namespace {

constexpr uint32_t kTileTokens = 64;                  // N of one GEMM tile
constexpr uint32_t kSkinny = 8;                       // tiles of <= 8 tokens take the mma.sync path
constexpr uint32_t kQStage = 128u * 144u;             // one superblock of 128 rows
constexpr uint32_t kSortThreads = 512;
constexpr uint32_t kSortWarps = kSortThreads / 32;
constexpr uint32_t kPackThreads = 256;

__host__ __device__ constexpr uint32_t round16(uint32_t n) { return (n + 15u) & ~15u; }
// Padded slots of an expert with c pairs: full tiles of 64, the last rounded to 16.
__host__ __device__ constexpr uint32_t padded_slots(uint32_t c) { return (c / 64u) * 64u + round16(c % 64u); }

__device__ __forceinline__ float silu_times(float g, float u, uint32_t flavour) {
    // Qwen3-MoE: g / (1 + exp(-g)) * u (qwen3_moe_runner.cpp:683);
    // Qwen3.5:   g * sigmoid(g) * u  (qwen35_runner.cpp:111-123).
    if (flavour == 0) return (g / (1.0f + expf(-g))) * u;
    float sg;
    if (g >= 0.0f) sg = 1.0f / (1.0f + expf(-g));
    else { const float e = expf(g); sg = e / (1.0f + e); }
    return (g * sg) * u;
}

// ---------------------------------------------------------------------------
// 1. Router logits for a batch: logits[t][e] = router[e] . x[t] in F32,
// tiled and split over the hidden dimension.  A CTA computes 64 tokens x 8
// experts over one slice of hidden (512 wide, or 256 when hidden is not a
// multiple of 512; chunks of 128 staged in shared memory) and writes its
// partial sums to partial[slice][t][e]; the
// routing kernel adds the slices in order, so the logits are reproducible.
// ---------------------------------------------------------------------------
constexpr uint32_t kRtTok = 64, kRtExp = 8, kRtChunk = 128;
__host__ __device__ constexpr uint32_t router_slice(uint32_t H) { return H % 512u == 0 ? 512u : 256u; }

__device__ __forceinline__ float4 load4(const void* x, uint32_t x_bf16, size_t at) {
    if (x_bf16) {
        const uint2 q = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(x) + at);
        return make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u),
                           __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u));
    }
    return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + at);
}

__global__ void __launch_bounds__(256) router_batch_kernel(const float* __restrict__ router,
                                                           const void* __restrict__ x, uint32_t x_bf16,
                                                           uint32_t T, uint32_t E, uint32_t H, uint32_t slice,
                                                           float* __restrict__ partial) {
    __shared__ float xs[kRtTok][kRtChunk + 1];
    __shared__ float ws[kRtExp][kRtChunk + 1];
    grid_dep_wait();      // x from the previous kernel (programmatic launch; no-op otherwise)
    grid_dep_launch();
    const uint32_t t0 = blockIdx.x * kRtTok, e0 = blockIdx.y * kRtExp, h0 = blockIdx.z * slice;
    const uint32_t ti = threadIdx.x >> 2, ej = threadIdx.x & 3;
    float a0 = 0.f, a1 = 0.f;
    for (uint32_t c = 0; c < slice; c += kRtChunk) {
        for (uint32_t i = threadIdx.x; i < kRtTok * kRtChunk / 4; i += 256) {
            const uint32_t row = i / (kRtChunk / 4), col = 4 * (i % (kRtChunk / 4)), t = t0 + row;
            const float4 v = t < T ? load4(x, x_bf16, static_cast<size_t>(t) * H + h0 + c + col)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            xs[row][col] = v.x; xs[row][col + 1] = v.y; xs[row][col + 2] = v.z; xs[row][col + 3] = v.w;
        }
        if (threadIdx.x < kRtExp * kRtChunk / 4) {
            const uint32_t row = threadIdx.x / (kRtChunk / 4), col = 4 * (threadIdx.x % (kRtChunk / 4));
            const uint32_t e = e0 + row;
            const float4 v = e < E ? *reinterpret_cast<const float4*>(router + static_cast<size_t>(e) * H + h0 + c + col)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            ws[row][col] = v.x; ws[row][col + 1] = v.y; ws[row][col + 2] = v.z; ws[row][col + 3] = v.w;
        }
        __syncthreads();
#pragma unroll 8
        for (uint32_t k = 0; k < kRtChunk; ++k) {
            const float xv = xs[ti][k];
            a0 = fmaf(ws[ej][k], xv, a0);
            a1 = fmaf(ws[ej + 4][k], xv, a1);
        }
        __syncthreads();
    }
    const uint32_t t = t0 + ti;
    if (t < T) {
        float* out = partial + (static_cast<size_t>(blockIdx.z) * T + t) * E;
        if (e0 + ej < E) out[e0 + ej] = a0;
        if (e0 + ej + 4 < E) out[e0 + ej + 4] = a1;
    }
}

// The router for a few tokens (T <= kRtSmall): one warp per (expert, hidden
// slice) computes the slice's dot with every token; the warp's loads (its
// router slice and the tokens' activations) all go out before any arithmetic,
// so the kernel costs about one memory latency.  Lane l takes the float4s l
// and l + 32 of the slice (slice 256) or l, l + 32, l + 64, l + 96 (512); the
// lanes are summed by the same butterfly for every token, so a partial does
// not depend on T, and the routing kernel adds the slices in order.
constexpr uint32_t kRtSmall = 8;
__global__ void __launch_bounds__(256) router_small_kernel(const float* __restrict__ router,
                                                           const void* __restrict__ x, uint32_t x_bf16,
                                                           uint32_t T, uint32_t E, uint32_t H, uint32_t slice,
                                                           float* __restrict__ partial) {
    grid_dep_wait();
    grid_dep_launch();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t e = blockIdx.x * 8 + warp, sl = blockIdx.y, h0 = sl * slice;
    if (e >= E) return;
    const uint32_t nq = slice / 128;   // float4s per lane: 2 or 4
    float4 w[4], xv[kRtSmall][4];
#pragma unroll
    for (uint32_t q = 0; q < 4; ++q) {
        if (q < nq) w[q] = *reinterpret_cast<const float4*>(router + static_cast<size_t>(e) * H + h0 + 4 * (lane + 32 * q));
#pragma unroll
        for (uint32_t t = 0; t < kRtSmall; ++t)
            if (q < nq && t < T) xv[t][q] = load4(x, x_bf16, static_cast<size_t>(t) * H + h0 + 4 * (lane + 32 * q));
    }
#pragma unroll
    for (uint32_t t = 0; t < kRtSmall; ++t) {
        if (t >= T) break;
        float a = 0.f;
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
            if (q < nq) {
                a = fmaf(w[q].x, xv[t][q].x, a);
                a = fmaf(w[q].y, xv[t][q].y, a);
                a = fmaf(w[q].z, xv[t][q].z, a);
                a = fmaf(w[q].w, xv[t][q].w, a);
            }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, d);
        if (lane == 0) partial[(static_cast<size_t>(sl) * T + t) * E + e] = a;
    }
}

// ---------------------------------------------------------------------------
// 3. Group: stable counting sort of pairs p = t * k + r by expert ids[p],
// keeping the pairs whose expert this device holds ([e_first, e_first + E));
// the sort runs over local expert indices ids[p] - e_first.  Pairs of one
// expert keep increasing p.  Writes the tile list and the slot -> pair map.
// One CTA.
// ---------------------------------------------------------------------------
struct GroupOut {
    uint32_t* plan;        // [0] tiles, [1] padded slots, [2] tiles of > kSkinny tokens, [3] the others
    uint32_t* tile_order;  // the large tiles, then the skinny ones
    uint32_t* tile_expert;
    uint32_t* tile_first;  // first slot (index into slot_pair)
    uint32_t* tile_n;      // tokens in the tile (1..64)
    uint32_t* tile_pad0;   // first padded slot
    uint32_t* slot_pair;
    uint32_t* rank;        // scratch [pairs]
};

__global__ void __launch_bounds__(kSortThreads, 1) group_kernel(const uint32_t* __restrict__ ids, uint32_t pairs,
                                                                uint32_t e_first, uint32_t E, GroupOut o) {
    extern __shared__ uint32_t sm[];
    uint32_t* wc = sm;                          // [kSortWarps][E]
    uint32_t* total = wc + kSortWarps * E;      // [E]
    uint32_t* off_slot = total + E;             // [E]
    uint32_t* off_tile = off_slot + E;          // [E]
    uint32_t* off_pad = off_tile + E;           // [E]
    uint32_t* off_thin = off_pad + E;           // [E] skinny tiles before expert e
    uint32_t* n_large = off_thin + E;           // [1]
    grid_dep_wait();
    grid_dep_launch();
    const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    for (uint32_t e = tid; e < E; e += kSortThreads) total[e] = 0;
    __syncthreads();
    for (uint32_t base = 0; base < pairs; base += kSortThreads) {
        const uint32_t p = base + tid;
        const uint32_t el = p < pairs ? ids[p] - e_first : 0xFFFFFFFFu;   // wraps when below e_first
        const bool valid = el < E;
        const uint32_t e = valid ? el : 0xFFFFFFFFu;
        for (uint32_t i = lane; i < E; i += 32) wc[warp * E + i] = 0;
        __syncwarp();
        const uint32_t m = __match_any_sync(0xFFFFFFFFu, e);
        const uint32_t lr = __popc(m & ((1u << lane) - 1u));
        if (valid && lr == 0) wc[warp * E + e] = __popc(m);
        __syncthreads();
        for (uint32_t i = tid; i < E; i += kSortThreads) {
            uint32_t run = total[i];
            for (uint32_t w = 0; w < kSortWarps; ++w) {
                const uint32_t c = wc[w * E + i];
                wc[w * E + i] = run;
                run += c;
            }
            total[i] = run;
        }
        __syncthreads();
        if (valid) o.rank[p] = wc[warp * E + e] + lr;
        __syncthreads();
    }
    if (warp == 0) {
        const uint32_t per = (E + 31) / 32, lo = min(E, lane * per), hi = min(E, lo + per);
        // An expert's last tile is skinny when it holds 1..kSkinny tokens.
        const auto thin = [](uint32_t c) -> uint32_t { return (c % kTileTokens) != 0 && (c % kTileTokens) <= kSkinny; };
        uint32_t sc = 0, st = 0, sp = 0, ss = 0;
        for (uint32_t e = lo; e < hi; ++e) {
            const uint32_t c = total[e];
            sc += c;
            st += (c + kTileTokens - 1) / kTileTokens;
            sp += padded_slots(c);
            ss += thin(c);
        }
        uint32_t ic = sc, it = st, ip = sp, is = ss;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t a = __shfl_up_sync(0xFFFFFFFFu, ic, d), b = __shfl_up_sync(0xFFFFFFFFu, it, d),
                           c = __shfl_up_sync(0xFFFFFFFFu, ip, d), f = __shfl_up_sync(0xFFFFFFFFu, is, d);
            if (lane >= static_cast<uint32_t>(d)) { ic += a; it += b; ip += c; is += f; }
        }
        uint32_t rc = ic - sc, rt = it - st, rp = ip - sp, rs = is - ss;
        for (uint32_t e = lo; e < hi; ++e) {
            const uint32_t c = total[e];
            off_slot[e] = rc;
            off_tile[e] = rt;
            off_pad[e] = rp;
            off_thin[e] = rs;
            rc += c;
            rt += (c + kTileTokens - 1) / kTileTokens;
            rp += padded_slots(c);
            rs += thin(c);
        }
        if (lane == 31) {
            o.plan[0] = it;
            o.plan[1] = ip;
            o.plan[2] = it - is;
            o.plan[3] = is;
            *n_large = it - is;
        }
    }
    __syncthreads();
    const uint32_t large = *n_large;
    for (uint32_t e = tid; e < E; e += kSortThreads) {
        const uint32_t c = total[e];
        for (uint32_t i = 0; i * kTileTokens < c; ++i) {
            const uint32_t tile = off_tile[e] + i;
            const uint32_t n = min(kTileTokens, c - i * kTileTokens);
            o.tile_expert[tile] = e;
            o.tile_first[tile] = off_slot[e] + i * kTileTokens;
            o.tile_n[tile] = n;
            o.tile_pad0[tile] = off_pad[e] + i * kTileTokens;
            // Large tiles before expert e: its tile index minus the skinny ones.
            o.tile_order[n <= kSkinny ? large + off_thin[e] : tile - off_thin[e]] = tile;
        }
    }
    for (uint32_t p = tid; p < pairs; p += kSortThreads) {
        const uint32_t e = ids[p] - e_first;
        if (e < E) o.slot_pair[off_slot[e] + o.rank[p]] = p;
    }
}

// ---------------------------------------------------------------------------
// 4/6. Pack GEMM activations.  One CTA per tile, a warp per (row, superblock).
// ---------------------------------------------------------------------------
struct PackArgs {
    const void* src;       // rows of `cols` elements (F32, or BF16 when src_bf16)
    uint32_t src_bf16;
    uint32_t by_token;     // 1: source row = token of the slot's pair; 0: row = padded slot
    uint32_t top_k;
    uint32_t cols;
    uint32_t split;        // 1: fp16 hi and lo parts
    const uint32_t* plan;
    const uint32_t* tile_first;
    const uint32_t* tile_n;
    const uint32_t* tile_pad0;
    const uint32_t* slot_pair;
    uint8_t* dst;
};

// Bytes of one packed superblock row: (kc8 + 2) chunks of 16 bytes + a scale.
__host__ __device__ constexpr uint32_t packed_row_bytes(uint32_t kc8) { return (kc8 + 2) * 16 + 4; }

// Skinny tiles (<= kSkinny tokens) are packed as mma.sync B fragments, per
// superblock s at tile base + s * thin_stage_bytes(split):
//   [0, 256)    sub-block sums, token n, lane quarter t: fp16 {hi(2t),
//               hi(2t+1), lo(2t), lo(2t+1)} at (4n + t) * 8
//   [256, 288)  the tokens' power-of-two scales (float)
//   [288, ...)  the hi parts, token n at 288 + n * 576 (kThinTokPitch),
//               then (split only) the lo parts at + kThinPart in the same
//               layout.  Lane quarter t's eight 16-byte chunks start at t *
//               144 (kThinSegPitch: 128 bytes and 16 of padding); chunk w
//               (the qs word w of Q4_K chunk t) holds the fp16 x of K
//               positions 64t + 4w + {0, 2, 1, 3} and 64t + 32 + 4w +
//               {0, 2, 1, 3}: the B registers of k-steps 2w (low nibbles) and
//               2w + 1 (high nibbles).  With segments 144 bytes and tokens
//               576 bytes (64 mod 128) apart, the eight (token, lane
//               quarter) reads of a quarter warp land on eight distinct
//               16-byte bank groups at constant offsets.
// The tile's region is the one the tensor-core layout would use (16 padded
// slots hold more than a superblock's 288 + 2 * 8 * 576 bytes).
constexpr uint32_t kThinTail = 288;
constexpr uint32_t kThinSegPitch = 144, kThinTokPitch = 4 * kThinSegPitch;
constexpr uint32_t kThinPart = kSkinny * kThinTokPitch;
__host__ __device__ constexpr uint32_t thin_stage_bytes(uint32_t split) {
    return kThinTail + (split ? 2u : 1u) * kThinPart;
}
static_assert(thin_stage_bytes(1) <= 16 * packed_row_bytes(64) && thin_stage_bytes(0) <= 16 * packed_row_bytes(32),
              "skinny packing fits a 16-slot tile");

__device__ __forceinline__ uint4 pack8_half(const float (&v)[8]) {
    uint4 r;
    r.x = pack_half2(v[0], v[1]);
    r.y = pack_half2(v[2], v[3]);
    r.z = pack_half2(v[4], v[5]);
    r.w = pack_half2(v[6], v[7]);
    return r;
}

// Loads lane's 8 elements of superblock s of a source row.
__device__ __forceinline__ void pack_load(const PackArgs& a, size_t at, float (&v)[8]) {
    if (a.src_bf16) {
        const uint4 q = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.src) + at);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    } else {
        const float4 p0 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.src) + at);
        const float4 p1 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.src) + at + 4);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
        v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
    }
}

// One warp per padded row n of a tile (grid: tiles x 8, 8 warps per CTA);
// the row's superblocks are loaded four at a time before any is packed.
__global__ void __launch_bounds__(kPackThreads) pack_kernel(PackArgs a) {
    __shared__ float stage[kPackThreads / 32][8 * 33];
    grid_dep_wait();
    grid_dep_launch();
    const uint32_t tile = blockIdx.x;
    if (tile >= a.plan[0]) return;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t n = blockIdx.y * (kPackThreads / 32) + warp;
    const uint32_t n_valid = a.tile_n[tile], np = round16(n_valid), pad0 = a.tile_pad0[tile];
    const bool thin = n_valid <= kSkinny;
    if (n >= (thin ? kSkinny : np)) return;
    const uint32_t S = a.cols / 256, kc8 = a.split ? 64u : 32u;
    const uint32_t stage_bytes = packed_row_bytes(kc8) * np;
    uint8_t* tile_base = a.dst + static_cast<size_t>(pad0) * S * packed_row_bytes(kc8);
    const bool valid = n < n_valid;
    const uint32_t row = !valid ? 0u : a.by_token ? a.slot_pair[a.tile_first[tile] + n] / a.top_k : pad0 + n;
    float* st = stage[warp];
    for (uint32_t s0 = 0; s0 < S; s0 += 4) {
        float v[4][8];
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[q][i] = 0.f;
            if (valid && s0 + q < S)
                pack_load(a, static_cast<size_t>(row) * a.cols + (s0 + q) * 256 + lane * 8, v[q]);
        }
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
            const uint32_t s = s0 + q;
            if (s >= S) break;
            // Power-of-two scale bringing max |v| of the superblock into
            // [512, 1024): sub-block sums stay below 2^15 and the scaling is exact.
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[q][i]));
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, d));
            int ex = 0;
            if (amax > 0.f && amax <= 3.0e38f) frexpf(amax, &ex);
            const int sig = max(-100, min(100, ex - 10));
            const float down = __int_as_float((127 - sig) << 23);
            float part = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float x = v[q][i] * down;
                part += x;
                st[33 * (lane / 4) + 8 * (lane % 4) + i] = x;
            }
            // Sub-block j = lane / 4 sums over its four lanes.
            part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
            part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
            __syncwarp();
            if (thin) {
                // Rows n_valid..7 are written as zeros, so every fragment of the tile is finite.
                uint8_t* region = tile_base + static_cast<size_t>(s) * thin_stage_bytes(a.split);
                const uint32_t t = lane >> 3, w = lane & 7;
                const float* b0 = st + 33 * (2 * t) + 4 * w;
                const float* b1 = st + 33 * (2 * t + 1) + 4 * w;
                const float e[8] = {b0[0], b0[2], b0[1], b0[3], b1[0], b1[2], b1[1], b1[3]};
                float hi[8], lo[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    hi[i] = __half2float(__float2half_rn(e[i]));
                    lo[i] = e[i] - hi[i];
                }
                uint8_t* tok = region + kThinTail + n * kThinTokPitch + t * kThinSegPitch + (w << 4);
                *reinterpret_cast<uint4*>(tok) = pack8_half(hi);
                if (a.split) *reinterpret_cast<uint4*>(tok + kThinPart) = pack8_half(lo);
                if ((lane & 3) == 0) {
                    const uint32_t j = lane >> 2;
                    const __half h = __float2half_rn(part);
                    const __half l = __float2half_rn(part - __half2float(h));
                    __half* sums = reinterpret_cast<__half*>(region) + (4 * n + (j >> 1)) * 4 + (j & 1);
                    sums[0] = h;
                    sums[2] = l;
                }
                if (lane == 0) reinterpret_cast<float*>(region + 256)[n] = __int_as_float((127 + sig) << 23);
                __syncwarp();
                continue;
            }
            uint8_t* region = tile_base + static_cast<size_t>(s) * stage_bytes;
            {
                const uint32_t c = lane >> 3, w = lane & 7;
                const float* b0 = st + 33 * (2 * c) + 4 * w;
                const float* b1 = st + 33 * (2 * c + 1) + 4 * w;
                const float e[8] = {b0[0], b0[2], b0[1], b0[3], b1[0], b1[2], b1[1], b1[3]};
                float hi[8], lo[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    hi[i] = __half2float(__float2half_rn(e[i]));
                    lo[i] = e[i] - hi[i];
                }
                *reinterpret_cast<uint4*>(region + (static_cast<size_t>(lane) * np + n) * 16) = pack8_half(hi);
                if (a.split)
                    *reinterpret_cast<uint4*>(region + (static_cast<size_t>(32 + lane) * np + n) * 16) =
                        pack8_half(lo);
            }
            if ((lane & 3) == 0) {
                const uint32_t j = lane >> 2;
                const __half h = __float2half_rn(part);
                const __half l = __float2half_rn(part - __half2float(h));
                reinterpret_cast<__half*>(region + (static_cast<size_t>(kc8) * np + n) * 16)[j] = h;
                reinterpret_cast<__half*>(region + (static_cast<size_t>(kc8 + 1) * np + n) * 16)[j] = l;
            }
            if (lane == 0)
                reinterpret_cast<float*>(region + static_cast<size_t>(kc8 + 2) * np * 16)[n] =
                    __int_as_float((127 + sig) << 23);
            __syncwarp();
        }
    }
}

// ---------------------------------------------------------------------------
// 5/7. The grouped GEMM.  Persistent: one CTA per SM takes units
// blockIdx.x, blockIdx.x + gridDim.x, ...  Warp roles:
//   warps 0..7    epilogue: two per tensor-memory lane quarter, each folds
//                 half of the tile's token columns of every superblock's
//                 accumulators into registers (d, dmin, activation scale)
//   warps 8..15   dequantise: two per lane quarter, each writes half of a
//                 superblock's K columns of A = s_j * q (fp16) into tensor
//                 memory, and the mins m_j into shared memory
//   warp 16       loader: TMA boxes of the Q4_K rows (144 bytes x 64 or 128
//                 rows), one bulk copy of packed activations per superblock
//   warp 17       owns tensor memory; one lane issues the MMAs
//
// Tensor memory (512 columns): A double-buffered in columns [0, 256); per
// buffer b the accumulators of the quants at 256 + 128b and of the mins at
// 256 + 128b + 64 (N <= 64 tokens).
//
// The tensor core takes ~68 cycles per M = 128, K = 16 MMA for any N <= 128
// (measured on B200), so a superblock costs 17 MMAs x 68 cycles whatever the
// tile's token count.
// ---------------------------------------------------------------------------
constexpr uint32_t kEpWarps = 8, kDqWarps = 8;
constexpr uint32_t kLoadWarp = kEpWarps + kDqWarps, kMmaWarp = kLoadWarp + 1;
constexpr uint32_t kGemmThreads = (kMmaWarp + 1) * 32;
constexpr uint32_t kDdRing = 4;   // (d, dmin) hand-off ring from dequantisers to epilogue

struct GemmArgs {
    CUtensorMap tm0;          // gate (mode 0) or down (mode 1)
    CUtensorMap tm1;          // up (mode 0)
    const uint8_t* b;         // packed activations (pack_kernel layout)
    const uint32_t* plan;
    const uint32_t* tile_order;   // [0, plan[2]): the tiles of > kSkinny tokens
    const uint32_t* tile_expert;
    const uint32_t* tile_first;
    const uint32_t* tile_n;
    const uint32_t* tile_pad0;
    const uint32_t* slot_pair;
    const float* route_w;     // [pairs] combine weights (mode 1)
    float* out;               // mode 0: act [padded][rows]; mode 1: pair_out [pairs][rows]
    uint32_t K;               // reduction length (hidden or inter)
    uint32_t rows;            // output rows per expert (inter or hidden)
    uint32_t flavour;
    uint32_t* status;
};

template <int kMode, int kSplit, int kQ, int kB>
struct GemmLayout {
    static constexpr uint32_t kc8 = kSplit ? 64u : 32u;
    static constexpr uint32_t bstage = packed_row_bytes(kc8) * kTileTokens;
    static constexpr uint32_t q_off = 0;
    static constexpr uint32_t b_off = q_off + kQ * kQStage;
    static constexpr uint32_t amin_off = b_off + kB * bstage;             // [2][2][128][16 B]
    static constexpr uint32_t dd_off = amin_off + 2 * 4096;                // [kDdRing][128] float2
    static constexpr uint32_t xch_off = dd_off + kDdRing * 128 * 8;        // [64 cols][64 rows] (mode 0)
    static constexpr uint32_t bar_off = xch_off + (kMode == 0 ? 64 * 64 * 4 : 0);
    static constexpr uint32_t nbars = 2 * kQ + 2 * kB + 8 + kDdRing + 3;
    static constexpr uint32_t misc_off = bar_off + nbars * 8;
    static constexpr uint32_t total = misc_off + 16;
};

// Eight fp16 pairs s * q of one 32-bit word of nibbles: byte pairs (0, 2) and
// (1, 3), low nibbles scaled by s_lo, high nibbles by s_hi.  A low nibble q
// becomes 1024 + q and a high nibble 1024 + 16 q (masked in place); one fp16
// FMA then gives q * s exactly.
struct NibbleScales {
    uint32_t lo_mul, lo_add, hi_mul, hi_add;
};
__device__ __forceinline__ NibbleScales nibble_scales(uint32_t s_lo, uint32_t s_hi) {
    const float lo = static_cast<float>(s_lo), hi = static_cast<float>(s_hi);
    NibbleScales n;
    n.lo_mul = pack_half2(lo, lo);
    n.lo_add = pack_half2(-1024.f * lo, -1024.f * lo);
    n.hi_mul = pack_half2(hi * 0.0625f, hi * 0.0625f);
    n.hi_add = pack_half2(-64.f * hi, -64.f * hi);
    return n;
}
__device__ __forceinline__ void dequant_word(uint32_t W, const NibbleScales& n, uint32_t* out4) {
    const uint32_t W8 = W >> 8;
    out4[0] = hfma2u((W & 0x000F000Fu) | kHalfMagic, n.lo_mul, n.lo_add);    // bytes 0, 2 low
    out4[1] = hfma2u((W8 & 0x000F000Fu) | kHalfMagic, n.lo_mul, n.lo_add);   // bytes 1, 3 low
    out4[2] = hfma2u((W & 0x00F000F0u) | kHalfMagic, n.hi_mul, n.hi_add);    // bytes 0, 2 high
    out4[3] = hfma2u((W8 & 0x00F000F0u) | kHalfMagic, n.hi_mul, n.hi_add);   // bytes 1, 3 high
}

template <int kMode, int kSplit, int kQ, int kB>
__global__ void __launch_bounds__(kGemmThreads, 1) grouped_gemm_kernel(const __grid_constant__ GemmArgs a) {
    using Lay = GemmLayout<kMode, kSplit, kQ, kB>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* qbuf = smem + Lay::q_off;
    uint8_t* bbuf = smem + Lay::b_off;
    uint8_t* amin = smem + Lay::amin_off;
    float2* dd = reinterpret_cast<float2*>(smem + Lay::dd_off);
    float* xch = reinterpret_cast<float*>(smem + Lay::xch_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::bar_off);
    uint64_t* q_full = bars;
    uint64_t* q_empty = q_full + kQ;
    uint64_t* b_full = q_empty + kQ;
    uint64_t* b_empty = b_full + kB;
    uint64_t* a_full = b_empty + kB;     // [2] dequantised A (and mins) ready
    uint64_t* a_free = a_full + 2;       // [2] MMAs reading A done
    uint64_t* acc_full = a_free + 2;     // [2] accumulators ready
    uint64_t* acc_free = acc_full + 2;   // [2] accumulators read
    uint64_t* dd_full = acc_free + 2;    // [kDdRing] (d, dmin) of a superblock written
    uint64_t* xch_full = dd_full + kDdRing;   // up rows written (mode 0)
    uint64_t* xch_free = xch_full + 1;        // up rows consumed (mode 0)
    uint64_t* drain = xch_free + 1;           // all MMAs complete
    uint32_t* misc = reinterpret_cast<uint32_t*>(smem + Lay::misc_off);
    volatile uint32_t* abort_flag = misc + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == kMmaWarp) {
        tmem_alloc(misc, 512);
        tmem_relinquish();
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kQ; ++i) { mbar_init(q_full + i, 1); mbar_init(q_empty + i, kDqWarps); }
        // A slot of packed activations is free once the MMAs read it (commit)
        // and the epilogue warps read its scales.
        for (int i = 0; i < kB; ++i) { mbar_init(b_full + i, 1); mbar_init(b_empty + i, 1 + kEpWarps); }
        for (int i = 0; i < 2; ++i) {
            mbar_init(a_full + i, kDqWarps);
            mbar_init(a_free + i, 1);
            mbar_init(acc_full + i, 1);
            mbar_init(acc_free + i, kEpWarps);
        }
        for (uint32_t i = 0; i < kDdRing; ++i) mbar_init(dd_full + i, kDqWarps);
        mbar_init(xch_full, kEpWarps / 2);
        mbar_init(xch_free, kEpWarps / 2);
        mbar_init(drain, 1);
        misc[1] = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = misc[0];
    // The tile list and packed activations come from the previous kernels
    // (programmatic launch: the set-up above overlapped their tail).
    grid_dep_wait();
    grid_dep_launch();

    const uint32_t S = a.K / 256;
    constexpr uint32_t kRowsPerUnit = kMode == 0 ? 64u : 128u;
    const uint32_t mblocks = a.rows / kRowsPerUnit;
    const uint32_t units = a.plan[2] * mblocks;

    const auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (*abort_flag) return false;
        if (mbar_wait_ns(bar, parity)) return true;
        atomicOr(a.status, kStatusWaitTimeout);
        *abort_flag = 1;
        return false;
    };
    // A warp's lanes take every wait together so that the warp-wide
    // tensor-memory instructions after it run converged.
    const auto wait_warp = [&](uint64_t* bar, uint32_t parity) -> bool {
        return __all_sync(0xFFFFFFFFu, wait(bar, parity)) != 0;
    };

    if (warp == kLoadWarp) {
        // ---------------- loader ----------------
        if (lane == 0) {
            int32_t last_q[kQ], last_b[kB];
            for (int i = 0; i < kQ; ++i) last_q[i] = -1;
            for (int i = 0; i < kB; ++i) last_b[i] = -1;
            uint32_t g = 0;
            bool ok = true;
            for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x) {
                const uint32_t tile = a.tile_order[u / mblocks], mb = u % mblocks;
                const uint32_t e = a.tile_expert[tile], np = round16(a.tile_n[tile]);
                const uint32_t stage = packed_row_bytes(Lay::kc8) * np;
                const uint8_t* bsrc = a.b + static_cast<size_t>(a.tile_pad0[tile]) * S * packed_row_bytes(Lay::kc8);
                for (uint32_t s = 0; s < S; ++s, ++g) {
                    const uint32_t qs = g % kQ, bs = g % kB;
                    if (!(ok = wait(q_empty + qs, ((g / kQ) & 1) ^ 1))) break;
                    mbar_expect_tx(q_full + qs, kQStage);
                    if (kMode == 0) {
                        tma_box_3d(qbuf + qs * kQStage, &a.tm0, s * 144, mb * 64, e, q_full + qs);
                        tma_box_3d(qbuf + qs * kQStage + 64 * 144, &a.tm1, s * 144, mb * 64, e, q_full + qs);
                    } else {
                        tma_box_3d(qbuf + qs * kQStage, &a.tm0, s * 144, mb * 128, e, q_full + qs);
                    }
                    last_q[qs] = static_cast<int32_t>(g);
                    if (!(ok = wait(b_empty + bs, ((g / kB) & 1) ^ 1))) break;
                    mbar_expect_tx(b_full + bs, stage);
                    bulk_g2s(bbuf + bs * Lay::bstage, bsrc + static_cast<size_t>(s) * stage, stage, b_full + bs);
                    last_b[bs] = static_cast<int32_t>(g);
                }
            }
            if (*abort_flag) {
                // Let the copies in flight land before the CTA exits.
                for (int i = 0; i < kQ; ++i)
                    if (last_q[i] >= 0) mbar_wait_ns(q_full + i, (static_cast<uint32_t>(last_q[i]) / kQ) & 1);
                for (int i = 0; i < kB; ++i)
                    if (last_b[i] >= 0) mbar_wait_ns(b_full + i, (static_cast<uint32_t>(last_b[i]) / kB) & 1);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x) {
                const uint32_t tile = a.tile_order[u / mblocks];
                const uint32_t np = round16(a.tile_n[tile]);
                const uint32_t idesc = tc_idesc_f16(128, np);
                const uint32_t lbo = np * 16;
                for (uint32_t s = 0; s < S; ++s, ++g) {
                    const uint32_t buf = g & 1, ph = (g >> 1) & 1, bs = g % kB;
                    if (!(ok = wait(a_full + buf, ph))) break;
                    if (!(ok = wait(b_full + bs, (g / kB) & 1))) break;
                    if (!(ok = wait(acc_free + buf, ph ^ 1))) break;
                    tc_fence_after();
                    const uint32_t a_col = tbase + buf * 128;
                    const uint32_t acc_q = tbase + 256 + buf * 128, acc_m = acc_q + 64;
                    const uint32_t bb = smem_addr(bbuf + bs * Lay::bstage);
#pragma unroll
                    for (uint32_t ks = 0; ks < 16; ++ks)
                        tc_mma_ts(acc_q, a_col + 8 * ks, tc_smem_desc(bb + 2 * ks * lbo, lbo, 128), idesc, ks > 0);
                    if (kSplit) {
#pragma unroll
                        for (uint32_t ks = 0; ks < 16; ++ks)
                            tc_mma_ts(acc_q, a_col + 8 * ks, tc_smem_desc(bb + (32 + 2 * ks) * lbo, lbo, 128), idesc,
                                      1);
                    }
                    tc_mma_ss(acc_m, tc_smem_desc(smem_addr(amin + buf * 4096), 2048, 128),
                              tc_smem_desc(bb + Lay::kc8 * lbo, lbo, 128), idesc, 0);
                    tc_commit(b_empty + bs);
                    tc_commit(a_free + buf);
                    tc_commit(acc_full + buf);
                }
            }
            tc_commit(drain);
            mbar_wait_ns(drain, 0);
        }
    } else if (warp >= kEpWarps) {
        // ---------------- dequantise ----------------
        const uint32_t dw = warp - kEpWarps;
        const uint32_t q4 = dw & 3, kh = dw >> 2;          // lane quarter, K half
        const uint32_t r = 32 * q4 + lane;                 // tile row = tensor-memory lane
        const uint32_t lane_base = (32 * q4) << 16;
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x) {
            for (uint32_t s = 0; s < S; ++s, ++g) {
                const uint32_t qs = g % kQ, buf = g & 1;
                if (!(ok = wait_warp(q_full + qs, (g / kQ) & 1))) break;
                if (!(ok = wait_warp(a_free + buf, ((g >> 1) & 1) ^ 1))) break;
                const uint8_t* row = qbuf + qs * kQStage + r * 144;
                // d, dmin and the 12 scale bytes in one 16-byte load (rows are 144 bytes
                // apart: a quarter warp's loads fall on distinct bank groups).
                const uint4 hdr = *reinterpret_cast<const uint4*>(row);
                const uint32_t dm = hdr.x, w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;
                // 6-bit scales / mins (k_scale_min): bytes q[0..11] = w0 | w1 | w2.
                uint32_t sc[8], mn[8];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t qj = (w0 >> (8 * j)) & 0xFF, qj4 = (w1 >> (8 * j)) & 0xFF;
                    const uint32_t qj8 = (w2 >> (8 * j)) & 0xFF;
                    sc[j] = qj & 63;
                    mn[j] = qj4 & 63;
                    sc[j + 4] = (qj8 & 0xF) | ((qj >> 6) << 4);
                    mn[j + 4] = (qj8 >> 4) | ((qj4 >> 6) << 4);
                }
                if (kh == 0)
                    dd[(g % kDdRing) * 128 + r] =
                        make_float2(half_bits_to_float(dm & 0xFFFF), half_bits_to_float(dm >> 16));
                {
                    uint4 mv;
                    mv.x = pack_half2(static_cast<float>(mn[0]), static_cast<float>(mn[1]));
                    mv.y = pack_half2(static_cast<float>(mn[2]), static_cast<float>(mn[3]));
                    mv.z = pack_half2(static_cast<float>(mn[4]), static_cast<float>(mn[5]));
                    mv.w = pack_half2(static_cast<float>(mn[6]), static_cast<float>(mn[7]));
                    *reinterpret_cast<uint4*>(amin + buf * 4096 + kh * 2048 + r * 16) = mv;
                }
#pragma unroll
                for (uint32_t cc = 0; cc < 2; ++cc) {
                    const uint32_t c = 2 * kh + cc;
                    const uint4 qa = *reinterpret_cast<const uint4*>(row + 16 + 32 * c);
                    const uint4 qb = *reinterpret_cast<const uint4*>(row + 16 + 32 * c + 16);
                    const uint32_t words[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    const NibbleScales ns = nibble_scales(sc[2 * c], sc[2 * c + 1]);
                    uint32_t v[32];
#pragma unroll
                    for (int w = 0; w < 8; ++w) dequant_word(words[w], ns, v + 4 * w);
                    tmem_st32(tbase + lane_base + buf * 128 + 32 * c, v);
                }
                tmem_wait_st();
                fence_async_shared();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(a_full + buf);
                    mbar_arrive(q_empty + qs);
                    mbar_arrive(dd_full + g % kDdRing);
                }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const uint32_t q4 = warp & 3, nh = warp >> 2;      // lane quarter, N half
        const uint32_t r = 32 * q4 + lane;
        const uint32_t lane_base = (32 * q4) << 16;
        float acc[32];
        uint32_t g = 0, ui = 0;
        bool ok = true;
        for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++ui) {
            const uint32_t tile = a.tile_order[u / mblocks], mb = u % mblocks;
            const uint32_t n_valid = a.tile_n[tile], np = round16(n_valid), pad0 = a.tile_pad0[tile];
            const uint32_t hn = np >> 1, c0 = nh * hn;
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0.f;
            for (uint32_t s = 0; s < S; ++s, ++g) {
                const uint32_t buf = g & 1, bs = g % kB;
                if (!(ok = wait_warp(acc_full + buf, (g >> 1) & 1))) break;
                if (!(ok = wait_warp(dd_full + g % kDdRing, (g / kDdRing) & 1))) break;
                if (!(ok = wait_warp(b_full + bs, (g / kB) & 1))) break;   // scales visible here
                tc_fence_after();
                const float2 dm = dd[(g % kDdRing) * 128 + r];
                const float* scl = reinterpret_cast<const float*>(bbuf + bs * Lay::bstage + (Lay::kc8 + 2) * np * 16);
                const uint32_t acc_q = tbase + lane_base + 256 + buf * 128 + c0, acc_m = acc_q + 64;
#pragma unroll
                for (uint32_t c2 = 0; c2 < 4; c2 += 2) {
                    if (8 * c2 < hn) {
                        uint32_t qv[2][8], mv[2][8];
#pragma unroll
                        for (uint32_t c = 0; c < 2; ++c) {
                            if (8 * (c2 + c) < hn) {
                                tmem_ld8(acc_q + 8 * (c2 + c), qv[c]);
                                tmem_ld8(acc_m + 8 * (c2 + c), mv[c]);
                            }
                        }
                        tmem_wait_ld();
#pragma unroll
                        for (uint32_t c = 0; c < 2; ++c) {
                            if (8 * (c2 + c) < hn) {
                                const float4 s0 = *reinterpret_cast<const float4*>(scl + c0 + 8 * (c2 + c));
                                const float4 s1 = *reinterpret_cast<const float4*>(scl + c0 + 8 * (c2 + c) + 4);
                                const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    float& A = acc[8 * (c2 + c) + i];
                                    A = fmaf(fmaf(dm.x, __uint_as_float(qv[c][i]), -dm.y * __uint_as_float(mv[c][i])),
                                             sv[i], A);
                                }
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(acc_free + buf);
                    mbar_arrive(b_empty + bs);
                }
            }
            if (!ok) break;
            if (kMode == 0) {
                // Rows 0..63 hold gate, 64..127 up: silu(gate) * up per token.
                if (q4 >= 2) {
                    if (!(ok = wait_warp(xch_free, (ui & 1) ^ 1))) break;
#pragma unroll
                    for (uint32_t c = 0; c < 4; ++c)
                        if (8 * c < hn)
#pragma unroll
                            for (int i = 0; i < 8; ++i) xch[(c0 + 8 * c + i) * 64 + (r - 64)] = acc[8 * c + i];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_full);
                } else {
                    if (!(ok = wait_warp(xch_full, ui & 1))) break;
#pragma unroll
                    for (uint32_t c = 0; c < 4; ++c) {
                        if (8 * c < hn) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const uint32_t col = c0 + 8 * c + i;
                                if (col < n_valid) {
                                    const float h = silu_times(acc[8 * c + i], xch[col * 64 + r], a.flavour);
                                    a.out[static_cast<size_t>(pad0 + col) * a.rows + mb * 64 + r] = h;
                                }
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_free);
                }
            } else {
                // The pair and combine weight of each of this warp's (<= 32)
                // columns: lane j loads column c0 + j once, the elements get
                // them by shuffle.
                const uint32_t first = a.tile_first[tile];
                const uint32_t lc = c0 + lane;
                const uint32_t pr = lc < n_valid ? a.slot_pair[first + lc] : 0u;
                const float wt = lc < n_valid ? a.route_w[pr] : 0.f;
#pragma unroll
                for (uint32_t c = 0; c < 4; ++c) {
                    if (8 * c < hn) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t col = c0 + 8 * c + i;
                            const uint32_t j = 8 * c + i;              // column within this warp's half
                            const uint32_t p = __shfl_sync(0xFFFFFFFFu, pr, j);
                            const float w = __shfl_sync(0xFFFFFFFFu, wt, j);
                            if (col < n_valid) a.out[static_cast<size_t>(p) * a.rows + mb * 128 + r] = w * acc[j];
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ---------------------------------------------------------------------------
// 5b/7b. Skinny tiles (<= kSkinny tokens) on mma.sync.m16n8k16 (fp16 in,
// F32 accumulate).  A tcgen05 MMA costs the same for 8 tokens as for 128, so
// a tile of a few tokens would leave the weights' HBM stream waiting on the
// tensor core; here the weights go straight from shared memory into A
// registers and each MMA multiplies 16 rows by the tile's 8 token columns.
//
// Persistent, one CTA per SM; a unit is (skinny tile, 128 rows of gate and the
// same 128 rows of up) or (skinny tile, 128 rows of down).  The last warp (one
// lane) loads each superblock of the unit into a ring stage: the Q4_K rows by
// TMA (144 bytes x 128 rows per matrix) and the tile's packed activations (the
// skinny layout above) by one bulk copy.  Two groups of eight warps take the
// unit's even and odd superblocks; in a group, warp w owns rows 16w..16w+15:
// thread (g = lane / 4, t = lane % 4) dequantises Q4_K chunk t (qs bytes
// 32t..32t+31: sub-blocks 2t, 2t+1) of rows g and g + 8 into fp16 s_j q
// (exact; the tensor-core path's nibble arithmetic) and feeds them as A with
// the activation fragments as B; one more MMA (A = m_j, B = the sub-block
// sums as hi + lo) gives the mins; d, dmin and the tokens' scales are applied
// per superblock in F32.  The odd group hands its sums to the even group,
// which writes the unit's outputs.
// ---------------------------------------------------------------------------
constexpr uint32_t kThinRowWarps = 8;                        // 16 rows each: 128 rows
constexpr uint32_t kThinWarps = 2 * kThinRowWarps;           // two superblock groups
constexpr uint32_t kThinThreads = (kThinWarps + 1) * 32;     // + the loader

template <int kMode, int kSplit>
struct ThinLayout {
    static constexpr uint32_t mats = kMode == 0 ? 2u : 1u;
    static constexpr uint32_t wbytes = mats * kQStage;
    static constexpr uint32_t stage = (wbytes + thin_stage_bytes(kSplit) + 127u) & ~127u;
    static constexpr uint32_t xch_bytes = kThinRowWarps * 32 * mats * 4 * 4;   // odd group's sums
    static constexpr uint32_t budget = 220u * 1024u - xch_bytes;
    static constexpr uint32_t stages = budget / stage < 8u ? budget / stage : 8u;
    static constexpr uint32_t xch_off = stages * stage;
    static constexpr uint32_t bar_off = xch_off + xch_bytes;
    static constexpr uint32_t total = bar_off + (2 * stages + 2) * 8 + 16;
};

struct ThinArgs {
    CUtensorMap tm0;          // gate (mode 0) or down (mode 1), 128-row boxes
    CUtensorMap tm1;          // up (mode 0)
    const uint8_t* b;         // packed activations
    const uint32_t* plan;
    const uint32_t* tile_order;   // [plan[2], plan[2] + plan[3]): the skinny tiles
    const uint32_t* tile_expert;
    const uint32_t* tile_first;
    const uint32_t* tile_n;
    const uint32_t* tile_pad0;
    const uint32_t* slot_pair;
    const float* route_w;
    float* out;               // mode 0: act [padded][rows]; mode 1: pair_out [pairs][rows]
    uint32_t K, rows, flavour;
    uint32_t* status;
};

// 6-bit scales (s0, s1) and mins (m0, m1) of sub-blocks 2t and 2t + 1 from a
// Q4_K header's scale words (hy, hz, hw = bytes 0..3, 4..7, 8..11), both
// sub-blocks at once and without a branch on t: the k_scale_min unpacking of
// decode_q4_k (src/quantized_linear.cpp:176-188).
__device__ __forceinline__ void q4k_pair_scales(uint32_t hy, uint32_t hz, uint32_t hw, uint32_t t, uint32_t& sc,
                                                uint32_t& mn) {
    const uint32_t sh = 16 * (t & 1);
    const uint32_t a = hy >> sh, b = hz >> sh, c = hw >> sh;
    const uint32_t sc_lo = a & 0x3F3Fu, mn_lo = b & 0x3F3Fu;                      // sub-blocks 0..3
    const uint32_t sc_hi = (c & 0x0F0Fu) | ((a >> 2) & 0x3030u);                   // sub-blocks 4..7
    const uint32_t mn_hi = ((c >> 4) & 0x0F0Fu) | ((b >> 2) & 0x3030u);
    sc = t >= 2 ? sc_hi : sc_lo;   // byte 0: sub-block 2t, byte 1: 2t + 1
    mn = t >= 2 ? mn_hi : mn_lo;
}
// (v, v) in fp16 for an integer v < 1024: 1024 + v has v as its mantissa.
__device__ __forceinline__ uint32_t half2_small(uint32_t v) {
    return hsub2u((v * 0x10001u) | kHalfMagic, kHalfMagic);
}
// nibble_scales for the 6-bit scales in bytes 0 (low nibbles) and 1 (high) of sc.
__device__ __forceinline__ NibbleScales nibble_scales_packed(uint32_t sc) {
    NibbleScales n;
    const uint32_t lo = half2_small(sc & 0xFFu), hi = half2_small((sc >> 8) & 0xFFu);
    n.lo_mul = lo;
    n.lo_add = hmul2u(lo, kHalfNeg1024);
    n.hi_mul = hmul2u(hi, kHalfInv16);
    n.hi_add = hmul2u(hi, kHalfNeg64);
    return n;
}

template <int kMode, int kSplit>
__global__ void __launch_bounds__(kThinThreads, 1) thin_gemm_kernel(const __grid_constant__ ThinArgs a) {
    using Lay = ThinLayout<kMode, kSplit>;
    constexpr uint32_t kMats = Lay::mats, kStages = Lay::stages;
    extern __shared__ __align__(1024) uint8_t smem[];
    float* xch = reinterpret_cast<float*>(smem + Lay::xch_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::bar_off);
    uint64_t* empty = full + kStages;
    uint64_t* xch_full = empty + kStages;   // odd group's sums written
    uint64_t* xch_free = xch_full + 1;      // ... and read
    volatile uint32_t* abort_flag = reinterpret_cast<uint32_t*>(xch_free + 1);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < kStages; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kThinRowWarps);
        }
        mbar_init(xch_full, kThinRowWarps);
        mbar_init(xch_free, kThinRowWarps);
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    grid_dep_wait();      // tile list and packed activations of the previous kernels
    grid_dep_launch();

    const uint32_t S = a.K / 256;
    const uint32_t mblocks = a.rows / 128;
    const uint32_t first_thin = a.plan[2];
    const uint32_t units = a.plan[3] * mblocks;
    const size_t tile_stride = static_cast<size_t>(S) * packed_row_bytes(kSplit ? 64u : 32u);

    const auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (*abort_flag) return false;
        if (mbar_wait_ns(bar, parity)) return true;
        atomicOr(a.status, kStatusWaitTimeout);
        *abort_flag = 1;
        return false;
    };
    const auto wait_warp = [&](uint64_t* bar, uint32_t parity) -> bool {
        return __all_sync(0xFFFFFFFFu, wait(bar, parity)) != 0;
    };

    if (warp == kThinWarps) {
        // ---------------- loader ----------------
        if (lane == 0) {
            int32_t last[kStages];
            for (uint32_t i = 0; i < kStages; ++i) last[i] = -1;
            uint32_t g = 0;
            bool ok = true;
            // A unit's expert and activation region, read one unit ahead so the
            // two dependent global loads overlap the previous unit's copies.
            const auto fetch = [&](uint32_t u) -> uint2 {
                if (u >= units) return make_uint2(0u, 0u);
                const uint32_t tile = a.tile_order[first_thin + u / mblocks];
                return make_uint2(a.tile_expert[tile], a.tile_pad0[tile]);
            };
            uint2 cur = fetch(blockIdx.x);
            for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x) {
                const uint2 nxt = fetch(u + gridDim.x);
                const uint32_t mb = u % mblocks, e = cur.x;
                const uint8_t* src = a.b + cur.y * tile_stride;
                cur = nxt;
                for (uint32_t s = 0; s < S; ++s, ++g) {
                    const uint32_t slot = g % kStages;
                    if (!(ok = wait(empty + slot, ((g / kStages) & 1) ^ 1))) break;
                    uint8_t* st = smem + slot * Lay::stage;
                    mbar_expect_tx(full + slot, Lay::wbytes + thin_stage_bytes(kSplit));
                    tma_box_3d(st, &a.tm0, s * 144, mb * 128, e, full + slot);
                    if (kMode == 0) tma_box_3d(st + kQStage, &a.tm1, s * 144, mb * 128, e, full + slot);
                    bulk_g2s(st + Lay::wbytes, src + static_cast<size_t>(s) * thin_stage_bytes(kSplit),
                             thin_stage_bytes(kSplit), full + slot);
                    last[slot] = static_cast<int32_t>(g);
                }
            }
            if (*abort_flag) {
                // Let the copies in flight land before the CTA exits.
                for (uint32_t i = 0; i < kStages; ++i)
                    if (last[i] >= 0) mbar_wait_ns(full + i, (static_cast<uint32_t>(last[i]) / kStages) & 1);
            }
        }
        return;
    }

    // ---------------- compute ----------------
    const uint32_t grp = warp / kThinRowWarps, rw = warp % kThinRowWarps;
    const uint32_t g8 = lane >> 2, t = lane & 3;
    const uint32_t r0 = 16 * rw + g8;
    uint32_t g = 0, ui = 0;
    bool ok = true;
    for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++ui) {
        const uint32_t tile = a.tile_order[first_thin + u / mblocks], mb = u % mblocks;
        float tot[kMats][4];
#pragma unroll
        for (uint32_t m = 0; m < kMats; ++m)
#pragma unroll
            for (int i = 0; i < 4; ++i) tot[m][i] = 0.f;
        for (uint32_t s = 0; s < S; ++s, ++g) {
            if ((s & 1) != grp) continue;
            const uint32_t slot = g % kStages;
            if (!(ok = wait_warp(full + slot, (g / kStages) & 1))) break;
            const uint8_t* st = smem + slot * Lay::stage;
            const uint8_t* xs = st + Lay::wbytes;
            const uint8_t* xt = xs + kThinTail + g8 * kThinTokPitch + t * kThinSegPitch;
            const uint2 bm = *reinterpret_cast<const uint2*>(xs + (4 * g8 + t) * 8);   // token g8's sums
            const float2 sc = *reinterpret_cast<const float2*>(xs + 256 + 8 * t);     // tokens 2t, 2t + 1
            // One matrix at a time (not unrolled): the registers of one set of rows.
#pragma unroll 1
            for (uint32_t m = 0; m < kMats; ++m) {
                const uint8_t* row0 = st + m * kQStage + r0 * 144;
                const uint8_t* row1 = row0 + 8 * 144;
                const uint4 h0 = *reinterpret_cast<const uint4*>(row0);
                const uint4 h1 = *reinterpret_cast<const uint4*>(row1);
                const uint4 qa0 = *reinterpret_cast<const uint4*>(row0 + 16 + 32 * t);
                const uint4 qa1 = *reinterpret_cast<const uint4*>(row0 + 32 + 32 * t);
                const uint4 qb0 = *reinterpret_cast<const uint4*>(row1 + 16 + 32 * t);
                const uint4 qb1 = *reinterpret_cast<const uint4*>(row1 + 32 + 32 * t);
                uint32_t sca, mna, scb, mnb;
                q4k_pair_scales(h0.y, h0.z, h0.w, t, sca, mna);
                q4k_pair_scales(h1.y, h1.z, h1.w, t, scb, mnb);
                const NibbleScales na = nibble_scales_packed(sca), nb = nibble_scales_packed(scb);
                const uint32_t wa[8] = {qa0.x, qa0.y, qa0.z, qa0.w, qa1.x, qa1.y, qa1.z, qa1.w};
                const uint32_t wb[8] = {qb0.x, qb0.y, qb0.z, qb0.w, qb1.x, qb1.y, qb1.z, qb1.w};
                // acc[parity]: low-nibble k-steps (parity 0) and high (1), hi and lo activations.
                float acc[2][4] = {};
#pragma unroll
                for (uint32_t w = 0; w < 8; ++w) {
                    const uint4 xh = *reinterpret_cast<const uint4*>(xt + (w << 4));
                    uint32_t ra[4], rb[4];   // rows g8 and g8 + 8
                    dequant_word(wa[w], na, ra);
                    dequant_word(wb[w], nb, rb);
                    mma16816(acc[0], ra[0], rb[0], ra[1], rb[1], xh.x, xh.y);
                    mma16816(acc[1], ra[2], rb[2], ra[3], rb[3], xh.z, xh.w);
                    if (kSplit) {
                        const uint4 xl = *reinterpret_cast<const uint4*>(xt + kThinPart + (w << 4));
                        mma16816(acc[0], ra[0], rb[0], ra[1], rb[1], xl.x, xl.y);
                        mma16816(acc[1], ra[2], rb[2], ra[3], rb[3], xl.z, xl.w);
                    }
                }
                float mn[4] = {0.f, 0.f, 0.f, 0.f};
                const uint32_t am0 = half2_small(mna & 0xFFu) & 0xFFFFu | (half2_small(mna >> 8) << 16);
                const uint32_t am1 = half2_small(mnb & 0xFFu) & 0xFFFFu | (half2_small(mnb >> 8) << 16);
                mma16816(mn, am0, am1, am0, am1, bm.x, bm.y);
                const float d0 = half_bits_to_float(h0.x), dm0 = half_bits_to_float(h0.x >> 16);
                const float d1 = half_bits_to_float(h1.x), dm1 = half_bits_to_float(h1.x >> 16);
                float part[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float q = acc[0][i] + acc[1][i];
                    const float d = i < 2 ? d0 : d1, dmin = i < 2 ? dm0 : dm1;
                    part[i] = fmaf(d, q, -dmin * mn[i]) * ((i & 1) ? sc.y : sc.x);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (m == 0) tot[0][i] += part[i];
                    else tot[kMats - 1][i] += part[i];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + slot);
        }
        if (!ok) break;
        // The odd group's sums go to the even group through shared memory.
        float* mine = xch + (rw * 32 + lane) * (kMats * 4);
        if (grp == 1) {
            if (!(ok = wait_warp(xch_free, (ui & 1) ^ 1))) break;
#pragma unroll
            for (uint32_t m = 0; m < kMats; ++m)
                *reinterpret_cast<float4*>(mine + 4 * m) = make_float4(tot[m][0], tot[m][1], tot[m][2], tot[m][3]);
            __syncwarp();
            if (lane == 0) mbar_arrive(xch_full);
            continue;
        }
        if (!(ok = wait_warp(xch_full, ui & 1))) break;
#pragma unroll
        for (uint32_t m = 0; m < kMats; ++m) {
            const float4 o = *reinterpret_cast<const float4*>(mine + 4 * m);
            tot[m][0] += o.x;
            tot[m][1] += o.y;
            tot[m][2] += o.z;
            tot[m][3] += o.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(xch_free);
        // Columns 2t, 2t + 1 of rows r0 and r0 + 8.
        const uint32_t n_valid = a.tile_n[tile], first = a.tile_first[tile], pad0 = a.tile_pad0[tile];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t col = 2 * t + (i & 1);
            const uint32_t row = mb * 128 + r0 + (i < 2 ? 0u : 8u);
            if (col < n_valid) {
                if (kMode == 0) {
                    a.out[static_cast<size_t>(pad0 + col) * a.rows + row] =
                        silu_times(tot[0][i], tot[kMats - 1][i], a.flavour);
                } else {
                    const uint32_t p = a.slot_pair[first + col];
                    a.out[static_cast<size_t>(p) * a.rows + row] = a.route_w[p] * tot[0][i];
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// 8. Combine: out[t] = sum_r pair_out[t * k + r] in rank order from 0
// (the reference adds w_r * y_r in that order, qwen3_moe_runner.cpp:688-690),
// over the ranks whose expert this device holds.
// ---------------------------------------------------------------------------
__global__ void combine_kernel(const float* __restrict__ pair_out, const uint32_t* __restrict__ ids,
                               uint32_t e_first, uint32_t e_count, uint32_t tokens, uint32_t k, uint32_t H,
                               float* __restrict__ out) {
    grid_dep_wait();
    grid_dep_launch();
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;   // float4 index
    const size_t per_token = H / 4;
    if (i >= static_cast<size_t>(tokens) * per_token) return;
    const size_t t = i / per_token, c = i % per_token;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t r = 0; r < k; ++r) {
        if (ids[t * k + r] - e_first >= e_count) continue;   // an expert of another shard
        const float4 v = reinterpret_cast<const float4*>(pair_out + (t * k + r) * H)[c];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    reinterpret_cast<float4*>(out + t * H)[c] = acc;
}

// ---------------------------------------------------------------------------
// 8'. Combine and exchange (expert parallelism over peer memory).  One kernel
// per block replaces the local combine and the all-reduce of the ranks'
// partial outputs:
//   1. this rank's partial (its experts' pairs, rank order) is stored into
//      slot [parity][rank] of every rank's exchange region (NVLink stores);
//   2. the CTA that arrives last raises flag [parity][rank] = call number on
//      every rank (release, after a system fence);
//   3. every CTA waits until all ranks' flags of this call are up (acquire;
//      at most ~1 s, then the status bit and no wait), then sums the ranks'
//      partials in rank order, so every rank writes the same values.
// The call number lives in device memory (read by every CTA before the last
// one advances it), so graph replays count correctly; the parity double
// buffer keeps a rank that runs one call ahead from overwriting a slot
// another rank is still reading.  All CTAs are co-resident (grid <= SMs),
// which the wait of step 3 needs.
// ---------------------------------------------------------------------------
struct ExchangeArgs {
    const float* pair_out;
    const uint32_t* ids;
    uint32_t e_first, e_count, tokens, k, H;
    float* out;
    uint32_t* status;
    EpExchange ex;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
constexpr uint32_t kExchangeSpins = 1u << 22;   // x >= 256 ns sleeps: about a second

__global__ void __launch_bounds__(256) exchange_combine_kernel(const __grid_constant__ ExchangeArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const EpExchange& ex = a.ex;
    __shared__ uint32_t s_target, s_last;
    if (threadIdx.x == 0) s_target = *reinterpret_cast<volatile const uint32_t*>(ex.epoch) + 1u;
    __syncthreads();
    const uint32_t target = s_target, par = target & 1u;
    const size_t slot = static_cast<size_t>(ex.max_tokens) * ex.hidden;   // floats per (parity, source) slot
    const size_t recv_floats = 2ull * ex.world * slot;
    const size_t per_token = a.H / 4, quads = static_cast<size_t>(a.tokens) * per_token;
    const size_t step = static_cast<size_t>(gridDim.x) * blockDim.x;
    // 1. The local partial into slot [par][rank] of every rank.
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < quads; i += step) {
        const size_t t = i / per_token, c = i % per_token;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t r = 0; r < a.k; ++r) {
            if (a.ids[t * a.k + r] - a.e_first >= a.e_count) continue;   // an expert of another shard
            const float4 v = reinterpret_cast<const float4*>(a.pair_out + (t * a.k + r) * a.H)[c];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        for (uint32_t d = 0; d < ex.world; ++d) {
            float* dst = reinterpret_cast<float*>(ex.peers[d]) + (static_cast<size_t>(par) * ex.world + ex.rank) * slot;
            reinterpret_cast<float4*>(dst)[t * per_token + c] = acc;
        }
    }
    __threadfence_system();
    __syncthreads();
    // 2. The last CTA raises this rank's flag on every rank.
    if (threadIdx.x == 0) s_last = atomicAdd(ex.arrive, 1u) == gridDim.x - 1u ? 1u : 0u;
    __syncthreads();
    if (s_last) {
        __threadfence_system();
        if (threadIdx.x < ex.world) {
            uint32_t* fl = reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(ex.peers[threadIdx.x]) + recv_floats);
            st_release_sys(fl + par * ex.world + ex.rank, target);
        }
        if (threadIdx.x == 0) {
            *ex.arrive = 0u;
            *ex.epoch = target;
        }
    }
    // 3. Wait for every rank's partial, then sum them in rank order.
    if (threadIdx.x == 0) {
        const uint32_t* fl =
            reinterpret_cast<const uint32_t*>(reinterpret_cast<const float*>(ex.peers[ex.rank]) + recv_floats) +
            par * ex.world;
        for (uint32_t src = 0; src < ex.world; ++src) {
            uint32_t spins = 0;
            while (ld_acquire_sys(fl + src) != target) {
                if (++spins > kExchangeSpins) {
                    atomicOr(a.status, kStatusWaitTimeout);
                    break;
                }
                __nanosleep(256);
            }
            if (spins > kExchangeSpins) break;
        }
    }
    __syncthreads();
    const float* mine = reinterpret_cast<const float*>(ex.peers[ex.rank]) + static_cast<size_t>(par) * ex.world * slot;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < quads; i += step) {
        const size_t t = i / per_token, c = i % per_token;
        float4 acc = __ldcg(reinterpret_cast<const float4*>(mine) + t * per_token + c);
        for (uint32_t src = 1; src < ex.world; ++src) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(mine + src * slot) + t * per_token + c);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        reinterpret_cast<float4*>(a.out + t * a.H)[c] = acc;
    }
}

// Gate/up operand from BF16 inputs (no lo part) or F32 inputs (hi + lo); the
// down operand always has the lo part.
using GateUpBf16 = GemmLayout<0, 0, 4, 3>;
using GateUpF32 = GemmLayout<0, 1, 3, 2>;
using DownLay = GemmLayout<1, 1, 4, 2>;
static_assert(GateUpBf16::total <= 227 * 1024, "gate/up (bf16) shared memory");
static_assert(GateUpF32::total <= 227 * 1024, "gate/up (f32) shared memory");
static_assert(DownLay::total <= 227 * 1024, "down shared memory");
static_assert(ThinLayout<0, 0>::total <= 227 * 1024 && ThinLayout<0, 1>::total <= 227 * 1024 &&
                  ThinLayout<1, 1>::total <= 227 * 1024,
              "skinny shared memory");

uint32_t max_tiles_for(uint32_t pairs, uint32_t E) { return pairs / kTileTokens + std::min(E, pairs) + 1; }

size_t al256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

struct BatchSizes {
    uint32_t pairs, max_tiles, max_padded;
    size_t logits, ids, weights, rank, plan, tiles, slot_pair, bgu, act, bdn, pair_out;
    size_t total;
};

BatchSizes batch_sizes(const MoeLayerDev& L, uint32_t T) {
    BatchSizes z{};
    z.pairs = T * L.top_k;
    z.max_tiles = max_tiles_for(z.pairs, L.expert_local);
    z.max_padded = z.pairs + 15u * z.max_tiles;
    const size_t Sg = L.hidden / 256, Sd = L.inter / 256;
    z.logits = al256(size_t(T) * L.experts * 4 * std::max<uint32_t>(1u, L.hidden / router_slice(L.hidden)));
    z.ids = al256(size_t(z.pairs) * 4);
    z.weights = z.ids;
    z.rank = z.ids;
    z.plan = 256;
    z.tiles = al256(size_t(z.max_tiles) * 4);
    z.slot_pair = z.ids;
    z.bgu = al256(size_t(z.max_padded) * Sg * packed_row_bytes(64));   // room for the hi + lo form
    z.act = al256(size_t(z.max_padded) * L.inter * 4);
    z.bdn = al256(size_t(z.max_padded) * Sd * packed_row_bytes(64));
    z.pair_out = al256(size_t(z.pairs) * L.hidden * 4);
    z.total = z.logits + z.ids + z.weights + z.rank + z.plan + 5 * z.tiles + z.slot_pair + z.bgu + z.act + z.bdn +
              z.pair_out;
    return z;
}

// Raises a kernel's dynamic shared-memory limit once per device (the call
// is then kept out of later launches, so they can be captured in graphs).
template <typename Kern>
cudaError_t set_smem(Kern k, uint32_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, uint32_t> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    uint32_t& have = done[{reinterpret_cast<const void*>(k), dev}];
    if (have >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) have = bytes;
    return e;
}

// Launches kernel k, as a programmatic dependent of the previous kernel in the
// stream when pdl (every kernel of the batched block waits for its
// predecessor with griddepcontrol.wait before reading what it wrote, and lets
// its own dependent start launching right after).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                     Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

}  // namespace

uint64_t ep_exchange_bytes(uint32_t world, uint32_t max_tokens, uint32_t hidden) {
    return al256(2ull * world * max_tokens * hidden * 4ull + 2ull * world * 4ull);
}

bool moe_batch_grouped(const MoeLayerDev& L) {
    const auto al16 = [](const void* p, uint64_t n) {
        return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (n & 15u) == 0;
    };
    return L.gate_type == kQ4_K && L.up_type == kQ4_K && L.down_type == kQ4_K && L.shared_inter == 0 &&
           L.hidden % 256 == 0 && L.inter % 256 == 0 && L.hidden >= 256 && L.inter >= 256 && L.gate && L.up &&
           L.down && al16(L.gate, L.gate_slice) && al16(L.up, L.up_slice) && al16(L.down, L.down_slice) &&
           L.experts >= 1 && L.experts <= 1024 && L.top_k >= 1 && L.top_k <= 64 && L.top_k <= L.experts &&
           L.expert_local >= 1 && L.expert_first + L.expert_local <= L.experts;
}

uint64_t moe_batch_scratch_bytes(const MoeLayerDev& L, uint32_t max_tokens) {
    return batch_sizes(L, max_tokens).total;
}

MoeBatchScratch moe_batch_scratch_carve(const MoeLayerDev& L, uint32_t max_tokens, void* base) {
    const BatchSizes z = batch_sizes(L, max_tokens);
    MoeBatchScratch S{};
    S.max_tokens = max_tokens;
    S.max_tiles = z.max_tiles;
    S.max_padded = z.max_padded;
    uint8_t* p = static_cast<uint8_t*>(base);
    const auto take = [&](size_t n) {
        uint8_t* q = p;
        p += n;
        return q;
    };
    S.logits = reinterpret_cast<float*>(take(z.logits));
    S.ids = reinterpret_cast<uint32_t*>(take(z.ids));
    S.weights = reinterpret_cast<float*>(take(z.weights));
    S.rank = reinterpret_cast<uint32_t*>(take(z.rank));
    S.plan = reinterpret_cast<uint32_t*>(take(z.plan));
    S.tile_order = reinterpret_cast<uint32_t*>(take(z.tiles));
    S.tile_expert = reinterpret_cast<uint32_t*>(take(z.tiles));
    S.tile_first = reinterpret_cast<uint32_t*>(take(z.tiles));
    S.tile_n = reinterpret_cast<uint32_t*>(take(z.tiles));
    S.tile_pad0 = reinterpret_cast<uint32_t*>(take(z.tiles));
    S.slot_pair = reinterpret_cast<uint32_t*>(take(z.slot_pair));
    S.b_gate_up = take(z.bgu);
    S.act = reinterpret_cast<float*>(take(z.act));
    S.b_down = take(z.bdn);
    S.pair_out = reinterpret_cast<float*>(take(z.pair_out));
    return S;
}

cudaError_t launch_moe_batch(const MoeLayerDev& L, const MoeBatchScratch& S, const void* x, uint32_t x_bf16,
                             uint32_t tokens, const float* logits, float* out, uint32_t* ids, float* weights,
                             uint32_t* status, cudaStream_t stream, uint32_t* launches, cudaEvent_t* marks,
                             const EpExchange* ex) {
    uint32_t n = 0, stage = 0;   // kernels launched; stage boundaries marked
    const bool pdl = marks == nullptr;   // per-stage events need the kernels serialised
    const auto mark = [&]() {
        if (marks) cudaEventRecord(marks[stage++], stream);
    };
    if (launches) *launches = 0;
    if (!moe_batch_grouped(L) || tokens == 0 || tokens > S.max_tokens || !x || !out || !status)
        return cudaErrorInvalidValue;
    if (ex && (ex->world < 1 || ex->world > kMaxExchangeRanks || ex->rank >= ex->world || tokens > ex->max_tokens ||
               ex->hidden != L.hidden || !ex->epoch || !ex->arrive))
        return cudaErrorInvalidValue;
    if (!logits && !L.router) return cudaErrorInvalidValue;
    const uint32_t E = L.experts, k = L.top_k, H = L.hidden, I = L.inter;
    const uint32_t EL = L.expert_local, E0 = L.expert_first;   // experts held here
    const uint32_t pairs = tokens * k;
    cudaError_t err;

    CUtensorMap tg{}, tu{}, td{}, tg128{}, tu128{};
    const uint64_t rb_in = row_bytes(kQ4_K, H), rb_dn = row_bytes(kQ4_K, I);
    if (!encode_expert_map(&tg, L.gate, rb_in, I, EL, L.gate_slice, 64) ||
        !encode_expert_map(&tu, L.up, rb_in, I, EL, L.up_slice, 64) ||
        !encode_expert_map(&tg128, L.gate, rb_in, I, EL, L.gate_slice, 128) ||
        !encode_expert_map(&tu128, L.up, rb_in, I, EL, L.up_slice, 128) ||
        !encode_expert_map(&td, L.down, rb_dn, H, EL, L.down_slice, 128))
        return cudaErrorInvalidValue;

    mark();
    // 1. router (partials over hidden slices when it runs here)
    const float* lg = logits;
    uint32_t splits = 1;
    if (!lg) {
        const uint32_t slice = router_slice(H);
        if (tokens <= kRtSmall) {
            if ((err = launch_k(router_small_kernel, dim3((E + 7) / 8, H / slice), dim3(256), 0, stream, pdl,
                                L.router, x, x_bf16, tokens, E, H, slice, S.logits)) != cudaSuccess)
                return err;
        } else {
            const dim3 rgrid((tokens + kRtTok - 1) / kRtTok, (E + kRtExp - 1) / kRtExp, H / slice);
            if ((err = launch_k(router_batch_kernel, rgrid, dim3(256), 0, stream, pdl, L.router, x, x_bf16, tokens, E,
                                H, slice, S.logits)) != cudaSuccess)
                return err;
        }
        splits = H / slice;
        ++n;
        mark();
        lg = S.logits;
    }
    // 2. routes
    if ((err = launch_route_experts(lg, E, k, L.flavour, L.normalize, L.expert_weights_scale, S.ids, S.weights,
                                    status, stream, tokens, splits, pdl)) != cudaSuccess)
        return err;
    ++n;
    mark();
    // 3. group
    {
        GroupOut o{S.plan, S.tile_order, S.tile_expert, S.tile_first, S.tile_n, S.tile_pad0, S.slot_pair, S.rank};
        const uint32_t smem = (kSortWarps + 5) * EL * 4 + 16;
        if ((err = set_smem(group_kernel, smem)) != cudaSuccess) return err;
        if ((err = launch_k(group_kernel, dim3(1), dim3(kSortThreads), smem, stream, pdl, S.ids, pairs, E0, EL, o)) !=
            cudaSuccess)
            return err;
        ++n;
        mark();
    }
    const int sms = device_sm_count();
    // 4. pack x
    PackArgs px{};
    px.src = x;
    px.src_bf16 = x_bf16;
    px.by_token = 1;
    px.top_k = k;
    px.cols = H;
    px.split = x_bf16 ? 0 : 1;
    px.plan = S.plan;
    px.tile_first = S.tile_first;
    px.tile_n = S.tile_n;
    px.tile_pad0 = S.tile_pad0;
    px.slot_pair = S.slot_pair;
    px.dst = S.b_gate_up;
    const uint32_t max_tiles = max_tiles_for(pairs, EL);
    const dim3 pack_grid(max_tiles, kTileTokens / (kPackThreads / 32));
    if ((err = launch_k(pack_kernel, pack_grid, dim3(kPackThreads), 0, stream, pdl, px)) != cudaSuccess) return err;
    ++n;
    mark();
    // 5. gate/up
    GemmArgs ga{};
    ga.tm0 = tg;
    ga.tm1 = tu;
    ga.b = S.b_gate_up;
    ga.plan = S.plan;
    ga.tile_order = S.tile_order;
    ga.tile_expert = S.tile_expert;
    ga.tile_first = S.tile_first;
    ga.tile_n = S.tile_n;
    ga.tile_pad0 = S.tile_pad0;
    ga.slot_pair = S.slot_pair;
    ga.route_w = S.weights;
    ga.out = S.act;
    ga.K = H;
    ga.rows = I;
    ga.flavour = L.flavour;
    ga.status = status;
    ThinArgs ta{};
    ta.tm0 = tg128;
    ta.tm1 = tu128;
    ta.b = S.b_gate_up;
    ta.plan = S.plan;
    ta.tile_order = S.tile_order;
    ta.tile_expert = S.tile_expert;
    ta.tile_first = S.tile_first;
    ta.tile_n = S.tile_n;
    ta.tile_pad0 = S.tile_pad0;
    ta.slot_pair = S.slot_pair;
    ta.route_w = S.weights;
    ta.out = S.act;
    ta.K = H;
    ta.rows = I;
    ta.flavour = L.flavour;
    ta.status = status;
    // A token's routes are distinct experts, so an expert holds at most `tokens`
    // pairs: with tokens <= kSkinny every tile is skinny and the tensor-core
    // GEMMs would find no unit.
    const bool any_large = tokens > kSkinny;
    if (x_bf16) {
        auto kern = grouped_gemm_kernel<0, 0, 4, 3>;
        if ((err = set_smem(kern, GateUpBf16::total)) != cudaSuccess) return err;
        if (any_large &&
            (err = launch_k(kern, dim3(sms), dim3(kGemmThreads), GateUpBf16::total, stream, pdl, ga)) != cudaSuccess)
            return err;
        auto thin = thin_gemm_kernel<0, 0>;
        if ((err = set_smem(thin, ThinLayout<0, 0>::total)) != cudaSuccess) return err;
        if ((err = launch_k(thin, dim3(sms), dim3(kThinThreads), ThinLayout<0, 0>::total, stream, pdl, ta)) !=
            cudaSuccess)
            return err;
    } else {
        auto kern = grouped_gemm_kernel<0, 1, 3, 2>;
        if ((err = set_smem(kern, GateUpF32::total)) != cudaSuccess) return err;
        if (any_large &&
            (err = launch_k(kern, dim3(sms), dim3(kGemmThreads), GateUpF32::total, stream, pdl, ga)) != cudaSuccess)
            return err;
        auto thin = thin_gemm_kernel<0, 1>;
        if ((err = set_smem(thin, ThinLayout<0, 1>::total)) != cudaSuccess) return err;
        if ((err = launch_k(thin, dim3(sms), dim3(kThinThreads), ThinLayout<0, 1>::total, stream, pdl, ta)) !=
            cudaSuccess)
            return err;
    }
    n += any_large ? 2u : 1u;
    mark();
    // 6. pack activations
    PackArgs pa = px;
    pa.src = S.act;
    pa.src_bf16 = 0;
    pa.by_token = 0;
    pa.cols = I;
    pa.split = 1;
    pa.dst = S.b_down;
    if ((err = launch_k(pack_kernel, pack_grid, dim3(kPackThreads), 0, stream, pdl, pa)) != cudaSuccess) return err;
    ++n;
    mark();
    // 7. down
    GemmArgs da = ga;
    da.tm0 = td;
    da.tm1 = td;
    da.b = S.b_down;
    da.out = S.pair_out;
    da.K = I;
    da.rows = H;
    {
        auto kern = grouped_gemm_kernel<1, 1, 4, 2>;
        if ((err = set_smem(kern, DownLay::total)) != cudaSuccess) return err;
        if (any_large &&
            (err = launch_k(kern, dim3(sms), dim3(kGemmThreads), DownLay::total, stream, pdl, da)) != cudaSuccess)
            return err;
        ThinArgs tda = ta;
        tda.tm0 = td;
        tda.tm1 = td;
        tda.b = S.b_down;
        tda.out = S.pair_out;
        tda.K = I;
        tda.rows = H;
        auto thin = thin_gemm_kernel<1, 1>;
        if ((err = set_smem(thin, ThinLayout<1, 1>::total)) != cudaSuccess) return err;
        if ((err = launch_k(thin, dim3(sms), dim3(kThinThreads), ThinLayout<1, 1>::total, stream, pdl, tda)) !=
            cudaSuccess)
            return err;
    }
    n += any_large ? 2u : 1u;
    mark();
    // 8. combine (and, with an exchange, the sum over the ranks)
    if (ex) {
        const size_t quads = static_cast<size_t>(tokens) * H / 4;
        const uint32_t grid = static_cast<uint32_t>(std::min<size_t>(static_cast<size_t>(sms), (quads + 255) / 256));
        ExchangeArgs xa{};
        xa.pair_out = S.pair_out;
        xa.ids = S.ids;
        xa.e_first = E0;
        xa.e_count = EL;
        xa.tokens = tokens;
        xa.k = k;
        xa.H = H;
        xa.out = out;
        xa.status = status;
        xa.ex = *ex;
        if ((err = launch_k(exchange_combine_kernel, dim3(grid), dim3(256), 0, stream, pdl, xa)) != cudaSuccess)
            return err;
        ++n;
        mark();
    } else {
        const size_t quads = static_cast<size_t>(tokens) * H / 4;
        if ((err = launch_k(combine_kernel, dim3(static_cast<uint32_t>((quads + 255) / 256)), dim3(256), 0, stream,
                            pdl, static_cast<const float*>(S.pair_out), static_cast<const uint32_t*>(S.ids), E0, EL,
                            tokens, k, H, out)) != cudaSuccess)
            return err;
        ++n;
        mark();
    }
    if (ids && ids != S.ids) {
        if ((err = cudaMemcpyAsync(ids, S.ids, size_t(pairs) * 4, cudaMemcpyDeviceToDevice, stream)) != cudaSuccess)
            return err;
    }
    if (weights && weights != S.weights) {
        if ((err = cudaMemcpyAsync(weights, S.weights, size_t(pairs) * 4, cudaMemcpyDeviceToDevice, stream)) !=
            cudaSuccess)
            return err;
    }
    if (launches) *launches = n;
    return cudaGetLastError();
}

}  // namespace pokit
