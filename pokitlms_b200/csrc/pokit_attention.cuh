// pokit_attention.cuh -- decode attention of the decoders (FP16 ring KV,
// GQA, Q/K RMSNorm, rotate-half or partial MRoPE, the Qwen3.5 output gate) and
// the attention block of one layer run by every CTA of a co-resident grid
// (the normed Q/K/V matvec, attention, the output projection into the
// residual) with tagged-word exchanges between its steps.  Included by the
// decoder (its attention kernels) and by the MoE chain kernel (a decoder's
// whole layer loop in one launch).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "pokit_mma.cuh"

namespace pokit {
namespace {

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce_all(T v, T* red, Op op) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    T r = red[0];
    for (int w = 1; w < nw; ++w) r = op(r, red[w]);
    return r;
}

// GQA decode attention of one query head over the ring's last min(pos + 1,
// window) positions, oldest first (KvCache::attend, kv_cache.cpp:185-294):
// scores = q . k * scale, softmax, out = sum_j (e_j / sum e) v_j.
// Scores: each lane takes a whole position (its key row as 16-byte loads, all
// in flight at once), one position per thread and pass.  Output: warp w sums
// positions w, w + warps, ... for four dimensions per lane, sixteen
// positions' loads in flight per round; the warps' partial sums are added in
// warp order.
constexpr uint32_t kAttendThreads = 256;
constexpr uint32_t kAttendMaxDim = 256;

// The CTA first forms its own query and its KV head's new key and value from
// the projected q|k|v (per-head RMSNorm with q_norm / k_norm, rotate-half
// RoPE, qwen3_moe_runner.cpp:141-172, 614-636; key and value rounded to FP16
// as the ring stores them, kv_cache.cpp:20-44); the group's first CTA writes
// them to the ring at slot position % window, and every CTA uses its own copy
// for the newest position (no CTA reads the slot being written).
// The query's and the key's scales in one reduction (red: 2 floats per warp).
__device__ __forceinline__ void head_rms_scale2(float xq, float xk, uint32_t d, float eps, float* red, float& sq,
                                                float& sk) {
    float vq = xq * xq, vk = xk * xk;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        vq += __shfl_xor_sync(0xffffffffu, vq, o);
        vk += __shfl_xor_sync(0xffffffffu, vk, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) {
        red[2 * warp] = vq;
        red[2 * warp + 1] = vk;
    }
    __syncthreads();
    float tq = 0.0f, tk = 0.0f;
    for (uint32_t w = 0; w < (d + 31) / 32; ++w) {
        tq += red[2 * w];
        tk += red[2 * w + 1];
    }
    sq = 1.0f / sqrtf(tq / static_cast<float>(d) + eps);
    sk = 1.0f / sqrtf(tk / static_cast<float>(d) + eps);
}

__device__ __forceinline__ float head_rms_scale(float x, uint32_t d, float eps, float* red) {
    float v = x * x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float total = 0.0f;
    for (uint32_t w = 0; w < (d + 31) / 32; ++w) total += red[w];
    return 1.0f / sqrtf(total / static_cast<float>(d) + eps);
}

// Geometry of one attention layer's projected [q (| gate) per head | k | v].
struct AttendShape {
    uint32_t qh, kvh, d;       // query heads, KV heads, head dimension (<= kAttendMaxDim)
    uint32_t q_stride;         // floats per query head in the projection: d, or 2 d with a gate
    uint32_t gated;            // Qwen3.5: out *= sigmoid(gate), gate = the head's second d floats
    uint32_t rh;               // rotary half: dimensions [0, 2 rh) rotate (rh = d / 2: all)
    uint32_t window;
    float eps, scale;
};

__device__ __forceinline__ float sigmoid_signed(float v) {
    if (v >= 0.0f) return 1.0f / (1.0f + expf(-v));
    const float e = expf(v);
    return e / (1.0f + e);
}

// Shared-memory floats attend_head needs beside the scores: reduction
// slots, query, normed key, new key and value, and one partial output row per
// warp.
__host__ __device__ constexpr uint32_t attend_scratch_floats(uint32_t d, uint32_t warps) {
    return 32u + 4u * d + warps * d;
}

// One query head of the layer: q_in / k_in / v_in are the head's projected
// query, its KV head's new key and value (d floats each, global or shared
// memory), gate_in the head's gate (Qwen3.5) or null, rope_cos / rope_sin the
// rotary half's table rows of this position; writes the head's d outputs to
// out.  sc: window floats and scratch: attend_scratch_floats(d, warps) floats
// of shared memory (16-byte aligned).  Every thread of the CTA (any multiple
// of 32 threads, at least d) calls it.
// kChunk: 16-byte key units a thread loads at once; kVals: positions whose
// values a warp loads at once (smaller in register-tight kernels).
template <uint32_t kChunk = 16, int kVals = 16>
__device__ void attend_head(const float* q_in, const float* k_in, const float* v_in, const float* gate_in,
                            const float* __restrict__ q_norm, const float* __restrict__ k_norm,
                            const float* rope_cos, const float* rope_sin,
                            __half* __restrict__ kc, __half* __restrict__ vc, uint32_t pos, const AttendShape& sh,
                            uint32_t h, float* sc, float* scratch, float* out) {
    const uint32_t d = sh.d, window = sh.window, qh = sh.qh, kvh = sh.kvh, rh = sh.rh;
    const uint32_t t = threadIdx.x, nthreads = blockDim.x;
    const int kW = static_cast<int>(nthreads >> 5);
    float* red = scratch;
    float* qs = scratch + 32;
    float* kn = qs + d;
    float* knew = kn + d;
    float* vnew = knew + d;
    float* part = vnew + d;                               // [warps][d]
    const uint32_t group = qh / kvh, kh = h / group;
    const uint32_t n = pos + 1 < window ? pos + 1 : window, first = pos + 1 - n;
    const int lane = t & 31, warp = t >> 5;
    const uint64_t row_stride = static_cast<uint64_t>(kvh) * d;
    const bool dim = t < d;
    const uint32_t units = d / 8;                         // 16-byte units of a key row
    const float xq = dim ? q_in[t] : 0.0f;
    const float xk = dim ? k_in[t] : 0.0f;
    float sq, sk;
    head_rms_scale2(xq, xk, d, sh.eps, red, sq, sk);
    if (dim) {
        qs[t] = __fmul_rn(__fmul_rn(xq, sq), q_norm[t]);
        kn[t] = __fmul_rn(__fmul_rn(xk, sk), k_norm[t]);
    }
    __syncthreads();
    float rq = 0.0f, rk = 0.0f;
    if (dim) {
        if (t < 2u * rh) {
            const uint32_t j = t < rh ? t : t - rh;
            const float c = rope_cos[j], s = rope_sin[j];
            const float aq = qs[j], bq = qs[j + rh], ak = kn[j], bk = kn[j + rh];
            rq = t < rh ? __fsub_rn(__fmul_rn(aq, c), __fmul_rn(bq, s)) : __fadd_rn(__fmul_rn(bq, c), __fmul_rn(aq, s));
            rk = t < rh ? __fsub_rn(__fmul_rn(ak, c), __fmul_rn(bk, s)) : __fadd_rn(__fmul_rn(bk, c), __fmul_rn(ak, s));
        } else {
            rq = qs[t];
            rk = kn[t];
        }
    }
    __syncthreads();
    if (dim) {
        qs[t] = rq;
        const __half hk = __float2half_rn(rk);
        const __half hv = __float2half_rn(v_in[t]);
        knew[t] = __half2float(hk);
        vnew[t] = __half2float(hv);
        if (h % group == 0) {
            const uint64_t at = static_cast<uint64_t>(pos % window) * row_stride + kh * d + t;
            kc[at] = hk;
            vc[at] = hv;
        }
    }
    __syncthreads();
    // Two threads per position (adjacent lanes), each dotting half the key
    // row; the halves are added at the end.
    const uint32_t half_units = units / 2, hsel = t & 1u;
    for (uint32_t j0 = 0; j0 < n; j0 += nthreads / 2) {
        const uint32_t j = j0 + t / 2;
        float dot = 0.0f;
        if (j + 1 == n) {
            for (uint32_t e = hsel * (d / 2); e < (hsel + 1) * (d / 2); ++e) dot = fmaf(qs[e], knew[e], dot);
        } else if (j < n) {
            const uint4* k = reinterpret_cast<const uint4*>(kc + ((first + j) % window) * row_stride + kh * d) +
                             hsel * half_units;
            const float* qh_ = qs + hsel * (d / 2);
            for (uint32_t c0 = 0; c0 < half_units; c0 += kChunk) {
                uint4 kv[kChunk];
#pragma unroll
                for (uint32_t u = 0; u < kChunk; ++u)
                    if (c0 + u < half_units) kv[u] = __ldg(k + c0 + u);
#pragma unroll
                for (uint32_t u = 0; u < kChunk; ++u) {
                    if (c0 + u < half_units) {
                        const __half2* hp = reinterpret_cast<const __half2*>(&kv[u]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(hp[e]);
                            dot = fmaf(qh_[(c0 + u) * 8 + 2 * e], f.x, dot);
                            dot = fmaf(qh_[(c0 + u) * 8 + 2 * e + 1], f.y, dot);
                        }
                    }
                }
            }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        if (j < n && hsel == 0) sc[j] = dot * sh.scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (uint32_t j = t; j < n; j += nthreads) m = fmaxf(m, sc[j]);
    m = block_reduce_all(m, red, [](float a, float b) { return fmaxf(a, b); });
    float den = 0.0f;
    for (uint32_t j = t; j < n; j += nthreads) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        den += e;
    }
    den = block_reduce_all(den, red, [](float a, float b) { return a + b; });
    // Each position's probability once: the reference's score / sum.
    for (uint32_t j = t; j < n; j += nthreads) sc[j] = sc[j] / den;
    __syncthreads();
    // Output: in segment g (dimensions 128 g .. 128 g + 127) lane covers
    // dimensions 128 g + 4 lane .. + 3; sixteen positions' loads in flight
    // per warp and round.
    for (uint32_t g0 = 0; g0 < d; g0 += 128u) {
        const bool active = g0 + static_cast<uint32_t>(lane) * 4u < d;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t j0 = warp; j0 < n; j0 += kVals * static_cast<uint32_t>(kW)) {
            uint2 vv[kVals];
#pragma unroll
            for (int u = 0; u < kVals; ++u) {
                const uint32_t j = j0 + u * static_cast<uint32_t>(kW);
                if (active && j + 1 < n)
                    vv[u] = __ldg(reinterpret_cast<const uint2*>(vc + ((first + j) % window) * row_stride + kh * d + g0) +
                                  lane);
            }
#pragma unroll
            for (int u = 0; u < kVals; ++u) {
                const uint32_t j = j0 + u * static_cast<uint32_t>(kW);
                if (active && j < n) {
                    const float p = sc[j];
                    float2 a, b;
                    if (j + 1 == n) {
                        a = make_float2(vnew[g0 + lane * 4], vnew[g0 + lane * 4 + 1]);
                        b = make_float2(vnew[g0 + lane * 4 + 2], vnew[g0 + lane * 4 + 3]);
                    } else {
                        a = __half22float2(*reinterpret_cast<const __half2*>(&vv[u].x));
                        b = __half22float2(*reinterpret_cast<const __half2*>(&vv[u].y));
                    }
                    acc.x = fmaf(p, a.x, acc.x);
                    acc.y = fmaf(p, a.y, acc.y);
                    acc.z = fmaf(p, b.x, acc.z);
                    acc.w = fmaf(p, b.y, acc.w);
                }
            }
        }
        if (active) *reinterpret_cast<float4*>(&part[warp * d + g0 + lane * 4]) = acc;
    }
    __syncthreads();
    if (t < d) {
        float o = part[t];
        for (int w = 1; w < kW; ++w) o += part[w * d + t];
        // qwen35_runner.cpp:577-580: the gated output attended * sigmoid(gate).
        if (gate_in) o = __fmul_rn(o, sigmoid_signed(gate_in[t]));
        out[t] = o;
    }
    __syncthreads();
}

struct AttnBlockArgs {
    const uint8_t* wqkv;             // Q4_K [rows][hidden]: q (| gate), k, v
    const uint8_t* wo;               // Q4_K [hidden][q_heads * d]
    const float* attn_norm;
    const float* q_norm;
    const float* k_norm;
    const float* rope_cos;           // [context][rotary half]
    const float* rope_sin;
    __half* kc;                      // this layer's rings
    __half* vc;
    const uint32_t* pos_p;
    AttendShape sh;
    float* hidden;
    unsigned long long* qkv_ll;      // [rows] words
    unsigned long long* att_ll;      // [q_heads * d] words
    uint32_t* status;                // timeout flag
    uint32_t H, rows, qd, layer, layers;
    float eps;
};

constexpr uint32_t kAttnBlockThreads = 256, kAttnBlockWarps = 8;
constexpr uint32_t kAttnStatusTimeout = 1u;
constexpr uint32_t kAttnMaxOutPerWarp = 2;          // output superblocks per warp of 8 warps: q_heads * d <= 4096

struct AttnBlockLayout {
    uint32_t nsb_in, nsb_o, pitch_in, pitch_o, blocks_max;
    uint32_t qtiles, otiles, xrec, arec, qpart, opart, stage, rope, scratch, sc, total;
};

__host__ __device__ inline AttnBlockLayout attn_block_layout(uint32_t H, uint32_t rows, uint32_t qd, uint32_t d,
                                                             uint32_t rh, uint32_t window, uint32_t grid,
                                                             uint32_t warps) {
    AttnBlockLayout c{};
    c.nsb_in = H / 256u;
    c.nsb_o = qd / 256u;
    c.pitch_in = c.nsb_in * 144u + 16u;
    c.pitch_o = c.nsb_o * 144u + 16u;
    c.blocks_max = (rows / 16u + grid - 1u) / grid;
    uint32_t off = 0;
    c.qtiles = off; off += c.blocks_max * 16u * c.pitch_in;
    off = (off + 127u) & ~127u;
    c.otiles = off; off += 16u * c.pitch_o;
    off = (off + 127u) & ~127u;
    c.xrec = off; off += c.nsb_in * kFragWords * 4u;
    c.arec = off; off += c.nsb_o * kFragWords * 4u;
    c.qpart = off; off += c.blocks_max * c.nsb_in * 16u * 4u;
    c.opart = off; off += c.nsb_o * 16u * 4u;
    c.stage = off; off += 5u * d * 4u;                   // query, gate, key, value, output of one head
    c.rope = off; off += 2u * rh * 4u;                   // this position's cos and sin rows
    off = (off + 15u) & ~15u;
    c.scratch = off; off += attend_scratch_floats(d, warps) * 4u;
    c.sc = off; off += window * 4u;
    c.total = (off + 127u) & ~127u;
    return c;
}

// Polls the words src[i] (where use[i]) until every tag is `tag`; false on a
// timeout (or another CTA's).
template <int N>
__device__ __forceinline__ bool await_words(const unsigned long long* const (&src)[N], unsigned long long (&v)[N],
                                            const bool (&use)[N], uint32_t tag, uint32_t* status) {
    long long t0 = 0;
    for (uint32_t polls = 0;; ++polls) {
        bool ready = true;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if (use[i] && static_cast<uint32_t>(v[i] >> 32) != tag) {
                ready = false;
                unsigned long long w;
                asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(src[i]) : "memory");
                v[i] = w;
            }
        }
        if (ready) return true;
        if (polls == 0) t0 = clock64();
        if ((polls & 63u) == 63u) {
            uint32_t st;
            asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(st) : "l"(status) : "memory");
            if (st || clock64() - t0 > 4000000000LL) {
                atomicOr(status, kAttnStatusTimeout);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void put_word(unsigned long long* p, uint32_t tag, float v) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// Shared state of one attention phase in the calling kernel.
struct AttnPhaseCtx {
    uint8_t* smem;                   // 128-byte aligned region of AttnBlockLayout::total bytes
    uint64_t* bars;                  // two initialised mbarriers (Q/K/V tiles, output tiles)
    uint32_t phase;                  // their parity for this use
    uint32_t* abort_sh;              // CTA-wide give-up flag
    float* red;                      // one float per warp
};

// The attention block of layer a.layer for the current position, run by every
// CTA of a co-resident grid (any multiple of 32 threads, at least head_dim):
// see attn_block_kernel.  h comes from hid_ll words tagged hid_tag when
// hid_ll is set (a fused decoder layer loop), else from a.hidden.  Returns,
// in threads tid < 16 of CTAs c < H/16, the new hidden value of row
// 16c + tid (also written to a.hidden); 0 elsewhere.
template <uint32_t kChunk = 16, int kVals = 16>
__device__ float attention_phase(const AttnBlockArgs& a, const AttnPhaseCtx& x, const unsigned long long* hid_ll,
                                 uint32_t hid_tag) {
    const AttendShape& sh = a.sh;
    const uint32_t G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x, d = sh.d;
    const uint32_t nw = blockDim.x >> 5;
    const int lane = tid & 31, warp = tid >> 5, g = lane >> 2;
    const AttnBlockLayout c = attn_block_layout(a.H, a.rows, a.qd, d, sh.rh, sh.window, G, nw);
    const uint32_t nblk = a.rows / 16u, units = a.H / 16u;
    const uint32_t mine = cta < nblk ? (nblk - cta + G - 1u) / G : 0u;
    const bool o_unit = cta < units, head = cta < sh.qh;
    const uint64_t rb_in = c.nsb_in * 144u, rb_o = c.nsb_o * 144u;
    uint8_t* smem = x.smem;
    uint8_t* qtiles = smem + c.qtiles;
    uint8_t* otiles = smem + c.otiles;
    uint32_t* xrec = reinterpret_cast<uint32_t*>(smem + c.xrec);
    uint32_t* arec = reinterpret_cast<uint32_t*>(smem + c.arec);
    float* qpart = reinterpret_cast<float*>(smem + c.qpart);
    float* opart = reinterpret_cast<float*>(smem + c.opart);
    float* stage = reinterpret_cast<float*>(smem + c.stage);
    float* rope = reinterpret_cast<float*>(smem + c.rope);
    float* sc = reinterpret_cast<float*>(smem + c.sc);
    uint64_t* bars = x.bars;
    // ---- entry: copies (after this CTA's generic reads of the region) ----
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (warp == 0 && mine) {
        if (lane == 0) mbar_expect_tx(&bars[0], mine * 16u * static_cast<uint32_t>(rb_in));
        __syncwarp();
        if (lane < 16)
            for (uint32_t i = 0; i < mine; ++i)
                bulk_copy_g2s(qtiles + (i * 16u + lane) * c.pitch_in,
                              a.wqkv + static_cast<uint64_t>((cta + G * i) * 16u + lane) * rb_in,
                              static_cast<uint32_t>(rb_in), &bars[0]);
    } else if (warp == 1 && o_unit) {
        if (lane == 0) mbar_expect_tx(&bars[1], 16u * static_cast<uint32_t>(rb_o));
        __syncwarp();
        if (lane < 16)
            bulk_copy_g2s(otiles + lane * c.pitch_o, a.wo + static_cast<uint64_t>(cta * 16u + lane) * rb_o,
                          static_cast<uint32_t>(rb_o), &bars[1]);
    }
    // ---- qkv: h staged once, x' records ----
    const uint32_t pos = *a.pos_p, tag = pos * a.layers + a.layer + 1u;
    const float resid = o_unit && tid < 16 ? __ldcg(a.hidden + cta * 16u + tid) : 0.0f;
    {
        // The warp's superblocks of h (two at most) into registers, then this
        // position's RoPE rows and the KV head's cached rows towards L2
        // (query-head CTAs) while they are in flight.
        float v[2][8];
        if (hid_ll) {
            const unsigned long long* src[16];
            unsigned long long w[16];
            bool use[16];
#pragma unroll
            for (uint32_t i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t sb = warp + nw * i;
                    use[i * 8 + j] = sb < c.nsb_in;
                    src[i * 8 + j] = hid_ll + (sb < c.nsb_in ? sb : 0u) * 256u + 32u * j + lane;
                    w[i * 8 + j] = 0ull;
                }
            if (!await_words<16>(src, w, use, hid_tag, a.status)) *x.abort_sh = 1u;
#pragma unroll
            for (uint32_t i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] = __uint_as_float(static_cast<uint32_t>(w[i * 8 + j]));
        } else {
#pragma unroll
            for (uint32_t i = 0; i < 2; ++i) {
                const uint32_t sb = warp + nw * i;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    v[i][j] = sb < c.nsb_in ? __ldcg(a.hidden + sb * 256u + 32u * j + lane) : 0.0f;
            }
        }
        if (head) {
            for (uint32_t j = tid; j < sh.rh; j += blockDim.x) {
                rope[j] = a.rope_cos[static_cast<uint64_t>(pos) * sh.rh + j];
                rope[sh.rh + j] = a.rope_sin[static_cast<uint64_t>(pos) * sh.rh + j];
            }
            const uint32_t group = sh.qh / sh.kvh, kh = cta / group;
            if (cta % group == 0) {
                const uint32_t n = pos + 1 < sh.window ? pos + 1 : sh.window, first = pos + 1 - n;
                const uint32_t lines = (d * 2u + 127u) / 128u;
                const uint64_t row_stride = static_cast<uint64_t>(sh.kvh) * d;
                for (uint32_t i = tid; i + lines < n * lines; i += blockDim.x) {
                    const uint64_t at = ((first + i / lines) % sh.window) * row_stride + kh * d + (i % lines) * 64u;
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(a.kc + at));
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(a.vc + at));
                }
            }
        }
        float ss = 0.0f;
#pragma unroll
        for (uint32_t i = 0; i < 2; ++i) {
            const uint32_t sb = warp + nw * i;
            if (sb < c.nsb_in) {
                float* st = reinterpret_cast<float*>(xrec + sb * kFragWords);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    ss = fmaf(v[i][j], v[i][j], ss);
                    st[32 * j + lane] = v[i][j];
                }
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) x.red[warp] = ss;
        __syncthreads();
        float total = 0.0f;
        for (uint32_t i = 0; i < nw; ++i) total += x.red[i];
        const float scale = 1.0f / sqrtf(total / static_cast<float>(a.H) + a.eps);
        for (uint32_t sb = warp; sb < c.nsb_in; sb += nw) {
            float* st = reinterpret_cast<float*>(xrec + sb * kFragWords);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t col = sb * 256u + 32u * j + lane;
                st[32 * j + lane] = __fmul_rn(__fmul_rn(st[32 * j + lane], scale), a.attn_norm[col]);
            }
            __syncwarp();
            q4k_frag_superblock(st, xrec + sb * kFragWords, lane);
        }
    }
    __syncthreads();
    // ---- qkv: multiply, publish ----
    if (mine) {
        if (!mbar_wait(&bars[0], x.phase)) {
            if (lane == 0) { atomicOr(a.status, kAttnStatusTimeout); *x.abort_sh = 1u; }
            mbar_wait(&bars[0], x.phase);
        }
        for (uint32_t task = warp; task < mine * c.nsb_in; task += nw) {
            const uint32_t i = task / c.nsb_in, sb = task % c.nsb_in;
            const uint8_t* t0 = qtiles + (i * 16u) * c.pitch_in + sb * 144u;
            float a0 = 0.0f, a1 = 0.0f;
            q4k_mma_superblock(t0 + g * c.pitch_in, t0 + (g + 8) * c.pitch_in, xrec + sb * kFragWords, a0, a1);
            a0 = quad_sum(a0);
            a1 = quad_sum(a1);
            if ((lane & 3) == 0) {
                qpart[(i * c.nsb_in + sb) * 16u + g] = a0;
                qpart[(i * c.nsb_in + sb) * 16u + g + 8] = a1;
            }
        }
        __syncthreads();
        for (uint32_t t = tid; t < mine * 16u; t += blockDim.x) {
            const uint32_t i = t / 16u, r = t % 16u;
            float v = qpart[(i * c.nsb_in) * 16u + r];
            for (uint32_t sb = 1; sb < c.nsb_in; ++sb) v += qpart[(i * c.nsb_in + sb) * 16u + r];
            put_word(a.qkv_ll + (cta + G * i) * 16u + r, tag, v);
        }
    }
    // ---- attend ----
    if (head) {
        const uint32_t h = cta, kh = h / (sh.qh / sh.kvh);
        const uint32_t kbase = sh.qh * sh.q_stride, vbase = kbase + sh.kvh * d;
        float* qin = stage;
        float* gin = stage + d;
        float* kin = stage + 2 * d;
        float* vin = stage + 3 * d;
        float* aout = stage + 4 * d;
        if (tid < d) {
            const unsigned long long* src[4] = {a.qkv_ll + h * sh.q_stride + tid, a.qkv_ll + h * sh.q_stride + d + tid,
                                                a.qkv_ll + kbase + kh * d + tid, a.qkv_ll + vbase + kh * d + tid};
            unsigned long long v[4] = {0ull, 0ull, 0ull, 0ull};
            const bool use[4] = {true, sh.gated != 0u, true, true};
            if (!await_words<4>(src, v, use, tag, a.status)) *x.abort_sh = 1u;
            qin[tid] = __uint_as_float(static_cast<uint32_t>(v[0]));
            gin[tid] = __uint_as_float(static_cast<uint32_t>(v[1]));
            kin[tid] = __uint_as_float(static_cast<uint32_t>(v[2]));
            vin[tid] = __uint_as_float(static_cast<uint32_t>(v[3]));
        }
        __syncthreads();
        if (!*x.abort_sh) {
            attend_head<kChunk, kVals>(qin, kin, vin, sh.gated ? gin : nullptr, a.q_norm, a.k_norm, rope,
                                       rope + sh.rh, a.kc, a.vc, pos, sh, h, sc,
                                       reinterpret_cast<float*>(smem + c.scratch), aout);
            if (tid < d) put_word(a.att_ll + h * d + tid, tag, aout[tid]);
        }
    }
    // ---- o ----
    float out = 0.0f;
    if (o_unit) {
        // All of the warp's output words in flight at once, then its records.
        const uint32_t per = (c.nsb_o + nw - 1) / nw;
        const uint32_t nmine = static_cast<uint32_t>(warp) < c.nsb_o ? (c.nsb_o - warp + nw - 1) / nw : 0u;
        if (nmine && !*x.abort_sh) {
            const unsigned long long* src[8 * kAttnMaxOutPerWarp];
            unsigned long long v[8 * kAttnMaxOutPerWarp];
            bool use[8 * kAttnMaxOutPerWarp];
#pragma unroll
            for (uint32_t i = 0; i < kAttnMaxOutPerWarp; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t sb = warp + i * nw;
                    use[i * 8 + j] = i < nmine;
                    src[i * 8 + j] = a.att_ll + (i < nmine ? sb : static_cast<uint32_t>(warp)) * 256u + 32u * j + lane;
                    v[i * 8 + j] = 0ull;
                }
            if (!await_words<8 * kAttnMaxOutPerWarp>(src, v, use, tag, a.status)) *x.abort_sh = 1u;
#pragma unroll
            for (uint32_t i = 0; i < kAttnMaxOutPerWarp; ++i) {
                if (i < nmine) {
                    const uint32_t sb = warp + i * nw;
                    float* st = reinterpret_cast<float*>(arec + sb * kFragWords);
#pragma unroll
                    for (int j = 0; j < 8; ++j) st[32 * j + lane] = __uint_as_float(static_cast<uint32_t>(v[i * 8 + j]));
                    __syncwarp();
                    q4k_frag_superblock(st, arec + sb * kFragWords, lane);
                }
            }
        }
        (void)per;
        __syncthreads();
        if (!mbar_wait(&bars[1], x.phase)) {
            if (lane == 0) { atomicOr(a.status, kAttnStatusTimeout); *x.abort_sh = 1u; }
            mbar_wait(&bars[1], x.phase);
        }
        __syncthreads();
        if (!*x.abort_sh) {
            for (uint32_t sb = warp; sb < c.nsb_o; sb += nw) {
                float a0 = 0.0f, a1 = 0.0f;
                const uint8_t* t0 = otiles + sb * 144u;
                q4k_mma_superblock(t0 + g * c.pitch_o, t0 + (g + 8) * c.pitch_o, arec + sb * kFragWords, a0, a1);
                a0 = quad_sum(a0);
                a1 = quad_sum(a1);
                if ((lane & 3) == 0) {
                    opart[sb * 16u + g] = a0;
                    opart[sb * 16u + g + 8] = a1;
                }
            }
            __syncthreads();
            if (tid < 16) {
                float v = opart[tid];
                for (uint32_t sb = 1; sb < c.nsb_o; ++sb) v += opart[sb * 16u + tid];
                out = resid + v;
                a.hidden[cta * 16u + tid] = out;
            }
        }
    }
    __syncthreads();
    return out;
}

}  // namespace
}  // namespace pokit
