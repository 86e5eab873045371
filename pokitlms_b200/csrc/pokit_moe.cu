// pokit_moe.cu -- the MoE FFN block for decode batch 1 on sm_100a.
//
// Three kernels per block (PokitLMs src/qwen3_moe_runner.cpp:643-692 and
// src/qwen35_runner.cpp:691-763):
//
//   route    rms_norm(hidden, ffn_norm) (decode chain only), router gemv split
//            over many CTAs; the last CTA to finish applies softmax, top-k (ties
//            to the lower expert id), renormalisation and the Qwen3.5 weight
//            scale / shared-expert sigmoid gate, on device.
//   gate_up  per routed slot (and the shared expert): g = W_g x, u = W_u x,
//            act = silu(g) * u.  Q4_K rows use the 128-bit "fast chunk" path;
//            other types the generic staged path.  Each CTA first asks the TMA
//            unit to stream its own gate/up rows and its share of the down rows
//            into L2, so HBM stays busy while warps compute.
//   down     y_s = W_d,s act_s for every slot, then out = sum_s w_s * y_s in
//            route order (shared expert last), then the residual add.
//
// No host round trip between the kernels: expert ids never leave the GPU.
#include "pokit_kernels.h"
#include "pokit_quant.cuh"

#include <algorithm>
#include <cfloat>

namespace pokit {
namespace {

constexpr int kRouteThreads = 256;
constexpr int kRouteColsPerWarp = 512;
constexpr int kGateUpThreads = 384;
constexpr int kDownThreads = 256;
constexpr int kDownRowsPerCta = 16;
constexpr int kMaxTopK = 64;

__host__ __device__ inline uint32_t route_splits(uint32_t H) {
    return (H + kRouteColsPerWarp - 1) / kRouteColsPerWarp;
}

struct RouteParams {
    const float* hidden;
    const float* ffn_norm;
    float eps;
    const float* x_in;
    float* x_out;
    const float* router;
    const float* shared_router;
    uint32_t H, E, k, splits, flavour, normalize;
    float ew_scale;
    float* partial;
    float* logits;
    uint32_t* ids;
    float* weights;
    uint32_t* counter;
    uint32_t* status;
};

__device__ __forceinline__ float sigmoid_qwen35(float v) {
    // src/qwen35_runner.cpp:111-115
    if (v >= 0.0f) return 1.0f / (1.0f + expf(-v));
    const float e = expf(v);
    return e / (1.0f + e);
}

// Rank order of both routers: higher logit first, equal logits -> lower id.
__device__ __forceinline__ bool route_before(float va, uint32_t ia, float vb, uint32_t ib) {
    return va > vb || (va == vb && ia < ib);
}

// Softmax top-k over E logits held in shared memory, executed by one warp.
// taken[0..E) must be zero on entry.  Writes k ids and combine weights (plus
// weights[k] = sigmoid(shared_logit) when has_shared); status may be null.
//   flavour 0: route_experts, src/qwen3_moe_runner.cpp:267-305
//   flavour 1: select_experts, src/qwen35_runner.cpp:131-173, weights * ew_scale
__device__ void route_warp(const float* lg, uint8_t* taken, uint32_t* sel, uint32_t E, uint32_t k,
                           uint32_t flavour, uint32_t normalize, float ew_scale, bool has_shared,
                           float shared_logit, uint32_t* ids, float* weights, uint32_t* status) {
    const int lane = threadIdx.x & 31;
    float mx = -FLT_MAX;
    bool bad = false;
    for (uint32_t e = lane; e < E; e += 32) {
        const float v = lg[e];
        bad |= !isfinite(v);
        mx = fmaxf(mx, v);
    }
    bad = __any_sync(0xffffffffu, bad);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (bad) {
        // The reference throws ("expert router produced non-finite logits").
        // Record it and emit in-bounds, zero-weight routes so later kernels stay safe.
        if (lane == 0 && status) atomicOr(status, kStatusNonFiniteLogits);
        for (uint32_t r = lane; r < k; r += 32) { ids[r] = r; weights[r] = 0.0f; }
        if (lane == 0 && has_shared) weights[k] = 0.0f;
        return;
    }
    // Softmax denominators: FP64 for Qwen3-MoE (qwen3_moe_runner.cpp:277-278),
    // FP32 for Qwen3.5 (qwen35_runner.cpp:139-144).
    double den_d = 0.0;
    float den_f = 0.0f;
    for (uint32_t e = lane; e < E; e += 32) {
        if (flavour == 0) den_d += exp(static_cast<double>(lg[e] - mx));
        else den_f += expf(lg[e] - mx);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        den_d += __shfl_xor_sync(0xffffffffu, den_d, o);
        den_f += __shfl_xor_sync(0xffffffffu, den_f, o);
    }
    // Top-k by repeated arg-max in the (logit desc, id asc) order: the same
    // set and order as the reference's insertion into a sorted vector.
    for (uint32_t r = 0; r < k; ++r) {
        float bv = -FLT_MAX;
        uint32_t bi = 0xffffffffu;
        for (uint32_t e = lane; e < E; e += 32) {
            if (taken[e]) continue;
            const float v = lg[e];
            if (bi == 0xffffffffu || route_before(v, e, bv, bi)) { bv = v; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0xffffffffu && (bi == 0xffffffffu || route_before(ov, oi, bv, bi))) {
                bv = ov; bi = oi;
            }
        }
        if (lane == 0) { sel[r] = bi; taken[bi] = 1; }
        __syncwarp();
    }
    if (lane == 0) {
        float probs[kMaxTopK];
        float sum = 0.0f;
        bool invalid = flavour == 1 && (!isfinite(den_f) || den_f <= 0.0f);
        for (uint32_t r = 0; r < k; ++r) {
            const float v = lg[sel[r]];
            probs[r] = flavour == 0 ? static_cast<float>(exp(static_cast<double>(v - mx)) / den_d)
                                    : expf(v - mx) / den_f;
            sum += probs[r];
        }
        if (normalize) {
            if (flavour == 1 && (!isfinite(sum) || sum <= 0.0f)) invalid = true;
            for (uint32_t r = 0; r < k; ++r) probs[r] /= sum;
        }
        if (invalid && status) atomicOr(status, kStatusBadSoftmax);
        for (uint32_t r = 0; r < k; ++r) {
            ids[r] = sel[r];
            weights[r] = invalid ? 0.0f : (flavour == 0 ? probs[r] : probs[r] * ew_scale);
        }
        if (has_shared) weights[k] = sigmoid_qwen35(shared_logit);
    }
    __syncwarp();
}

__global__ void __launch_bounds__(kRouteThreads)
moe_route_kernel(RouteParams p) {
    extern __shared__ float xs[];   // max(H, E) floats
    __shared__ float red[kRouteThreads / 32];
    __shared__ uint32_t last_flag;
    __shared__ uint8_t taken[1024];
    __shared__ uint32_t sel[kMaxTopK];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t H = p.H;

    // 1. The block input: rms_norm(hidden) * ffn_norm, or the caller's x.
    if (p.hidden) {
        float ss = 0.0f;
        for (uint32_t i = tid; i < H; i += kRouteThreads) {
            const float v = p.hidden[i];
            xs[i] = v;
            ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int w = 0; w < kRouteThreads / 32; ++w) total += red[w];
        // src/rms_norm.cpp:20-26: scale = 1 / sqrt(mean + eps); y = x * scale * w
        const float scale = 1.0f / sqrtf(total / static_cast<float>(H) + p.eps);
        for (uint32_t i = tid; i < H; i += kRouteThreads) xs[i] = xs[i] * scale * p.ffn_norm[i];
    } else {
        for (uint32_t i = tid; i < H; i += kRouteThreads) xs[i] = p.x_in[i];
    }
    __syncthreads();
    if (blockIdx.x == 0 && p.x_out)
        for (uint32_t i = tid; i < H; i += kRouteThreads) p.x_out[i] = xs[i];

    // 2. Partial router dots: task = (row, split); row E is the shared-expert gate.
    const uint32_t rows = p.E + (p.shared_router ? 1u : 0u);
    const uint32_t tasks = rows * p.splits;
    for (uint32_t t = blockIdx.x * (kRouteThreads / 32) + warp; t < tasks;
         t += gridDim.x * (kRouteThreads / 32)) {
        const uint32_t row = t / p.splits, sp = t % p.splits;
        const float* w = row < p.E ? p.router + static_cast<uint64_t>(row) * H : p.shared_router;
        const uint32_t c0 = sp * kRouteColsPerWarp;
        const uint32_t c1 = min(c0 + kRouteColsPerWarp, H);
        float acc = 0.0f;
        if ((H & 3u) == 0) {
#pragma unroll 4
            for (uint32_t i = c0 + lane * 4u; i < c1; i += 128u) {
                const uint4 v = ldg_stream128(w + i);
                acc = fmaf(__uint_as_float(v.x), xs[i], acc);
                acc = fmaf(__uint_as_float(v.y), xs[i + 1], acc);
                acc = fmaf(__uint_as_float(v.z), xs[i + 2], acc);
                acc = fmaf(__uint_as_float(v.w), xs[i + 3], acc);
            }
        } else {
            for (uint32_t i = c0 + lane; i < c1; i += 32u) acc = fmaf(__ldg(w + i), xs[i], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) p.partial[t] = acc;
    }

    // 3. Last CTA to arrive performs the routing.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomic_add_acq_rel_gpu(p.counter, 1u);
        last_flag = (old == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    float* lg = xs;   // reuse: E logits
    __syncthreads();
    for (uint32_t e = tid; e < p.E; e += kRouteThreads) {
        float s = __ldcg(p.partial + e * p.splits);
        for (uint32_t sp = 1; sp < p.splits; ++sp) s += __ldcg(p.partial + e * p.splits + sp);
        lg[e] = s;
        p.logits[e] = s;
        taken[e] = 0;
    }
    __syncthreads();
    if (warp != 0) return;

    float shared_logit = 0.0f;
    if (p.shared_router) {
        shared_logit = __ldcg(p.partial + p.E * p.splits);
        for (uint32_t sp = 1; sp < p.splits; ++sp)
            shared_logit += __ldcg(p.partial + p.E * p.splits + sp);
    }
    route_warp(lg, taken, sel, p.E, p.k, p.flavour, p.normalize, p.ew_scale,
               p.shared_router != nullptr, shared_logit, p.ids, p.weights, p.status);
    if (lane == 0) *p.counter = 0u;
}

// Routing of a standalone logits vector (pokit_cuda_route_experts).
__global__ void __launch_bounds__(32)
route_logits_kernel(const float* __restrict__ logits, uint32_t E, uint32_t k, uint32_t flavour,
                    uint32_t normalize, float ew_scale, uint32_t* ids, float* weights,
                    uint32_t* status) {
    __shared__ float lg[1024];
    __shared__ uint8_t taken[1024];
    __shared__ uint32_t sel[kMaxTopK];
    for (uint32_t e = threadIdx.x; e < E; e += 32) { lg[e] = logits[e]; taken[e] = 0; }
    __syncwarp();
    route_warp(lg, taken, sel, E, k, flavour, normalize, ew_scale, false, 0.0f, ids, weights,
               status);
}

// ---------------------------------------------------------------------------
struct SlotMats {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    uint32_t gate_type, up_type, down_type, rows;   // rows = inter of this slot
};

struct BlockParams {
    MoeLayerDev L;
    const float* x;
    const uint32_t* ids;
    const float* weights;
    float* act;
    uint32_t act_stride;
    float* hidden;
    float* moe_out;
    const float* next_router;
};

__device__ __forceinline__ SlotMats slot_mats(const BlockParams& p, uint32_t s) {
    SlotMats m;
    if (s < p.L.top_k) {
        const uint64_t id = p.ids[s];
        m.gate = p.L.gate + id * p.L.gate_slice;
        m.up = p.L.up + id * p.L.up_slice;
        m.down = p.L.down + id * p.L.down_slice;
        m.gate_type = p.L.gate_type; m.up_type = p.L.up_type; m.down_type = p.L.down_type;
        m.rows = p.L.inter;
    } else {
        m.gate = p.L.shared_gate; m.up = p.L.shared_up; m.down = p.L.shared_down;
        m.gate_type = p.L.shared_gate_type; m.up_type = p.L.shared_up_type;
        m.down_type = p.L.shared_down_type;
        m.rows = p.L.shared_inter;
    }
    return m;
}

__device__ __forceinline__ float silu_mul(float g, float u, uint32_t flavour) {
    // Qwen3-MoE: g / (1 + exp(-g)) * u (qwen3_moe_runner.cpp:683);
    // Qwen3.5:   g * sigmoid(g) * u   (qwen35_runner.cpp:123, 733-735).
    return flavour == 0 ? (g / (1.0f + expf(-g))) * u : (g * sigmoid_qwen35(g)) * u;
}

__device__ float generic_row_dot(uint32_t type, const uint8_t* row_g, uint32_t cols,
                                 const float* xs, uint8_t* stage, int lane) {
    const uint32_t rb = static_cast<uint32_t>(row_bytes(type, cols));
    warp_stage_row(row_g, rb, stage, lane);
    __syncwarp();
    float acc = 0.0f;
    const int groups = static_cast<int>(cols >> 5);
    for (int g = lane; g < groups; g += 32) {
        switch (type) {
            case kQ4_K: acc += group_dot<kQ4_K>(stage, g, xs); break;
            case kQ5_K: acc += group_dot<kQ5_K>(stage, g, xs); break;
            case kQ6_K: acc += group_dot<kQ6_K>(stage, g, xs); break;
            case kQ8_0: acc += group_dot<kQ8_0>(stage, g, xs); break;
            default: acc += group_dot<kF32>(stage, g, xs); break;
        }
    }
    acc = warp_sum(acc);
    __syncwarp();
    return acc;
}

__device__ __forceinline__ bool q4k_fast(uint32_t t1, uint32_t t2) { return t1 == kQ4_K && t2 == kQ4_K; }

// gate/up task space: [fast quads of all fast slots][generic rows of the rest].
__global__ void __launch_bounds__(kGateUpThreads)
moe_gate_up_kernel(BlockParams p, uint32_t stage_bytes) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t H = p.L.hidden;
    const int nsb = static_cast<int>(H >> 8);
    float* xp = sm;                                   // nsb*4*68
    float* gsum = xp + nsb * 4 * kQ4kChunkStride;     // H/32
    float* xs = gsum + (H >> 5);                      // H
    uint8_t* stage = reinterpret_cast<uint8_t*>(xs + H);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = kGateUpThreads / 32;
    const uint32_t slots = p.L.top_k + (p.L.shared_inter ? 1u : 0u);

    // Task bookkeeping (uniform across the grid).
    uint32_t n_fast = 0, n_gen = 0;
    for (uint32_t s = 0; s < slots; ++s) {
        const bool routed = s < p.L.top_k;
        const uint32_t gt = routed ? p.L.gate_type : p.L.shared_gate_type;
        const uint32_t ut = routed ? p.L.up_type : p.L.shared_up_type;
        const uint32_t rows = routed ? p.L.inter : p.L.shared_inter;
        if (q4k_fast(gt, ut) && (rows & 3u) == 0) n_fast += rows >> 2; else n_gen += rows;
    }
    const uint32_t total = n_fast + n_gen;
    const uint32_t t0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * total / gridDim.x);
    const uint32_t t1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * total / gridDim.x);

    // Map a task index to (slot, first row, fast?).
    auto locate = [&](uint32_t t, uint32_t& slot, uint32_t& row, bool& fast) {
        uint32_t acc_fast = 0, acc_gen = n_fast;
        for (uint32_t s = 0; s < slots; ++s) {
            const bool routed = s < p.L.top_k;
            const uint32_t gt = routed ? p.L.gate_type : p.L.shared_gate_type;
            const uint32_t ut = routed ? p.L.up_type : p.L.shared_up_type;
            const uint32_t rows = routed ? p.L.inter : p.L.shared_inter;
            if (q4k_fast(gt, ut) && (rows & 3u) == 0) {
                const uint32_t n = rows >> 2;
                if (t < n_fast && t < acc_fast + n) { slot = s; row = (t - acc_fast) * 4u; fast = true; return; }
                acc_fast += n;
            } else {
                if (t >= n_fast && t < acc_gen + rows) { slot = s; row = t - acc_gen; fast = false; return; }
                acc_gen += rows;
            }
        }
        slot = 0; row = 0; fast = false;
    };

    // L2 prefetch: this CTA's gate/up rows, and its share of every slot's down rows.
    if (warp == 0 && t1 > t0) {
        for (uint32_t t = t0 + lane; t < t1; t += 32) {
            uint32_t s, row; bool fast;
            locate(t, s, row, fast);
            const SlotMats m = slot_mats(p, s);
            const uint32_t nrows = fast ? 4u : 1u;
            const uint64_t rg = row_bytes(m.gate_type, H), ru = row_bytes(m.up_type, H);
            prefetch_l2_range(m.gate + row * rg, nrows * rg);
            prefetch_l2_range(m.up + row * ru, nrows * ru);
        }
        for (uint32_t s = lane; s < slots; s += 32) {
            const SlotMats m = slot_mats(p, s);
            const uint64_t rd = row_bytes(m.down_type, m.rows);
            const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * H / gridDim.x;
            const uint64_t r1 = static_cast<uint64_t>(blockIdx.x + 1) * H / gridDim.x;
            if (r1 > r0) prefetch_l2_range(m.down + r0 * rd, (r1 - r0) * rd);
        }
    }

    q4k_prepare_x(p.x, static_cast<int>(H), xp, gsum);
    for (uint32_t i = tid; i < H; i += kGateUpThreads) xs[i] = p.x[i];
    __syncthreads();

    const int r = (lane >> 2) & 3, mat = lane >> 4, c = lane & 3;
    for (uint32_t t = t0 + warp; t < t1; t += nwarps) {
        uint32_t s, row0; bool fast;
        locate(t, s, row0, fast);
        const SlotMats m = slot_mats(p, s);
        const uint32_t flavour = p.L.flavour;
        if (fast) {
            const uint64_t rb = static_cast<uint64_t>(nsb) * 144u;
            const uint8_t* rp = (mat ? m.up : m.gate) + (row0 + r) * rb;
            float acc = 0.0f;
#pragma unroll 2
            for (int sb = 0; sb < nsb; ++sb) {
                const uint8_t* blk = rp + sb * 144;
                const uint4 hdr = ldg_stream128(blk);
                const uint4 q0 = ldg_stream128(blk + 16 + 32 * c);
                const uint4 q1 = ldg_stream128(blk + 32 + 32 * c);
                acc += q4k_chunk_dot(hdr, q0, q1, c, xp + (sb * 4 + c) * kQ4kChunkStride,
                                     gsum[sb * 8 + 2 * c], gsum[sb * 8 + 2 * c + 1]);
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            const float u = __shfl_down_sync(0xffffffffu, acc, 16);
            if (mat == 0 && c == 0)
                p.act[s * p.act_stride + row0 + r] = silu_mul(acc, u, s < p.L.top_k ? flavour : 1u);
        } else {
            uint8_t* my_stage = stage + warp * stage_bytes;
            const float g = generic_row_dot(m.gate_type, m.gate + row0 * row_bytes(m.gate_type, H),
                                            H, xs, my_stage, lane);
            const float u = generic_row_dot(m.up_type, m.up + row0 * row_bytes(m.up_type, H),
                                            H, xs, my_stage, lane);
            if (lane == 0)
                p.act[s * p.act_stride + row0] = silu_mul(g, u, s < p.L.top_k ? flavour : 1u);
        }
    }
}

// down + combine: CTA = 16 output rows; task = (row octet, slot).
__global__ void __launch_bounds__(kDownThreads)
moe_down_kernel(BlockParams p, uint32_t max_inter, uint32_t stage_bytes) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t H = p.L.hidden;
    const uint32_t slots = p.L.top_k + (p.L.shared_inter ? 1u : 0u);
    const int msb = static_cast<int>((max_inter + 255) >> 8);
    const uint32_t prep_len = msb * 4 * kQ4kChunkStride;
    const uint32_t gs_len = max_inter >> 5;
    float* xp_all = sm;                               // slots * prep_len
    float* gs_all = xp_all + slots * prep_len;        // slots * gs_len
    float* xs_all = gs_all + slots * gs_len;          // slots * max_inter
    float* ybuf = xs_all + slots * max_inter;         // slots * 16
    uint8_t* stage = reinterpret_cast<uint8_t*>(ybuf + slots * kDownRowsPerCta);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = kDownThreads / 32;
    const uint32_t j0 = blockIdx.x * kDownRowsPerCta;

    if (p.next_router && tid == 0) {
        const uint64_t bytes = static_cast<uint64_t>(p.L.experts) * H * 4u;
        const uint64_t a = (bytes * blockIdx.x / gridDim.x) & ~uint64_t(15);
        const uint64_t b = blockIdx.x + 1 == gridDim.x ? bytes
                                                       : (bytes * (blockIdx.x + 1) / gridDim.x) & ~uint64_t(15);
        if (b > a) prefetch_l2_range(reinterpret_cast<const uint8_t*>(p.next_router) + a, b - a);
    }

    for (uint32_t s = 0; s < slots; ++s) {
        const SlotMats m = slot_mats(p, s);
        const float* a = p.act + s * p.act_stride;
        if (m.down_type == kQ4_K)
            q4k_prepare_x(a, static_cast<int>(m.rows), xp_all + s * prep_len, gs_all + s * gs_len);
        else
            for (uint32_t i = tid; i < m.rows; i += kDownThreads) xs_all[s * max_inter + i] = a[i];
    }
    __syncthreads();

    const int r = lane >> 2, c = lane & 3;
    const uint32_t tasks = 2u * slots;
    for (uint32_t t = warp; t < tasks; t += nwarps) {
        const uint32_t o = t & 1u, s = t >> 1;
        const SlotMats m = slot_mats(p, s);
        const uint32_t I = m.rows;
        if (m.down_type == kQ4_K) {
            const int nsb = static_cast<int>(I >> 8);
            const uint64_t rb = static_cast<uint64_t>(nsb) * 144u;
            const uint32_t j = j0 + o * 8u + r;
            float acc = 0.0f;
            if (j < H) {
                const uint8_t* rp = m.down + j * rb;
                const float* xp = xp_all + s * prep_len;
                const float* gs = gs_all + s * gs_len;
#pragma unroll 2
                for (int sb = 0; sb < nsb; ++sb) {
                    const uint8_t* blk = rp + sb * 144;
                    const uint4 hdr = ldg_stream128(blk);
                    const uint4 q0 = ldg_stream128(blk + 16 + 32 * c);
                    const uint4 q1 = ldg_stream128(blk + 32 + 32 * c);
                    acc += q4k_chunk_dot(hdr, q0, q1, c, xp + (sb * 4 + c) * kQ4kChunkStride,
                                         gs[sb * 8 + 2 * c], gs[sb * 8 + 2 * c + 1]);
                }
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (c == 0) ybuf[s * kDownRowsPerCta + o * 8 + r] = acc;
        } else {
            uint8_t* my_stage = stage + warp * stage_bytes;
            const uint64_t rb = row_bytes(m.down_type, I);
            for (uint32_t rr = 0; rr < 8; ++rr) {
                const uint32_t j = j0 + o * 8u + rr;
                if (j >= H) break;
                const float y = generic_row_dot(m.down_type, m.down + j * rb, I,
                                                xs_all + s * max_inter, my_stage, lane);
                if (lane == 0) ybuf[s * kDownRowsPerCta + o * 8 + rr] = y;
            }
        }
    }
    __syncthreads();
    if (tid < kDownRowsPerCta) {
        const uint32_t j = j0 + tid;
        if (j < H) {
            float acc = 0.0f;
            for (uint32_t s = 0; s < p.L.top_k; ++s) acc += p.weights[s] * ybuf[s * kDownRowsPerCta + tid];
            if (p.L.shared_inter) acc = acc + p.weights[p.L.top_k] * ybuf[p.L.top_k * kDownRowsPerCta + tid];
            if (p.moe_out) p.moe_out[j] = acc;
            else p.hidden[j] += acc;
        }
    }
}

template <typename K>
cudaError_t ensure_smem(K kernel, size_t bytes) {
    if (bytes <= 48u * 1024u) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(bytes));
}

uint32_t max_slot_inter(const MoeLayerDev& L) {
    return L.shared_inter > L.inter ? L.shared_inter : L.inter;
}

uint64_t align256(uint64_t v) { return (v + 255u) & ~uint64_t(255); }

bool q4k_fast_host(uint32_t a, uint32_t b) { return a == kQ4_K && b == kQ4_K; }

}  // namespace

uint64_t moe_scratch_bytes(const MoeLayerDev& L) {
    const uint64_t slots = L.top_k + 1u;
    uint64_t b = 0;
    b += align256(L.hidden * 4u);                                         // x
    b += align256((L.experts + 1u) * route_splits(L.hidden) * 4u);        // partial
    b += align256(L.experts * 4u);                                        // logits
    b += align256(L.top_k * 4u);                                          // ids
    b += align256(slots * 4u);                                            // weights
    b += align256(slots * max_slot_inter(L) * 4u);                        // act
    b += align256(4u);                                                    // counter
    b += align256(4u);                                                    // status
    return b;
}

MoeScratch moe_scratch_carve(const MoeLayerDev& L, void* base) {
    const uint64_t slots = L.top_k + 1u;
    uint8_t* p = static_cast<uint8_t*>(base);
    MoeScratch s;
    s.x = reinterpret_cast<float*>(p); p += align256(L.hidden * 4u);
    s.partial = reinterpret_cast<float*>(p); p += align256((L.experts + 1u) * route_splits(L.hidden) * 4u);
    s.logits = reinterpret_cast<float*>(p); p += align256(L.experts * 4u);
    s.ids = reinterpret_cast<uint32_t*>(p); p += align256(L.top_k * 4u);
    s.weights = reinterpret_cast<float*>(p); p += align256(slots * 4u);
    s.act = reinterpret_cast<float*>(p); p += align256(slots * max_slot_inter(L) * 4u);
    s.counter = reinterpret_cast<uint32_t*>(p); p += align256(4u);
    s.status = reinterpret_cast<uint32_t*>(p);
    return s;
}

cudaError_t launch_route_experts(const float* logits, uint32_t E, uint32_t k, uint32_t flavour,
                                 uint32_t normalize, float ew_scale, uint32_t* ids, float* weights,
                                 uint32_t* status, cudaStream_t stream) {
    if (k == 0 || k > E || k > kMaxTopK || E > 1024) return cudaErrorInvalidValue;
    route_logits_kernel<<<1, 32, 0, stream>>>(logits, E, k, flavour, normalize, ew_scale, ids,
                                              weights, status);
    return cudaGetLastError();
}

cudaError_t launch_moe_block(const MoeLayerDev& L, const MoeScratch& S, const float* x_in,
                             float* hidden, float* moe_out, const float* next_router,
                             cudaStream_t stream) {
    if (L.top_k == 0 || L.top_k > L.experts || L.top_k > kMaxTopK || L.experts > 1024 ||
        L.hidden == 0 || (L.hidden & 255u) || L.inter == 0 || (L.inter & 255u) ||
        (L.shared_inter & 255u))
        return cudaErrorInvalidValue;
    if (!hidden && !x_in) return cudaErrorInvalidValue;
    if (!hidden && !moe_out) return cudaErrorInvalidValue;
    const int sms = device_sm_count();
    cudaError_t e;

    // 1. route
    RouteParams rp{};
    rp.hidden = hidden;
    rp.ffn_norm = L.ffn_norm;
    rp.eps = L.rms_eps;
    rp.x_in = x_in;
    rp.x_out = S.x;
    rp.router = L.router;
    rp.shared_router = L.shared_inter ? L.shared_router : nullptr;
    rp.H = L.hidden;
    rp.E = L.experts;
    rp.k = L.top_k;
    rp.splits = route_splits(L.hidden);
    rp.flavour = L.flavour;
    rp.normalize = L.normalize;
    rp.ew_scale = L.expert_weights_scale;
    rp.partial = S.partial;
    rp.logits = S.logits;
    rp.ids = S.ids;
    rp.weights = S.weights;
    rp.counter = S.counter;
    rp.status = S.status;
    if (hidden && !L.ffn_norm) return cudaErrorInvalidValue;
    {
        const uint32_t tasks = (L.experts + 1u) * rp.splits;
        uint32_t grid = (tasks + 7u) / 8u;
        if (grid > static_cast<uint32_t>(sms)) grid = static_cast<uint32_t>(sms);
        const size_t smem = static_cast<size_t>(L.hidden > L.experts ? L.hidden : L.experts) * 4u;
        e = ensure_smem(moe_route_kernel, smem);
        if (e != cudaSuccess) return e;
        moe_route_kernel<<<grid, kRouteThreads, smem, stream>>>(rp);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }

    BlockParams bp{};
    bp.L = L;
    bp.x = S.x;
    bp.ids = S.ids;
    bp.weights = S.weights;
    bp.act = S.act;
    bp.act_stride = max_slot_inter(L);
    bp.hidden = hidden;
    bp.moe_out = moe_out;
    bp.next_router = next_router;

    // Largest staged row (generic path) across every matrix of the block.
    auto rb = [](uint32_t t, uint32_t cols) { return static_cast<uint32_t>((row_bytes(t, cols) + 15u) & ~uint64_t(15)); };
    uint32_t stage_gu = 16u;
    if (!q4k_fast_host(L.gate_type, L.up_type))
        stage_gu = std::max(stage_gu, std::max(rb(L.gate_type, L.hidden), rb(L.up_type, L.hidden)));
    if (L.shared_inter && !q4k_fast_host(L.shared_gate_type, L.shared_up_type))
        stage_gu = std::max(stage_gu, std::max(rb(L.shared_gate_type, L.hidden), rb(L.shared_up_type, L.hidden)));
    uint32_t stage_dn = 16u;
    if (L.down_type != kQ4_K) stage_dn = std::max(stage_dn, rb(L.down_type, L.inter));
    if (L.shared_inter && L.shared_down_type != kQ4_K)
        stage_dn = std::max(stage_dn, rb(L.shared_down_type, L.shared_inter));

    // 2. gate/up
    {
        const uint32_t H = L.hidden;
        const size_t smem = (static_cast<size_t>(H >> 8) * 4u * kQ4kChunkStride + (H >> 5) + H) * 4u +
                            static_cast<size_t>(stage_gu) * (kGateUpThreads / 32);
        if (smem > 220u * 1024u) return cudaErrorInvalidValue;
        e = ensure_smem(moe_gate_up_kernel, smem);
        if (e != cudaSuccess) return e;
        moe_gate_up_kernel<<<sms, kGateUpThreads, smem, stream>>>(bp, stage_gu);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    // 3. down + combine (+ residual)
    {
        const uint32_t slots = L.top_k + (L.shared_inter ? 1u : 0u);
        const uint32_t mi = max_slot_inter(L);
        const size_t prep_len = static_cast<size_t>((mi + 255u) >> 8) * 4u * kQ4kChunkStride;
        const size_t smem = (slots * (prep_len + (mi >> 5) + mi + kDownRowsPerCta)) * 4u +
                            static_cast<size_t>(stage_dn) * (kDownThreads / 32);
        if (smem > 220u * 1024u) return cudaErrorInvalidValue;
        e = ensure_smem(moe_down_kernel, smem);
        if (e != cudaSuccess) return e;
        const uint32_t grid = (L.hidden + kDownRowsPerCta - 1) / kDownRowsPerCta;
        moe_down_kernel<<<grid, kDownThreads, smem, stream>>>(bp, mi, stage_dn);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace pokit
