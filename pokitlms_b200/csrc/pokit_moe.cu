// pokit_moe.cu -- the MoE FFN block for decode batch 1 on sm_100a.
//
// One block (PokitLMs src/qwen3_moe_runner.cpp:643-692, src/qwen35_runner.cpp:691-763)
// is five phases:
//
//   R0  x = rms_norm(hidden, ffn_norm) (decode chain) or the caller's x
//   R1  router partial dots (F32 [E, H] . x), split over every CTA
//   R2  softmax + top-k (ties to the lower expert id) + renormalisation (+ the
//       Qwen3.5 weight scale and shared-expert sigmoid gate); every CTA
//       computes it redundantly from the partials, so no CTA waits on another
//   G   per routed slot (and the shared expert): act = silu(W_g x) * (W_u x)
//   D   y_s = W_d,s act_s per slot, out = sum_s w_s y_s in route order (shared
//       expert last), then the residual add
//
// Two drivers share these phases:
//   * launch_moe_block: three kernels (R0+R1 | R2+G | D) for one block;
//   * launch_moe_decode: one persistent cooperative kernel that runs a range of
//     layers for one token with three bounded-spin grid barriers per layer.
//     Each phase issues its weight loads before the barrier that precedes its
//     compute, so barrier latency overlaps memory latency, and the TMA unit
//     streams the next phase's bytes (down rows, next router) into L2.
//
// Data written by other CTAs of the same kernel (h, partials, act) is read with
// ld.global.cg so a stale L1 line can never be observed.  Weights are read-only
// for the kernel's lifetime and use the non-coherent path.
#include "pokit_kernels.h"
#include "pokit_mma.cuh"
#include "pokit_quant.cuh"

#include <algorithm>
#include <cfloat>

namespace pokit {
namespace {

constexpr int kThreads = 384;
constexpr int kWarps = kThreads / 32;
constexpr int kRouteColsPerWarp = 512;
constexpr int kMaxTopK = 64;
constexpr int kMaxExperts = 1024;
constexpr int kSbChunk = 8;                 // gate/up superblocks whose loads go out together
constexpr int kSbChunkDown = 4;             // down superblocks whose loads go out together
constexpr long long kBarrierTimeoutCycles = 4000000000LL;   // ~2 s at 2 GHz

__host__ __device__ inline uint32_t route_splits(uint32_t H) {
    return (H + kRouteColsPerWarp - 1) / kRouteColsPerWarp;
}
__host__ __device__ inline uint32_t slots_of(const MoeLayerDev& L) {
    return L.top_k + (L.shared_inter ? 1u : 0u);
}
__host__ __device__ inline uint32_t max_inter_of(const MoeLayerDev& L) {
    return L.shared_inter > L.inter ? L.shared_inter : L.inter;
}
__host__ __device__ inline uint32_t prep_len_of(uint32_t inter) {
    return ((inter + 255u) >> 8) * 4u * kQ4kChunkStride;
}
__host__ __device__ inline bool fast_pair(uint32_t a, uint32_t b) { return a == kQ4_K && b == kQ4_K; }

// Rows of the D phase owned by CTA b of n (contiguous, balanced).
__host__ __device__ inline void down_rows(uint32_t H, uint32_t b, uint32_t n, uint32_t& r0,
                                          uint32_t& r1) {
    r0 = static_cast<uint32_t>(static_cast<uint64_t>(b) * H / n);
    r1 = static_cast<uint32_t>(static_cast<uint64_t>(b + 1) * H / n);
}
__host__ __device__ inline uint32_t max_down_rows(uint32_t H, uint32_t n) {
    return (H + n - 1) / n;
}

// Dynamic shared memory layout (byte offsets), identical on host and device.
struct SmemLayout {
    uint32_t xs, xp, gsum, lg, red, sel_id, sel_w, act_plain, act_prep, act_gsum, ybuf, stage;
    uint32_t total, rows_cap, stage_bytes;
};

__host__ __device__ inline uint32_t al16(uint32_t v) { return (v + 15u) & ~15u; }
__host__ __device__ inline uint32_t umax(uint32_t a, uint32_t b) { return a > b ? a : b; }

__host__ __device__ inline uint32_t stage_bytes_of(const MoeLayerDev& L) {
    uint32_t s = 16u;
    if (!fast_pair(L.gate_type, L.up_type))
        s = umax(s, umax(al16(static_cast<uint32_t>(row_bytes(L.gate_type, L.hidden))),
                         al16(static_cast<uint32_t>(row_bytes(L.up_type, L.hidden)))));
    if (L.down_type != kQ4_K) s = umax(s, al16(static_cast<uint32_t>(row_bytes(L.down_type, L.inter))));
    if (L.shared_inter) {
        if (!fast_pair(L.shared_gate_type, L.shared_up_type))
            s = umax(s, umax(al16(static_cast<uint32_t>(row_bytes(L.shared_gate_type, L.hidden))),
                             al16(static_cast<uint32_t>(row_bytes(L.shared_up_type, L.hidden)))));
        if (L.shared_down_type != kQ4_K)
            s = umax(s, al16(static_cast<uint32_t>(row_bytes(L.shared_down_type, L.shared_inter))));
    }
    return s;
}

__host__ __device__ inline SmemLayout make_layout(const MoeLayerDev& L, uint32_t down_ctas) {
    SmemLayout m{};
    const uint32_t H = L.hidden, slots = slots_of(L), mi = max_inter_of(L);
    uint32_t off = 0;
    m.xs = off; off += al16(H * 4u);
    m.xp = off; off += al16((H >> 8) * 4u * kQ4kChunkStride * 4u);
    m.gsum = off; off += al16((H >> 5) * 4u);
    m.lg = off; off += al16(L.experts * 4u);
    m.red = off; off += al16(64u * 8u);
    m.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    m.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    // act_plain also holds the router partials during R2.
    m.act_plain = off; off += al16(umax(slots * mi, (L.experts + 1u) * route_splits(H)) * 4u);
    m.act_prep = off; off += al16(slots * prep_len_of(mi) * 4u);
    m.act_gsum = off; off += al16(slots * (mi >> 5) * 4u);
    m.rows_cap = (max_down_rows(H, down_ctas) + 7u) & ~7u;
    m.ybuf = off; off += al16(slots * m.rows_cap * 4u);
    m.stage_bytes = stage_bytes_of(L);
    m.stage = off; off += m.stage_bytes * kWarps;
    m.total = off;
    return m;
}

struct Shared {
    float* xs;
    float* xp;
    float* gsum;
    float* lg;
    double* red;
    uint32_t* sel_id;
    float* sel_w;
    float* act_plain;
    float* act_prep;
    float* act_gsum;
    float* ybuf;
    uint8_t* stage;
    SmemLayout m;
};

__device__ inline Shared carve(uint8_t* base, const SmemLayout& m) {
    Shared s;
    s.xs = reinterpret_cast<float*>(base + m.xs);
    s.xp = reinterpret_cast<float*>(base + m.xp);
    s.gsum = reinterpret_cast<float*>(base + m.gsum);
    s.lg = reinterpret_cast<float*>(base + m.lg);
    s.red = reinterpret_cast<double*>(base + m.red);
    s.sel_id = reinterpret_cast<uint32_t*>(base + m.sel_id);
    s.sel_w = reinterpret_cast<float*>(base + m.sel_w);
    s.act_plain = reinterpret_cast<float*>(base + m.act_plain);
    s.act_prep = reinterpret_cast<float*>(base + m.act_prep);
    s.act_gsum = reinterpret_cast<float*>(base + m.act_gsum);
    s.ybuf = reinterpret_cast<float*>(base + m.ybuf);
    s.stage = base + m.stage;
    s.m = m;
    return s;
}

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoid_qwen35(float v) {
    // src/qwen35_runner.cpp:111-115
    if (v >= 0.0f) return 1.0f / (1.0f + expf(-v));
    const float e = expf(v);
    return e / (1.0f + e);
}

__device__ __forceinline__ float silu_mul(float g, float u, uint32_t flavour) {
    // Qwen3-MoE: g / (1 + exp(-g)) * u (qwen3_moe_runner.cpp:683);
    // Qwen3.5:   g * sigmoid(g) * u   (qwen35_runner.cpp:123, 733-735).
    return flavour == 0 ? (g / (1.0f + expf(-g))) * u : (g * sigmoid_qwen35(g)) * u;
}

// Rank order of both routers: higher logit first, equal logits -> lower id.
__device__ __forceinline__ bool route_before(float va, uint32_t ia, float vb, uint32_t ib) {
    return va > vb || (va == vb && ia < ib);
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* red, Op op) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    T r = red[0];
    for (int w = 1; w < kWarps; ++w) r = op(r, red[w]);
    return r;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier for a co-resident (cooperative) grid.  `counter` only
// grows; barrier number `index` (1-based within this launch) completes when
// it reaches base + index * gridDim.x.  The wait is bounded: after ~2 s (or as
// soon as another CTA has flagged a timeout) the CTA records
// kStatusWaitTimeout and returns false, and the caller abandons the launch.
__device__ bool grid_barrier(uint32_t* counter, uint32_t base, uint32_t index, uint32_t* status,
                             uint32_t* abort_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_gpu_add(counter, 1u);
        const uint32_t target = base + index * gridDim.x;
        const long long t0 = clock64();
        uint32_t polls = 0;
        while (static_cast<int32_t>(ld_acquire_gpu(counter) - target) < 0) {
            if ((++polls & 255u) == 0) {
                if (ld_acquire_gpu(status) & kStatusWaitTimeout) { *abort_flag = 1u; break; }
                if (clock64() - t0 > kBarrierTimeoutCycles) {
                    atomicOr(status, kStatusWaitTimeout);
                    *abort_flag = 1u;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return *abort_flag == 0u;
}

// ---------------------------------------------------------------------------
// R0: the block input into shared memory (every CTA).
// ---------------------------------------------------------------------------
constexpr int kMaxPerThread = 12;          // ceil(max hidden 4096 / kThreads)

// Copies n floats written by other CTAs (ld.global.cg) into shared memory, all
// loads of a thread in flight together.
__device__ __forceinline__ void copy_coherent(const float* __restrict__ src, float* dst, uint32_t n) {
    for (uint32_t base = 0; base < n; base += kThreads * kMaxPerThread) {
        float v[kMaxPerThread];
#pragma unroll
        for (int j = 0; j < kMaxPerThread; ++j) {
            const uint32_t i = base + threadIdx.x + j * kThreads;
            v[j] = i < n ? __ldcg(src + i) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kMaxPerThread; ++j) {
            const uint32_t i = base + threadIdx.x + j * kThreads;
            if (i < n) dst[i] = v[j];
        }
    }
}

// The tensor-core path (gate_up_mma / down_mma) serves blocks whose expert
// matrices are all Q4_K, without a shared expert, with at most one slot per
// warp and whole superblocks of the intermediate.
__host__ __device__ inline bool mma_path_ok(const MoeLayerDev& L) {
    return L.gate_type == kQ4_K && L.up_type == kQ4_K && L.down_type == kQ4_K && L.shared_inter == 0 &&
           L.top_k <= static_cast<uint32_t>(kWarps) && (L.inter % 256u) == 0;
}

// Same as copy_coherent for 16-byte aligned buffers of n4 uint4 elements.
__device__ __forceinline__ void copy_coherent4(const uint4* __restrict__ src, uint4* dst, uint32_t n4) {
    constexpr int kPer = 6;
    for (uint32_t base = 0; base < n4; base += kThreads * kPer) {
        uint4 v[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const uint32_t i = base + threadIdx.x + j * kThreads;
            v[j] = i < n4 ? __ldcg(src + i) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const uint32_t i = base + threadIdx.x + j * kThreads;
            if (i < n4) dst[i] = v[j];
        }
    }
}

__device__ void phase_input(const MoeLayerDev& L, const float* hidden, const float* x_in,
                            Shared& s) {
    const uint32_t H = L.hidden;
    if (hidden) {
        float v[kMaxPerThread], w[kMaxPerThread];
#pragma unroll
        for (int j = 0; j < kMaxPerThread; ++j) {
            const uint32_t i = threadIdx.x + j * kThreads;
            v[j] = i < H ? __ldcg(hidden + i) : 0.0f;
            w[j] = i < H ? __ldg(L.ffn_norm + i) : 0.0f;
        }
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxPerThread; ++j) ss = fmaf(v[j], v[j], ss);
        float* redf = reinterpret_cast<float*>(s.red);
        const float total = block_reduce(ss, redf, [](float a, float b) { return a + b; });
        // src/rms_norm.cpp:20-26: scale = 1 / sqrt(mean + eps); y = x * scale * w
        const float scale = 1.0f / sqrtf(total / static_cast<float>(H) + L.rms_eps);
#pragma unroll
        for (int j = 0; j < kMaxPerThread; ++j) {
            const uint32_t i = threadIdx.x + j * kThreads;
            if (i < H) s.xs[i] = v[j] * scale * w[j];
        }
    } else {
        copy_coherent(x_in, s.xs, H);
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// R1: router partial dots.  Task t = (row, split) over (E + shared) rows and
// 512-column splits; warp `gw` of `nw` grid warps takes t = gw, gw + nw, ...
// Loads for up to two tasks are issued by router_issue (which may run before
// the input is ready); router_finish consumes them.
// ---------------------------------------------------------------------------
struct RouterRegs {
    uint4 w[2][4];
    uint32_t task[2];
    uint32_t n;
};

__device__ __forceinline__ void router_issue(const MoeLayerDev& L, uint32_t gw, uint32_t nw,
                                             RouterRegs& rr) {
    const int lane = threadIdx.x & 31;
    const uint32_t splits = route_splits(L.hidden);
    const uint32_t tasks = (L.experts + (L.shared_inter ? 1u : 0u)) * splits;
    rr.n = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint32_t t = gw + j * nw;
        rr.task[j] = t;
        if (t < tasks) {
            rr.n = j + 1;
            const uint32_t row = t / splits, sp = t % splits;
            const float* w = row < L.experts ? L.router + static_cast<uint64_t>(row) * L.hidden
                                             : L.shared_router;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t col = sp * kRouteColsPerWarp + q * 128u + lane * 4u;
                rr.w[j][q] = col < L.hidden ? ldg_stream128(w + col) : make_uint4(0, 0, 0, 0);
            }
        }
    }
}

__device__ __forceinline__ void router_finish(const MoeLayerDev& L, uint32_t gw, uint32_t nw,
                                              RouterRegs& rr, const Shared& s, float* partial) {
    const int lane = threadIdx.x & 31;
    const uint32_t splits = route_splits(L.hidden);
    const uint32_t tasks = (L.experts + (L.shared_inter ? 1u : 0u)) * splits;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        if (j < static_cast<int>(rr.n)) {
            const uint32_t sp = rr.task[j] % splits;
            float acc = 0.0f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t col = sp * kRouteColsPerWarp + q * 128u + lane * 4u;
                if (col < L.hidden) {
                    const float4 xv = *reinterpret_cast<const float4*>(s.xs + col);
                    acc = fmaf(__uint_as_float(rr.w[j][q].x), xv.x, acc);
                    acc = fmaf(__uint_as_float(rr.w[j][q].y), xv.y, acc);
                    acc = fmaf(__uint_as_float(rr.w[j][q].z), xv.z, acc);
                    acc = fmaf(__uint_as_float(rr.w[j][q].w), xv.w, acc);
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) partial[rr.task[j]] = acc;
        }
    }
    // Tasks beyond two per warp (only for very large E): finish them directly.
    for (uint32_t t = gw + 2 * nw; t < tasks; t += nw) {
        const uint32_t row = t / splits, sp = t % splits;
        const float* w = row < L.experts ? L.router + static_cast<uint64_t>(row) * L.hidden
                                         : L.shared_router;
        float acc = 0.0f;
        for (uint32_t q = 0; q < 4; ++q) {
            const uint32_t col = sp * kRouteColsPerWarp + q * 128u + lane * 4u;
            if (col < L.hidden) {
                const uint4 v = ldg_stream128(w + col);
                const float4 xv = *reinterpret_cast<const float4*>(s.xs + col);
                acc = fmaf(__uint_as_float(v.x), xv.x, acc);
                acc = fmaf(__uint_as_float(v.y), xv.y, acc);
                acc = fmaf(__uint_as_float(v.z), xv.z, acc);
                acc = fmaf(__uint_as_float(v.w), xv.w, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) partial[t] = acc;
    }
}

// ---------------------------------------------------------------------------
// R2: routing from the partials, by every thread of the CTA.
//   flavour 0: route_experts, src/qwen3_moe_runner.cpp:267-305 (FP64 denominator)
//   flavour 1: select_experts, src/qwen35_runner.cpp:131-173 (FP32), weights
//              times expert_weights_scale, shared gate sigmoid(w_s . x)
// Top-k by rank: expert e is selected at position rank(e) = #{e' before e}
// when rank(e) < k -- the same set and order as the reference's insertion into
// a sorted vector.  Non-finite logits (the reference throws) set the status
// bit and give in-bounds zero-weight routes.
// Results: s.sel_id[0..k), s.sel_w[0..k] (sel_w[k] = shared gate).
// ---------------------------------------------------------------------------
__device__ void route_core(const float* lg, uint32_t E, uint32_t k, uint32_t flavour,
                           uint32_t normalize, float ew_scale, bool has_shared, float shared_logit,
                           Shared& s, uint32_t* status) {
    const int tid = threadIdx.x;
    float* redf = reinterpret_cast<float*>(s.red + 16);
    float mx = -FLT_MAX;
    int bad = 0;
    for (uint32_t e = tid; e < E; e += kThreads) {
        const float v = lg[e];
        bad |= !isfinite(v);
        mx = fmaxf(mx, v);
    }
    bad = __syncthreads_or(bad);
    mx = block_reduce(mx, redf, [](float a, float b) { return fmaxf(a, b); });
    if (bad) {
        if (tid == 0 && status) atomicOr(status, kStatusNonFiniteLogits);
        for (uint32_t r = tid; r < k; r += kThreads) { s.sel_id[r] = r; s.sel_w[r] = 0.0f; }
        if (tid == 0) s.sel_w[k] = 0.0f;
        __syncthreads();
        return;
    }
    double den_d = 0.0;
    float den_f = 0.0f;
    for (uint32_t e = tid; e < E; e += kThreads) {
        if (flavour == 0) den_d += exp(static_cast<double>(lg[e] - mx));
        else den_f += expf(lg[e] - mx);
    }
    if (flavour == 0) den_d = block_reduce(den_d, s.red, [](double a, double b) { return a + b; });
    else den_f = block_reduce(den_f, redf, [](float a, float b) { return a + b; });
    for (uint32_t e = tid; e < E; e += kThreads) {
        const float v = lg[e];
        uint32_t rank = 0;
        uint32_t f = 0;
        if ((reinterpret_cast<uintptr_t>(lg) & 15u) == 0) {
            for (; f + 8 <= E; f += 8) {
                const float4 a = *reinterpret_cast<const float4*>(lg + f);
                const float4 c = *reinterpret_cast<const float4*>(lg + f + 4);
                rank += (route_before(a.x, f, v, e) ? 1u : 0u) + (route_before(a.y, f + 1, v, e) ? 1u : 0u) +
                        (route_before(a.z, f + 2, v, e) ? 1u : 0u) + (route_before(a.w, f + 3, v, e) ? 1u : 0u) +
                        (route_before(c.x, f + 4, v, e) ? 1u : 0u) + (route_before(c.y, f + 5, v, e) ? 1u : 0u) +
                        (route_before(c.z, f + 6, v, e) ? 1u : 0u) + (route_before(c.w, f + 7, v, e) ? 1u : 0u);
            }
        }
        for (; f < E; ++f) rank += route_before(lg[f], f, v, e) ? 1u : 0u;
        if (rank < k) {
            s.sel_id[rank] = e;
            s.sel_w[rank] = flavour == 0
                ? static_cast<float>(exp(static_cast<double>(v - mx)) / den_d)
                : expf(v - mx) / den_f;
        }
    }
    __syncthreads();
    if (tid == 0) {
        bool invalid = flavour == 1 && (!isfinite(den_f) || den_f <= 0.0f);
        if (normalize) {
            float sum = 0.0f;
            for (uint32_t r = 0; r < k; ++r) sum += s.sel_w[r];
            if (flavour == 1 && (!isfinite(sum) || sum <= 0.0f)) invalid = true;
            for (uint32_t r = 0; r < k; ++r) s.sel_w[r] /= sum;
        }
        if (invalid && status) atomicOr(status, kStatusBadSoftmax);
        for (uint32_t r = 0; r < k; ++r)
            s.sel_w[r] = invalid ? 0.0f : (flavour == 0 ? s.sel_w[r] : s.sel_w[r] * ew_scale);
        s.sel_w[k] = has_shared ? sigmoid_qwen35(shared_logit) : 0.0f;
    }
    __syncthreads();
}

// Logits from the router partials (summed in split order), then route_core.
// The `writer` CTA also stores logits, ids and weights to global memory.
__device__ void phase_route(const MoeLayerDev& L, const float* partial, Shared& s,
                            uint32_t* status, bool writer, const MoeScratch& S) {
    const uint32_t splits = route_splits(L.hidden);
    const uint32_t rows = L.experts + (L.shared_inter ? 1u : 0u);
    // All partials into shared memory first (the act buffer is free here),
    // then per-row sums in split order.
    float* pbuf = s.act_plain;
    copy_coherent(partial, pbuf, rows * splits);
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < L.experts; e += kThreads) {
        float v = pbuf[e * splits];
        for (uint32_t sp = 1; sp < splits; ++sp) v += pbuf[e * splits + sp];
        s.lg[e] = v;
    }
    float shared_logit = 0.0f;
    if (L.shared_inter) {
        const float* p = pbuf + L.experts * splits;
        shared_logit = p[0];
        for (uint32_t sp = 1; sp < splits; ++sp) shared_logit += p[sp];
    }
    __syncthreads();
    route_core(s.lg, L.experts, L.top_k, L.flavour, L.normalize, L.expert_weights_scale,
               L.shared_inter != 0, shared_logit, s, status);
    if (writer) {
        for (uint32_t e = threadIdx.x; e < L.experts; e += kThreads) S.logits[e] = s.lg[e];
        for (uint32_t r = threadIdx.x; r <= L.top_k; r += kThreads) {
            if (r < L.top_k) S.ids[r] = s.sel_id[r];
            S.weights[r] = s.sel_w[r];
        }
    }
}

// ---------------------------------------------------------------------------
// Expert slot matrices.
// ---------------------------------------------------------------------------
struct SlotMats {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    uint32_t gate_type, up_type, down_type, rows;
};

__device__ __forceinline__ SlotMats slot_mats(const MoeLayerDev& L, const uint32_t* ids, uint32_t s) {
    SlotMats m;
    if (s < L.top_k) {
        const uint64_t id = ids[s];
        m.gate = L.gate + id * L.gate_slice;
        m.up = L.up + id * L.up_slice;
        m.down = L.down + id * L.down_slice;
        m.gate_type = L.gate_type; m.up_type = L.up_type; m.down_type = L.down_type;
        m.rows = L.inter;
    } else {
        m.gate = L.shared_gate; m.up = L.shared_up; m.down = L.shared_down;
        m.gate_type = L.shared_gate_type; m.up_type = L.shared_up_type;
        m.down_type = L.shared_down_type;
        m.rows = L.shared_inter;
    }
    return m;
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

// Q4_K loads of N superblocks starting at sb0 of one row, for chunk c.
template <int N>
struct Q4kChunkRegs {
    uint4 hdr[N], q0[N], q1[N];
};

template <int N>
__device__ __forceinline__ void q4k_issue(const uint8_t* rowp, int c, int sb0, int nsb,
                                          Q4kChunkRegs<N>& r) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
        if (sb0 + i < nsb) {
            const uint8_t* blk = rowp + (sb0 + i) * 144;
            r.hdr[i] = ldg_stream128(blk);
            r.q0[i] = ldg_stream128(blk + 16 + 32 * c);
            r.q1[i] = ldg_stream128(blk + 32 + 32 * c);
        }
    }
}

template <int N>
__device__ __forceinline__ float q4k_consume(const Q4kChunkRegs<N>& r, int c, int sb0, int nsb,
                                             const float* xp, const float* gsum) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int sb = sb0 + i;
        if (sb < nsb)
            acc += q4k_chunk_dot(r.hdr[i], r.q0[i], r.q1[i], c, xp + (sb * 4 + c) * kQ4kChunkStride,
                                 gsum[sb * 8 + 2 * c], gsum[sb * 8 + 2 * c + 1]);
    }
    return acc;
}

// ---------------------------------------------------------------------------
// G: gate/up.  Task space = [fast Q4_K quads of every fast slot][generic rows of
// the other slots]; CTA b of n owns tasks [b*T/n, (b+1)*T/n), warp w takes
// t0 + w, t0 + w + kWarps, ...  A fast quad: lanes (row r 0..3, matrix
// gate/up, chunk c 0..3) each own one 64-weight chunk of every superblock of
// their row.  Before computing, the CTA asks the TMA unit to stream its share
// of the down rows into L2.
// ---------------------------------------------------------------------------
struct GateUpTasks {
    uint32_t n_fast, n_gen, total;
};

__device__ __forceinline__ GateUpTasks gate_up_tasks(const MoeLayerDev& L) {
    GateUpTasks t{0, 0, 0};
    const uint32_t slots = slots_of(L);
    for (uint32_t s = 0; s < slots; ++s) {
        const bool routed = s < L.top_k;
        const uint32_t gt = routed ? L.gate_type : L.shared_gate_type;
        const uint32_t ut = routed ? L.up_type : L.shared_up_type;
        const uint32_t rows = routed ? L.inter : L.shared_inter;
        if (fast_pair(gt, ut)) t.n_fast += rows >> 2; else t.n_gen += rows;
    }
    t.total = t.n_fast + t.n_gen;
    return t;
}

__device__ __forceinline__ void gate_up_locate(const MoeLayerDev& L, const GateUpTasks& T,
                                               uint32_t t, uint32_t& slot, uint32_t& row,
                                               bool& fast) {
    const uint32_t slots = slots_of(L);
    uint32_t acc_fast = 0, acc_gen = T.n_fast;
    slot = 0; row = 0; fast = false;
    for (uint32_t s = 0; s < slots; ++s) {
        const bool routed = s < L.top_k;
        const uint32_t gt = routed ? L.gate_type : L.shared_gate_type;
        const uint32_t ut = routed ? L.up_type : L.shared_up_type;
        const uint32_t rows = routed ? L.inter : L.shared_inter;
        if (fast_pair(gt, ut)) {
            const uint32_t n = rows >> 2;
            if (t < T.n_fast && t < acc_fast + n) { slot = s; row = (t - acc_fast) * 4u; fast = true; return; }
            acc_fast += n;
        } else {
            if (t >= T.n_fast && t < acc_gen + rows) { slot = s; row = t - acc_gen; return; }
            acc_gen += rows;
        }
    }
}

__device__ void phase_gate_up(const MoeLayerDev& L, Shared& s, float* act, uint32_t act_stride,
                              uint32_t b, uint32_t n, uint32_t down_ctas) {
    const uint32_t H = L.hidden;
    const int nsb = static_cast<int>(H >> 8);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const GateUpTasks T = gate_up_tasks(L);
    const uint32_t t0 = static_cast<uint32_t>(static_cast<uint64_t>(b) * T.total / n);
    const uint32_t t1 = static_cast<uint32_t>(static_cast<uint64_t>(b + 1) * T.total / n);
    const int r = (lane >> 2) & 3, mat = lane >> 4, c = lane & 3;

    // First task of this warp: issue its loads before anything else.
    const uint32_t first = t0 + warp;
    uint32_t slot0 = 0, row0 = 0;
    bool fast0 = false;
    Q4kChunkRegs<kSbChunk> regs;
    if (first < t1) {
        gate_up_locate(L, T, first, slot0, row0, fast0);
        if (fast0) {
            const SlotMats m = slot_mats(L, s.sel_id, slot0);
            const uint8_t* rp = (mat ? m.up : m.gate) + static_cast<uint64_t>(row0 + r) * (nsb * 144u);
            q4k_issue(rp, c, 0, nsb, regs);
        }
    }
    // Stream this CTA's share of every slot's down rows into L2 (D reads them next).
    if (b < down_ctas) {
        const uint32_t slots = slots_of(L);
        uint32_t r0, r1;
        down_rows(H, b, down_ctas, r0, r1);
        if (static_cast<uint32_t>(tid) < slots && r1 > r0) {
            const SlotMats m = slot_mats(L, s.sel_id, tid);
            const uint64_t rd = row_bytes(m.down_type, m.rows);
            prefetch_l2_range(m.down + r0 * rd, (r1 - r0) * rd);
        }
    }
    q4k_prepare_x(s.xs, static_cast<int>(H), s.xp, s.gsum);
    __syncthreads();

    for (uint32_t t = first; t < t1; t += kWarps) {
        uint32_t slot = slot0, row = row0;
        bool fast = fast0;
        if (t != first) gate_up_locate(L, T, t, slot, row, fast);
        const SlotMats m = slot_mats(L, s.sel_id, slot);
        const uint32_t flavour = slot < L.top_k ? L.flavour : 1u;
        if (fast) {
            float acc = 0.0f;
            const uint8_t* rp = (mat ? m.up : m.gate) + static_cast<uint64_t>(row + r) * (nsb * 144u);
            for (int sb0 = 0; sb0 < nsb; sb0 += kSbChunk) {
                if (!(t == first && sb0 == 0)) q4k_issue(rp, c, sb0, nsb, regs);
                acc += q4k_consume(regs, c, sb0, nsb, s.xp, s.gsum);
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            const float u = __shfl_down_sync(0xffffffffu, acc, 16);
            if (mat == 0 && c == 0) act[slot * act_stride + row + r] = silu_mul(acc, u, flavour);
        } else {
            uint8_t* my_stage = s.stage + warp * s.m.stage_bytes;
            const float g = generic_row_dot(m.gate_type, m.gate + row * row_bytes(m.gate_type, H),
                                            H, s.xs, my_stage, lane);
            const float u = generic_row_dot(m.up_type, m.up + row * row_bytes(m.up_type, H), H,
                                            s.xs, my_stage, lane);
            if (lane == 0) act[slot * act_stride + row] = silu_mul(g, u, flavour);
        }
    }
}

// ---------------------------------------------------------------------------
// D: down + combine (+ residual) for CTA b's rows [r0, r1).  Warp tasks =
// (slot, octet of rows); a fast (Q4_K down) task: lanes (row r 0..7, chunk c)
// own one 64-weight chunk of every superblock of their row.  The loads of the
// warp's first task are issued before `wait_for_act()` runs, so the caller's
// grid barrier overlaps them.
// ---------------------------------------------------------------------------
template <typename Wait>
__device__ void phase_down(const MoeLayerDev& L, Shared& s, const float* act, uint32_t act_stride,
                           uint32_t b, uint32_t n, float* hidden, float* moe_out,
                           const float* next_router, uint64_t next_router_bytes, Wait wait_for_act,
                           bool& ok) {
    const uint32_t H = L.hidden;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t slots = slots_of(L);
    uint32_t r0, r1;
    down_rows(H, b, n, r0, r1);
    const uint32_t nrows = r1 - r0;
    const uint32_t octets = (nrows + 7u) >> 3;
    const uint32_t tasks = slots * octets;
    const int r = lane >> 2, c = lane & 3;

    // Pre-issue the warp's first fast task (its first kSbChunkDown superblocks).
    Q4kChunkRegs<kSbChunkDown> pre;
    if (static_cast<uint32_t>(warp) < tasks) {
        const uint32_t slot = warp / octets, o = warp % octets;
        const SlotMats m = slot_mats(L, s.sel_id, slot);
        const uint32_t row = r0 + o * 8u + r;
        if (m.down_type == kQ4_K && row < r1) {
            const int nsb = static_cast<int>(m.rows >> 8);
            q4k_issue(m.down + static_cast<uint64_t>(row) * (nsb * 144u), c, 0, nsb, pre);
        }
    }
    if (next_router && tid == 0) {
        const uint64_t a = (next_router_bytes * b / n) & ~uint64_t(15);
        const uint64_t e = b + 1 == n ? next_router_bytes : (next_router_bytes * (b + 1) / n) & ~uint64_t(15);
        if (e > a) prefetch_l2_range(reinterpret_cast<const uint8_t*>(next_router) + a, e - a);
    }

    ok = wait_for_act();
    if (!ok) return;

    // act of every slot -> shared memory (plain + Q4_K-prepared layouts).
    const uint32_t mi = max_inter_of(L);
    const uint32_t prep_len = prep_len_of(mi);
    // act rows are stored with stride mi == act_stride (max_inter_of), so one
    // flat copy moves every slot (the shared slot's tail beyond its rows is unused).
    copy_coherent(act, s.act_plain, slots * act_stride);
    __syncthreads();
    for (uint32_t sl = 0; sl < slots; ++sl) {
        const bool routed = sl < L.top_k;
        const uint32_t dt = routed ? L.down_type : L.shared_down_type;
        const uint32_t rows = routed ? L.inter : L.shared_inter;
        if (dt == kQ4_K)
            q4k_prepare_x(s.act_plain + sl * mi, static_cast<int>(rows), s.act_prep + sl * prep_len,
                          s.act_gsum + sl * (mi >> 5));
    }
    __syncthreads();

    const uint32_t cap = s.m.rows_cap;
    for (uint32_t t = warp; t < tasks; t += kWarps) {
        const uint32_t slot = t / octets, o = t % octets;
        const SlotMats m = slot_mats(L, s.sel_id, slot);
        if (m.down_type == kQ4_K) {
            const int nsb = static_cast<int>(m.rows >> 8);
            const uint32_t row = r0 + o * 8u + r;
            float acc = 0.0f;
            if (row < r1) {
                const uint8_t* rp = m.down + static_cast<uint64_t>(row) * (nsb * 144u);
                const float* xp = s.act_prep + slot * prep_len;
                const float* gs = s.act_gsum + slot * (mi >> 5);
                for (int sb0 = 0; sb0 < nsb; sb0 += kSbChunkDown) {
                    if (t == static_cast<uint32_t>(warp) && sb0 == 0) {
                        acc += q4k_consume(pre, c, sb0, nsb, xp, gs);
                    } else {
                        Q4kChunkRegs<kSbChunkDown> regs;
                        q4k_issue(rp, c, sb0, nsb, regs);
                        acc += q4k_consume(regs, c, sb0, nsb, xp, gs);
                    }
                }
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (c == 0 && row < r1) s.ybuf[slot * cap + (row - r0)] = acc;
        } else {
            uint8_t* my_stage = s.stage + warp * s.m.stage_bytes;
            const uint64_t rb = row_bytes(m.down_type, m.rows);
            for (uint32_t rr = 0; rr < 8; ++rr) {
                const uint32_t row = r0 + o * 8u + rr;
                if (row >= r1) break;
                const float y = generic_row_dot(m.down_type, m.down + row * rb, m.rows,
                                                s.act_plain + slot * mi, my_stage, lane);
                if (lane == 0) s.ybuf[slot * cap + (row - r0)] = y;
            }
        }
    }
    __syncthreads();
    for (uint32_t i = tid; i < nrows; i += kThreads) {
        float acc = 0.0f;
        for (uint32_t sl = 0; sl < L.top_k; ++sl) acc += s.sel_w[sl] * s.ybuf[sl * cap + i];
        if (L.shared_inter) acc = acc + s.sel_w[L.top_k] * s.ybuf[L.top_k * cap + i];
        const uint32_t row = r0 + i;
        if (moe_out) moe_out[row] = acc;
        else hidden[row] = __ldcg(hidden + row) + acc;
    }
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
struct BlockArgs {
    MoeLayerDev L;
    MoeScratch S;
    const float* x_in;
    float* hidden;
    float* moe_out;
    const float* next_router;
    SmemLayout m;
    uint32_t down_ctas;
};

// Kernel 1 of a block: R0 + R1 (CTA 0 also publishes x).
__global__ void __launch_bounds__(kThreads, 1) moe_route_kernel(BlockArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    Shared s = carve(smem, a.m);
    const uint32_t gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
    RouterRegs rr;
    router_issue(a.L, gw, nw, rr);
    phase_input(a.L, a.hidden, a.x_in, s);
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < a.L.hidden; i += kThreads) a.S.x[i] = s.xs[i];
    // Tensor-core fragments of x: superblock sb is built by warp 0 of CTA sb mod grid.
    if ((threadIdx.x >> 5) == 0 && mma_path_ok(a.L))
        for (uint32_t sb = blockIdx.x; sb < (a.L.hidden >> 8); sb += gridDim.x)
            q4k_frag_superblock(s.xs + sb * 256u, a.S.xfrag + sb * kFragWords, threadIdx.x & 31);
    router_finish(a.L, gw, nw, rr, s, a.S.partial);
}

// Kernel 2: R2 (every CTA; CTA 0 publishes the routes) + G.
__global__ void __launch_bounds__(kThreads, 1) moe_gate_up_kernel(BlockArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    Shared s = carve(smem, a.m);
    phase_route(a.L, a.S.partial, s, a.S.status, blockIdx.x == 0, a.S);
    copy_coherent(a.S.x, s.xs, a.L.hidden);
    __syncthreads();
    phase_gate_up(a.L, s, a.S.act, max_inter_of(a.L), blockIdx.x, gridDim.x, a.down_ctas);
}

// Kernel 3: D.
__global__ void __launch_bounds__(kThreads, 1) moe_down_kernel(BlockArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    Shared s = carve(smem, a.m);
    for (uint32_t r = threadIdx.x; r <= a.L.top_k; r += kThreads) {
        if (r < a.L.top_k) s.sel_id[r] = __ldcg(a.S.ids + r);
        s.sel_w[r] = __ldcg(a.S.weights + r);
    }
    __syncthreads();
    bool ok = true;
    const uint64_t nrb = static_cast<uint64_t>(a.L.experts) * a.L.hidden * 4u;
    phase_down(a.L, s, a.S.act, max_inter_of(a.L), blockIdx.x, gridDim.x, a.hidden, a.moe_out,
               a.next_router, nrb, [] { return true; }, ok);
}

// Routing of a standalone logits vector (pokit_cuda_route_experts).
__global__ void __launch_bounds__(kThreads, 1)
route_logits_kernel(const float* __restrict__ logits, uint32_t E, uint32_t k, uint32_t flavour,
                    uint32_t normalize, float ew_scale, uint32_t* ids, float* weights,
                    uint32_t* status) {
    __shared__ float lg[kMaxExperts];
    __shared__ double red[64];
    __shared__ uint32_t sel_id[kMaxTopK + 1];
    __shared__ float sel_w[kMaxTopK + 1];
    Shared s{};
    s.red = red;
    s.sel_id = sel_id;
    s.sel_w = sel_w;
    for (uint32_t e = threadIdx.x; e < E; e += kThreads) lg[e] = logits[e];
    __syncthreads();
    route_core(lg, E, k, flavour, normalize, ew_scale, false, 0.0f, s, status);
    for (uint32_t r = threadIdx.x; r < k; r += kThreads) {
        ids[r] = sel_id[r];
        weights[r] = sel_w[r];
    }
}

// The decode chain for one token: layers [first, first + count) of `layers`,
// hidden += MoE_l(rms_norm(hidden, ffn_norm_l)).  Cooperative launch only.
struct DecodeArgs {
    const MoeLayerDev* layers;
    uint32_t first, count;
    MoeScratch S;
    float* hidden;
    SmemLayout m;
    uint32_t barrier_base;
};

__global__ void __launch_bounds__(kThreads, 1) moe_decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint32_t abort_flag;
    Shared s = carve(smem, a.m);
    if (threadIdx.x == 0) abort_flag = 0u;
    const uint32_t b = blockIdx.x, n = gridDim.x;
    const uint32_t gw = b * kWarps + (threadIdx.x >> 5), nw = n * kWarps;
    uint32_t barrier = 0;
    RouterRegs rr;
    router_issue(a.layers[a.first], gw, nw, rr);
    __syncthreads();
    static_assert(sizeof(MoeLayerDev) % 4 == 0 && sizeof(MoeLayerDev) / 4 <= kThreads, "descriptor copy");
    __shared__ __align__(16) uint32_t lsh[sizeof(MoeLayerDev) / 4];
    for (uint32_t i = 0; i < a.count; ++i) {
        // The layer descriptor lives in shared memory for the whole layer.
        __syncthreads();
        if (threadIdx.x < sizeof(MoeLayerDev) / 4)
            lsh[threadIdx.x] = reinterpret_cast<const uint32_t*>(&a.layers[a.first + i])[threadIdx.x];
        __syncthreads();
        const MoeLayerDev& L = *reinterpret_cast<const MoeLayerDev*>(lsh);
        // R0 + R1
        phase_input(L, a.hidden, nullptr, s);
        router_finish(L, gw, nw, rr, s, a.S.partial);
        if (!grid_barrier(a.S.counter, a.barrier_base, ++barrier, a.S.status, &abort_flag)) return;
        // R2 + G
        const bool last = i + 1 == a.count;
        phase_route(L, a.S.partial, s, a.S.status, b == 0 && last, a.S);
        phase_gate_up(L, s, a.S.act, max_inter_of(L), b, n, n);
        // D (its loads go out before the barrier that publishes act)
        const MoeLayerDev* next = last ? nullptr : &a.layers[a.first + i + 1];
        bool ok = true;
        phase_down(L, s, a.S.act, max_inter_of(L), b, n, a.hidden, nullptr,
                   next ? next->router : nullptr,
                   next ? static_cast<uint64_t>(next->experts) * next->hidden * 4u : 0u,
                   [&] { return grid_barrier(a.S.counter, a.barrier_base, ++barrier, a.S.status,
                                             &abort_flag); },
                   ok);
        if (!ok) return;
        if (!last) router_issue(*next, gw, nw, rr);
        if (!grid_barrier(a.S.counter, a.barrier_base, ++barrier, a.S.status, &abort_flag)) return;
    }
}

// ---------------------------------------------------------------------------
// Tensor-core path: every routed matrix Q4_K, no shared expert.
//
// gate_up: CTA b of n owns tiles [b*T/n, (b+1)*T/n) of the T = k * 2 * (I/16)
// (slot, gate|up, 16-row) tiles, at most kMmaTilesPerCta of them.  Tile p is
// computed by warps 2p and 2p+1, one half of the superblocks each; each warp
// TMA-copies its half of the 16 rows into padded shared memory as soon as the
// routes are known, so the copies overlap the activation preparation.
// down: CTA b owns output rows [16b, 16b+16); warp w < k computes slot w's
// 16 rows (TMA-copied, L2-resident after gate_up's prefetch), then the rows
// are combined in route order and added to the residual.
// ---------------------------------------------------------------------------
constexpr int kMmaTilesPerCta = kWarps / 2;

struct MmaLayout {
    uint32_t bars, recs, lg, red, sel_id, sel_w, pbuf, tmp, part, flags, tiles;
    uint32_t total, nsb, stride;
};

__host__ __device__ inline MmaLayout mma_gate_up_layout(const MoeLayerDev& L) {
    MmaLayout m{};
    const uint32_t H = L.hidden, nsb = H >> 8;
    m.nsb = nsb;
    m.stride = q4k_tile_stride(nsb * 144u);
    uint32_t off = 0;
    m.bars = off; off += 128;
    m.recs = off; off += al16(nsb * kFragWords * 4u);
    m.lg = off; off += al16(L.experts * 4u);
    m.red = off; off += al16(64u * 8u);
    m.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    m.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    m.pbuf = off; off += al16((L.experts + 1u) * route_splits(H) * 4u);
    m.tmp = off; off += al16(256u * 4u);
    m.part = off; off += al16(kWarps * 16u * 4u);
    m.flags = off; off += al16(kMmaTilesPerCta * 4u + 4u);
    off = (off + 127u) & ~127u;
    m.tiles = off; off += kMmaTilesPerCta * 16u * m.stride;
    m.total = off;
    return m;
}

__host__ __device__ inline MmaLayout mma_down_layout(const MoeLayerDev& L) {
    MmaLayout m{};
    const uint32_t I = L.inter, nsb = I >> 8, k = L.top_k;
    m.nsb = nsb;
    m.stride = q4k_tile_stride(nsb * 144u);
    uint32_t off = 0;
    m.bars = off; off += 128;
    m.recs = off; off += al16(k * nsb * kFragWords * 4u);
    m.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    m.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    m.part = off; off += al16(k * 16u * 4u);
    off = (off + 127u) & ~127u;
    m.tiles = off; off += k * 16u * m.stride;
    m.total = off;
    return m;
}

struct MmaArgs {
    MoeLayerDev L;
    MoeScratch S;
    float* hidden;
    float* moe_out;
    const float* next_router;
    MmaLayout m;
    uint32_t down_ctas;   // CTAs of the down kernel (gate_up prefetches their rows)
};

__device__ __forceinline__ void gate_up_tile_coords(uint32_t tile, uint32_t tiles_per_mat, uint32_t& slot,
                                                    uint32_t& mat, uint32_t& row0) {
    slot = tile / (2u * tiles_per_mat);
    const uint32_t rem = tile % (2u * tiles_per_mat);
    mat = rem / tiles_per_mat;
    row0 = (rem % tiles_per_mat) * 16u;
}

__global__ void __launch_bounds__(kThreads, 1) moe_gate_up_mma_kernel(MmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const MoeLayerDev& L = a.L;
    const MmaLayout& m = a.m;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + m.bars);
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + m.recs);
    float* tmp = reinterpret_cast<float*>(smem + m.tmp);
    float* part = reinterpret_cast<float*>(smem + m.part);
    uint32_t* flags = reinterpret_cast<uint32_t*>(smem + m.flags);
    uint8_t* tiles = smem + m.tiles;
    Shared s{};
    s.lg = reinterpret_cast<float*>(smem + m.lg);
    s.red = reinterpret_cast<double*>(smem + m.red);
    s.sel_id = reinterpret_cast<uint32_t*>(smem + m.sel_id);
    s.sel_w = reinterpret_cast<float*>(smem + m.sel_w);
    s.act_plain = reinterpret_cast<float*>(smem + m.pbuf);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int i = 0; i < kWarps; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    // R2: the routes, from the router partials (every CTA; CTA 0 publishes them).
    phase_route(L, a.S.partial, s, a.S.status, blockIdx.x == 0, a.S);

    const uint32_t I = L.inter, nsb = m.nsb, nsbI = I >> 8;
    const uint32_t row_bytes_g = nsb * 144u;
    const uint32_t tiles_per_mat = I / 16u;
    const uint32_t T = L.top_k * 2u * tiles_per_mat;
    const uint32_t t0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * T / gridDim.x);
    const uint32_t t1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * T / gridDim.x);
    const uint32_t p = warp >> 1, half = warp & 1;
    const uint32_t sb_split = nsb / 2;
    const uint32_t sb0 = half ? sb_split : 0u, sb1 = half ? nsb : sb_split;
    const uint32_t tile = t0 + p;
    const bool has_tile = p < static_cast<uint32_t>(kMmaTilesPerCta) && tile < t1 && sb1 > sb0;
    uint8_t* mytile = tiles + p * 16u * m.stride;
    if (has_tile && lane == 0) {
        uint32_t slot, mat, row0;
        gate_up_tile_coords(tile, tiles_per_mat, slot, mat, row0);
        const uint64_t id = s.sel_id[slot];
        const uint8_t* base = (mat ? L.up + id * L.up_slice : L.gate + id * L.gate_slice) +
                              static_cast<uint64_t>(row0) * row_bytes_g + sb0 * 144u;
        const uint32_t bytes = (sb1 - sb0) * 144u;
        mbar_expect_tx(&bars[warp], 16u * bytes);
        for (uint32_t r = 0; r < 16u; ++r)
            tma_load(mytile + r * m.stride + sb0 * 144u, base + static_cast<uint64_t>(r) * row_bytes_g,
                     bytes, &bars[warp]);
    }
    // Stream this CTA's share of every slot's down rows into L2.
    if (blockIdx.x < a.down_ctas && tid < static_cast<int>(L.top_k)) {
        uint32_t r0, r1;
        down_rows(L.hidden, blockIdx.x, a.down_ctas, r0, r1);
        if (r1 > r0) {
            const uint64_t rd = row_bytes(L.down_type, I);
            prefetch_l2_range(L.down + s.sel_id[tid] * L.down_slice + r0 * rd, (r1 - r0) * rd);
        }
    }
    // x fragments (published by the route kernel).
    copy_coherent4(reinterpret_cast<const uint4*>(a.S.xfrag), reinterpret_cast<uint4*>(recs),
                   nsb * kFragWords / 4u);
    __syncthreads();

    if (has_tile) {
        float acc0 = 0.0f, acc1 = 0.0f;
        if (mbar_wait(&bars[warp], 0)) {
            q4k_mma_tile(mytile + sb0 * 144u, m.stride, static_cast<int>(sb1 - sb0), recs + sb0 * kFragWords,
                         acc0, acc1);
        } else if (lane == 0) {
            atomicOr(a.S.status, kStatusWaitTimeout);
        }
        if ((lane & 3) == 0) {
            part[warp * 16 + (lane >> 2)] = acc0;
            part[warp * 16 + (lane >> 2) + 8] = acc1;
        }
    } else if (lane < 16) {
        part[warp * 16 + lane] = 0.0f;
    }
    __syncthreads();
    // Rows of every tile: sum of the two halves, to the gate (act) or up (act2) buffer.
    for (uint32_t i = tid; i < kMmaTilesPerCta * 16u; i += kThreads) {
        const uint32_t pp = i >> 4, r = i & 15u, tt = t0 + pp;
        if (tt >= t1) continue;
        uint32_t sl, mt, rw;
        gate_up_tile_coords(tt, tiles_per_mat, sl, mt, rw);
        const float v = part[(2 * pp) * 16 + r] + part[(2 * pp + 1) * 16 + r];
        (mt ? a.S.act2 : a.S.act)[sl * I + rw + r] = v;
    }
    __syncthreads();
    // Count finished tiles per (slot, superblock of the intermediate); the CTA
    // that completes a superblock (16 gate + 16 up tiles) builds its activation
    // fragments.  No CTA waits for another.
    if (tid < kMmaTilesPerCta) {
        uint32_t done = 0xffffffffu;
        const uint32_t tt = t0 + tid;
        if (tt < t1) {
            uint32_t sl, mt, rw;
            gate_up_tile_coords(tt, tiles_per_mat, sl, mt, rw);
            const uint32_t key = sl * nsbI + (rw >> 8);
            __threadfence();
            if (atomicAdd(&a.S.sbcnt[key], 1u) == 31u) done = key;
            __threadfence();
        }
        flags[tid] = done;
    }
    __syncthreads();
    for (int f = 0; f < kMmaTilesPerCta; ++f) {
        const uint32_t key = flags[f];
        if (key == 0xffffffffu) continue;
        __threadfence();
        const uint32_t sl = key / nsbI, sb = key % nsbI;
        for (uint32_t i = tid; i < 256u; i += kThreads) {
            const uint32_t idx = sl * I + sb * 256u + i;
            tmp[i] = silu_mul(__ldcg(a.S.act + idx), __ldcg(a.S.act2 + idx), L.flavour);
        }
        __syncthreads();
        if (warp == 0) {
            q4k_frag_superblock(tmp, a.S.afrag + key * kFragWords, lane);
            if (lane == 0) a.S.sbcnt[key] = 0u;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kThreads, 1) moe_down_mma_kernel(MmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const MoeLayerDev& L = a.L;
    const MmaLayout& m = a.m;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + m.bars);
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + m.recs);
    uint32_t* sel_id = reinterpret_cast<uint32_t*>(smem + m.sel_id);
    float* sel_w = reinterpret_cast<float*>(smem + m.sel_w);
    float* part = reinterpret_cast<float*>(smem + m.part);
    uint8_t* tiles = smem + m.tiles;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t k = L.top_k, nsb = m.nsb, H = L.hidden;
    const uint32_t j0 = blockIdx.x * 16u;

    if (tid == 0) {
        for (int i = 0; i < kWarps; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    for (uint32_t r = tid; r < k; r += kThreads) {
        sel_id[r] = __ldcg(a.S.ids + r);
        sel_w[r] = __ldcg(a.S.weights + r);
    }
    __syncthreads();
    const uint32_t rbd = nsb * 144u;
    if (static_cast<uint32_t>(warp) < k && lane == 0) {
        const uint8_t* base = L.down + static_cast<uint64_t>(sel_id[warp]) * L.down_slice +
                              static_cast<uint64_t>(j0) * rbd;
        mbar_expect_tx(&bars[warp], 16u * rbd);
        for (uint32_t r = 0; r < 16u; ++r)
            tma_load(tiles + (warp * 16u + r) * m.stride, base + static_cast<uint64_t>(r) * rbd, rbd,
                     &bars[warp]);
    }
    if (a.next_router && tid == 0) {
        const uint64_t bytes = static_cast<uint64_t>(L.experts) * H * 4u;
        const uint64_t lo = (bytes * blockIdx.x / gridDim.x) & ~uint64_t(15);
        const uint64_t hi = blockIdx.x + 1 == gridDim.x ? bytes : (bytes * (blockIdx.x + 1) / gridDim.x) & ~uint64_t(15);
        if (hi > lo) prefetch_l2_range(reinterpret_cast<const uint8_t*>(a.next_router) + lo, hi - lo);
    }
    // Activation fragments of every slot (built by the gate/up kernel).
    copy_coherent4(reinterpret_cast<const uint4*>(a.S.afrag), reinterpret_cast<uint4*>(recs),
                   k * nsb * kFragWords / 4u);
    __syncthreads();
    if (static_cast<uint32_t>(warp) < k) {
        float acc0 = 0.0f, acc1 = 0.0f;
        if (mbar_wait(&bars[warp], 0)) {
            q4k_mma_tile(tiles + warp * 16u * m.stride, m.stride, static_cast<int>(nsb),
                         recs + warp * nsb * kFragWords, acc0, acc1);
        } else if (lane == 0) {
            atomicOr(a.S.status, kStatusWaitTimeout);
        }
        if ((lane & 3) == 0) {
            part[warp * 16 + (lane >> 2)] = acc0;
            part[warp * 16 + (lane >> 2) + 8] = acc1;
        }
    }
    __syncthreads();
    if (tid < 16) {
        float acc = 0.0f;
        for (uint32_t sl = 0; sl < k; ++sl) acc += sel_w[sl] * part[sl * 16 + tid];
        const uint32_t row = j0 + tid;
        if (a.moe_out) a.moe_out[row] = acc;
        else a.hidden[row] = __ldcg(a.hidden + row) + acc;
    }
}

// ---------------------------------------------------------------------------
template <typename K>
cudaError_t ensure_smem(K kernel, size_t bytes, size_t& granted) {
    if (bytes <= 48u * 1024u || bytes <= granted) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(bytes));
    if (e == cudaSuccess) granted = bytes;
    return e;
}

size_t g_route_smem = 0, g_gate_up_smem = 0, g_down_smem = 0, g_decode_smem = 0;
size_t g_gate_up_mma_smem = 0, g_down_mma_smem = 0;

uint64_t align256(uint64_t v) { return (v + 255u) & ~uint64_t(255); }

bool layer_valid(const MoeLayerDev& L) {
    return !(L.top_k == 0 || L.top_k > L.experts || L.top_k > kMaxTopK || L.experts > kMaxExperts ||
             L.hidden == 0 || (L.hidden & 255u) || L.inter == 0 || (L.inter & 255u) ||
             (L.shared_inter & 255u));
}

uint32_t block_down_ctas(const MoeLayerDev& L) { return (L.hidden + 15u) / 16u; }

}  // namespace

uint32_t moe_barriers_per_layer() { return 3u; }

uint64_t moe_scratch_bytes(const MoeLayerDev& L) {
    const uint64_t slots = L.top_k + 1u;
    uint64_t b = 0;
    b += align256(L.hidden * 4u);                                         // x
    b += align256((L.experts + 1u) * route_splits(L.hidden) * 4u);        // partial
    b += align256(L.experts * 4u);                                        // logits
    b += align256(L.top_k * 4u);                                          // ids
    b += align256(slots * 4u);                                            // weights
    b += align256(slots * max_inter_of(L) * 4u);                          // act
    b += align256(slots * max_inter_of(L) * 4u);                          // act2
    b += align256((L.hidden >> 8) * kFragWords * 4u);                     // xfrag
    b += align256(slots * ((max_inter_of(L) + 255u) >> 8) * kFragWords * 4u);  // afrag
    b += align256(slots * ((max_inter_of(L) + 255u) >> 8) * 4u);         // sbcnt
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
    s.act = reinterpret_cast<float*>(p); p += align256(slots * max_inter_of(L) * 4u);
    s.act2 = reinterpret_cast<float*>(p); p += align256(slots * max_inter_of(L) * 4u);
    s.xfrag = reinterpret_cast<uint32_t*>(p); p += align256((L.hidden >> 8) * kFragWords * 4u);
    s.afrag = reinterpret_cast<uint32_t*>(p);
    p += align256(slots * ((max_inter_of(L) + 255u) >> 8) * kFragWords * 4u);
    s.sbcnt = reinterpret_cast<uint32_t*>(p); p += align256(slots * ((max_inter_of(L) + 255u) >> 8) * 4u);
    s.counter = reinterpret_cast<uint32_t*>(p); p += align256(4u);
    s.status = reinterpret_cast<uint32_t*>(p);
    return s;
}

cudaError_t launch_route_experts(const float* logits, uint32_t E, uint32_t k, uint32_t flavour,
                                 uint32_t normalize, float ew_scale, uint32_t* ids, float* weights,
                                 uint32_t* status, cudaStream_t stream) {
    if (k == 0 || k > E || k > kMaxTopK || E > kMaxExperts) return cudaErrorInvalidValue;
    route_logits_kernel<<<1, kThreads, 0, stream>>>(logits, E, k, flavour, normalize, ew_scale,
                                                    ids, weights, status);
    return cudaGetLastError();
}

static cudaError_t block_impl(const MoeLayerDev& L, const MoeScratch& S, const float* x_in,
                              float* hidden, float* moe_out, const float* next_router,
                              cudaStream_t stream, bool dry_run) {
    if (!layer_valid(L)) return cudaErrorInvalidValue;
    if (!hidden && (!x_in || !moe_out)) return cudaErrorInvalidValue;
    if (hidden && !L.ffn_norm) return cudaErrorInvalidValue;
    const int sms = device_sm_count();
    const uint32_t down_ctas = block_down_ctas(L);
    BlockArgs a{};
    a.L = L;
    a.S = S;
    a.x_in = x_in;
    a.hidden = hidden;
    a.moe_out = moe_out;
    a.next_router = next_router;
    a.down_ctas = down_ctas;
    // Kernel 1 uses enough CTAs to give every router task its own warp.
    const uint32_t tasks = (L.experts + (L.shared_inter ? 1u : 0u)) * route_splits(L.hidden);
    const uint32_t g1 = std::min<uint32_t>(static_cast<uint32_t>(sms), (tasks + kWarps - 1) / kWarps);
    a.m = make_layout(L, down_ctas);
    if (a.m.total > 227u * 1024u) return cudaErrorInvalidValue;
    cudaError_t e = ensure_smem(moe_route_kernel, a.m.total, g_route_smem);
    if (e == cudaSuccess) e = ensure_smem(moe_gate_up_kernel, a.m.total, g_gate_up_smem);
    if (e == cudaSuccess) e = ensure_smem(moe_down_kernel, a.m.total, g_down_smem);
    if (e != cudaSuccess) return e;
    if (mma_path_ok(L)) {
        MmaArgs ma{};
        ma.L = L;
        ma.S = S;
        ma.hidden = hidden;
        ma.moe_out = moe_out;
        ma.next_router = next_router;
        const MmaLayout gl = mma_gate_up_layout(L), dl = mma_down_layout(L);
        if (gl.total > 227u * 1024u || dl.total > 227u * 1024u) return cudaErrorInvalidValue;
        e = ensure_smem(moe_gate_up_mma_kernel, gl.total, g_gate_up_mma_smem);
        if (e == cudaSuccess) e = ensure_smem(moe_down_mma_kernel, dl.total, g_down_mma_smem);
        if (e != cudaSuccess || dry_run) return e;
        const uint32_t T = L.top_k * 2u * (L.inter / 16u);
        const uint32_t g2 = std::max<uint32_t>(static_cast<uint32_t>(sms),
                                               (T + kMmaTilesPerCta - 1) / kMmaTilesPerCta);
        const uint32_t g3 = L.hidden / 16u;
        ma.down_ctas = g3;
        moe_route_kernel<<<g1, kThreads, a.m.total, stream>>>(a);
        ma.m = gl;
        moe_gate_up_mma_kernel<<<g2, kThreads, gl.total, stream>>>(ma);
        ma.m = dl;
        moe_down_mma_kernel<<<g3, kThreads, dl.total, stream>>>(ma);
        return cudaGetLastError();
    }
    if (dry_run) return cudaSuccess;
    moe_route_kernel<<<g1, kThreads, a.m.total, stream>>>(a);
    moe_gate_up_kernel<<<sms, kThreads, a.m.total, stream>>>(a);
    moe_down_kernel<<<down_ctas, kThreads, a.m.total, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_moe_block(const MoeLayerDev& L, const MoeScratch& S, const float* x_in,
                             float* hidden, float* moe_out, const float* next_router,
                             cudaStream_t stream) {
    return block_impl(L, S, x_in, hidden, moe_out, next_router, stream, false);
}

cudaError_t prepare_moe_block(const MoeLayerDev& L) {
    MoeScratch none;
    float dummy = 0.0f;
    cudaError_t e = block_impl(L, none, &dummy, nullptr, &dummy, nullptr, nullptr, true);
    if (e != cudaSuccess) return e;
    const SmemLayout m = make_layout(L, static_cast<uint32_t>(device_sm_count()));
    if (m.total > 227u * 1024u) return cudaErrorInvalidValue;
    return ensure_smem(moe_decode_kernel, m.total, g_decode_smem);
}

uint32_t moe_decode_grid(const MoeLayerDev& L) {
    const uint32_t sms = static_cast<uint32_t>(device_sm_count());
    const SmemLayout m = make_layout(L, sms);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_decode_kernel, kThreads, m.total) !=
            cudaSuccess || per_sm < 1)
        return 0;
    return sms;
}

cudaError_t launch_moe_decode(const MoeLayerDev* layers_dev, const MoeLayerDev& shape,
                              uint32_t first, uint32_t count, const MoeScratch& S, float* hidden,
                              uint32_t barrier_base, uint32_t grid, cudaStream_t stream) {
    if (!layer_valid(shape) || !hidden || count == 0 || grid == 0) return cudaErrorInvalidValue;
    DecodeArgs a{};
    a.layers = layers_dev;
    a.first = first;
    a.count = count;
    a.S = S;
    a.hidden = hidden;
    a.m = make_layout(shape, grid);
    a.barrier_base = barrier_base;
    if (a.m.total > 227u * 1024u) return cudaErrorInvalidValue;
    cudaError_t e = ensure_smem(moe_decode_kernel, a.m.total, g_decode_smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = a.m.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, moe_decode_kernel, a);
}

}  // namespace pokit
