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
#include "pokit_attention.cuh"
#include "pokit_deltablock.cuh"
#include "pokit_kernels.h"
#include "pokit_mma.cuh"
#include "pokit_quant.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>
#include <vector>

namespace pokit {
namespace {

constexpr int kThreads = 384;
constexpr int kWarps = kThreads / 32;
constexpr int kRouteColsPerWarp = 512;
constexpr uint32_t kMaxRouteSplits = 8;       // route_warp: hidden <= 8 * 512
constexpr uint32_t kRouteWarpMaxSlots = 8;    // tensor-core path routing: experts <= 8 * 32
constexpr uint32_t kTailLogitWarps = 4;       // routing tail: warps reading the accumulators
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
    // Generic down rows are staged eight at a time (one warp task = 8 contiguous
    // rows, from a 16-byte boundary).
    if (L.down_type != kQ4_K) s = umax(s, al16(8u * static_cast<uint32_t>(row_bytes(L.down_type, L.inter)) + 16u));
    if (L.shared_inter) {
        if (!fast_pair(L.shared_gate_type, L.shared_up_type))
            s = umax(s, umax(al16(static_cast<uint32_t>(row_bytes(L.shared_gate_type, L.hidden))),
                             al16(static_cast<uint32_t>(row_bytes(L.shared_up_type, L.hidden)))));
        if (L.shared_down_type != kQ4_K)
            s = umax(s, al16(8u * static_cast<uint32_t>(row_bytes(L.shared_down_type, L.shared_inter)) + 16u));
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

// Layout of the route kernel: input, logits, reductions, routes and the
// router partials only.
__host__ __device__ inline SmemLayout route_layout(const MoeLayerDev& L) {
    SmemLayout m{};
    uint32_t off = 0;
    m.xs = off; off += al16(L.hidden * 4u);
    m.lg = off; off += al16(L.experts * 4u);
    m.red = off; off += al16(64u * 8u);
    m.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    m.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    m.act_plain = off; off += al16((L.experts + 1u) * route_splits(L.hidden) * 4u);
    m.xp = m.gsum = m.act_prep = m.act_gsum = m.ybuf = m.stage = off;
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
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
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
           L.top_k <= static_cast<uint32_t>(kWarps) && (L.inter % 256u) == 0 &&
           route_splits(L.hidden) <= kMaxRouteSplits && L.experts <= 32u * kRouteWarpMaxSlots;
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
template <uint32_t kSlots>
__device__ void route_select_regs(const MoeLayerDev& L, const float (&lgv)[kSlots], float shared_logit,
                                  uint32_t* sel_id, float* sel_w, uint32_t* status, bool writer,
                                  const MoeScratch& S);

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
    if (L.experts <= 32u * 16u && L.top_k < 32u) {
        // One warp selects from logits held in registers (k rounds of a warp
        // maximum); the rest of the CTA waits.
        if (threadIdx.x < 32) {
            const uint32_t lane = threadIdx.x;
            if (L.experts <= 32u * 8u) {
                float lgv[8];
#pragma unroll
                for (uint32_t i = 0; i < 8; ++i) lgv[i] = lane + 32u * i < L.experts ? s.lg[lane + 32u * i] : 0.0f;
                route_select_regs<8>(L, lgv, shared_logit, s.sel_id, s.sel_w, status, writer, S);
            } else {
                float lgv[16];
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) lgv[i] = lane + 32u * i < L.experts ? s.lg[lane + 32u * i] : 0.0f;
                route_select_regs<16>(L, lgv, shared_logit, s.sel_id, s.sel_w, status, writer, S);
            }
        }
        __syncthreads();
        return;
    }
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

// R2 in one warp, from logits already in shared memory.  Same selection as
// phase_route: expert f precedes e when its logit is larger, ties to the
// lower id.  Lane l holds the logits of experts l, l + 32, ... in registers;
// each of the k rounds takes the warp maximum of the order-preserving logit
// bits (redux.sync) and, among the lanes at that maximum, the lowest id.  With
// renormalisation the softmax denominator cancels and is not formed: the
// weights are exp(l - max) / sum over the selection (the reference's two
// divisions folded, equal to rounding).  Writes sel_id[0..k), sel_w[0..k]
// (sel_w[k] = shared gate) and, for `writer`, logits, ids and weights to S.
// Requires E <= 32 * kSlots and top_k < 32.
__device__ __forceinline__ uint32_t route_ord(float v) {
    const uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);      // -0 ranks as +0
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <uint32_t kSlots>
__device__ void route_select_regs(const MoeLayerDev& L, const float (&lgv)[kSlots], float shared_logit,
                                  uint32_t* sel_id, float* sel_w, uint32_t* status, bool writer,
                                  const MoeScratch& S) {
    const int lane = threadIdx.x & 31;
    const uint32_t E = L.experts, k = L.top_k;
    int bad = 0;
#pragma unroll
    for (uint32_t i = 0; i < kSlots; ++i)
        if (lane + 32u * i < E) bad |= !isfinite(lgv[i]);
    bad = __any_sync(0xffffffffu, bad);
    if (writer) {
#pragma unroll
        for (uint32_t i = 0; i < kSlots; ++i)
            if (lane + 32u * i < E) S.logits[lane + 32u * i] = lgv[i];
    }
    if (bad) {
        if (lane == 0 && status) atomicOr(status, kStatusNonFiniteLogits);
        if (static_cast<uint32_t>(lane) < k) { sel_id[lane] = lane; sel_w[lane] = 0.0f; }
        if (static_cast<uint32_t>(lane) == k) sel_w[k] = 0.0f;
    } else {
        // Order-preserving keys; 0 marks a taken or absent slot (a real key
        // has bit 31 set or is the complement of a negative float, never 0
        // for finite logits).
        uint32_t ord[kSlots];
#pragma unroll
        for (uint32_t i = 0; i < kSlots; ++i) ord[i] = lane + 32u * i < E ? route_ord(lgv[i]) : 0u;
        uint32_t my_id = 0;
        float my_v = 0.0f, mx = 0.0f;
        for (uint32_t r = 0; r < k; ++r) {
            uint32_t best_ord = 0, best_e = 0xffffffffu;
#pragma unroll
            for (uint32_t i = 0; i < kSlots; ++i)
                if (ord[i] > best_ord) { best_ord = ord[i]; best_e = lane + 32u * i; }
            const uint32_t top = __reduce_max_sync(0xffffffffu, best_ord);
            // The lowest id among the lanes at the maximum.
            const uint32_t win = __reduce_min_sync(0xffffffffu, best_ord == top ? best_e : 0xffffffffu);
#pragma unroll
            for (uint32_t i = 0; i < kSlots; ++i)
                if (lane + 32u * i == win) ord[i] = 0u;
            // The logit back from its key.
            const float v = __uint_as_float((top & 0x80000000u) ? (top & 0x7fffffffu) : ~top);
            if (r == 0) mx = v;
            if (static_cast<uint32_t>(lane) == r) { my_id = win; my_v = v; }
        }
        double den_d = 0.0;
        float den_f = 0.0f;
        if (!L.normalize) {
#pragma unroll
            for (uint32_t i = 0; i < kSlots; ++i)
                if (lane + 32u * i < E) {
                    if (L.flavour == 0) den_d += exp(static_cast<double>(lgv[i] - mx));
                    else den_f += expf(lgv[i] - mx);
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                if (L.flavour == 0) den_d += __shfl_xor_sync(0xffffffffu, den_d, o);
                else den_f += __shfl_xor_sync(0xffffffffu, den_f, o);
            }
        }
        float p = 0.0f;
        if (static_cast<uint32_t>(lane) < k) {
            if (L.normalize) p = expf(my_v - mx);
            else p = L.flavour == 0 ? static_cast<float>(exp(static_cast<double>(my_v - mx)) / den_d)
                                    : expf(my_v - mx) / den_f;
        }
        float sum = p;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        bool invalid = L.flavour == 1 && !L.normalize && (!isfinite(den_f) || den_f <= 0.0f);
        if (L.normalize) {
            if (L.flavour == 1 && (!isfinite(sum) || sum <= 0.0f)) invalid = true;
            p *= 1.0f / sum;                 // one division for the warp
        }
        if (invalid && lane == 0 && status) atomicOr(status, kStatusBadSoftmax);
        if (static_cast<uint32_t>(lane) < k) {
            sel_id[lane] = my_id;
            sel_w[lane] = invalid ? 0.0f : (L.flavour == 0 ? p : p * L.expert_weights_scale);
        }
        if (static_cast<uint32_t>(lane) == k) sel_w[k] = L.shared_inter ? sigmoid_qwen35(shared_logit) : 0.0f;
    }
    __syncwarp();
    if (writer) {
        if (static_cast<uint32_t>(lane) < k) S.ids[lane] = sel_id[lane];
        if (static_cast<uint32_t>(lane) <= k) S.weights[lane] = sel_w[lane];
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
    warp_stage_row<2>(row_g, rb, stage, lane);  // a small batch: the kernel is at its register limit
    __syncwarp();
    float acc = warp_sum(lane_row_dot_any(type, stage, cols, xs, lane));
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
            // The task's (up to) 8 rows staged together: one memory latency,
            // then one warp-wide dot per row.
            // The rows of a down matrix are contiguous: one span of nr rows.
            uint8_t* my_stage = s.stage + warp * s.m.stage_bytes;
            const uint64_t rb = row_bytes(m.down_type, m.rows);
            const uint32_t row0 = r0 + o * 8u;
            const uint32_t nr = min(8u, r1 - row0);
            const uint32_t delta = warp_stage_span(m.down + row0 * rb, static_cast<uint32_t>(nr * rb), my_stage, lane);
            __syncwarp();
            const float* xa = s.act_plain + slot * mi;
            for (uint32_t rr = 0; rr < nr; ++rr) {
                const float acc =
                    warp_sum(lane_row_dot_any(m.down_type, my_stage + delta + rr * rb, m.rows, xa, lane));
                if (lane == 0) s.ybuf[slot * cap + (row0 + rr - r0)] = acc;
            }
            __syncwarp();
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

// Returns true in every thread of the CTA that arrives last at `count`
// (after all of this CTA's global writes), and resets the counter there.
__device__ __forceinline__ bool last_cta_arrival(uint32_t* count, uint32_t* flag) {
    __syncthreads();
    if (threadIdx.x == 0) *flag = atomic_add_acq_rel_gpu(count, 1u) == gridDim.x - 1u ? 1u : 0u;
    __syncthreads();
    const bool last = *flag != 0u;
    if (last && threadIdx.x == 0) *count = 0u;
    return last;
}

// Kernel 1 of a block: R0 + R1 (CTA 0 also publishes x), then R2 in the last CTA.
__global__ void __launch_bounds__(kThreads, 1) moe_route_kernel(BlockArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    Shared s = carve(smem, a.m);
    const uint32_t gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
    RouterRegs rr;
    router_issue(a.L, gw, nw, rr);
    // The router weights' loads above may overlap the previous kernel (a
    // programmatic dependent launch); the hidden state is read after it ends.
    grid_dep_wait();
    grid_dep_launch();
    phase_input(a.L, a.hidden, a.x_in, s);
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < a.L.hidden; i += kThreads) a.S.x[i] = s.xs[i];
    router_finish(a.L, gw, nw, rr, s, a.S.partial);
    // R2 once per block: the CTA that finishes last sums the partials and
    // routes; the gate/up kernel's CTAs read the routes it publishes.
    __shared__ uint32_t last;
    __threadfence();
    if (last_cta_arrival(a.S.route_count, &last)) phase_route(a.L, a.S.partial, s, a.S.status, true, a.S);
}

// Kernel 2: G, on the routes the route kernel's last CTA published.
__global__ void __launch_bounds__(kThreads, 1) moe_gate_up_kernel(BlockArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    Shared s = carve(smem, a.m);
    grid_dep_wait();      // routes and input of the route kernel
    grid_dep_launch();
    for (uint32_t r = threadIdx.x; r <= a.L.top_k; r += kThreads) {
        if (r < a.L.top_k) s.sel_id[r] = __ldcg(a.S.ids + r);
        s.sel_w[r] = __ldcg(a.S.weights + r);
    }
    copy_coherent(a.S.x, s.xs, a.L.hidden);
    __syncthreads();
    phase_gate_up(a.L, s, a.S.act, max_inter_of(a.L), blockIdx.x, gridDim.x, a.down_ctas);
}

// Kernel 3: D.
__global__ void __launch_bounds__(kThreads, 1) moe_down_kernel(BlockArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    Shared s = carve(smem, a.m);
    for (uint32_t r = threadIdx.x; r <= a.L.top_k; r += kThreads) {
        if (r < a.L.top_k) s.sel_id[r] = __ldcg(a.S.ids + r);
        s.sel_w[r] = __ldcg(a.S.weights + r);
    }
    __syncthreads();
    bool ok = true;
    const uint64_t nrb = static_cast<uint64_t>(a.L.experts) * a.L.hidden * 4u;
    // The routes were published two kernels back; the first task's weight loads
    // go out before the wait for the gate/up kernel's act.
    phase_down(a.L, s, a.S.act, max_inter_of(a.L), blockIdx.x, gridDim.x, a.hidden, a.moe_out,
               a.next_router, nrb, [] { grid_dep_wait(); grid_dep_launch(); return true; }, ok);
}

// Routing of standalone logits vectors (pokit_cuda_route_experts; the
// batched MoE forward routes one row per token).
__global__ void __launch_bounds__(kThreads, 1)
route_logits_kernel(const float* __restrict__ logits, uint32_t E, uint32_t k, uint32_t flavour,
                    uint32_t normalize, float ew_scale, uint32_t* ids, float* weights,
                    uint32_t* status, uint32_t splits) {
    __shared__ float lg[kMaxExperts];
    __shared__ double red[64];
    __shared__ uint32_t sel_id[kMaxTopK + 1];
    __shared__ float sel_w[kMaxTopK + 1];
    grid_dep_wait();      // logits of the previous kernel (programmatic launch; no-op otherwise)
    grid_dep_launch();
    Shared s{};
    s.red = red;
    s.sel_id = sel_id;
    s.sel_w = sel_w;
    // One CTA per logits row (a batch of tokens routes row by row); a row may
    // arrive as `splits` partial rows (slices of the hidden dimension, split s
    // at logits + (s * rows + row) * E), added here in slice order.
    const size_t rows = gridDim.x;
    ids += static_cast<size_t>(blockIdx.x) * k;
    weights += static_cast<size_t>(blockIdx.x) * k;
    for (uint32_t e = threadIdx.x; e < E; e += kThreads) {
        float v = logits[static_cast<size_t>(blockIdx.x) * E + e];
        for (uint32_t sp = 1; sp < splits; ++sp) v += logits[(sp * rows + blockIdx.x) * E + e];
        lg[e] = v;
    }
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
    extern __shared__ __align__(128) uint8_t smem[];
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
// Tensor-core path: every routed matrix Q4_K, no shared expert.  Two
// launches per block; the router runs inside them:
//   partials  (only for a block whose predecessor did not produce them) CTA c
//             adds sum_{j in [16c, 16c+16)} W_r[e][j] * x'[j] to logit e,
//             x' = ffn_norm * hidden (decode) or x_in (forward).
//   gate_up   every CTA sums the partials in chunk order, applies the rms
//             scale (linearity: W (s x') = s (W x')), selects the routes in
//             one warp (CTA 0 publishes them) and builds the fragment records
//             of x'; CTA b then owns row groups [3b, 3b+3) of the k * I/16
//             (slot, 16-row) groups, four warps per group computing gate and
//             up over the two halves of the superblocks; act = silu(s g) * (s u).
//   down      CTA b owns output rows [16b, 16b+16): it requests its k down
//             tiles, builds the activation fragments of every slot, runs the
//             (slot, superblock) units over all warps and combines the rows
//             in route order into the output (or the residual).  In a decode
//             chain it then writes the next block's router partials for its
//             16 new hidden rows.
// ---------------------------------------------------------------------------
constexpr uint32_t kGuGroups = kWarps / 4;
constexpr uint32_t kPartRows = 16;             // hidden rows per router-partial chunk

__host__ __device__ inline uint32_t al128(uint32_t v) { return (v + 127u) & ~127u; }

// Router partial dots are summed across CTAs exactly and independently of
// arrival order: each float m * 2^ex is added to a carry-save fixed-point
// accumulator of kRaccLimbs 64-bit limbs, limb i holding bits
// [32 i + kRaccBase, 32 i + kRaccBase + 32) with 31 bits of headroom for
// carries (at most 2^31 additions), resolved when the sum is read.  The
// 24-bit mantissa lands in at most two adjacent limbs; bits below 2^kRaccBase
// are dropped (below 1e-19 in absolute value).  Non-finite partials set a flag.
constexpr int kRaccLimbs = 8;                  // covers 2^-64 .. 2^192
constexpr int kRaccBase = -64;
__device__ __forceinline__ void racc_add(unsigned long long* limbs, uint32_t* bad, float p) {
    const uint32_t b = __float_as_uint(p);
    const uint32_t eb = (b >> 23) & 0xffu;
    if (eb == 0xffu) {
        atomicOr(bad, 1u);
        return;
    }
    uint32_t m = b & 0x7fffffu;
    int ex;
    if (eb == 0u) {
        if (m == 0u) return;
        ex = -149;
    } else {
        m |= 0x800000u;
        ex = static_cast<int>(eb) - 150;
    }
    int pos = ex - kRaccBase;
    if (pos < 0) {
        if (pos <= -24) return;
        m >>= -pos;
        pos = 0;
        if (m == 0u) return;
    }
    const int i = pos >> 5, o = pos & 31;
    long long v = static_cast<long long>(m) << o;            // below 2^55
    if (b >> 31) v = -v;
    const unsigned long long lo = static_cast<unsigned long long>(v & 0xffffffffll);
    const long long hi = v >> 32;                             // floor division
    if (lo) atomicAdd(limbs + i, lo);
    if (hi) atomicAdd(limbs + i + 1, static_cast<unsigned long long>(hi));
}

// racc_add with one atomic: the whole signed m 2^o (|v| < 2^55) into limb i.
// The limbs then hold larger values (up to units x 2^55 < 2^63 for at most
// 256 adding units) but the same integer sum over limbs; racc_value reads
// either form, rounding a limb beyond 2^53 to double (relative 2^-53), which
// stays far below a float's unit in the last place unless the exact sum
// cancels to about 2^-29 of its largest limb term.  The value still depends
// only on the limbs, not on the order of the additions.
__device__ __forceinline__ void racc_add1(unsigned long long* limbs, uint32_t* bad, float p) {
    const uint32_t b = __float_as_uint(p);
    const uint32_t eb = (b >> 23) & 0xffu;
    if (eb == 0xffu) {
        atomicOr(bad, 1u);
        return;
    }
    uint32_t m = b & 0x7fffffu;
    int ex;
    if (eb == 0u) {
        if (m == 0u) return;
        ex = -149;
    } else {
        m |= 0x800000u;
        ex = static_cast<int>(eb) - 150;
    }
    int pos = ex - kRaccBase;
    if (pos < 0) {
        if (pos <= -24) return;
        m >>= -pos;
        pos = 0;
        if (m == 0u) return;
    }
    long long v = static_cast<long long>(m) << (pos & 31);
    if (b >> 31) v = -v;
    atomicAdd(limbs + (pos >> 5), static_cast<unsigned long long>(v));
}

// The accumulated value of the limbs (as loaded): Horner's rule in double from
// the top limb, without resolving carries first.  Each step is exact until
// the running value passes 2^53, after which every step rounds relative to
// the value itself, so the float result is within one unit in the last place
// of the exact sum and depends only on the limbs (not on arrival order).
__device__ __forceinline__ float racc_value(const ulonglong2 (&v)[kRaccLimbs / 2]) {
    double d = static_cast<double>(static_cast<long long>(v[kRaccLimbs / 2 - 1].y));
#pragma unroll
    for (int i = kRaccLimbs - 2; i >= 0; --i) {
        const unsigned long long li = (i & 1) ? v[i / 2].y : v[i / 2].x;
        d = fma(d, 4294967296.0, static_cast<double>(static_cast<long long>(li)));
    }
    // 2^kRaccBase from its exponent bits.
    return static_cast<float>(d * __longlong_as_double(static_cast<long long>(1023 + kRaccBase) << 52));
}

// Shared memory of the routing tail (run by the last CTA of the partials
// kernel or of a down kernel), at byte offset `base`.
struct TailLayout {
    uint32_t lg, sel_id, sel_w, stage, end;
};
__host__ __device__ inline TailLayout tail_layout(const MoeLayerDev& L, uint32_t base) {
    TailLayout t{};
    uint32_t off = base;
    t.lg = off; off += al16(L.experts * 4u);
    t.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    t.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    t.stage = off; off += (kWarps - kTailLogitWarps) * 1024u;
    t.end = off;
    return t;
}

struct MmaLayout {
    uint32_t bars, recs, sel_id, sel_w, part, comb, hrow, tiles;
    TailLayout tail;
    uint32_t total, nsb, boxes;      // boxes: superblock boxes (and mbarriers) per warp or slot
};

__host__ __device__ inline MmaLayout mma_gate_up_layout(const MoeLayerDev& L) {
    MmaLayout m{};
    const uint32_t nsb = L.hidden >> 8, half_sb = (nsb + 1u) / 2u;
    m.nsb = nsb;
    m.boxes = half_sb;
    uint32_t off = 0;
    m.bars = off; off += al16(kWarps * half_sb * 8u);
    m.recs = off; off += al16(nsb * kFragWords * 4u);
    m.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    m.sel_w = off;
    m.part = off; off += al16(kWarps * 16u * 4u);
    m.comb = m.hrow = off;
    off = al128(off);
    m.tiles = off; off += kWarps * half_sb * kBoxBytes;
    m.total = off;
    return m;
}

// The down kernel's routing tail reuses the record space.
__host__ __device__ inline MmaLayout mma_down_layout(const MoeLayerDev& L, const MoeLayerDev& next) {
    MmaLayout m{};
    const uint32_t nsb = L.inter >> 8, k = L.top_k;
    m.nsb = nsb;
    m.boxes = nsb;
    uint32_t off = 0;
    m.bars = off; off += al16(k * nsb * 8u);
    m.recs = off;
    m.tail = tail_layout(next, off);
    off = umax(off + al16(k * nsb * kFragWords * 4u), m.tail.end);
    m.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    m.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    m.part = off; off += al16(k * nsb * 16u * 4u);
    m.comb = off; off += al16(k * 16u * 4u);
    m.hrow = off; off += al16(2u * kPartRows * 4u);
    off = al128(off);
    m.tiles = off; off += k * nsb * kBoxBytes;
    m.total = off;
    return m;
}

struct MmaArgs {
    // 3-D tensor maps (byte column, row, expert) of the block's Q4_K gate, up
    // and down tensors; boxes of 144 bytes x 16 rows.
    CUtensorMap tm_gate, tm_up, tm_down;
    MoeLayerDev L;
    MoeLayerDev next;           // decode chain: the following block (valid when has_next)
    MoeScratch S;
    const float* x_in;          // forward: the normalised input
    float* hidden;              // decode: the residual stream (rms_norm'd on the way in)
    float* moe_out;             // forward: the block output
    uint32_t has_next;          // the down kernel routes `next` (partials, tail)
    MmaLayout m;
};

// Router weights W_r[e][16c .. 16c+16) and their dot with x'[0..16) in row
// order.
struct RouterSlice {
    float4 w[4];
};
__device__ __forceinline__ RouterSlice router_slice(const float* router, uint32_t H, uint32_t e, uint32_t c) {
    const float4* p = reinterpret_cast<const float4*>(router + static_cast<uint64_t>(e) * H + c * kPartRows);
    return RouterSlice{{__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3)}};
}
__device__ __forceinline__ float router_dot16(const RouterSlice& r, const float* xr) {
    const float wv[16] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w, r.w[1].x, r.w[1].y, r.w[1].z, r.w[1].w,
                          r.w[2].x, r.w[2].y, r.w[2].z, r.w[2].w, r.w[3].x, r.w[3].y, r.w[3].z, r.w[3].w};
    float p = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) p = fmaf(wv[i], xr[i], p);
    return p;
}

// A read-only 16-byte load issued where it stands: the compiler keeps the
// order of volatile asm, so the load is not sunk to its first use (which
// would expose its latency in a later phase).
__device__ __forceinline__ float4 ldg_f4_issue_here(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ float ldcg_f32_issue_here(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ RouterSlice router_slice_issue_here(const float* router, uint32_t H, uint32_t e,
                                                               uint32_t c) {
    const float* p = router + static_cast<uint64_t>(e) * H + c * kPartRows;
    return RouterSlice{{ldg_f4_issue_here(p), ldg_f4_issue_here(p + 4), ldg_f4_issue_here(p + 8),
                        ldg_f4_issue_here(p + 12)}};
}


// The routing tail's selection in warp 0 (lane l owns experts l, l + 32, ...):
// the rms scale from the per-chunk sums of squares (hidden_mode), the exact
// logits from the accumulators (left zero), then route_select_regs.  The
// selection order does not depend on the scale, which only enters the
// weights.  Writes S.scale.
// The routing tail of block L, run by the one CTA that finished last after
// every chunk added its router partials.  Warps 0..kTailLogitWarps-1 read the
// accumulators (one expert per lane, leaving them zero) into exact-order-free
// logits in shared memory, warp 0 also the per-chunk sums of squares for the
// rms scale (1 for a normalised input); after a barrier of those warps, warp
// 0 selects the routes and publishes them with the scale (S.ids / S.weights /
// S.logits / S.scale).  The other warps build the fragment records of
// x' = ffn_norm * hidden (or x_in) for the gate/up kernel (S.xrec).  The
// selection order does not depend on the scale, which only enters the
// weights.
__device__ void route_tail(const MoeLayerDev& L, const MoeScratch& S, const float* x, bool hidden_mode,
                           uint8_t* smem, const TailLayout& t) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp < static_cast<int>(kTailLogitWarps)) {
        float* lg = reinterpret_cast<float*>(smem + t.lg);
        const uint32_t E = L.experts;
        __shared__ float tail_scale;
        __shared__ uint32_t tail_bad;
        if (warp == 0) {
            const uint32_t chunks = L.hidden / kPartRows;
            float sq = 0.0f;
            for (uint32_t c = lane; c < chunks; c += 32) sq += __ldcg(S.rsq + c);
            uint32_t bad = lane == 0 ? __ldcg(S.rbad) : 0u;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            if (lane == 0) {
                // rms_norm scale (src/rms_norm.cpp:20-26).
                tail_scale = hidden_mode ? 1.0f / sqrtf(sq / static_cast<float>(L.hidden) + L.rms_eps) : 1.0f;
                tail_bad = bad;
                if (bad) *S.rbad = 0u;
            }
        }
        for (uint32_t e0 = warp * 32u; e0 < E; e0 += kTailLogitWarps * 32u) {
            const uint32_t e = e0 + lane;
            ulonglong2 limbs[kRaccLimbs / 2];
            ulonglong2* p = reinterpret_cast<ulonglong2*>(S.racc + static_cast<uint64_t>(e) * kRaccLimbs);
#pragma unroll
            for (int h = 0; h < kRaccLimbs / 2; ++h) limbs[h] = e < E ? __ldcg(p + h) : make_ulonglong2(0ull, 0ull);
            if (e < E) {
#pragma unroll
                for (int h = 0; h < kRaccLimbs / 2; ++h) p[h] = make_ulonglong2(0ull, 0ull);
                lg[e] = racc_value(limbs);
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kTailLogitWarps * 32u) : "memory");
        if (warp != 0) return;
        uint32_t* sel_id = reinterpret_cast<uint32_t*>(smem + t.sel_id);
        float* sel_w = reinterpret_cast<float*>(smem + t.sel_w);
        const float scale = tail_scale;
        const bool bad = tail_bad != 0u;
        const auto select = [&](auto slots) {
            constexpr uint32_t kSlots = decltype(slots)::value;
            float lgv[kSlots];
#pragma unroll
            for (uint32_t i = 0; i < kSlots; ++i) {
                const uint32_t e = lane + 32u * i;
                lgv[i] = e < E ? (bad ? __int_as_float(0x7fc00000) : lg[e] * scale) : 0.0f;
            }
            route_select_regs<kSlots>(L, lgv, 0.0f, sel_id, sel_w, S.status, true, S);
        };
        if (E <= 128u) select(std::integral_constant<uint32_t, 4>{});
        else select(std::integral_constant<uint32_t, kRouteWarpMaxSlots>{});
        if (lane == 0) *S.scale = scale;
        return;
    }
    const uint32_t nsb = L.hidden >> 8, builders = static_cast<uint32_t>(kWarps) - kTailLogitWarps;
    const uint32_t b = static_cast<uint32_t>(warp) - kTailLogitWarps;
    float* stage = reinterpret_cast<float*>(smem + t.stage) + b * 256u;
    for (uint32_t q = b; q < nsb; q += builders) {
        float hv[8], nv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t i = q * 256u + 32u * j + lane;
            hv[j] = __ldcg(x + i);
            nv[j] = hidden_mode ? __ldg(L.ffn_norm + i) : 1.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) stage[32 * j + lane] = hidden_mode ? nv[j] * hv[j] : hv[j];
        __syncwarp();
        q4k_frag_superblock(stage, S.xrec + q * kFragWords, lane);
        __syncwarp();
    }
}


// Router partials of block L for the first block of a chain or a single
// block, then its routing tail.
__global__ void __launch_bounds__(kThreads, 1) moe_partials_kernel(const __grid_constant__ MmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float xr[kPartRows];
    __shared__ uint32_t flag;
    const MoeLayerDev& L = a.L;
    const uint32_t c = blockIdx.x, j0 = c * kPartRows;
    const float* x = a.hidden ? a.hidden : a.x_in;
    grid_dep_launch();
    if (threadIdx.x < 32) {
        const uint32_t r = threadIdx.x & 15u;
        const float h = __ldcg(x + j0 + r);
        float sq = threadIdx.x < 16 ? h * h : 0.0f;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (threadIdx.x < 16) xr[r] = a.hidden ? __ldg(L.ffn_norm + j0 + r) * h : h;
        if (threadIdx.x == 0) a.S.rsq[c] = sq;
    }
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < L.experts; e += kThreads)
        racc_add(a.S.racc + static_cast<uint64_t>(e) * kRaccLimbs, a.S.rbad,
                 router_dot16(router_slice(L.router, L.hidden, e, c), xr));
    if (last_cta_arrival(a.S.route_count, &flag))
        route_tail(L, a.S, x, a.hidden != nullptr, smem, a.m.tail);
}

// Kernel 2 (tensor-core path): act = silu(s g) * (s u) for the CTA's row
// groups, with the routes, s and the x records from the routing tail.  Each
// warp's superblocks arrive in their own cp.async group and are multiplied
// as they land.
__global__ void __launch_bounds__(kThreads, 1) moe_gate_up_mma_kernel(const __grid_constant__ MmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const MoeLayerDev& L = a.L;
    const MmaLayout& m = a.m;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + m.bars);
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + m.recs);
    uint32_t* sel_id = reinterpret_cast<uint32_t*>(smem + m.sel_id);
    float* part = reinterpret_cast<float*>(smem + m.part);
    uint8_t* tiles = smem + m.tiles;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t H = L.hidden, I = L.inter, nsb = m.nsb, per_slot = I / 16u;
    const uint32_t groups = L.top_k * per_slot;

    if (lane == 0) {
        for (uint32_t i = 0; i < m.boxes; ++i) mbar_init(&bars[warp * m.boxes + i], 1);
        mbar_fence_init();
    }
    // Launched early behind the routing tail of the previous kernel: nothing
    // above reads its results.  The down kernel may launch once every CTA is
    // past this point (the routes it reads are then complete).
    grid_dep_wait();
    grid_dep_launch();
    for (uint32_t p = tid; p < nsb * (kFragWords / 4u); p += kThreads)
        cp_async16(recs + p * 4u, a.S.xrec + p * 4u);
    cp_async_commit();
    for (uint32_t r = tid; r < L.top_k; r += kThreads) sel_id[r] = __ldcg(a.S.ids + r);
    const float scale = __ldcg(a.S.scale);
    __syncthreads();

    const uint32_t rg = blockIdx.x * kGuGroups + static_cast<uint32_t>(warp >> 2);
    const uint32_t mat = (warp >> 1) & 1, half = warp & 1;
    const uint32_t split = (nsb + 1u) / 2u;
    const uint32_t sb0 = half ? split : 0u, sb1 = half ? nsb : split;
    const uint32_t nmine = (rg < groups && sb1 > sb0) ? sb1 - sb0 : 0u;
    uint8_t* mytile = tiles + warp * m.boxes * kBoxBytes;
    uint64_t* mybars = bars + warp * m.boxes;
    // One TMA box per superblock of the warp's half, each on its own
    // mbarrier: the mma on superblock i overlaps the copies of i+1...
    if (nmine && lane == 0) {
        const uint32_t slot = rg / per_slot, row0 = (rg % per_slot) * 16u;
        const int id = static_cast<int>(sel_id[slot]);
        const CUtensorMap* map = mat ? &a.tm_up : &a.tm_gate;
        for (uint32_t i = 0; i < nmine; ++i) {
            mbar_expect_tx(&mybars[i], kBoxBytes);
            tma_box_3d(mytile + i * kBoxBytes, map, static_cast<int>((sb0 + i) * 144u), static_cast<int>(row0), id,
                       &mybars[i]);
        }
    }
    // Warm L2 with the next block's router slice the down CTA with this index
    // reads (16 floats of every expert row).
    if (a.has_next && blockIdx.x < H / kPartRows)
        for (uint32_t e = tid; e < a.next.experts; e += kThreads)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(a.next.router + static_cast<uint64_t>(e) * H +
                                                          blockIdx.x * kPartRows));
    // Warm L2 with the down rows of the down CTA with this index.
    if (blockIdx.x < H / 16u && tid < static_cast<int>(L.top_k)) {
        const uint64_t rd = static_cast<uint64_t>(I >> 8) * 144u;
        prefetch_l2_range(L.down + static_cast<uint64_t>(sel_id[tid]) * L.down_slice +
                              static_cast<uint64_t>(blockIdx.x) * 16u * rd,
                          16u * rd);
    }
    cp_async_wait_all();      // the x records
    __syncthreads();
    const int g = lane >> 2;
    const auto wait_box = [&](uint32_t i) {
        if (!mbar_wait(&mybars[i], 0)) {
            if (lane == 0) atomicOr(a.S.status, kStatusWaitTimeout);
            mbar_wait(&mybars[i], 0);          // the copy may still land: wait once more
        }
    };
    // Superblocks two at a time with separate accumulators: two independent
    // dependency chains per warp.
    float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
    uint32_t i = 0;
    for (; i + 2 <= nmine; i += 2) {
        wait_box(i);
        wait_box(i + 1);
        const uint8_t* b0 = mytile + i * kBoxBytes;
        const uint8_t* b1 = b0 + kBoxBytes;
        q4k_mma_superblock(b0 + g * 144u, b0 + (g + 8) * 144u, recs + (sb0 + i) * kFragWords, acc0, acc1);
        q4k_mma_superblock(b1 + g * 144u, b1 + (g + 8) * 144u, recs + (sb0 + i + 1) * kFragWords, acc2, acc3);
    }
    if (i < nmine) {
        wait_box(i);
        const uint8_t* b0 = mytile + i * kBoxBytes;
        q4k_mma_superblock(b0 + g * 144u, b0 + (g + 8) * 144u, recs + (sb0 + i) * kFragWords, acc0, acc1);
    }
    acc0 = quad_sum(acc0 + acc2);
    acc1 = quad_sum(acc1 + acc3);
    if ((lane & 3) == 0) {
        part[warp * 16 + g] = acc0;
        part[warp * 16 + g + 8] = acc1;
    }
    __syncthreads();
    if (tid < static_cast<int>(kGuGroups * 16u)) {
        const uint32_t gl = tid >> 4, r = tid & 15, rgx = blockIdx.x * kGuGroups + gl;
        if (rgx < groups) {
            const float gv = part[(gl * 4 + 0) * 16 + r] + part[(gl * 4 + 1) * 16 + r];
            const float uv = part[(gl * 4 + 2) * 16 + r] + part[(gl * 4 + 3) * 16 + r];
            const uint32_t slot = rgx / per_slot, row0 = (rgx % per_slot) * 16u;
            const float av = silu_mul(gv * scale, uv * scale, L.flavour);
            for (uint32_t cp = 0; cp < a.S.rep; ++cp)
                a.S.actr[static_cast<uint64_t>(cp) * L.top_k * I + slot * I + row0 + r] = av;
        }
    }
}

// Kernel 3 (tensor-core path): 16 rows of the block output per CTA; in a
// decode chain also the next block's router partials for those rows, and in
// the CTA that finishes last the next block's routing tail.
// At most 88 registers a thread: with the gate/up kernel's 80 both CTAs fit
// one SM's register file, so the down grid can start behind the gate/up one.
__global__ void __maxnreg__(88) moe_down_mma_kernel(const __grid_constant__ MmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t flag;
    const MoeLayerDev& L = a.L;
    const MmaLayout& m = a.m;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + m.bars);
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + m.recs);
    uint32_t* sel_id = reinterpret_cast<uint32_t*>(smem + m.sel_id);
    float* sel_w = reinterpret_cast<float*>(smem + m.sel_w);
    float* part = reinterpret_cast<float*>(smem + m.part);
    float* hrow = reinterpret_cast<float*>(smem + m.hrow);
    uint8_t* tiles = smem + m.tiles;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t k = L.top_k, nsb = m.nsb, H = L.hidden;
    const uint32_t units = k * nsb;
    const uint32_t j0 = blockIdx.x * 16u;
    const MoeLayerDev& N = a.next;
    // Launched early behind the gate/up kernel: the routes, the residual and
    // the weights are complete; act is read after grid_dep_wait.  The next
    // gate/up kernel may launch right away (it waits for this grid).
    grid_dep_launch();

    for (uint32_t r = tid; r < k; r += kThreads) {
        sel_id[r] = __ldcg(a.S.ids + r);
        sel_w[r] = __ldcg(a.S.weights + r);
    }
    if (tid == 0) {
        for (uint32_t i = 0; i < units; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    const float resid = (!a.moe_out && tid < 16) ? __ldcg(a.hidden + j0 + tid) : 0.0f;
    const float nnorm = (a.has_next && tid < 16) ? __ldg(N.ffn_norm + j0 + tid) : 0.0f;
    // The next block's router weights for these 16 rows (thread e; E above
    // the block size loads the rest at the end).
    const bool slice_now = a.has_next && static_cast<uint32_t>(tid) < N.experts;
    RouterSlice rs{};
    if (slice_now) rs = router_slice(N.router, H, tid, blockIdx.x);
    __syncthreads();
    // Box (slot, superblock) u = slot * nsb + sb on mbarrier u.
    if (static_cast<uint32_t>(warp) < k && lane == 0) {
        const int id = static_cast<int>(sel_id[warp]);
        for (uint32_t sb = 0; sb < nsb; ++sb) {
            const uint32_t u = warp * nsb + sb;
            mbar_expect_tx(&bars[u], kBoxBytes);
            tma_box_3d(tiles + u * kBoxBytes, &a.tm_down, static_cast<int>(sb * 144u), static_cast<int>(j0), id, &bars[u]);
        }
    }
    grid_dep_wait();          // act of the gate/up kernel
    // Activation values of this warp's records (q = warp, warp + kWarps, ...
    // of k * nsb), from this CTA's replica.
    const float* act = a.S.actr + static_cast<uint64_t>(blockIdx.x % a.S.rep) * k * L.inter;
    constexpr int kRecPerWarp = 2;
    float v[kRecPerWarp][8];
#pragma unroll
    for (int i = 0; i < kRecPerWarp; ++i) {
        const uint32_t q = warp + i * kWarps;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            v[i][j] = q < units ? __ldcg(act + static_cast<uint64_t>(q) * 256u + 32 * j + lane) : 0.0f;
    }
    // Records staged in their own space, then built in place.
#pragma unroll
    for (int i = 0; i < kRecPerWarp; ++i) {
        const uint32_t q = warp + i * kWarps;
        if (q < units) {
            float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
#pragma unroll
            for (int j = 0; j < 8; ++j) stage[32 * j + lane] = v[i][j];
        }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < kRecPerWarp; ++i) {
        const uint32_t q = warp + i * kWarps;
        if (q < units) q4k_frag_superblock(reinterpret_cast<float*>(recs + q * kFragWords), recs + q * kFragWords, lane);
    }
    for (uint32_t q = warp + kRecPerWarp * kWarps; q < units; q += kWarps) {
        float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
#pragma unroll
        for (int j = 0; j < 8; ++j) stage[32 * j + lane] = __ldcg(act + static_cast<uint64_t>(q) * 256u + 32 * j + lane);
        __syncwarp();
        q4k_frag_superblock(stage, recs + q * kFragWords, lane);
    }
    __syncthreads();
    const int g = lane >> 2;
    const auto wait_box = [&](uint32_t u) {
        if (!mbar_wait(&bars[u], 0)) {
            if (lane == 0) atomicOr(a.S.status, kStatusWaitTimeout);
            mbar_wait(&bars[u], 0);            // the copy may still land: wait once more
        }
    };
    // Units u and u + kWarps side by side (two independent chains).
    for (uint32_t u = warp; u < units; u += 2 * kWarps) {
        const uint32_t v2 = u + kWarps;
        float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
        wait_box(u);
        if (v2 < units) wait_box(v2);
        const uint8_t* bx = tiles + u * kBoxBytes;
        q4k_mma_superblock(bx + g * 144u, bx + (g + 8) * 144u, recs + u * kFragWords, a0, a1);
        if (v2 < units) {
            const uint8_t* by = tiles + v2 * kBoxBytes;
            q4k_mma_superblock(by + g * 144u, by + (g + 8) * 144u, recs + v2 * kFragWords, b0, b1);
        }
        a0 = quad_sum(a0);
        a1 = quad_sum(a1);
        b0 = quad_sum(b0);
        b1 = quad_sum(b1);
        if ((lane & 3) == 0) {
            part[u * 16 + g] = a0;
            part[u * 16 + g + 8] = a1;
            if (v2 < units) {
                part[v2 * 16 + g] = b0;
                part[v2 * 16 + g + 8] = b1;
            }
        }
    }
    __syncthreads();
    // Weighted slot rows (row, slot) in parallel, then the sum over slots in
    // route order.
    float* comb = reinterpret_cast<float*>(smem + m.comb);
    for (uint32_t t = tid; t < 16u * k; t += kThreads) {
        const uint32_t row = t & 15u, sl = t >> 4;
        float y = 0.0f;
        for (uint32_t sb = 0; sb < nsb; ++sb) y += part[(sl * nsb + sb) * 16 + row];
        comb[sl * 16 + row] = sel_w[sl] * y;
    }
    __syncthreads();
    if (tid < 16) {
        float acc = 0.0f;
        for (uint32_t sl = 0; sl < k; ++sl) acc += comb[sl * 16 + tid];
        const uint32_t row = j0 + tid;
        if (a.moe_out) {
            a.moe_out[row] = acc;
        } else {
            const float h = resid + acc;
            a.hidden[row] = h;
            hrow[tid] = nnorm * h;
            hrow[kPartRows + tid] = h * h;
        }
    }
    if (!a.has_next) return;
    __syncthreads();
    if (slice_now) racc_add(a.S.racc + static_cast<uint64_t>(tid) * kRaccLimbs, a.S.rbad, router_dot16(rs, hrow));
    for (uint32_t e = tid + kThreads; e < N.experts; e += kThreads)
        racc_add(a.S.racc + static_cast<uint64_t>(e) * kRaccLimbs, a.S.rbad,
                 router_dot16(router_slice(N.router, H, e, blockIdx.x), hrow));
    if (tid == 0) {
        float sq = 0.0f;
        for (uint32_t r = 0; r < kPartRows; ++r) sq += hrow[kPartRows + r];
        a.S.rsq[blockIdx.x] = sq;
    }
    if (last_cta_arrival(a.S.route_count, &flag)) route_tail(N, a.S, a.hidden, true, smem, m.tail);
}

// ---------------------------------------------------------------------------
// Persistent decode chain (tensor-core path): one cooperative launch carries
// one token through a range of layers.  Every CTA is resident for the whole
// launch; the phases of a layer hand off through three monotonic counters
// instead of kernel boundaries, and each phase issues its weight loads as
// soon as the routes are known:
//
//   route  wait until every D unit of the previous layer (or the prologue)
//          has added its router partials; then EVERY CTA reads the exact
//          router accumulators of this layer (parity layer & 1) and the
//          per-chunk sums of squares, selects the routes in one warp (the
//          reference's order, route_select_regs) and builds the x' fragment
//          records of the hidden state in its own shared memory.  No CTA
//          publishes routes to another: nothing waits on a single tail CTA.
//   G      CTA c owns gate/up row groups c, c + G, c + 2G of the k * I/16
//          (slot, 16-row) groups (4 warps each: gate/up x two superblock
//          halves); its TMA boxes go out right after the selection, together
//          with its D unit's down boxes (all k slots x I/256 superblocks of
//          its 16 output rows) and the next layer's router slice (registers).
//          act = silu(s g) * (s u) goes to global memory as 8-byte words
//          (the layer's sequence number << 32 | the float's bits): no fence
//          or counter between producer and consumer.
//   D      CTA c < H/16 owns hidden rows [16c, 16c + 16): it reads the k x I
//          activation words until every tag is this layer's (every CTA's G
//          done), builds the activation records, multiplies its already-
//          landed down boxes, combines the slots in route order into the
//          residual, and adds the next layer's router partials for its 16
//          rows into the other parity's accumulators before arriving on the
//          route counter.
//
// Buffer reuse: layer l's router accumulators sit in parity l % 3.  The D
// units zero parity (l - 1) % 3 during layer l (every CTA has read it:
// passing layer l's route wait implies every D unit saw every CTA's layer
// l - 1 activation words, written after that CTA's routing reads); their
// layer l route arrivals (fence, release) publish the zeros before any CTA
// adds into that parity again, in layer l + 1's D.  Each activation word is
// rewritten every layer, and a CTA writes layer l + 1's only after every D
// unit finished reading layer l's.  The last CTA to leave zeroes the
// accumulators read last, resets the counters and advances the sequence
// number, so the next launch finds them ready.  Every wait is bounded (~2 s):
// a timeout sets kStatusWaitTimeout (a sticky failure on the host), the CTA
// drains its in-flight copies and returns.
// ---------------------------------------------------------------------------
constexpr uint32_t kChainGroupsPerCta = kWarps / 4;
constexpr uint32_t kChainStamps = 8;

// The chain kernel's TMA boxes span two superblocks of 16 rows (288 bytes a
// row, 8-byte elements): half the box count of single-superblock boxes, and
// the 288-byte row pitch keeps the fragment reads free of bank conflicts.  A
// pair that runs past the end of a row reads zeros there.
constexpr uint32_t kPairRowBytes = 288u, kPairBytes = 16u * kPairRowBytes;

struct ChainLayout {
    uint32_t gbars, dbars, abars, recs, lg, sel_id, sel_w, part, dpart, comb, hrow, gtiles, dtiles, total;
    uint32_t nsb, half_sb, nsd, gpairs, dpairs;
};

__host__ __device__ inline ChainLayout chain_layout(const MoeLayerDev& L) {
    ChainLayout c{};
    const uint32_t nsb = L.hidden >> 8, half = (nsb + 1u) / 2u, nsd = L.inter >> 8, k = L.top_k;
    c.nsb = nsb;
    c.half_sb = half;
    c.nsd = nsd;
    c.gpairs = (half + 1u) / 2u;
    c.dpairs = (nsd + 1u) / 2u;
    uint32_t off = 0;
    c.gbars = off; off += al16(kWarps * c.gpairs * 8u);
    c.dbars = off; off += al16(k * c.dpairs * 8u);
    c.abars = off; off += 16u;
    c.recs = off; off += al16(umax(nsb, k * nsd) * kFragWords * 4u);
    c.lg = off; off += al16(L.experts * 4u);
    c.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    c.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    c.part = off; off += al16(kWarps * 16u * 4u);
    c.dpart = off; off += al16(k * nsd * 16u * 4u);
    c.comb = off; off += al16(k * 16u * 4u);
    c.hrow = off; off += al16(2u * kPartRows * 4u);
    off = al128(off);
    c.gtiles = off; off += kWarps * c.gpairs * kPairBytes;
    c.dtiles = off; off += k * c.dpairs * kPairBytes;
    c.total = off;
    return c;
}

struct ChainArgs {
    // 4-D tensor maps (byte column, row, expert, layer) over the pool's gate,
    // up and down tensors of every layer; boxes of 144 bytes x 16 rows.
    CUtensorMap tm_gate, tm_up, tm_down;
    const float* router0;        // layer 0's router and ffn_norm; layer l's sit
    const float* norm0;          // `stride` bytes further per layer
    uint64_t stride;
    MoeLayerDev shape;           // the common shape of the layers
    uint32_t first, count;
    MoeScratch S;                // ids / weights / logits of the last layer, act replicas, status
    ChainScratch C;
    float* hidden;
    ChainLayout c;
    // Measurement: when non-null, thread 0 of each CTA stores kChainStamps
    // globaltimer readings (ns) and then kChainStamps clock64 readings per
    // layer at [(l * grid + cta) * 2 * kChainStamps + i].
    unsigned long long* trace;
    // A decoder's attention blocks before each MoE block (with_att != 0).
    ChainAttnDesc att;
    uint32_t with_att;
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void tma_box_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                           uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
        : "memory");
}

// Thread 0 waits (bounded) until *ctr >= target, then the CTA goes on; false
// when this or another CTA gave up.
__device__ bool chain_wait(const uint32_t* ctr, uint32_t target, uint32_t* status, uint32_t* abort_sh) {
    if (threadIdx.x == 0) {
        const long long t0 = clock64();
        uint32_t polls = 0;
        while (static_cast<int32_t>(ld_acquire_gpu(ctr) - target) < 0) {
            if ((++polls & 63u) == 0) {
                if (ld_acquire_gpu(status) & kStatusWaitTimeout) { *abort_sh = 1u; break; }
                if (clock64() - t0 > kBarrierTimeoutCycles) {
                    atomicOr(status, kStatusWaitTimeout);
                    *abort_sh = 1u;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return *abort_sh == 0u;
}

// All of the CTA's writes so far become visible before the counter moves.
__device__ __forceinline__ void chain_arrive(uint32_t* ctr) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_gpu_add(ctr, 1u);
    }
}

// Router partial dots of 16 hidden rows (hrow[0..16) = ffn_norm * h, with
// hrow[16..32) = h^2) into the accumulators `racc` (E x kRaccLimbs) and the
// chunk's sum of squares into rsq[chunk]; rs holds thread e's router slice.
__device__ __forceinline__ void chain_partials(const float* router, uint32_t E, const RouterSlice& rs,
                                               const float* hrow, unsigned long long* racc, uint32_t* rbad, float* rsq,
                                               uint32_t chunk, uint32_t H) {
    const uint32_t tid = threadIdx.x;
    if (tid < E) racc_add1(racc + static_cast<uint64_t>(tid) * kRaccLimbs, rbad, router_dot16(rs, hrow));
    for (uint32_t e = tid + kThreads; e < E; e += kThreads)
        racc_add1(racc + static_cast<uint64_t>(e) * kRaccLimbs, rbad,
                  router_dot16(router_slice(router, H, e, chunk), hrow));
    if (tid == 0) {
        float sq = 0.0f;
        for (uint32_t r = 0; r < kPartRows; ++r) sq += hrow[kPartRows + r];
        rsq[chunk] = sq;
    }
}

// kAtt: a decoder's attention blocks before each MoE block (a separate
// instantiation, so the MoE-only chain keeps its registers).
template <bool kAtt>
__global__ void __launch_bounds__(kThreads, 1) moe_chain_kernel(const __grid_constant__ ChainArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t abort_sh, bad_sh, last_sh;
    __shared__ float scale_sh;
    __shared__ float attn_red[kWarps];
    const ChainLayout& c = a.c;
    const MoeLayerDev& Ls = a.shape;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = gridDim.x, cta = blockIdx.x;
    const uint32_t H = Ls.hidden, I = Ls.inter, E = Ls.experts, k = Ls.top_k;
    const uint32_t nsb = c.nsb, nsd = c.nsd, half = c.half_sb;
    const uint32_t per_slot = I / 16u, groups = k * per_slot, units = H / kPartRows;
    const bool has_unit = cta < units;
    const uint32_t j0 = cta * kPartRows;
    uint64_t* gbars = reinterpret_cast<uint64_t*>(smem + c.gbars);
    uint64_t* dbars = reinterpret_cast<uint64_t*>(smem + c.dbars);
    uint64_t* abars = reinterpret_cast<uint64_t*>(smem + c.abars);
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + c.recs);
    float* lg = reinterpret_cast<float*>(smem + c.lg);
    uint32_t* sel_id = reinterpret_cast<uint32_t*>(smem + c.sel_id);
    float* sel_w = reinterpret_cast<float*>(smem + c.sel_w);
    float* part = reinterpret_cast<float*>(smem + c.part);
    float* dpart = reinterpret_cast<float*>(smem + c.dpart);
    float* comb = reinterpret_cast<float*>(smem + c.comb);
    float* hrow = reinterpret_cast<float*>(smem + c.hrow);
    uint8_t* gtiles = smem + c.gtiles;
    uint8_t* dtiles = smem + c.dtiles;
    uint32_t* ctr_route = a.C.counters;
    uint32_t* ctr_exit = a.C.counters + 2u * kChainCounterStride;
    uint32_t* ctr_seq = a.C.counters + 3u * kChainCounterStride;
    uint32_t* status = a.S.status;
    const uint64_t racc_span = static_cast<uint64_t>(E) * kRaccLimbs;
    // x' = ffn_norm * hidden of the layer being routed, in kChainXReplicas
    // copies (CTA c reads copy c % kChainXReplicas).
    const float* xrep = a.C.xrep + static_cast<uint64_t>(cta % kChainXReplicas) * H;
    // Layer l's router and ffn_norm sit at a constant stride from layer 0's.
    const auto router_of = [&](uint32_t layer) {
        return reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.router0) + a.stride * layer);
    };
    const auto norm_of = [&](uint32_t layer) {
        return reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.norm0) + a.stride * layer);
    };
    const auto stamp = [&](uint32_t l, uint32_t i) {
        if (a.trace && tid == 0) {
            unsigned long long* t = a.trace + (static_cast<uint64_t>(l) * G + cta) * (2u * kChainStamps);
            t[i] = global_ns();
            t[kChainStamps + i] = static_cast<unsigned long long>(clock64());
        }
    };

    if (tid == 0) abort_sh = 0u;
    const uint32_t gpairs = c.gpairs, dpairs = c.dpairs;
    if (lane == 0) {
        for (uint32_t i = 0; i < gpairs; ++i) mbar_init(&gbars[warp * gpairs + i], 1);
        if (warp == 0) {
            for (uint32_t u = 0; u < k * dpairs; ++u) mbar_init(&dbars[u], 1);
            mbar_init(&abars[0], 1);
            mbar_init(&abars[1], 1);
        }
        mbar_fence_init();
    }
    // This CTA's gate/up row group and superblock half per warp (the same
    // every layer, so an mbarrier's phase flips once per layer it is used).
    const uint32_t rg = cta + G * static_cast<uint32_t>(warp >> 2);
    const uint32_t mat = (warp >> 1) & 1, hsel = warp & 1;
    const uint32_t split = (nsb + 1u) / 2u;
    const uint32_t sb0 = hsel ? split : 0u, sb1 = hsel ? nsb : split;
    const uint32_t nmine = (rg < groups && sb1 > sb0) ? sb1 - sb0 : 0u;
    const uint32_t npairs = (nmine + 1u) / 2u;
    uint8_t* mytile = gtiles + warp * gpairs * kPairBytes;
    uint64_t* mybars = gbars + warp * gpairs;
    const int g = lane >> 2;
    (void)half;

    // Prologue: the first layer's router partials and x' rows from the input
    // hidden state (with attention blocks, the first attention phase adds them).
    if (has_unit && !kAtt) {
        if (tid < 16) {
            const float h = __ldcg(a.hidden + j0 + tid);
            const float xn = __ldg(norm_of(a.first) + j0 + tid) * h;
            hrow[tid] = xn;
            hrow[kPartRows + tid] = h * h;
            for (uint32_t r = 0; r < kChainXReplicas; ++r) a.C.xrep[static_cast<uint64_t>(r) * H + j0 + tid] = xn;
        }
        __syncthreads();
        RouterSlice rs{};
        if (static_cast<uint32_t>(tid) < E) rs = router_slice(router_of(a.first), H, tid, cta);
        const uint32_t p = a.first & 1u;
        const uint32_t r0 = a.first % 3u;
        chain_partials(router_of(a.first), E, rs, hrow, a.C.racc + r0 * racc_span, a.C.rbad + r0, a.C.rsq + p * units,
                       cta, H);
        chain_arrive(ctr_route);
    }

    uint32_t phase = 0;
    bool ok = true;
    // Activation words carry the sequence number of the layer that wrote
    // them (launches advance it by their layer count; zero-filled memory
    // never matches).
    const uint32_t seq0 = __ldcg(ctr_seq);
    // With attention blocks: the decoder's position (hidden-row word tags) and
    // the router slice of the layer whose partials the next attention phase adds.
    const uint32_t att_pos = kAtt ? *a.att.pos : 0u;
    RouterSlice rs_att{};
    if (kAtt && has_unit && static_cast<uint32_t>(tid) < E) rs_att = router_slice(router_of(a.first), H, tid, cta);
    for (uint32_t l = 0; l < a.count && ok; ++l, phase ^= 1u) {
        const uint32_t layer = a.first + l, p = layer & 1u, pr = layer % 3u, tag = seq0 + l + 1u;
        const bool has_next = l + 1 < a.count;
        const uint32_t nlayer = has_next ? layer + 1 : layer;
        // ---- attention (decoder layer loop) ----
        if constexpr (kAtt) {
            const ChainAttnDesc& d = a.att;
            const uint64_t wo = static_cast<uint64_t>(layer) * d.w_stride;
            AttnBlockArgs aa{};
            aa.wqkv = d.wqkv + wo;
            aa.wo = d.wo + wo;
            aa.attn_norm = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(d.attn_norm) + wo);
            aa.q_norm = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(d.q_norm) + wo);
            aa.k_norm = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(d.k_norm) + wo);
            aa.rope_cos = d.rope_cos;
            aa.rope_sin = d.rope_sin;
            aa.kc = static_cast<__half*>(d.kc) + static_cast<uint64_t>(layer) * d.kv_stride;
            aa.vc = static_cast<__half*>(d.vc) + static_cast<uint64_t>(layer) * d.kv_stride;
            aa.pos_p = d.pos;
            aa.sh = AttendShape{d.q_heads, d.kv_heads, d.head_dim, d.q_stride, d.gated, d.rotary_half, d.window,
                                d.eps, d.scale};
            aa.hidden = a.hidden;
            aa.qkv_ll = d.qkv_words;
            aa.att_ll = d.att_words;
            aa.status = d.status;
            aa.H = H;
            aa.rows = d.rows;
            aa.qd = d.q_heads * d.head_dim;
            aa.layer = layer;
            aa.layers = d.layers_total;
            aa.eps = d.eps;
            const AttnPhaseCtx x{smem + c.gtiles, abars, phase, &abort_sh, attn_red};
            // Smaller load batches keep the attention inside the chain's
            // register budget (384 threads).
            const float hn = attention_phase<8, 8>(aa, x, l > 0 ? d.hidden_words : nullptr,
                                                   att_pos * d.layers_total + layer + 1u);
            if (abort_sh) { ok = false; break; }
            // This layer's router partials from the D unit's new rows.
            if (has_unit) {
                if (tid < 16) {
                    const float xn = __ldg(norm_of(layer) + j0 + tid) * hn;
                    hrow[tid] = xn;
                    hrow[kPartRows + tid] = hn * hn;
                    for (uint32_t r = 0; r < kChainXReplicas; ++r) a.C.xrep[static_cast<uint64_t>(r) * H + j0 + tid] = xn;
                }
                __syncthreads();
                chain_partials(router_of(layer), E, rs_att, hrow, a.C.racc + pr * racc_span, a.C.rbad + pr,
                               a.C.rsq + p * units, cta, H);
                chain_arrive(ctr_route);
            }
        }
        // ---- route ----
        if (!chain_wait(ctr_route, units * (l + 1u), status, &abort_sh)) { ok = false; break; }
        stamp(l, 0);
        const unsigned long long* racc = a.C.racc + pr * racc_span;
        if (warp < static_cast<int>(kTailLogitWarps)) {
            // The first expert's limbs, then (warp 0) the per-chunk sums of
            // squares: both loads in flight before either is used.
            const uint32_t e_first = warp * 32u + lane;
            ulonglong2 limbs[kRaccLimbs / 2];
            if (e_first < E) {
                const ulonglong2* q = reinterpret_cast<const ulonglong2*>(racc + static_cast<uint64_t>(e_first) * kRaccLimbs);
#pragma unroll
                for (int h2 = 0; h2 < kRaccLimbs / 2; ++h2) limbs[h2] = __ldcg(q + h2);
            }
            if (warp == 0) {
                float sq = 0.0f;
                for (uint32_t u = lane; u < units; u += 32) sq += __ldcg(a.C.rsq + p * units + u);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane == 0) {
                    // rms_norm scale (src/rms_norm.cpp:20-26).
                    scale_sh = 1.0f / sqrtf(sq / static_cast<float>(H) + Ls.rms_eps);
                    bad_sh = __ldcg(a.C.rbad + pr);
                }
            }
            if (e_first < E) lg[e_first] = racc_value(limbs);
            for (uint32_t e0 = warp * 32u + kTailLogitWarps * 32u; e0 < E; e0 += kTailLogitWarps * 32u) {
                const uint32_t e = e0 + lane;
                if (e < E) {
                    const ulonglong2* q = reinterpret_cast<const ulonglong2*>(racc + static_cast<uint64_t>(e) * kRaccLimbs);
#pragma unroll
                    for (int h2 = 0; h2 < kRaccLimbs / 2; ++h2) limbs[h2] = __ldcg(q + h2);
                    lg[e] = racc_value(limbs);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kTailLogitWarps * 32u) : "memory");
            if (warp == 0) {
                const float scale = scale_sh;
                const bool bad = bad_sh != 0u;
                const auto select = [&](auto slots) {
                    constexpr uint32_t kSlots = decltype(slots)::value;
                    float lgv[kSlots];
#pragma unroll
                    for (uint32_t i = 0; i < kSlots; ++i) {
                        const uint32_t e = lane + 32u * i;
                        lgv[i] = e < E ? (bad ? __int_as_float(0x7fc00000) : lg[e] * scale) : 0.0f;
                    }
                    route_select_regs<kSlots>(Ls, lgv, 0.0f, sel_id, sel_w, status, cta == 0, a.S);
                };
                if (E <= 128u) select(std::integral_constant<uint32_t, 4>{});
                else select(std::integral_constant<uint32_t, kRouteWarpMaxSlots>{});
            }
        } else {
            // x' fragment records, one superblock per builder warp.
            const uint32_t builders = static_cast<uint32_t>(kWarps) - kTailLogitWarps;
            for (uint32_t q = static_cast<uint32_t>(warp) - kTailLogitWarps; q < nsb; q += builders) {
                float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
                float xv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) xv[j] = __ldcg(xrep + q * 256u + 32u * j + lane);
#pragma unroll
                for (int j = 0; j < 8; ++j) stage[32 * j + lane] = xv[j];
                __syncwarp();
                q4k_frag_superblock(stage, recs + q * kFragWords, lane);
                __syncwarp();
            }
        }
        __syncthreads();
        stamp(l, 1);
        const float scale = scale_sh;
        // ---- G: the gate/up boxes out first ----
        if (nmine && lane == 0) {
            const int id = static_cast<int>(sel_id[rg / per_slot]);
            const int row0 = static_cast<int>((rg % per_slot) * 16u);
            const CUtensorMap* map = mat ? &a.tm_up : &a.tm_gate;
            for (uint32_t i = 0; i < npairs; ++i) {
                mbar_expect_tx(&mybars[i], kPairBytes);
                tma_box_4d(mytile + i * kPairBytes, map, static_cast<int>((sb0 + 2u * i) * 18u), row0, id,
                           static_cast<int>(layer), &mybars[i]);
            }
        }
        // The down boxes (needed after the act wait).  MoE-only chain: right
        // behind the gate/up boxes -- its gate/up phase is latency-bound, so
        // they do not slow it, and they land before the activations do.  With
        // attention: once the warp's gate/up work is done (measured no gain).
        const auto issue_down = [&]() {
            if (!(has_unit && static_cast<uint32_t>(warp) < k && lane == 0)) return;
            const int id = static_cast<int>(sel_id[warp]);
            for (uint32_t j = 0; j < dpairs; ++j) {
                const uint32_t u = warp * dpairs + j;
                mbar_expect_tx(&dbars[u], kPairBytes);
                tma_box_4d(dtiles + u * kPairBytes, &a.tm_down, static_cast<int>(j * 36u), static_cast<int>(j0), id,
                           static_cast<int>(layer), &dbars[u]);
            }
        };
        if (!kAtt) issue_down();
        // The previous layer's accumulators and flag (every CTA has read
        // them), zeroed by the D units: their route arrivals publish the
        // zeros before anyone adds into this parity again (the layer after next).
        if (has_unit) {
            const uint32_t pz = (layer + 2u) % 3u;
            for (uint32_t i = cta * kThreads + tid; i < racc_span; i += units * kThreads)
                a.C.racc[pz * racc_span + i] = 0ull;
            if (cta == 0 && tid == 0) a.C.rbad[pz] = 0u;
        }
        // The next layer's router slice and ffn_norm, this unit's residual rows.
        RouterSlice rs{};
        if (has_unit && has_next && static_cast<uint32_t>(tid) < E)
            rs = router_slice_issue_here(router_of(nlayer), H, tid, cta);
        if (kAtt) rs_att = rs;
        const float resid = (has_unit && tid < 16) ? __ldcg(a.hidden + j0 + tid) : 0.0f;
        const float nnorm = (has_unit && has_next && tid < 16) ? __ldg(norm_of(nlayer) + j0 + tid) : 0.0f;
        // ---- G: multiply the boxes as they land ----
        const auto wait_bar = [&](uint64_t* bar) {
            if (!mbar_wait(bar, phase)) {
                if (lane == 0) atomicOr(status, kStatusWaitTimeout);
                mbar_wait(bar, phase);         // the copy may still land: wait once more
            }
        };
        {
            float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
            for (uint32_t i = 0; i < npairs; ++i) {
                wait_bar(&mybars[i]);
                const uint8_t* bx = mytile + i * kPairBytes;
                const uint32_t s0 = sb0 + 2u * i;
                q4k_mma_superblock(bx + g * kPairRowBytes, bx + (g + 8) * kPairRowBytes, recs + s0 * kFragWords, acc0,
                                   acc1);
                if (2u * i + 1u < nmine)
                    q4k_mma_superblock(bx + g * kPairRowBytes + 144u, bx + (g + 8) * kPairRowBytes + 144u,
                                       recs + (s0 + 1u) * kFragWords, acc2, acc3);
            }
            acc0 = quad_sum(acc0 + acc2);
            acc1 = quad_sum(acc1 + acc3);
            if ((lane & 3) == 0) {
                part[warp * 16 + g] = acc0;
                part[warp * 16 + g + 8] = acc1;
            }
        }
        if (kAtt) issue_down();
        __syncthreads();
        stamp(l, 2);
        if (tid < static_cast<int>(kChainGroupsPerCta * 16u)) {
            const uint32_t gl = tid >> 4, r = tid & 15, rgx = cta + G * gl;
            if (rgx < groups) {
                const float gv = part[(gl * 4 + 0) * 16 + r] + part[(gl * 4 + 1) * 16 + r];
                const float uv = part[(gl * 4 + 2) * 16 + r] + part[(gl * 4 + 3) * 16 + r];
                const uint32_t slot = rgx / per_slot, row = (rgx % per_slot) * 16u + r;
                const float av = silu_mul(gv * scale, uv * scale, Ls.flavour);
                const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(av);
                for (uint32_t r = 0; r < kChainXReplicas; ++r)
                    st_relaxed_gpu_u64(a.C.act + (static_cast<uint64_t>(r) * k + slot) * I + row, w);
            }
        }
        stamp(l, 3);
        if (!has_unit) continue;
        // ---- D ----
        {
            // Every activation word of this layer, read as it arrives: a word
            // is current once its tag is this layer's sequence number (each
            // word is one 8-byte store, so tag and value arrive together).
            const uint32_t nrec = k * nsd;
            // Two records per warp per pass, all of their loads in flight together.
            for (uint32_t q0 = warp; q0 < nrec; q0 += 2 * kWarps) {
                unsigned long long v[2][8];
                const auto word = [&](int i, int j) {
                    return a.C.act + static_cast<uint64_t>(cta % kChainXReplicas) * k * I +
                           static_cast<uint64_t>(q0 + i * kWarps) * 256u + 32 * j + lane;
                };
#pragma unroll
                for (int i = 0; i < 2; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        v[i][j] = q0 + i * kWarps < nrec ? ld_relaxed_gpu_u64(word(i, j))
                                                         : static_cast<unsigned long long>(tag) << 32;
                long long t0 = 0;
                for (uint32_t polls = 0;; ++polls) {
                    bool ready = true;
#pragma unroll
                    for (int i = 0; i < 2; ++i)
#pragma unroll
                        for (int j = 0; j < 8; ++j) ready = ready && static_cast<uint32_t>(v[i][j] >> 32) == tag;
                    if (__all_sync(0xffffffffu, ready)) break;
                    if (polls == 0) t0 = clock64();
                    if ((polls & 63u) == 63u &&
                        ((ld_acquire_gpu(status) & kStatusWaitTimeout) || clock64() - t0 > kBarrierTimeoutCycles)) {
                        if (lane == 0) {
                            atomicOr(status, kStatusWaitTimeout);
                            abort_sh = 1u;
                        }
                        break;
                    }
#pragma unroll
                    for (int i = 0; i < 2; ++i)
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (static_cast<uint32_t>(v[i][j] >> 32) != tag) v[i][j] = ld_relaxed_gpu_u64(word(i, j));
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const uint32_t q = q0 + i * kWarps;
                    if (q < nrec) {
                        float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
#pragma unroll
                        for (int j = 0; j < 8; ++j) stage[32 * j + lane] = __uint_as_float(static_cast<uint32_t>(v[i][j]));
                    }
                }
                __syncwarp();
                if (!kAtt && q0 + kWarps < nrec) {
                    // Both records' steps interleaved (the attention instantiation
                    // keeps one at a time: it is at its register cap).
                    const float* const vp[2] = {reinterpret_cast<const float*>(recs + q0 * kFragWords),
                                                reinterpret_cast<const float*>(recs + (q0 + kWarps) * kFragWords)};
                    uint32_t* const rp[2] = {recs + q0 * kFragWords, recs + (q0 + kWarps) * kFragWords};
                    q4k_frag_superblocks<2>(vp, rp, lane);
                } else {
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const uint32_t q = q0 + i * kWarps;
                        if (q < nrec)
                            q4k_frag_superblock(reinterpret_cast<float*>(recs + q * kFragWords), recs + q * kFragWords,
                                                lane);
                    }
                }
                __syncwarp();
                // The warp multiplies the records it just built (no wait for
                // the CTA's other warps): unit (slot, sb) lives in pair box
                // slot * dpairs + sb / 2.
                const uint32_t u = q0, v2 = q0 + kWarps;
                float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
                const auto unit_box = [&](uint32_t q) {
                    const uint32_t sl = q / nsd, sb = q % nsd, bi = sl * dpairs + (sb >> 1);
                    wait_bar(&dbars[bi]);
                    return dtiles + bi * kPairBytes + (sb & 1u) * 144u;
                };
                const uint8_t* bx = unit_box(u);
                q4k_mma_superblock(bx + g * kPairRowBytes, bx + (g + 8) * kPairRowBytes, recs + u * kFragWords, a0, a1);
                if (v2 < nrec) {
                    const uint8_t* by = unit_box(v2);
                    q4k_mma_superblock(by + g * kPairRowBytes, by + (g + 8) * kPairRowBytes, recs + v2 * kFragWords,
                                       b0, b1);
                }
                a0 = quad_sum(a0);
                a1 = quad_sum(a1);
                b0 = quad_sum(b0);
                b1 = quad_sum(b1);
                if ((lane & 3) == 0) {
                    dpart[u * 16 + g] = a0;
                    dpart[u * 16 + g + 8] = a1;
                    if (v2 < nrec) {
                        dpart[v2 * 16 + g] = b0;
                        dpart[v2 * 16 + g + 8] = b1;
                    }
                }
            }
            stamp(l, 4);
            __syncthreads();
            if (abort_sh) {
                if (static_cast<uint32_t>(warp) < k && lane == 0)
                    for (uint32_t j = 0; j < dpairs; ++j) mbar_wait(&dbars[warp * dpairs + j], phase);
                ok = false;
                break;
            }
            stamp(l, 5);
            // Weighted slot rows, then the sum over slots in route order.
            for (uint32_t t = tid; t < 16u * k; t += kThreads) {
                const uint32_t row = t & 15u, sl = t >> 4;
                float y = 0.0f;
                for (uint32_t sb = 0; sb < nsd; ++sb) y += dpart[(sl * nsd + sb) * 16 + row];
                comb[sl * 16 + row] = sel_w[sl] * y;
            }
            __syncthreads();
            stamp(l, 6);
            if (tid < 16) {
                float acc = 0.0f;
                for (uint32_t sl = 0; sl < k; ++sl) acc += comb[sl * 16 + tid];
                const float h = resid + acc;
                a.hidden[j0 + tid] = h;
                if (has_next && kAtt) {
                    // The next attention phase stages every row from these words.
                    put_word(a.att.hidden_words + j0 + tid, att_pos * a.att.layers_total + nlayer + 1u, h);
                } else if (has_next) {
                    const float xn = nnorm * h;
                    hrow[tid] = xn;
                    hrow[kPartRows + tid] = h * h;
                    for (uint32_t r = 0; r < kChainXReplicas; ++r)
                        a.C.xrep[static_cast<uint64_t>(r) * H + j0 + tid] = xn;
                }
            }
            if (has_next && !kAtt) {
                __syncthreads();
                const uint32_t pn = (layer + 1u) % 3u;
                chain_partials(router_of(nlayer), E, rs, hrow, a.C.racc + pn * racc_span, a.C.rbad + pn,
                               a.C.rsq + (p ^ 1u) * units, cta, H);
            }
        }
        // With attention blocks the next layer's attention phase arrives.
        if (!kAtt) chain_arrive(ctr_route);
        else __syncthreads();
        stamp(l, 7);
    }
    if (!ok) return;
    // The last CTA out leaves the accumulators and counters at zero.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        last_sh = atomicAdd(ctr_exit, 1u) == G - 1u ? 1u : 0u;
    }
    __syncthreads();
    if (!last_sh) return;
    __threadfence();
    const uint32_t plast = (a.first + a.count - 1u) % 3u;
    for (uint32_t i = tid; i < racc_span; i += kThreads) a.C.racc[plast * racc_span + i] = 0ull;
    __syncthreads();
    if (tid == 0) {
        a.C.rbad[plast] = 0u;
        *ctr_route = 0u;
        *ctr_exit = 0u;
        *ctr_seq = seq0 + a.count;
        __threadfence();
    }
}

// ---------------------------------------------------------------------------
// moe_chain35_kernel: the decode chain for Qwen3.5-MoE blocks (configuration
// 3): Q4_K gate/up and Q4_K / Q5_K / Q6_K down (per layer) on the integer
// tensor path, and the sigmoid-gated Q8_0 shared expert (src/qwen35_runner.cpp:
// 691-763).  The same phases and hand-offs as moe_chain_kernel, with:
//   route  E + 1 accumulator rows (the shared expert's gate row last), at
//          most two per thread with all loads in flight; one warp selects, the
//          selection taking sigmoid(scale * that logit) as the shared weight,
//          while eight build the x' records
//   G      routed 16-row groups as in the chain, a tensor-map box per
//          two-superblock tile from the layer's own maps (the layers' tensors
//          need not sit at one stride); the shared expert's gate/up in 8-row
//          groups, a box of half rows per warp, dotted in FP32 with x'
//   D      every slot's 16 down rows by one bulk copy; the routed slots'
//          activation records built as they arrive and multiplied on the
//          tensor path (q4k / q5k / q6k_mma_superblock); the shared slot as
//          FP32 row dots by the last four warps; the combine in route order,
//          then + sigmoid gate * shared output, into the residual; the next
//          layer's router partials (E + 1 rows)
// ---------------------------------------------------------------------------
constexpr uint32_t kChain35SharedRows = 8;       // rows per shared-expert gate/up group
constexpr uint32_t kChain35SharedWarps = 4;      // warps taking the shared slot in D

struct Chain35Layout {
    uint32_t gbars, dbars, recs, xf, lg, sel_id, sel_w, part, dpart, hrow, gtiles, dtiles, total;
    uint32_t nsb, nsd, gpairs, slots, rb_down_max, rb_shared, nrec;
};

__host__ __device__ inline Chain35Layout chain35_layout(const MoeLayerDev& L, uint32_t rb_down_max) {
    Chain35Layout c{};
    const uint32_t nsb = L.hidden >> 8, half = (nsb + 1u) / 2u;
    c.nsb = nsb;
    c.nsd = L.inter >> 8;
    c.gpairs = (half + 1u) / 2u;
    c.slots = L.top_k + 1u;
    c.nrec = L.top_k * c.nsd;
    c.rb_down_max = rb_down_max;
    c.rb_shared = static_cast<uint32_t>(row_bytes(L.shared_down_type, L.shared_inter));
    uint32_t off = 0;
    c.gbars = off; off += al16(kWarps * c.gpairs * 8u);
    c.dbars = off; off += al16(c.slots * 8u);
    c.recs = off; off += al16(umax(nsb, c.nrec) * kFragWords * 4u);
    c.xf = off; off += al16(L.hidden * 4u);
    c.lg = off; off += al16((L.experts + 1u) * 4u);
    c.sel_id = off; off += al16((kMaxTopK + 1) * 4u);
    c.sel_w = off; off += al16((kMaxTopK + 1) * 4u);
    c.part = off; off += al16(kWarps * 16u * 4u);
    c.dpart = off; off += al16((c.nrec + 1u) * 16u * 4u);
    c.hrow = off; off += al16(2u * kPartRows * 4u);
    off = al128(off);
    // Tile space: the gate/up tiles and the shared slot's activation floats
    // (D) in turn.
    c.gtiles = off;
    off += umax(kWarps * c.gpairs * kPairBytes, al16(L.inter * 4u));
    off = al128(off);
    c.dtiles = off; off += L.top_k * 16u * rb_down_max + 16u * c.rb_shared;
    c.total = off;
    return c;
}

struct Chain35Args {
    const MoeLayerDev* layers;   // device table
    MoeLayerDev shape;           // the common shape (hidden, inter, experts, top_k, flavour, ...)
    uint32_t first, count;
    MoeScratch S;
    ChainScratch C;
    float* hidden;
    Chain35Layout c;
    const Chain35Maps* maps;     // per-layer tensor maps (device memory)
    unsigned long long* trace;   // optional per-(layer, CTA) phase stamps (measurement)
    DeltaBlockArgs delta;        // with_delta: the layer's Gated DeltaNet mixer runs first
    uint32_t with_delta;
    AttnBlockArgs att;           // with_att: the layer's attention block runs first
    uint32_t with_att;
};

// Thread t's router slices of a layer: expert t (rs) and expert t + kThreads,
// or for the last thread the shared expert's gate row (rs2).  E <= 2 kThreads - 1.
__device__ __forceinline__ void chain35_slices(const MoeLayerDev& L, uint32_t E, uint32_t H, uint32_t chunk,
                                               RouterSlice& rs, RouterSlice& rs2) {
    const uint32_t tid = threadIdx.x;
    if (tid < E) rs = router_slice_issue_here(L.router, H, tid, chunk);
    if (tid + kThreads < E) rs2 = router_slice_issue_here(L.router, H, tid + kThreads, chunk);
    else if (tid == kThreads - 1u) rs2 = router_slice_issue_here(L.shared_router, H, 0, chunk);
}

// Router partials of 16 hidden rows for E experts and the shared gate row
// (accumulator row E), from the slices chain35_slices loaded.
__device__ __forceinline__ void chain35_partials(uint32_t E, const RouterSlice& rs, const RouterSlice& rs2,
                                                 const float* hrow, unsigned long long* racc, uint32_t* rbad,
                                                 float* rsq, uint32_t chunk) {
    const uint32_t tid = threadIdx.x;
    if (tid < E) racc_add1(racc + static_cast<uint64_t>(tid) * kRaccLimbs, rbad, router_dot16(rs, hrow));
    if (tid + kThreads < E)
        racc_add1(racc + static_cast<uint64_t>(tid + kThreads) * kRaccLimbs, rbad, router_dot16(rs2, hrow));
    else if (tid == kThreads - 1u)
        racc_add1(racc + static_cast<uint64_t>(E) * kRaccLimbs, rbad, router_dot16(rs2, hrow));
    if (tid == 0) {
        float sq = 0.0f;
        for (uint32_t r = 0; r < kPartRows; ++r) sq += hrow[kPartRows + r];
        rsq[chunk] = sq;
    }
}

__device__ __forceinline__ void chain35_down_mma(uint32_t type, const uint8_t* b0p, const uint8_t* b1p,
                                                 const uint32_t* rec, float& acc0, float& acc1) {
    if (type == kQ6_K) q6k_mma_superblock(b0p, b1p, rec, acc0, acc1);
    else if (type == kQ5_K) q5k_mma_superblock(b0p, b1p, rec, acc0, acc1);
    else q4k_mma_superblock(b0p, b1p, rec, acc0, acc1);
}

__global__ void __launch_bounds__(kThreads, 1) moe_chain35_kernel(const __grid_constant__ Chain35Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t abort_sh, bad_sh, last_sh;
    __shared__ float scale_sh;
    const Chain35Layout& c = a.c;
    const MoeLayerDev& Ls = a.shape;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = gridDim.x, cta = blockIdx.x;
    const uint32_t H = Ls.hidden, I = Ls.inter, E = Ls.experts, k = Ls.top_k;
    const uint32_t nsb = c.nsb, nsd = c.nsd, slots = c.slots, nrec = c.nrec;
    const uint32_t per_slot = I / 16u, routed_groups = k * per_slot;
    const uint32_t groups = routed_groups + Ls.shared_inter / kChain35SharedRows;
    const uint32_t units = H / kPartRows;
    const bool has_unit = cta < units;
    const uint32_t j0 = cta * kPartRows;
    uint64_t* gbars = reinterpret_cast<uint64_t*>(smem + c.gbars);
    uint64_t* dbars = reinterpret_cast<uint64_t*>(smem + c.dbars);
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + c.recs);
    float* xf = reinterpret_cast<float*>(smem + c.xf);
    float* lg = reinterpret_cast<float*>(smem + c.lg);
    uint32_t* sel_id = reinterpret_cast<uint32_t*>(smem + c.sel_id);
    float* sel_w = reinterpret_cast<float*>(smem + c.sel_w);
    float* part = reinterpret_cast<float*>(smem + c.part);
    float* dpart = reinterpret_cast<float*>(smem + c.dpart);
    float* dsh = dpart + nrec * 16u;                               // the shared slot's 16 rows
    float* hrow = reinterpret_cast<float*>(smem + c.hrow);
    uint8_t* gtiles = smem + c.gtiles;
    float* actsh = reinterpret_cast<float*>(smem + c.gtiles);      // D: the shared slot's activations
    uint8_t* dtiles = smem + c.dtiles;
    uint32_t* ctr_route = a.C.counters;
    uint32_t* ctr_exit = a.C.counters + 2u * kChainCounterStride;
    uint32_t* ctr_seq = a.C.counters + 3u * kChainCounterStride;
    uint32_t* status = a.S.status;
    const uint32_t Er = E + 1u;                                     // accumulator rows
    const uint64_t racc_span = static_cast<uint64_t>(Er) * kRaccLimbs;
    const float* xrep = a.C.xrep + static_cast<uint64_t>(cta % kChainXReplicas) * H;
    const uint64_t act_span = static_cast<uint64_t>(slots) * I;
    const unsigned long long* act_mine = a.C.act + static_cast<uint64_t>(cta % kChainXReplicas) * act_span;
    const auto stamp = [&](uint32_t l, uint32_t i) {
        if (a.trace && tid == 0) {
            unsigned long long* t = a.trace + (static_cast<uint64_t>(l) * G + cta) * (2u * kChainStamps);
            t[i] = global_ns();
            t[kChainStamps + i] = static_cast<unsigned long long>(clock64());
        }
    };
    if (a.with_att) {
        // A decoder's attention layer ahead of its MoE block (count 1): its
        // output units leave this CTA's D-unit rows of the residual (rows
        // [16c, 16c + 16), the prologue's), and every CTA has read all of
        // hidden before any CTA reaches the route below.  It runs in the
        // tile space.
        __shared__ uint64_t att_bars[2];
        __shared__ float att_red[kWarps];
        __shared__ uint32_t att_abort;
        if (tid == 0) {
            mbar_init(&att_bars[0], 1);
            mbar_init(&att_bars[1], 1);
            mbar_fence_init();
            att_abort = 0u;
        }
        __syncthreads();
        const AttnPhaseCtx x{smem + c.gtiles, att_bars, 0u, &att_abort, att_red};
        attention_phase<8, 8>(a.att, x, nullptr, 0u);
        if (att_abort) return;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
    }
    // A decoder's DeltaNet layer ahead of its MoE block (one launch, count 1):
    // its phase 3 leaves this CTA's D-unit rows of the residual, read by the
    // prologue below after a CTA barrier.  The mixer runs in the tile space.
    if (a.with_delta) {
        if (!delta_layer_run(a.delta, smem + c.gtiles)) return;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
    }
    if (tid == 0) abort_sh = 0u;
    const uint32_t gpairs = c.gpairs;
    if (lane == 0) {
        for (uint32_t i = 0; i < gpairs; ++i) mbar_init(&gbars[warp * gpairs + i], 1);
        if (warp == 0)
            for (uint32_t u = 0; u < slots; ++u) mbar_init(&dbars[u], 1);
        mbar_fence_init();
    }
    // This CTA's row group and superblock half per warp (as in the chain).
    const uint32_t rg = cta + G * static_cast<uint32_t>(warp >> 2);
    const uint32_t mat = (warp >> 1) & 1, hsel = warp & 1;
    const uint32_t split = (nsb + 1u) / 2u;
    const uint32_t sb0 = hsel ? split : 0u, sb1 = hsel ? nsb : split;
    const bool routed_group = rg < routed_groups;
    const bool shared_group = !routed_group && rg < groups;
    const uint32_t nmine = (routed_group && sb1 > sb0) ? sb1 - sb0 : 0u;
    const uint32_t npairs = (nmine + 1u) / 2u;
    uint8_t* mytile = gtiles + warp * gpairs * kPairBytes;
    uint64_t* mybars = gbars + warp * gpairs;
    const int g = lane >> 2;
    // Shared-expert gate/up rows (Q8_0): a warp's half row is shalf bytes.
    const uint32_t srb = static_cast<uint32_t>(row_bytes(kQ8_0, H)), shalf = srb / 2u;

    // Prologue: the first layer's router partials and x' rows.
    if (has_unit) {
        const MoeLayerDev L0 = a.layers[a.first];
        if (tid < 16) {
            const float h = __ldcg(a.hidden + j0 + tid);
            const float xn = __ldg(L0.ffn_norm + j0 + tid) * h;
            hrow[tid] = xn;
            hrow[kPartRows + tid] = h * h;
            for (uint32_t r = 0; r < kChainXReplicas; ++r) a.C.xrep[static_cast<uint64_t>(r) * H + j0 + tid] = xn;
        }
        __syncthreads();
        RouterSlice rs{}, rs2{};
        chain35_slices(L0, E, H, cta, rs, rs2);
        const uint32_t r0 = a.first % 3u;
        chain35_partials(E, rs, rs2, hrow, a.C.racc + r0 * racc_span, a.C.rbad + r0, a.C.rsq + (a.first & 1u) * units,
                         cta);
        chain_arrive(ctr_route);
    }

    uint32_t phase = 0;
    bool ok = true;
    const uint32_t seq0 = __ldcg(ctr_seq);
    const auto wait_bar = [&](uint64_t* bar) {
        if (!mbar_wait(bar, phase)) {
            if (lane == 0) atomicOr(status, kStatusWaitTimeout);
            mbar_wait(bar, phase);
        }
    };
    for (uint32_t l = 0; l < a.count && ok; ++l, phase ^= 1u) {
        const uint32_t layer = a.first + l, p = layer & 1u, pr = layer % 3u, tag = seq0 + l + 1u;
        const bool has_next = l + 1 < a.count;
        const MoeLayerDev L = a.layers[layer];
        // The tile space's generic accesses so far come before this layer's
        // bulk copies into it.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        // ---- route ----
        if (!chain_wait(ctr_route, units * (l + 1u), status, &abort_sh)) { ok = false; break; }
        stamp(l, 0);
        {
            // Every thread turns at most two accumulator rows into logits, all
            // of their loads in flight together (E + 1 <= 2 x kThreads rows).
            const unsigned long long* racc = a.C.racc + pr * racc_span;
            ulonglong2 limbs[2][kRaccLimbs / 2];
#pragma unroll
            for (uint32_t i = 0; i < 2; ++i) {
                const uint32_t e = static_cast<uint32_t>(tid) + i * kThreads;
                if (e < Er) {
                    const ulonglong2* q = reinterpret_cast<const ulonglong2*>(racc + static_cast<uint64_t>(e) * kRaccLimbs);
#pragma unroll
                    for (int h2 = 0; h2 < kRaccLimbs / 2; ++h2) limbs[i][h2] = __ldcg(q + h2);
                }
            }
            if (warp == 0) {
                float sq = 0.0f;
                for (uint32_t u = lane; u < units; u += 32) sq += __ldcg(a.C.rsq + p * units + u);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane == 0) {
                    scale_sh = 1.0f / sqrtf(sq / static_cast<float>(H) + Ls.rms_eps);
                    bad_sh = __ldcg(a.C.rbad + pr);
                }
            }
#pragma unroll
            for (uint32_t i = 0; i < 2; ++i) {
                const uint32_t e = static_cast<uint32_t>(tid) + i * kThreads;
                if (e < Er) lg[e] = racc_value(limbs[i]);
            }
        }
        __syncthreads();
        if (warp < static_cast<int>(kTailLogitWarps)) {
            if (warp == 0) {
                const float scale = scale_sh;
                const bool bad = bad_sh != 0u;
                const float shared_logit = bad ? __int_as_float(0x7fc00000) : lg[E] * scale;
                const auto select = [&](auto slots_c) {
                    constexpr uint32_t kSlots = decltype(slots_c)::value;
                    float lgv[kSlots];
#pragma unroll
                    for (uint32_t i = 0; i < kSlots; ++i) {
                        const uint32_t e = lane + 32u * i;
                        lgv[i] = e < E ? (bad ? __int_as_float(0x7fc00000) : lg[e] * scale) : 0.0f;
                    }
                    route_select_regs<kSlots>(Ls, lgv, shared_logit, sel_id, sel_w, status, cta == 0, a.S);
                };
                if (E <= 128u) select(std::integral_constant<uint32_t, 4>{});
                else if (E <= 256u) select(std::integral_constant<uint32_t, 8>{});
                else select(std::integral_constant<uint32_t, 16>{});
            }
        } else {
            // x' floats (for the shared expert's rows) and fragment records.
            const uint32_t builders = static_cast<uint32_t>(kWarps) - kTailLogitWarps;
            for (uint32_t q = static_cast<uint32_t>(warp) - kTailLogitWarps; q < nsb; q += builders) {
                float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
                float xv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) xv[j] = __ldcg(xrep + q * 256u + 32u * j + lane);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    stage[32 * j + lane] = xv[j];
                    xf[q * 256u + 32u * j + lane] = xv[j];
                }
                __syncwarp();
                q4k_frag_superblock(stage, recs + q * kFragWords, lane);
                __syncwarp();
            }
        }
        // The staged accumulator rows are read before the gate/up copies
        // overwrite them.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        stamp(l, 1);
        const float scale = scale_sh;
        // ---- G: the gate/up boxes of this layer's maps ----
        const Chain35Maps* maps = a.maps + layer;
        if (nmine && lane == 0) {
            const int id = static_cast<int>(sel_id[rg / per_slot]);
            const int row0 = static_cast<int>((rg % per_slot) * 16u);
            const CUtensorMap* map = mat ? &maps->up : &maps->gate;
            for (uint32_t i = 0; i < npairs; ++i) {
                mbar_expect_tx(&mybars[i], kPairBytes);
                tma_box_3d(mytile + i * kPairBytes, map, static_cast<int>((sb0 + 2u * i) * 18u), row0, id, &mybars[i]);
            }
        } else if (shared_group && lane == 0) {
            // 8 half rows of the shared expert's gate or up.
            const int srow0 = static_cast<int>((rg - routed_groups) * kChain35SharedRows);
            mbar_expect_tx(&mybars[0], kChain35SharedRows * shalf);
            tma_box_2d(mytile, mat ? &maps->shared_up : &maps->shared_gate, static_cast<int>(hsel * (shalf / 8u)), srow0,
                       &mybars[0]);
        }
        // The previous layer's accumulators (zeroed by the D units).
        if (has_unit) {
            const uint32_t pz = (layer + 2u) % 3u;
            for (uint32_t i = cta * kThreads + tid; i < racc_span; i += units * kThreads)
                a.C.racc[pz * racc_span + i] = 0ull;
            if (cta == 0 && tid == 0) a.C.rbad[pz] = 0u;
        }
        const MoeLayerDev Ln = has_next ? a.layers[layer + 1] : L;
        RouterSlice rs{}, rs2{};
        if (has_unit && has_next) chain35_slices(Ln, E, H, cta, rs, rs2);
        const float resid = (has_unit && tid < 16) ? ldcg_f32_issue_here(a.hidden + j0 + tid) : 0.0f;
        const float nnorm = (has_unit && has_next && tid < 16) ? ldcg_f32_issue_here(Ln.ffn_norm + j0 + tid) : 0.0f;
        if (routed_group) {
            float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
            for (uint32_t i = 0; i < npairs; ++i) {
                wait_bar(&mybars[i]);
                const uint8_t* bx = mytile + i * kPairBytes;
                const uint32_t s0 = sb0 + 2u * i;
                q4k_mma_superblock(bx + g * kPairRowBytes, bx + (g + 8) * kPairRowBytes, recs + s0 * kFragWords,
                                   acc0, acc1);
                if (2u * i + 1u < nmine)
                    q4k_mma_superblock(bx + g * kPairRowBytes + 144u, bx + (g + 8) * kPairRowBytes + 144u,
                                       recs + (s0 + 1u) * kFragWords, acc2, acc3);
            }
            acc0 = quad_sum(acc0 + acc2);
            acc1 = quad_sum(acc1 + acc3);
            if ((lane & 3) == 0) {
                part[warp * 16 + g] = acc0;
                part[warp * 16 + g + 8] = acc1;
            }
        } else if (shared_group) {
            wait_bar(&mybars[0]);
            const float* xs = xf + hsel * (H / 2u);
#pragma unroll 1
            for (uint32_t r = 0; r < kChain35SharedRows; r += 2u) {
                float v0 = lane_row_dot4<kQ8_0>(mytile + r * shalf, H / 2u, xs, lane);
                float v1 = lane_row_dot4<kQ8_0>(mytile + (r + 1u) * shalf, H / 2u, xs, lane);
                v0 = warp_sum(v0);
                v1 = warp_sum(v1);
                if (lane == 0) {
                    part[warp * 16 + r] = v0;
                    part[warp * 16 + r + 1] = v1;
                }
            }
        }
        stamp(l, 2);
        // Every slot's 16 down rows of this D unit: one bulk copy per slot,
        // once the warp's own gate/up work is done (issued with the gate/up
        // copies they slow this kernel's bandwidth-sensitive gate/up phase).
        if (has_unit && static_cast<uint32_t>(warp) < slots && lane == 0) {
            const uint32_t sl = warp;
            const bool shared = sl == k;
            const uint32_t rbd = shared ? c.rb_shared : static_cast<uint32_t>(row_bytes(L.down_type, I));
            const uint8_t* src = shared ? L.shared_down + static_cast<uint64_t>(j0) * rbd
                                        : L.down + static_cast<uint64_t>(sel_id[sl]) * L.down_slice +
                                              static_cast<uint64_t>(j0) * rbd;
            mbar_expect_tx(&dbars[sl], 16u * rbd);
            bulk_copy_g2s(dtiles + sl * 16u * c.rb_down_max, src, 16u * rbd, &dbars[sl]);
        }
        __syncthreads();
        if (tid < static_cast<int>(kChainGroupsPerCta * 16u)) {
            const uint32_t gl = tid >> 4, r = tid & 15, rgx = cta + G * gl;
            uint32_t slot = 0, row = 0;
            bool mine = false;
            if (rgx < routed_groups) {
                slot = rgx / per_slot;
                row = (rgx % per_slot) * 16u + r;
                mine = true;
            } else if (rgx < groups && r < kChain35SharedRows) {
                slot = k;
                row = (rgx - routed_groups) * kChain35SharedRows + r;
                mine = true;
            }
            if (mine) {
                const float gv = part[(gl * 4 + 0) * 16 + r] + part[(gl * 4 + 1) * 16 + r];
                const float uv = part[(gl * 4 + 2) * 16 + r] + part[(gl * 4 + 3) * 16 + r];
                const float av = silu_mul(gv * scale, uv * scale, Ls.flavour);
                const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(av);
                for (uint32_t rr = 0; rr < kChainXReplicas; ++rr)
                    st_relaxed_gpu_u64(a.C.act + rr * act_span + slot * I + row, w);
            }
        }
        stamp(l, 3);
        if (!has_unit) continue;
        // ---- D ----
        {
            const uint32_t dtype = L.down_type;
            const uint32_t rbd = static_cast<uint32_t>(row_bytes(dtype, I));
            const uint32_t sbb = dtype == kQ6_K ? 210u : (dtype == kQ5_K ? 176u : 144u);
            // Routed units (slot, superblock): two per warp and pass, every
            // activation word read as it arrives (tag = this layer's sequence
            // number), the records built and multiplied by the same warp.
            for (uint32_t q0 = warp; q0 < nrec; q0 += 2 * kWarps) {
                unsigned long long v[2][8];
                const auto word = [&](int i, int j) {
                    return act_mine + static_cast<uint64_t>(q0 + i * kWarps) * 256u + 32 * j + lane;
                };
#pragma unroll
                for (int i = 0; i < 2; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        v[i][j] = q0 + i * kWarps < nrec ? ld_relaxed_gpu_u64(word(i, j))
                                                         : static_cast<unsigned long long>(tag) << 32;
                long long t0 = 0;
                for (uint32_t polls = 0;; ++polls) {
                    bool ready = true;
#pragma unroll
                    for (int i = 0; i < 2; ++i)
#pragma unroll
                        for (int j = 0; j < 8; ++j) ready = ready && static_cast<uint32_t>(v[i][j] >> 32) == tag;
                    if (__all_sync(0xffffffffu, ready)) break;
                    if (polls == 0) t0 = clock64();
                    if ((polls & 63u) == 63u &&
                        ((ld_acquire_gpu(status) & kStatusWaitTimeout) || clock64() - t0 > kBarrierTimeoutCycles)) {
                        if (lane == 0) {
                            atomicOr(status, kStatusWaitTimeout);
                            abort_sh = 1u;
                        }
                        break;
                    }
#pragma unroll
                    for (int i = 0; i < 2; ++i)
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (static_cast<uint32_t>(v[i][j] >> 32) != tag) v[i][j] = ld_relaxed_gpu_u64(word(i, j));
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const uint32_t q = q0 + i * kWarps;
                    if (q < nrec) {
                        float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
#pragma unroll
                        for (int j = 0; j < 8; ++j) stage[32 * j + lane] = __uint_as_float(static_cast<uint32_t>(v[i][j]));
                    }
                }
                __syncwarp();
                if (q0 + kWarps < nrec) {
                    const float* const vp[2] = {reinterpret_cast<const float*>(recs + q0 * kFragWords),
                                                reinterpret_cast<const float*>(recs + (q0 + kWarps) * kFragWords)};
                    uint32_t* const rp[2] = {recs + q0 * kFragWords, recs + (q0 + kWarps) * kFragWords};
                    q4k_frag_superblocks<2>(vp, rp, lane);       // both records' steps interleaved
                } else {
                    q4k_frag_superblock(reinterpret_cast<float*>(recs + q0 * kFragWords), recs + q0 * kFragWords, lane);
                }
                __syncwarp();
                const auto unit = [&](uint32_t q, float& r0, float& r1) {
                    const uint32_t sl = q / nsd, sb = q % nsd;
                    wait_bar(&dbars[sl]);
                    const uint8_t* bx = dtiles + sl * 16u * c.rb_down_max + sb * sbb;
                    chain35_down_mma(dtype, bx + g * rbd, bx + (g + 8) * rbd, recs + q * kFragWords, r0, r1);
                    r0 = quad_sum(r0);
                    r1 = quad_sum(r1);
                    if ((lane & 3) == 0) {
                        dpart[q * 16 + g] = r0;
                        dpart[q * 16 + g + 8] = r1;
                    }
                };
                float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
                unit(q0, a0, a1);
                if (q0 + kWarps < nrec) unit(q0 + kWarps, b0, b1);
            }
            // The shared slot: its activations into shared memory, then a
            // (row) FP32 dot per warp and pass.
            if (warp >= kWarps - static_cast<int>(kChain35SharedWarps)) {
                const uint32_t sw = static_cast<uint32_t>(warp) - (kWarps - kChain35SharedWarps);
                const unsigned long long* src = act_mine + static_cast<uint64_t>(k) * I;
                for (uint32_t w0 = sw * 32u + lane; w0 < I; w0 += 4u * kChain35SharedWarps * 32u) {
                    unsigned long long v[4];
                    bool use[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t w = w0 + i * kChain35SharedWarps * 32u;
                        use[i] = w < I;
                        v[i] = use[i] ? ld_relaxed_gpu_u64(src + w) : static_cast<unsigned long long>(tag) << 32;
                    }
                    long long t0 = 0;
                    for (uint32_t polls = 0;; ++polls) {
                        bool ready = true;
#pragma unroll
                        for (int i = 0; i < 4; ++i) ready = ready && static_cast<uint32_t>(v[i] >> 32) == tag;
                        if (__all_sync(0xffffffffu, ready)) break;
                        if (polls == 0) t0 = clock64();
                        if ((polls & 63u) == 63u &&
                            ((ld_acquire_gpu(status) & kStatusWaitTimeout) || clock64() - t0 > kBarrierTimeoutCycles)) {
                            if (lane == 0) {
                                atomicOr(status, kStatusWaitTimeout);
                                abort_sh = 1u;
                            }
                            break;
                        }
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            if (use[i] && static_cast<uint32_t>(v[i] >> 32) != tag)
                                v[i] = ld_relaxed_gpu_u64(src + w0 + i * kChain35SharedWarps * 32u);
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (use[i]) actsh[w0 + i * kChain35SharedWarps * 32u] = __uint_as_float(static_cast<uint32_t>(v[i]));
                }
                asm volatile("bar.sync 2, %0;" ::"r"(kChain35SharedWarps * 32u) : "memory");
                wait_bar(&dbars[k]);
                for (uint32_t r = sw; r < 16u; r += kChain35SharedWarps) {
                    float v = lane_row_dot_any(L.shared_down_type, dtiles + k * 16u * c.rb_down_max + r * c.rb_shared,
                                               I, actsh, lane);
                    v = warp_sum(v);
                    if (lane == 0) dsh[r] = v;
                }
            }
            stamp(l, 4);
            __syncthreads();
            if (abort_sh) {
                if (static_cast<uint32_t>(warp) < slots && lane == 0) mbar_wait(&dbars[warp], phase);
                ok = false;
                break;
            }
            stamp(l, 5);
            // Weighted slot rows (a thread per slot and row; the gate/up
            // partials' space is free), then in route order (qwen35_runner.cpp
            // :738-741) the gated shared expert (:760-763) and the residual.
            float* comb = part;
            if (static_cast<uint32_t>(tid) < k * 16u) {
                const uint32_t sl = static_cast<uint32_t>(tid) >> 4, row = tid & 15;
                float y = 0.0f;
                for (uint32_t sb = 0; sb < nsd; ++sb) y += dpart[(sl * nsd + sb) * 16u + row];
                comb[tid] = sel_w[sl] * y;
            }
            __syncthreads();
            if (tid < 16) {
                float moe = 0.0f;
                for (uint32_t sl = 0; sl < k; ++sl) moe += comb[sl * 16u + tid];
                const float sh = sel_w[k] * dsh[tid];
                const float h = resid + (moe + sh);
                a.hidden[j0 + tid] = h;
                if (has_next) {
                    const float xn = nnorm * h;
                    hrow[tid] = xn;
                    hrow[kPartRows + tid] = h * h;
                    for (uint32_t r = 0; r < kChainXReplicas; ++r)
                        a.C.xrep[static_cast<uint64_t>(r) * H + j0 + tid] = xn;
                }
            }
            if (has_next) {
                __syncthreads();
                stamp(l, 6);
                const uint32_t pn = (layer + 1u) % 3u;
                chain35_partials(E, rs, rs2, hrow, a.C.racc + pn * racc_span, a.C.rbad + pn,
                                 a.C.rsq + (p ^ 1u) * units, cta);
            }
        }
        chain_arrive(ctr_route);
        stamp(l, 7);
    }
    if (!ok) return;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        last_sh = atomicAdd(ctr_exit, 1u) == G - 1u ? 1u : 0u;
    }
    __syncthreads();
    if (!last_sh) return;
    __threadfence();
    const uint32_t plast = (a.first + a.count - 1u) % 3u;
    for (uint32_t i = tid; i < racc_span; i += kThreads) a.C.racc[plast * racc_span + i] = 0ull;
    __syncthreads();
    if (tid == 0) {
        a.C.rbad[plast] = 0u;
        *ctr_route = 0u;
        *ctr_exit = 0u;
        *ctr_seq = seq0 + a.count;
        if (a.with_delta) {
            a.delta.counters[0] = 0u;
            a.delta.counters[1] = 0u;
        }
        __threadfence();
    }
}

// ---------------------------------------------------------------------------
// Raises a kernel's dynamic shared-memory limit once per (kernel, device):
// cudaFuncSetAttribute applies to the current device only, so a grant made
// on one GPU says nothing about another.  Later launches skip the call, so
// they can be captured in graphs.
template <typename K>
cudaError_t ensure_smem(K kernel, size_t bytes) {
    if (bytes <= 48u * 1024u) return cudaSuccess;
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> granted;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    size_t& have = granted[{reinterpret_cast<const void*>(kernel), dev}];
    if (bytes <= have) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) have = bytes;
    return e;
}

uint64_t align256(uint64_t v) { return (v + 255u) & ~uint64_t(255); }

bool layer_valid(const MoeLayerDev& L) {
    return !(L.top_k == 0 || L.top_k > L.experts || L.top_k > kMaxTopK || L.experts > kMaxExperts ||
             L.hidden == 0 || (L.hidden & 255u) || L.inter == 0 || (L.inter & 255u) ||
             (L.shared_inter & 255u));
}

uint32_t block_down_ctas(const MoeLayerDev& L) { return (L.hidden + 15u) / 16u; }

}  // namespace

uint32_t moe_barriers_per_layer() { return 3u; }

uint64_t moe_scratch_bytes(const MoeLayerDev& L, uint32_t rep) {
    const uint64_t slots = L.top_k + 1u;
    uint64_t b = 0;
    b += align256(L.hidden * 4u);                                         // x
    b += align256((L.experts + 1u) * route_splits(L.hidden) * 4u);        // partial
    b += align256(L.experts * 4u);                                        // logits
    b += align256(L.top_k * 4u);                                          // ids
    b += align256(slots * 4u);                                            // weights
    b += align256(slots * max_inter_of(L) * 4u);                          // act
    b += align256((L.hidden >> 8) * kFragWords * 4u);                     // xrec
    b += align256(static_cast<uint64_t>(rep) * L.top_k * L.inter * 4u);  // actr
    b += align256(4u);                                                    // scale
    b += align256((L.hidden / kPartRows) * 4u);                           // rsq
    b += align256(L.experts * kRaccLimbs * 8u);                           // racc
    b += align256(4u);                                                    // rbad
    b += align256(4u);                                                    // route_count
    b += align256(4u);                                                    // counter
    b += align256(4u);                                                    // status
    return b;
}

MoeScratch moe_scratch_carve(const MoeLayerDev& L, void* base, uint32_t rep) {
    const uint64_t slots = L.top_k + 1u;
    uint8_t* p = static_cast<uint8_t*>(base);
    MoeScratch s;
    s.x = reinterpret_cast<float*>(p); p += align256(L.hidden * 4u);
    s.partial = reinterpret_cast<float*>(p); p += align256((L.experts + 1u) * route_splits(L.hidden) * 4u);
    s.logits = reinterpret_cast<float*>(p); p += align256(L.experts * 4u);
    s.ids = reinterpret_cast<uint32_t*>(p); p += align256(L.top_k * 4u);
    s.weights = reinterpret_cast<float*>(p); p += align256(slots * 4u);
    s.act = reinterpret_cast<float*>(p); p += align256(slots * max_inter_of(L) * 4u);
    s.xrec = reinterpret_cast<uint32_t*>(p); p += align256((L.hidden >> 8) * kFragWords * 4u);
    s.rep = rep;
    s.actr = reinterpret_cast<float*>(p); p += align256(static_cast<uint64_t>(rep) * L.top_k * L.inter * 4u);
    s.scale = reinterpret_cast<float*>(p); p += align256(4u);
    s.rsq = reinterpret_cast<float*>(p); p += align256((L.hidden / kPartRows) * 4u);
    // racc .. status end the carve and must be zero before a launch.
    s.racc = reinterpret_cast<unsigned long long*>(p); p += align256(L.experts * kRaccLimbs * 8u);
    s.rbad = reinterpret_cast<uint32_t*>(p); p += align256(4u);
    s.route_count = reinterpret_cast<uint32_t*>(p); p += align256(4u);
    s.counter = reinterpret_cast<uint32_t*>(p); p += align256(4u);
    s.status = reinterpret_cast<uint32_t*>(p);
    return s;
}

cudaError_t launch_route_experts(const float* logits, uint32_t E, uint32_t k, uint32_t flavour,
                                 uint32_t normalize, float ew_scale, uint32_t* ids, float* weights,
                                 uint32_t* status, cudaStream_t stream, uint32_t rows, uint32_t splits,
                                 bool pdl) {
    if (k == 0 || k > E || k > kMaxTopK || E > kMaxExperts || rows == 0 || splits == 0)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, route_logits_kernel, logits, E, k, flavour, normalize, ew_scale, ids, weights,
                              status, splits);
}

// ---------------------------------------------------------------------------
// Tensor maps of the expert tensors, encoded once per (tensor, shape).
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// (byte column, row, expert) view of a Q4_K expert tensor: `rows` rows of
// `row_bytes` per expert, experts `slice` bytes apart; boxes of one
// superblock (144 bytes) by `box_rows` rows.
bool encode_expert_map(CUtensorMap* map, const uint8_t* base, uint64_t row_bytes, uint64_t rows,
                       uint64_t experts, uint64_t slice, uint32_t box_rows) {
    static std::mutex mu;
    static std::map<std::tuple<const uint8_t*, uint64_t, uint64_t, uint64_t, uint64_t, uint32_t>, CUtensorMap>
        cache;
    const auto key = std::make_tuple(base, row_bytes, rows, experts, slice, box_rows);
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) {
        *map = it->second;
        return true;
    }
    const auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[3] = {row_bytes, rows, experts};
    const cuuint64_t strides[2] = {row_bytes, slice};
    if (box_rows == 0 || box_rows > 256 || box_rows > rows) return false;
    const cuuint32_t box[3] = {144u, box_rows, 1u};
    const cuuint32_t elem[3] = {1u, 1u, 1u};
    if (encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    // Callers of the handle-free entry pass their own tensors, so the key set
    // is open-ended: the cache is dropped whole once it holds kMaxMaps maps
    // (an encode is a host computation of about a microsecond).
    constexpr size_t kMaxMaps = 4096;
    if (cache.size() >= kMaxMaps) cache.clear();
    cache.emplace(key, *map);
    return true;
}

static bool aligned16(const void* p, uint64_t slice) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (slice & 15u) == 0;
}

// The tensor-core path serves the block (shapes, TMA alignment and
// shared-memory budgets).
static bool tensor_path(const MoeLayerDev& L) {
    return mma_path_ok(L) && aligned16(L.gate, L.gate_slice) && aligned16(L.up, L.up_slice) &&
           aligned16(L.down, L.down_slice) && mma_gate_up_layout(L).total <= 227u * 1024u &&
           mma_down_layout(L, L).total <= 227u * 1024u && tail_layout(L, 0).end <= 227u * 1024u;
}

static cudaError_t block_impl(const MoeLayerDev& L, const MoeScratch& S, const float* x_in,
                              float* hidden, float* moe_out, const MoeLayerDev* prev,
                              const MoeLayerDev* next, cudaStream_t stream, bool dry_run,
                              uint32_t* launches, cudaEvent_t* marks) {
    const auto mark = [&](uint32_t i) {
        if (marks) cudaEventRecord(marks[i], stream);
    };
    if (launches) *launches = 0;
    if (!layer_valid(L)) return cudaErrorInvalidValue;
    if (!hidden && (!x_in || !moe_out)) return cudaErrorInvalidValue;
    if (hidden && !L.ffn_norm) return cudaErrorInvalidValue;
    const int sms = device_sm_count();
    if (tensor_path(L)) {
        // In a decode chain of tensor-path blocks of one shape, each down
        // kernel routes the next block (partials and tail).
        const auto chains = [&](const MoeLayerDev* o) {
            return hidden && o && tensor_path(*o) && o->hidden == L.hidden && o->experts == L.experts &&
                   o->inter == L.inter && o->top_k == L.top_k;
        };
        const bool from_prev = chains(prev), to_next = chains(next);
        const MoeLayerDev& nx = to_next ? *next : L;
        const MmaLayout gl = mma_gate_up_layout(L), dl = mma_down_layout(L, nx);
        MmaLayout pl{};
        pl.tail = tail_layout(L, 0);
        pl.total = pl.tail.end;
        cudaError_t e = ensure_smem(moe_gate_up_mma_kernel, gl.total);
        if (e == cudaSuccess) e = ensure_smem(moe_down_mma_kernel, dl.total);
        if (e == cudaSuccess) e = ensure_smem(moe_partials_kernel, pl.total);
        if (e != cudaSuccess || dry_run) return e;
        MmaArgs ma{};
        const uint64_t rb_in = static_cast<uint64_t>(L.hidden >> 8) * 144u;
        const uint64_t rb_down = static_cast<uint64_t>(L.inter >> 8) * 144u;
        if (!encode_expert_map(&ma.tm_gate, L.gate, rb_in, L.inter, L.experts, L.gate_slice, kBoxRows) ||
            !encode_expert_map(&ma.tm_up, L.up, rb_in, L.inter, L.experts, L.up_slice, kBoxRows) ||
            !encode_expert_map(&ma.tm_down, L.down, rb_down, L.hidden, L.experts, L.down_slice, kBoxRows))
            return cudaErrorInvalidValue;
        ma.L = L;
        ma.next = nx;
        ma.has_next = to_next ? 1u : 0u;
        ma.S = S;
        ma.x_in = x_in;
        ma.hidden = hidden;
        ma.moe_out = hidden ? nullptr : moe_out;
        const uint32_t chunks = L.hidden / kPartRows;
        const uint32_t groups = L.top_k * (L.inter / 16u);
        uint32_t n = 0;
        mark(0);
        if (!from_prev) {
            ma.m = pl;
            moe_partials_kernel<<<chunks, kThreads, pl.total, stream>>>(ma);
            mark(++n);
        }
        ma.m = gl;
        {
            // The gate/up grid may launch while the routing tail (one CTA of
            // the previous kernel) finishes; it waits for it in-kernel.
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3((groups + kGuGroups - 1u) / kGuGroups);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = gl.total;
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = marks ? 0 : 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            const cudaError_t le = cudaLaunchKernelEx(&cfg, moe_gate_up_mma_kernel, ma);
            if (le != cudaSuccess) return le;
        }
        mark(++n);
        ma.m = dl;
        {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(chunks);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = dl.total;
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = marks ? 0 : 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            const cudaError_t le = cudaLaunchKernelEx(&cfg, moe_down_mma_kernel, ma);
            if (le != cudaSuccess) return le;
        }
        mark(++n);
        if (launches) *launches = n;
        return cudaGetLastError();
    }
    const uint32_t down_ctas = block_down_ctas(L);
    BlockArgs a{};
    a.L = L;
    a.S = S;
    a.x_in = x_in;
    a.hidden = hidden;
    a.moe_out = moe_out;
    a.next_router = next ? next->router : nullptr;
    a.down_ctas = down_ctas;
    // Kernel 1 uses enough CTAs to give every router task its own warp.
    const uint32_t tasks = (L.experts + (L.shared_inter ? 1u : 0u)) * route_splits(L.hidden);
    const uint32_t g1 = std::min<uint32_t>(static_cast<uint32_t>(sms), (tasks + kWarps - 1) / kWarps);
    const SmemLayout rl = route_layout(L);
    a.m = make_layout(L, down_ctas);
    if (a.m.total > 227u * 1024u || rl.total > 227u * 1024u) return cudaErrorInvalidValue;
    cudaError_t e = ensure_smem(moe_route_kernel, rl.total);
    if (e == cudaSuccess) e = ensure_smem(moe_gate_up_kernel, a.m.total);
    if (e == cudaSuccess) e = ensure_smem(moe_down_kernel, a.m.total);
    if (e != cudaSuccess || dry_run) return e;
    BlockArgs ra = a;
    ra.m = rl;
    // Each kernel is a programmatic dependent of the one before (it waits in-
    // kernel before reading its predecessor's output); plain launches when
    // per-kernel events are recorded.
    const auto launch = [&](void (*k)(BlockArgs), uint32_t grid, uint32_t smem, const BlockArgs& args) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = marks ? 0 : 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, k, args);
    };
    mark(0);
    if ((e = launch(moe_route_kernel, g1, rl.total, ra)) != cudaSuccess) return e;
    mark(1);
    if ((e = launch(moe_gate_up_kernel, sms, a.m.total, a)) != cudaSuccess) return e;
    mark(2);
    if ((e = launch(moe_down_kernel, down_ctas, a.m.total, a)) != cudaSuccess) return e;
    mark(3);
    if (launches) *launches = 3;
    return cudaGetLastError();
}

cudaError_t launch_moe_block(const MoeLayerDev& L, const MoeScratch& S, const float* x_in,
                             float* hidden, float* moe_out, const MoeLayerDev* prev,
                             const MoeLayerDev* next, cudaStream_t stream, uint32_t* launches,
                             cudaEvent_t* marks) {
    return block_impl(L, S, x_in, hidden, moe_out, prev, next, stream, false, launches, marks);
}

cudaError_t time_moe_kernel(const MoeLayerDev* layers, uint32_t count, const MoeScratch& S, uint32_t which,
                            uint32_t reps, float* out, cudaStream_t stream, float* avg_us) {
    if (!layers || count == 0 || reps == 0 || !out || !avg_us || which > 1) return cudaErrorInvalidValue;
    for (uint32_t l = 0; l < count; ++l)
        if (!tensor_path(layers[l])) return cudaErrorNotSupported;
    // Routes, x records and scale of layers[0] for every launch.
    cudaError_t e = block_impl(layers[0], S, out, nullptr, out, nullptr, nullptr, stream, false, nullptr, nullptr);
    if (e != cudaSuccess) return e;
    std::vector<MmaArgs> args(count);
    for (uint32_t l = 0; l < count; ++l) {
        const MoeLayerDev& L = layers[l];
        MmaArgs& ma = args[l];
        const uint64_t rb_in = static_cast<uint64_t>(L.hidden >> 8) * 144u;
        const uint64_t rb_down = static_cast<uint64_t>(L.inter >> 8) * 144u;
        if (!encode_expert_map(&ma.tm_gate, L.gate, rb_in, L.inter, L.experts, L.gate_slice, kBoxRows) ||
            !encode_expert_map(&ma.tm_up, L.up, rb_in, L.inter, L.experts, L.up_slice, kBoxRows) ||
            !encode_expert_map(&ma.tm_down, L.down, rb_down, L.hidden, L.experts, L.down_slice, kBoxRows))
            return cudaErrorInvalidValue;
        ma.L = L;
        ma.next = L;
        ma.S = S;
        ma.x_in = out;
        ma.moe_out = out;
        ma.m = which == 0 ? mma_gate_up_layout(L) : mma_down_layout(L, L);
    }
    const uint32_t groups = layers[0].top_k * (layers[0].inter / 16u);
    const uint32_t g_gate_up = (groups + kGuGroups - 1u) / kGuGroups, g_down = layers[0].hidden / kPartRows;
    // The repetitions replay from a CUDA graph (captured on a private stream)
    // so the host launch rate does not pace the device.
    e = cudaStreamSynchronize(stream);
    cudaStream_t cap = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        for (uint32_t i = 0; i < reps; ++i) {
            const MmaArgs& ma = args[i % count];
            if (which == 0) moe_gate_up_mma_kernel<<<g_gate_up, kThreads, ma.m.total, cap>>>(ma);
            else moe_down_mma_kernel<<<g_down, kThreads, ma.m.total, cap>>>(ma);
        }
        const cudaError_t end = cudaStreamEndCapture(cap, &graph);
        e = end;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, cap);          // warm-up replay
    if (e == cudaSuccess) e = cudaEventCreate(&a);
    if (e == cudaSuccess) e = cudaEventCreate(&b);
    if (e == cudaSuccess) e = cudaEventRecord(a, cap);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, cap);
    if (e == cudaSuccess) e = cudaEventRecord(b, cap);
    if (e == cudaSuccess) e = cudaEventSynchronize(b);
    float ms = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (cap) cudaStreamDestroy(cap);
    if (e == cudaSuccess) *avg_us = ms * 1e3f / static_cast<float>(reps);
    return e;
}

// Router accumulators cover the experts and, with a shared expert, its gate
// row (index `experts`); activation words cover the routed slots and the
// shared expert's.
static uint64_t chain_router_rows(const MoeLayerDev& L) { return L.experts + (L.shared_inter ? 1u : 0u); }
static uint64_t chain_act_words(const MoeLayerDev& L) {
    return static_cast<uint64_t>(L.top_k + (L.shared_inter ? 1u : 0u)) * umax(L.inter, L.shared_inter);
}

uint64_t moe_chain_scratch_bytes(const MoeLayerDev& L) {
    return align256(3ull * chain_router_rows(L) * kRaccLimbs * 8u) + align256(2ull * (L.hidden / kPartRows) * 4u) +
           align256(3u * 4u) + align256(static_cast<uint64_t>(kChainXReplicas) * L.hidden * 4u) +
           align256(static_cast<uint64_t>(kChainXReplicas) * chain_act_words(L) * 8u) + 4u * kChainCounterStride * 4u;
}

ChainScratch moe_chain_scratch_carve(const MoeLayerDev& L, void* base) {
    uint8_t* p = static_cast<uint8_t*>(base);
    ChainScratch c;
    c.racc = reinterpret_cast<unsigned long long*>(p); p += align256(3ull * chain_router_rows(L) * kRaccLimbs * 8u);
    c.rsq = reinterpret_cast<float*>(p); p += align256(2ull * (L.hidden / kPartRows) * 4u);
    c.rbad = reinterpret_cast<uint32_t*>(p); p += align256(3u * 4u);
    c.xrep = reinterpret_cast<float*>(p); p += align256(static_cast<uint64_t>(kChainXReplicas) * L.hidden * 4u);
    c.act = reinterpret_cast<unsigned long long*>(p);
    p += align256(static_cast<uint64_t>(kChainXReplicas) * chain_act_words(L) * 8u);
    c.counters = reinterpret_cast<uint32_t*>(p);
    return c;
}

// (8-byte column, row, expert, layer) view of one Q4_K tensor kind across
// the layers of a pool: `rows` rows of `row_bytes` per expert, experts
// `slice` bytes apart, layers `layer_stride` bytes apart; boxes of two
// superblocks (288 bytes) by 16 rows.
static bool encode_pool_map(CUtensorMap* map, const uint8_t* base, uint64_t row_bytes, uint64_t rows,
                            uint64_t experts, uint64_t slice, uint64_t layers, uint64_t layer_stride) {
    const auto encode = tensor_map_encoder();
    if (!encode || (reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes & 15u) || (slice & 15u) ||
        (layer_stride & 15u))
        return false;
    if (row_bytes % 8u) return false;
    const cuuint64_t dims[4] = {row_bytes / 8u, rows, experts, layers};
    const cuuint64_t strides[3] = {row_bytes, slice, layers > 1 ? layer_stride : slice * experts};
    const cuuint32_t box[4] = {kPairRowBytes / 8u, kBoxRows, 1u, 1u};
    const cuuint32_t elem[4] = {1u, 1u, 1u, 1u};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<uint8_t*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool moe_chain_plan(const MoeLayerDev* layers, uint32_t n, ChainPlan* plan) {
    if (!layers || n == 0 || !plan) return false;
    const MoeLayerDev& L0 = layers[0];
    if (!layer_valid(L0) || !tensor_path(L0) || !L0.ffn_norm || L0.expert_local != 0 && L0.expert_local != L0.experts)
        return false;
    const int64_t stride = n > 1 ? layers[1].gate - layers[0].gate : 0;
    for (uint32_t l = 0; l < n; ++l) {
        const MoeLayerDev& L = layers[l];
        const auto at = [&](const void* q, const void* q0) {
            return static_cast<const uint8_t*>(q) - static_cast<const uint8_t*>(q0) == stride * l;
        };
        if (!tensor_path(L) || !L.ffn_norm || !L.router || L.hidden != L0.hidden || L.inter != L0.inter ||
            L.experts != L0.experts || L.top_k != L0.top_k || L.flavour != L0.flavour ||
            L.normalize != L0.normalize || L.expert_weights_scale != L0.expert_weights_scale ||
            L.rms_eps != L0.rms_eps || L.gate_slice != L0.gate_slice || L.up_slice != L0.up_slice ||
            L.down_slice != L0.down_slice || !at(L.gate, L0.gate) || !at(L.up, L0.up) || !at(L.down, L0.down) ||
            !at(L.router, L0.router) || !at(L.ffn_norm, L0.ffn_norm) || (reinterpret_cast<uintptr_t>(L.router) & 15u))
            return false;
    }
    if (stride < 0) return false;
    const uint32_t sms = static_cast<uint32_t>(device_sm_count());
    const uint32_t units = L0.hidden / kPartRows, groups = L0.top_k * (L0.inter / 16u);
    const ChainLayout c = chain_layout(L0);
    // Every CTA owns at least one gate/up row group (its activation words
    // order its routing reads before the D units' next writes).
    if (units > sms || groups > kChainGroupsPerCta * sms || groups < sms || L0.experts > kThreads ||
        c.total > 227u * 1024u || (L0.hidden >> 8) > 64u)
        return false;
    if (ensure_smem(moe_chain_kernel<false>, c.total) != cudaSuccess ||
        ensure_smem(moe_chain_kernel<true>, c.total) != cudaSuccess)
        return false;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_chain_kernel<false>, kThreads, c.total) != cudaSuccess ||
        per_sm < 1)
        return false;
    const uint64_t rb_in = static_cast<uint64_t>(L0.hidden >> 8) * 144u;
    const uint64_t rb_down = static_cast<uint64_t>(L0.inter >> 8) * 144u;
    if (!encode_pool_map(&plan->tm_gate, L0.gate, rb_in, L0.inter, L0.experts, L0.gate_slice, n, stride) ||
        !encode_pool_map(&plan->tm_up, L0.up, rb_in, L0.inter, L0.experts, L0.up_slice, n, stride) ||
        !encode_pool_map(&plan->tm_down, L0.down, rb_down, L0.hidden, L0.experts, L0.down_slice, n, stride))
        return false;
    plan->shape = L0;
    plan->stride = static_cast<uint64_t>(stride);
    plan->layers = n;
    plan->grid = sms;
    plan->smem = c.total;
    return true;
}

// (8-byte column, row) view of a shared expert's Q8_0 gate or up: boxes of
// kChain35SharedRows rows by half a row.
static bool encode_shared_half_map(CUtensorMap* map, const uint8_t* base, uint64_t row_bytes, uint64_t rows) {
    const auto encode = tensor_map_encoder();
    if (!encode || (reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes % 16u) || ((row_bytes / 2u) % 16u) ||
        row_bytes / 16u > 256u || rows < kChain35SharedRows)
        return false;
    const cuuint64_t dims[2] = {row_bytes / 8u, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(row_bytes / 16u), kChain35SharedRows};
    const cuuint32_t elem[2] = {1u, 1u};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// (8-byte column, row, expert) view of a layer's routed Q4_K gate or up:
// boxes of two superblocks (288 bytes) by 16 rows.
static bool encode_pair_map(CUtensorMap* map, const uint8_t* base, uint64_t row_bytes, uint64_t rows,
                            uint64_t experts, uint64_t slice) {
    const auto encode = tensor_map_encoder();
    if (!encode || (reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes & 15u) || (slice & 15u)) return false;
    const cuuint64_t dims[3] = {row_bytes / 8u, rows, experts};
    const cuuint64_t strides[2] = {row_bytes, slice};
    const cuuint32_t box[3] = {kPairRowBytes / 8u, kBoxRows, 1u};
    const cuuint32_t elem[3] = {1u, 1u, 1u};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool moe_chain35_plan(const MoeLayerDev* layers, uint32_t n, Chain35Plan* plan, std::vector<Chain35Maps>* maps) {
    if (!layers || n == 0 || !plan || !maps) return false;
    const MoeLayerDev& L0 = layers[0];
    const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const auto down_ok = [](uint32_t t) { return t == kQ4_K || t == kQ5_K || t == kQ6_K; };
    if (!layer_valid(L0) || L0.flavour != 1u || L0.shared_inter == 0 || L0.shared_inter != L0.inter ||
        (L0.expert_local != 0 && L0.expert_local != L0.experts) || L0.experts > 512u ||
        L0.top_k + 1u > static_cast<uint32_t>(kWarps) || L0.top_k > static_cast<uint32_t>(kMaxTopK) ||
        L0.hidden % 512u || (L0.hidden >> 8) > 64u || L0.inter % 256u)
        return false;
    uint32_t rb_max = 0;
    for (uint32_t l = 0; l < n; ++l) {
        const MoeLayerDev& L = layers[l];
        if (L.hidden != L0.hidden || L.inter != L0.inter || L.experts != L0.experts || L.top_k != L0.top_k ||
            L.flavour != L0.flavour || L.normalize != L0.normalize ||
            L.expert_weights_scale != L0.expert_weights_scale || L.rms_eps != L0.rms_eps ||
            L.shared_inter != L0.shared_inter || L.gate_type != kQ4_K || L.up_type != kQ4_K ||
            !down_ok(L.down_type) || L.shared_gate_type != kQ8_0 || L.shared_up_type != kQ8_0 ||
            L.shared_down_type != kQ8_0 || !L.router || !L.ffn_norm || !L.shared_router || !L.gate || !L.up ||
            !L.down || !L.shared_gate || !L.shared_up || !L.shared_down || !a16(L.gate) || !a16(L.up) ||
            !a16(L.down) || !a16(L.shared_down) || !a16(L.router) || !a16(L.shared_router) || !a16(L.shared_gate) ||
            !a16(L.shared_up) || L.gate_slice % 16u || L.up_slice % 16u || L.down_slice % 16u)
            return false;
        rb_max = umax(rb_max, static_cast<uint32_t>(row_bytes(L.down_type, L.inter)));
    }
    const uint32_t sms = static_cast<uint32_t>(device_sm_count());
    const uint32_t units = L0.hidden / kPartRows;
    const uint32_t groups = L0.top_k * (L0.inter / 16u) + L0.shared_inter / kChain35SharedRows;
    const Chain35Layout c = chain35_layout(L0, rb_max);
    // A shared-expert group's half rows fill at most one warp's tile space.
    const uint64_t shared_tile = kChain35SharedRows * (row_bytes(kQ8_0, L0.hidden) / 2u);
    if (units > sms || groups > kChainGroupsPerCta * sms || groups < sms || c.total > 227u * 1024u ||
        shared_tile > static_cast<uint64_t>(c.gpairs) * kPairBytes || (row_bytes(kQ8_0, L0.hidden) / 2u) % 16u)
        return false;
    if (ensure_smem(moe_chain35_kernel, c.total) != cudaSuccess) return false;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_chain35_kernel, kThreads, c.total) != cudaSuccess ||
        per_sm < 1)
        return false;
    std::vector<Chain35Maps> m(n);
    const uint64_t rb_in = row_bytes(kQ4_K, L0.hidden), rb_shared = row_bytes(kQ8_0, L0.hidden);
    for (uint32_t l = 0; l < n; ++l) {
        const MoeLayerDev& L = layers[l];
        if (!encode_pair_map(&m[l].gate, L.gate, rb_in, L.inter, L.experts, L.gate_slice) ||
            !encode_pair_map(&m[l].up, L.up, rb_in, L.inter, L.experts, L.up_slice) ||
            !encode_shared_half_map(&m[l].shared_gate, L.shared_gate, rb_shared, L.shared_inter) ||
            !encode_shared_half_map(&m[l].shared_up, L.shared_up, rb_shared, L.shared_inter))
            return false;
    }
    plan->shape = L0;
    plan->layers = n;
    plan->grid = sms;
    plan->smem = c.total;
    plan->rb_down_max = rb_max;
    *maps = std::move(m);
    return true;
}

bool moe_chain35_delta_fits(const Chain35Plan& plan, const DeltaBlockShape& d) {
    const Chain35Layout c = chain35_layout(plan.shape, plan.rb_down_max);
    return plan.grid != 0 && d.hidden == plan.shape.hidden &&
           db_layout(d.hidden, d.value_heads * kDbHeadDim).total <= c.total - c.gtiles;
}

bool moe_chain35_attention_fits(const Chain35Plan& plan, const void* att_args, size_t bytes) {
    if (!att_args || bytes != sizeof(AttnBlockArgs) || plan.grid == 0) return false;
    AttnBlockArgs at;
    std::memcpy(&at, att_args, sizeof at);
    const Chain35Layout c = chain35_layout(plan.shape, plan.rb_down_max);
    // The attention phase's own limits (as the standalone block's planner
    // sets them): a Q/K/V row block per CTA, an output unit and query head
    // per CTA at most, two output superblocks per warp.
    const uint32_t G = plan.grid;
    if (at.rows % 16u || at.qd % 256u || at.H % 256u || at.rows / 16u < G || at.H / 16u > G || at.sh.qh > G ||
        at.qd / 256u > 8u * kAttnMaxOutPerWarp || at.H / 256u > 2u * kWarps || at.layers > 255u)
        return false;
    return at.H == plan.shape.hidden && at.sh.d <= static_cast<uint32_t>(kThreads) &&
           attn_block_layout(at.H, at.rows, at.qd, at.sh.d, at.sh.rh, at.sh.window, plan.grid, kWarps).total <=
               c.total - c.gtiles;
}

cudaError_t launch_moe_chain35(const Chain35Plan& plan, const MoeLayerDev* layers_dev, const Chain35Maps* maps_dev,
                               uint32_t first, uint32_t count, const MoeScratch& S, const ChainScratch& C,
                               float* hidden, cudaStream_t stream, unsigned long long* trace,
                               const DeltaBlockShape* delta_shape, const DeltaBlockTensors* delta,
                               const void* att_args, size_t att_bytes) {
    if (!hidden || !layers_dev || !maps_dev || count == 0 || first >= plan.layers || count > plan.layers - first ||
        plan.grid == 0)
        return cudaErrorInvalidValue;
    if (delta_shape || delta) {
        const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
        if (!delta_shape || !delta || count != 1 || !moe_chain35_delta_fits(plan, *delta_shape) ||
            delta->hidden != hidden || !a16(delta->w_in) || !a16(delta->w_out) || !a16(delta->state) ||
            !delta->counters || !delta->timeout || !delta->gates_bad || !delta->proj || !delta->att ||
            !delta->ms_part)
            return cudaErrorInvalidValue;
    }
    Chain35Args a{};
    a.layers = layers_dev;
    a.shape = plan.shape;
    a.first = first;
    a.count = count;
    a.S = S;
    a.C = C;
    a.hidden = hidden;
    a.c = chain35_layout(plan.shape, plan.rb_down_max);
    a.maps = maps_dev;
    a.trace = trace;
    if (delta) {
        a.delta = make_delta_args(*delta_shape, *delta);
        a.with_delta = 1u;
    }
    if (att_args) {
        if (delta || count != 1 || !moe_chain35_attention_fits(plan, att_args, att_bytes))
            return cudaErrorInvalidValue;
        std::memcpy(&a.att, att_args, sizeof a.att);
        if (a.att.hidden != hidden) return cudaErrorInvalidValue;
        a.with_att = 1u;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, moe_chain35_kernel, a);
}

uint32_t chain_tile_offset(const ChainPlan& plan) { return chain_layout(plan.shape).gtiles; }

uint32_t chain_attention_smem(const ChainPlan& plan, const ChainAttnDesc& att) {
    return attn_block_layout(plan.shape.hidden, att.rows, att.q_heads * att.head_dim, att.head_dim, att.rotary_half,
                             att.window, plan.grid, kWarps)
        .total;
}

cudaError_t launch_moe_chain(const ChainPlan& plan, const MoeLayerDev* layers_dev, uint32_t first, uint32_t count,
                             const MoeScratch& S, const ChainScratch& C, float* hidden, cudaStream_t stream,
                             unsigned long long* trace, const ChainAttnDesc* attention) {
    (void)layers_dev;
    if (!hidden || count == 0 || first >= plan.layers || count > plan.layers - first || plan.grid == 0)
        return cudaErrorInvalidValue;
    if (attention) {
        // The attention phase runs in the tile region (gate/up and down tiles
        // are not live then); every CTA owns a Q/K/V row block, the output
        // units are the chain's D units and the query heads fit the grid.
        const ChainAttnDesc& t = *attention;
        const ChainLayout cl = chain_layout(plan.shape);
        const uint32_t qd = t.q_heads * t.head_dim;
        if (!t.wqkv || !t.wo || !t.pos || !t.qkv_words || !t.att_words || !t.hidden_words || !t.status ||
            t.rows % 16u || t.rows / 16u < plan.grid || plan.shape.hidden / 16u > plan.grid || t.q_heads > plan.grid ||
            t.head_dim == 0 || t.head_dim > kAttendMaxDim || t.head_dim > kThreads || qd % 256u ||
            qd / 256u > kWarps * kAttnMaxOutPerWarp || plan.shape.hidden / 256u > 2u * kWarps ||
            chain_attention_smem(plan, t) > plan.smem - cl.gtiles)
            return cudaErrorInvalidValue;
    }
    ChainArgs a{};
    a.tm_gate = plan.tm_gate;
    a.tm_up = plan.tm_up;
    a.tm_down = plan.tm_down;
    a.router0 = plan.shape.router;
    a.norm0 = plan.shape.ffn_norm;
    a.stride = plan.stride;
    a.shape = plan.shape;
    a.first = first;
    a.count = count;
    a.S = S;
    a.C = C;
    a.hidden = hidden;
    a.c = chain_layout(plan.shape);
    a.trace = trace;
    if (attention) {
        a.att = *attention;
        a.with_att = 1u;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return attention ? cudaLaunchKernelEx(&cfg, moe_chain_kernel<true>, a)
                     : cudaLaunchKernelEx(&cfg, moe_chain_kernel<false>, a);
}

cudaError_t prepare_moe_block(const MoeLayerDev& L) {
    MoeScratch none;
    float dummy = 0.0f;
    cudaError_t e = block_impl(L, none, &dummy, nullptr, &dummy, nullptr, nullptr, nullptr, true, nullptr, nullptr);
    if (e != cudaSuccess) return e;
    const SmemLayout m = make_layout(L, static_cast<uint32_t>(device_sm_count()));
    if (m.total > 227u * 1024u) return cudaErrorInvalidValue;
    return ensure_smem(moe_decode_kernel, m.total);
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
    cudaError_t e = ensure_smem(moe_decode_kernel, a.m.total);
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
