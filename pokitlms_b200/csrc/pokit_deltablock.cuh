// pokit_deltablock.cuh -- the Gated DeltaNet layer's mixer as device code
// (delta_layer_run), shared by its own cooperative kernel (pokit_deltablock.cu)
// and the Qwen3.5-MoE decode chain, which runs it ahead of a MoE block in the
// same launch.  Phases, layout and waits: pokit_deltablock.cu.
#pragma once

#include "pokit_kernels.h"
#include "pokit_mma.cuh"

namespace pokit {
namespace {


constexpr int kDbThreads = 384, kDbWarps = kDbThreads / 32;
constexpr uint32_t kDbMaxTiles = 6;               // in-projection tiles per CTA
constexpr uint32_t kDbPitchPad = 32;
constexpr uint32_t kDbHeadDim = 128;              // key and value head dims this kernel takes
constexpr uint32_t kDbMaxConv = 8;
constexpr uint32_t kDbSplit = 4;                  // CTAs per value head in phase 2 (32 rows each)
constexpr long long kDbTimeoutCycles = 4000000000LL;   // ~2 s at 2 GHz

struct DeltaBlockArgs {
    const uint8_t* w_in;      // Q4_K [rows_in][H]: q | k | v | z | alpha | beta
    const uint8_t* w_out;     // Q4_K [H][vw]
    const float* attn_norm;   // [H]
    const float* conv_w;      // [conv_ch][K]
    float* conv_state;        // [conv_ch][K - 1]
    const float* ssm_a;       // [hv]
    const float* dt_bias;     // [hv]
    const float* ssm_norm;    // [dv]
    float* state;             // [hv][dv][dk]
    float* hidden;            // [H], the residual (in and out)
    float* proj;              // [rows_in] scratch: conv'd q|k|v, raw z|alpha|beta
    float* att;               // [vw] scratch: the heads' raw outputs o
    float* ms_part;           // [hv * kDbSplit] scratch: per quarter-head sums of o^2 (-1: invalid gates)
    uint32_t* counters;       // [2] arrivals and exits (zero between launches)
    uint32_t* timeout;        // set when a bounded wait gives up
    uint32_t* gates_bad;      // bit 0: an invalid decay or beta (the step kernel's status)
    uint32_t H, rows_in, conv_ch, kh, hv, K;
    float norm_eps, eps;
};

struct DbLayout {
    uint32_t tiles, state, recs, part, xs, zs, total;
    uint32_t pitch_in, pitch_out;
};

__host__ __device__ inline DbLayout db_layout(uint32_t H, uint32_t vw) {
    DbLayout L{};
    L.pitch_in = (H / 256u) * 144u + kDbPitchPad;
    L.pitch_out = (vw / 256u) * 144u + kDbPitchPad;
    const uint32_t tiles = kDbMaxTiles * 16u * L.pitch_in, out_tile = 16u * L.pitch_out;
    const uint32_t nrec = (H / 256u) > (vw / 256u) ? H / 256u : vw / 256u;
    uint32_t off = 0;
    L.tiles = off; off += (tiles > out_tile ? tiles : out_tile);
    off = (off + 127u) & ~127u;
    // The head quarter's state in phase 2, then z (the output gate) in phase 3.
    const uint32_t st = (kDbHeadDim / kDbSplit) * kDbHeadDim * 4u, zb = vw * 4u;
    L.state = off; off += (st > zb ? st : zb);
    L.recs = off; off += nrec * kFragWords * 4u;
    L.part = off;
    const uint32_t p1 = kDbMaxTiles * (H / 256u) * 16u * 4u, p3 = (vw / 256u) * 16u * 4u;
    off += (p1 > p3 ? p1 : p3);
    L.xs = off; off += H * 4u;
    L.zs = off; off += vw * 4u;
    L.total = off;
    return L;
}

__device__ __forceinline__ uint32_t db_ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier `n` (1, 2, ...): every CTA's writes so far before any CTA
// goes on.  False when the wait gave up (or another CTA did).
__device__ bool db_grid_barrier(uint32_t* ctr, uint32_t target, uint32_t* timeout, uint32_t* abort_sh) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        const long long t0 = clock64();
        uint32_t polls = 0;
        while (static_cast<int32_t>(db_ld_acquire(ctr) - target) < 0) {
            if ((++polls & 63u) == 0) {
                if (db_ld_acquire(timeout)) { *abort_sh = 1u; break; }
                if (clock64() - t0 > kDbTimeoutCycles) {
                    atomicOr(timeout, 1u);
                    *abort_sh = 1u;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return *abort_sh == 0u;
}

__device__ __forceinline__ float db_sigmoid(float v) {
    if (v >= 0.0f) return 1.0f / (1.0f + expf(-v));
    const float e = expf(v);
    return e / (1.0f + e);
}
__device__ __forceinline__ float db_softplus(float v) {
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return log1pf(expf(v));
}
__device__ float db_block_sum(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = 0.0f;
    for (int w = 0; w < kDbWarps; ++w) r += red[w];
    return r;
}

// The wait on a bulk copy: bounded; on a timeout the flag is set and the
// wait repeated once more (a copy may still write the buffer).
__device__ __forceinline__ bool db_wait_copy(uint64_t* bar, uint32_t* timeout) {
    if (mbar_wait(bar, 0)) return true;
    if ((threadIdx.x & 31) == 0) atomicOr(timeout, 1u);
    mbar_wait(bar, 0);
    return false;
}

// One DeltaNet layer's mixer over the grid (every CTA calls it): phases 1-3
// in the dynamic shared memory at `smem` (db_layout's bytes).  False when a
// bounded wait gave up; the counters are left for the caller to reset.
__device__ __forceinline__ bool delta_layer_run(const DeltaBlockArgs& a, uint8_t* smem) {
    __shared__ uint64_t bars[3];                 // in-projection tiles, head state, ssm_out tile
    __shared__ float red[32], nq[kDbHeadDim], nk[kDbHeadDim], ob[kDbHeadDim];
    __shared__ uint32_t abort_sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2;
    const uint32_t G = gridDim.x, cta = blockIdx.x;
    const uint32_t H = a.H, nsb_in = H / 256u, dk = kDbHeadDim, dv = kDbHeadDim, vw = a.hv * dv;
    const uint32_t nsb_out = vw / 256u, K = a.K, sl = K - 1u;
    const DbLayout Ly = db_layout(H, vw);
    uint8_t* tiles = smem + Ly.tiles;
    float* S = reinterpret_cast<float*>(smem + Ly.state);
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + Ly.recs);
    float* part = reinterpret_cast<float*>(smem + Ly.part);
    float* xs = reinterpret_cast<float*>(smem + Ly.xs);
    float* zs = reinterpret_cast<float*>(smem + Ly.zs);
    const uint32_t ntiles_in = a.rows_in / 16u;
    const uint32_t mine = cta < ntiles_in ? (ntiles_in - cta + G - 1u) / G : 0u;   // <= kDbMaxTiles
    const uint64_t rb_in = static_cast<uint64_t>(nsb_in) * 144u, rb_out = static_cast<uint64_t>(nsb_out) * 144u;
    const uint32_t rows2 = dv / kDbSplit;
    const bool head = cta < a.hv * kDbSplit, out_tile = cta < H / 16u;
    const uint32_t h2 = cta / kDbSplit, r0 = (cta % kDbSplit) * rows2;    // phase 2: head, first row
    if (tid == 0) {
        abort_sh = 0u;
        for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
        // Byte counts first, then the copies (which may land at once).
        if (mine) mbar_expect_tx(&bars[0], mine * 16u * static_cast<uint32_t>(rb_in));
        if (head) mbar_expect_tx(&bars[1], rows2 * dk * 4u);
    }
    __syncthreads();
    // The in-projection tiles (a lane per row) and this head's state.
    if (static_cast<uint32_t>(warp) < mine && lane < 16) {
        const uint32_t t = cta + G * static_cast<uint32_t>(warp);
        bulk_copy_g2s(tiles + (warp * 16u + lane) * Ly.pitch_in, a.w_in + static_cast<uint64_t>(t * 16u + lane) * rb_in,
                      static_cast<uint32_t>(rb_in), &bars[0]);
    }
    if (head && tid == kDbThreads - 1)
        bulk_copy_g2s(S, a.state + (static_cast<uint64_t>(h2) * dv + r0) * dk, rows2 * dk * 4u, &bars[1]);

    // ---- phase 1: x' records, the in-projection, conv1d ----
    {
        // This thread's conv row (if any): weights and history, early.
        const bool conv_row = static_cast<uint32_t>(tid) < mine * 16u &&
                              (cta + G * (static_cast<uint32_t>(tid) >> 4)) * 16u + (tid & 15) < a.conv_ch;
        float cw[kDbMaxConv], hist[kDbMaxConv];
        if (conv_row) {
            const uint32_t row = (cta + G * (static_cast<uint32_t>(tid) >> 4)) * 16u + (tid & 15);
#pragma unroll
            for (uint32_t t = 0; t < kDbMaxConv; ++t) {
                cw[t] = t < K ? a.conv_w[static_cast<uint64_t>(row) * K + t] : 0.0f;
                hist[t] = t < sl ? a.conv_state[static_cast<uint64_t>(row) * sl + t] : 0.0f;
            }
        }
        float ss = 0.0f;
        for (uint32_t i = tid * 4u; i < H; i += kDbThreads * 4u) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(a.hidden + i));
            *reinterpret_cast<float4*>(xs + i) = v;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        const float total = db_block_sum(ss, red);
        const float scale = 1.0f / sqrtf(total / static_cast<float>(H) + a.norm_eps);
        for (uint32_t q = warp; q < nsb_in; q += kDbWarps) {
            float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t c = q * 256u + 32u * j + lane;
                v[j] = __fmul_rn(__fmul_rn(xs[c], scale), a.attn_norm[c]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) stage[32 * j + lane] = v[j];
            __syncwarp();
            q4k_frag_superblock(stage, recs + q * kFragWords, lane);
            __syncwarp();
        }
        __syncthreads();
        if (mine && !db_wait_copy(&bars[0], a.timeout) && lane == 0) abort_sh = 1u;
        for (uint32_t p = warp; p < mine * nsb_in; p += kDbWarps) {
            const uint32_t i = p / nsb_in, sb = p % nsb_in;
            const uint8_t* t = tiles + i * 16u * Ly.pitch_in + sb * 144u;
            float acc0 = 0.0f, acc1 = 0.0f;
            q4k_mma_superblock(t + g * Ly.pitch_in, t + (g + 8) * Ly.pitch_in, recs + sb * kFragWords, acc0, acc1);
            acc0 = quad_sum(acc0);
            acc1 = quad_sum(acc1);
            if ((lane & 3) == 0) {
                part[p * 16u + g] = acc0;
                part[p * 16u + g + 8] = acc1;
            }
        }
        __syncthreads();
        if (static_cast<uint32_t>(tid) < mine * 16u) {
            const uint32_t i = tid >> 4, r = tid & 15;
            const uint32_t row = (cta + G * i) * 16u + r;
            float v = part[(i * nsb_in) * 16u + r];
            for (uint32_t sb = 1; sb < nsb_in; ++sb) v += part[(i * nsb_in + sb) * 16u + r];
            if (conv_row) {
                // causal_depthwise_conv1d_step + SiLU (delta_conv_kernel's arithmetic).
                float* st = a.conv_state + static_cast<uint64_t>(row) * sl;
                float sum = 0.0f;
#pragma unroll
                for (uint32_t t = 0; t < kDbMaxConv; ++t)
                    if (t == sl) sum = __fmul_rn(v, cw[t]);
#pragma unroll
                for (uint32_t t = 0; t < kDbMaxConv; ++t)
                    if (t < sl) sum = __fadd_rn(sum, __fmul_rn(hist[t], cw[t]));
#pragma unroll
                for (uint32_t t = 0; t + 1 < kDbMaxConv; ++t)
                    if (t + 1 < sl) st[t] = hist[t + 1];
                if (sl) st[sl - 1] = v;
                float s;
                if (sum >= 0.0f) {
                    s = sum / (1.0f + expf(-sum));
                } else {
                    const float e = expf(sum);
                    s = sum * e / (1.0f + e);
                }
                v = s;
            }
            a.proj[row] = v;
        }
    }
    // The tile space is free: ssm_out's 16 rows of this CTA, copied now.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (out_tile) {
        if (tid == 0) mbar_expect_tx(&bars[2], 16u * static_cast<uint32_t>(rb_out));
        __syncthreads();
        if (warp == 0 && lane < 16)
            bulk_copy_g2s(tiles + lane * Ly.pitch_out, a.w_out + static_cast<uint64_t>(cta * 16u + lane) * rb_out,
                          static_cast<uint32_t>(rb_out), &bars[2]);
    }
    bool ok = abort_sh == 0u && db_grid_barrier(a.counters, G, a.timeout, &abort_sh);
    // The output gate's silu(z) = z sigmoid(z), in place in the projection,
    // a slice per CTA (phase 3 reads it after the next barrier).
    if (ok) {
        const uint32_t chunk = (vw + G - 1u) / G, i = cta * chunk + static_cast<uint32_t>(tid);
        if (static_cast<uint32_t>(tid) < chunk && i < vw) {
            float* zp = a.proj + a.conv_ch + i;
            const float z = __ldcg(zp);
            *zp = __fmul_rn(z, db_sigmoid(z));
        }
    }

    // ---- phase 2: the delta rule on rows [r0, r0 + 32) of value head h2 ----
    if (ok && head) {
        const uint32_t h = h2, kq = h % a.kh;
        // Every projected input of the rows in one round of loads.
        const float* q = a.proj + static_cast<uint64_t>(kq) * dk;
        const float* k = a.proj + static_cast<uint64_t>(a.kh) * dk + static_cast<uint64_t>(kq) * dk;
        const float* v = a.proj + 2ull * a.kh * dk + static_cast<uint64_t>(h) * dv + r0;
        const bool in_head = static_cast<uint32_t>(tid) < dk;
        const float qv = in_head ? __ldcg(q + tid) : 0.0f;
        const float kv = in_head ? __ldcg(k + tid) : 0.0f;
        const float vv = static_cast<uint32_t>(tid) < rows2 ? __ldcg(v + tid) : 0.0f;
        const float al = __ldcg(a.proj + a.conv_ch + vw + h), be = __ldcg(a.proj + a.conv_ch + vw + a.hv + h);
        const float log_decay = a.ssm_a[h] * db_softplus(al + a.dt_bias[h]);
        const float b = db_sigmoid(be);
        const bool bad = !isfinite(log_decay) || log_decay > 0.0f || !isfinite(b) || b < 0.0f || b > 1.0f;
        if (static_cast<uint32_t>(tid) < rows2) ob[tid] = vv;
        const float sq = db_block_sum(qv * qv, red);
        const float sk = db_block_sum(kv * kv, red);
        if (in_head) {
            nq[tid] = __fmul_rn(__fmul_rn(qv, 1.0f / sqrtf(sq + 1.0e-6f)), 1.0f / sqrtf(static_cast<float>(dk)));
            nk[tid] = __fmul_rn(kv, 1.0f / sqrtf(sk + 1.0e-6f));
        }
        __syncthreads();
        if (!db_wait_copy(&bars[1], a.timeout)) ok = false;
        float* o_out = a.att + static_cast<uint64_t>(h) * dv + r0;
        if (bad) {
            if (r0 == 0 && tid == 0) atomicOr(a.gates_bad, 1u);
            if (tid == 0) a.ms_part[cta] = -1.0f;
            for (uint32_t i = tid; i < rows2; i += kDbThreads) o_out[i] = 0.0f;
        } else {
            const float decay = expf(log_decay);
            float kk[4], qq[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                kk[i] = nk[lane + 32 * i];
                qq[i] = nq[lane + 32 * i];
            }
            float* Sg = a.state + (static_cast<uint64_t>(h) * dv + r0) * dk;
            for (uint32_t r = warp; r < rows2; r += kDbWarps) {
                float c[4], mem = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    c[i] = __fmul_rn(S[r * dk + lane + 32 * i], decay);
                    mem = fmaf(c[i], kk[i], mem);
                }
                mem = warp_sum(mem);
                const float delta = __fmul_rn(__fsub_rn(ob[r], mem), b);
                float acc = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    c[i] = __fadd_rn(c[i], __fmul_rn(kk[i], delta));
                    acc = fmaf(c[i], qq[i], acc);
                    __stcs(Sg + static_cast<uint64_t>(r) * dk + lane + 32 * i, c[i]);
                }
                acc = warp_sum(acc);
                if (lane == 0) {
                    o_out[r] = acc;                  // the head's raw output o; phase 3 norms it
                    red[r] = acc;
                }
            }
            // These 32 rows' share of the head's sum of squares: the lane
            // butterfly of delta_step_regs_kernel's block_sum over rows r0..r0+31.
            __syncthreads();
            if (warp == 0) {
                const float x = red[lane];
                const float sq = warp_sum(x * x);
                if (lane == 0) a.ms_part[cta] = sq;
            }
        }
    } else if (head) {
        if (!db_wait_copy(&bars[1], a.timeout)) ok = false;     // the state copy lands before the CTA leaves
    }
    if (ok) ok = db_grid_barrier(a.counters, 2u * G, a.timeout, &abort_sh);

    // ---- phase 3: ssm_out rows of this CTA into the residual ----
    if (out_tile) {
        const bool landed = db_wait_copy(&bars[2], a.timeout);
        if (ok && landed) {
            const float resid = tid < 16 ? __ldcg(a.hidden + cta * 16u + tid) : 0.0f;
            // The heads' raw outputs into the record space, silu(z) beside
            // them and the quarter-head sums of squares, in one round of loads.
            float* hscale = nq;
            const auto stage_at = [&](uint32_t i) {
                return reinterpret_cast<float*>(recs + (i >> 8) * kFragWords) + (i & 255u);
            };
            for (uint32_t i = tid * 4u; i < vw; i += kDbThreads * 4u) {
                *reinterpret_cast<float4*>(stage_at(i)) = __ldcg(reinterpret_cast<const float4*>(a.att + i));
                *reinterpret_cast<float4*>(zs + i) = __ldcg(reinterpret_cast<const float4*>(a.proj + a.conv_ch + i));
            }
            float* nw = ob;
            if (static_cast<uint32_t>(tid) < dv) nw[tid] = a.ssm_norm[tid];
            if (static_cast<uint32_t>(tid) < a.hv) {
                // rms_norm_gated's scale (the four warp sums in order); -1 marks
                // a head with invalid gates, whose output is zero.
                float ms = 0.0f;
                bool bad = false;
#pragma unroll
                for (uint32_t c = 0; c < kDbSplit; ++c) {
                    const float p = __ldcg(a.ms_part + tid * kDbSplit + c);
                    bad = bad || p < 0.0f;
                    ms += p;
                }
                hscale[tid] = bad ? -1.0f : 1.0f / sqrtf(ms / static_cast<float>(dv) + a.eps);
            }
            __syncthreads();
            for (uint32_t i = tid; i < vw; i += kDbThreads) {
                const float sc = hscale[i / dv];
                float* x = stage_at(i);
                *x = sc < 0.0f ? 0.0f : __fmul_rn(__fmul_rn(__fmul_rn(*x, sc), nw[i % dv]), zs[i]);
            }
            __syncthreads();
            for (uint32_t q = warp; q < nsb_out; q += kDbWarps) {
                float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
                q4k_frag_superblock(stage, recs + q * kFragWords, lane);
                __syncwarp();
            }
            __syncthreads();
            for (uint32_t q = warp; q < nsb_out; q += kDbWarps) {
                const uint8_t* t = tiles + q * 144u;
                float acc0 = 0.0f, acc1 = 0.0f;
                q4k_mma_superblock(t + g * Ly.pitch_out, t + (g + 8) * Ly.pitch_out, recs + q * kFragWords, acc0, acc1);
                acc0 = quad_sum(acc0);
                acc1 = quad_sum(acc1);
                if ((lane & 3) == 0) {
                    part[q * 16u + g] = acc0;
                    part[q * 16u + g + 8] = acc1;
                }
            }
            __syncthreads();
            if (tid < 16) {
                float y = part[tid];
                for (uint32_t q = 1; q < nsb_out; ++q) y += part[q * 16u + tid];
                a.hidden[cta * 16u + tid] = resid + y;
            }
        }
    }
    return ok;
}

// The kernel arguments from the host-side shape and tensors.
inline DeltaBlockArgs make_delta_args(const DeltaBlockShape& s, const DeltaBlockTensors& t) {
    DeltaBlockArgs a{};
    a.w_in = static_cast<const uint8_t*>(t.w_in);
    a.w_out = static_cast<const uint8_t*>(t.w_out);
    a.attn_norm = t.attn_norm;
    a.conv_w = t.conv_w;
    a.conv_state = t.conv_state;
    a.ssm_a = t.ssm_a;
    a.dt_bias = t.dt_bias;
    a.ssm_norm = t.ssm_norm;
    a.state = t.state;
    a.hidden = t.hidden;
    a.proj = t.proj;
    a.att = t.att;
    a.ms_part = t.ms_part;
    a.counters = t.counters;
    a.timeout = t.timeout;
    a.gates_bad = t.gates_bad;
    a.H = s.hidden;
    a.rows_in = s.rows_in;
    a.conv_ch = 2u * s.key_heads * kDbHeadDim + s.value_heads * kDbHeadDim;
    a.kh = s.key_heads;
    a.hv = s.value_heads;
    a.K = s.conv_kernel;
    a.norm_eps = s.norm_eps;
    a.eps = s.eps;
    return a;
}

}  // namespace
}  // namespace pokit
