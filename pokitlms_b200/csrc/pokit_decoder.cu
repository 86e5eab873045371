// pokit_decoder.cu -- the whole Qwen3-MoE decoder of one sequence on the GPU:
// the reference's Qwen3MoeRunner (src/qwen3_moe_runner.cpp) with every
// matrix, norm, attention and MoE step in HBM, so that greedy decoding runs
// with no host round trip per layer.
//
// One token step (Qwen3MoeRunner::Impl::forward_into, qwen3_moe_runner.cpp:580-704):
//   embed     the token's row of token_embd (any GGUF type, bit-exact decode)
//   per layer rms_norm(attn_norm) -> one Q/K/V matvec over the concatenated
//             [q | k | v] rows -> per-head RMSNorm of q and k, rotate-half
//             RoPE from a position table, K/V appended to an FP16 ring (RNE,
//             kv_cache.cpp:20-44) -> GQA attention over the ring
//             (kv_cache.cpp:185-294) -> output projection added into the
//             residual -> the MoE block (pokit_cuda_moe_decode_layers: rms_norm,
//             router, top-k, experts, combine, residual)
//   logits    rms_norm(output_norm) -> LM head -> greedy argmax (first maximum,
//             :320-333) written as the next token of the sequence
// The Qwen3.5-MoE hybrid (Qwen35Runner::Impl::forward_into,
// src/qwen35_runner.cpp:538-777) runs in the same frame: its full-attention
// layers project a gated query (per head: query, then gate), rotate the first
// rotary_dim dimensions with the text-position MRoPE table and multiply the
// attention output by sigmoid(gate); its Gated DeltaNet layers project
// [qkv | gate | alpha | beta] in one matvec, run the conv1d + delta-rule step
// (pokit_cuda_delta_net_step) on per-layer states and add ssm_out's product;
// the MoE blocks add the sigmoid-gated shared expert.
// The token and position live in device memory, so a step is position-free
// and runs as one CUDA graph replay (captured on first use).
#include "../../include/pokit_cuda.h"
#include "pokit_attention.cuh"
#include "pokit_kernels.h"
#include "pokit_mma.cuh"
#include "pokit_quant.cuh"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace pokit {
namespace {

constexpr uint32_t kStatusDecoderNonFinite = 1u;   // LM head produced NaN/Inf (the reference throws)
constexpr uint32_t kMaxWindow = 8192;
constexpr uint32_t kArgmaxCtas = 148;

// The token's embedding row, decoded exactly as dequantize_quantized_row.
template <uint32_t T>
__global__ void embed_kernel(const uint8_t* __restrict__ table, uint32_t cols, const uint32_t* __restrict__ seq,
                             const uint32_t* __restrict__ pos, float* __restrict__ out) {
    const uint32_t token = seq[*pos];
    const uint8_t* row = table + static_cast<uint64_t>(token) * row_bytes(T, cols);
    for (uint32_t g = threadIdx.x; g < cols / 32u; g += blockDim.x) group_decode<T>(row, static_cast<int>(g), out + g * 32u);
}

// out = x * (1 / sqrt(mean(x^2) + eps)) * w   (src/rms_norm.cpp:9-27)
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps,
                                float* __restrict__ out, uint32_t n) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    const float total = block_reduce_all(ss, red, [](float a, float b) { return a + b; });
    const float scale = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
}

__global__ void __launch_bounds__(kAttendThreads, 1)
attend_kernel(const float* __restrict__ qkv, const float* __restrict__ q_norm, const float* __restrict__ k_norm,
              const float* __restrict__ rope_cos, const float* __restrict__ rope_sin, __half* __restrict__ kc,
              __half* __restrict__ vc, const uint32_t* __restrict__ pos_p, const AttendShape sh,
              float* __restrict__ out) {
    extern __shared__ __align__(16) float dyn[];
    float* scratch = dyn;
    float* sc = dyn + attend_scratch_floats(sh.d, kAttendThreads / 32);
    // The position counter changes only at the end of a token step, so it and
    // the cached keys and values of earlier positions are read before waiting
    // for the Q/K/V projection: the first CTA of each query group pulls its
    // head's cached rows towards L2 while the projection finishes.
    const uint32_t t = threadIdx.x, h = blockIdx.x, pos = *pos_p, d = sh.d, window = sh.window;
    const uint32_t group = sh.qh / sh.kvh, kh = h / group;
    const uint32_t n = pos + 1 < window ? pos + 1 : window, first = pos + 1 - n;
    const uint64_t row_stride = static_cast<uint64_t>(sh.kvh) * d;
    if (h % group == 0) {
        const uint32_t lines = (d * 2u + 127u) / 128u;
        for (uint32_t i = t; i + lines < n * lines; i += kAttendThreads) {
            const uint64_t at = ((first + i / lines) % window) * row_stride + kh * d + (i % lines) * 64u;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(kc + at));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(vc + at));
        }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t kbase = sh.qh * sh.q_stride, vbase = kbase + sh.kvh * d;
    attend_head(qkv + h * sh.q_stride, qkv + kbase + kh * d, qkv + vbase + kh * d,
                sh.gated ? qkv + h * sh.q_stride + d : nullptr, q_norm, k_norm,
                rope_cos + static_cast<uint64_t>(pos) * sh.rh, rope_sin + static_cast<uint64_t>(pos) * sh.rh, kc, vc,
                pos, sh, h, sc, scratch, out + h * d);
}

// ---------------------------------------------------------------------------
// The attention block of one layer in one cooperative launch (Q4_K
// projections): rms_norm(attn_norm) -> the [q (| gate) | k | v] matvec ->
// attention per query head -> the output projection added into the residual.
// Steps and who runs them (G CTAs, one per SM):
//   entry   every CTA bulk-copies its Q/K/V row blocks (16 rows each: blocks
//           c, c + G, ...) and, for c < H/16, its 16 rows of attn_output into
//           shared memory (rows padded by 16 bytes so the fragment reads
//           spread over the banks); query-head CTAs load this position's RoPE
//           rows and pull their KV head's cached rows towards L2
//   qkv     every CTA stages h once, forms x' = attn_norm * h / rms(h)
//           records, multiplies its blocks on the integer tensor path
//           (q4k_mma_superblock), adds each row's superblock partials in
//           order and publishes the rows as 8-byte words (tag << 32 | bits)
//   attend  CTA h < q_heads reads its query (and gate) and its KV head's key
//           and value words as they arrive and runs attend_head (norms,
//           RoPE, FP16 ring append, softmax, values); publishes its d outputs
//   o       CTA c < H/16 reads all output words of its records at once as
//           they arrive, multiplies its attn_output rows and writes hidden
//           rows [16c, 16c + 16) = their staged residual + the product
// Order: every CTA publishes Q/K/V words only after reading all of hidden,
// and attention needs words from the CTAs owning every row, so no CTA writes
// hidden before all have read it.  The tag is position * layers + layer + 1
// (unique within a sequence; the words are cleared with the decode state), so
// words of another layer or step never match.  Waits are bounded (~2 s); a
// timeout sets the status word and the CTA drains its copies and leaves.
__global__ void __launch_bounds__(kAttnBlockThreads, 1) attn_block_kernel(const __grid_constant__ AttnBlockArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[2];
    __shared__ float red[kAttnBlockWarps];
    __shared__ uint32_t abort_sh;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
        abort_sh = 0u;
    }
    __syncthreads();
    const AttnPhaseCtx x{smem, bars, 0u, &abort_sh, red};
    attention_phase(a, x, nullptr, 0u);
}

// Greedy sampling (qwen3_moe_runner.cpp:320-333): the first maximum of the
// logits becomes token position + 1 of the sequence; a non-finite logit sets
// the status word (the reference throws).  Each CTA reduces a slice to its
// (value, index) pair; the CTA that arrives last combines them, larger value
// first and the lower index on ties, and leaves the arrival counter at zero.
__device__ __forceinline__ void better(float& v, uint32_t& i, float ov, uint32_t oi) {
    if (oi != 0xffffffffu && (i == 0xffffffffu || ov > v || (ov == v && oi < i))) {
        v = ov;
        i = oi;
    }
}

__device__ void block_best(float& v, uint32_t& i, float* rv, uint32_t* ri) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
        better(v, i, ov, oi);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) { rv[warp] = v; ri[warp] = i; }
    __syncthreads();
    v = rv[0];
    i = ri[0];
    for (int w = 1; w < static_cast<int>((blockDim.x + 31) >> 5); ++w) better(v, i, rv[w], ri[w]);
}

__global__ void argmax_kernel(const float* __restrict__ logits, uint32_t n, float* __restrict__ part_v,
                              uint32_t* __restrict__ part_i, uint32_t* __restrict__ arrivals,
                              uint32_t* __restrict__ seq, const uint32_t* __restrict__ pos_p, uint32_t seq_cap,
                              uint32_t* __restrict__ status) {
    __shared__ float rv[32];
    __shared__ uint32_t ri[32];
    __shared__ uint32_t last;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t per = (n + gridDim.x - 1) / gridDim.x, lo = blockIdx.x * per, hi = min(n, lo + per);
    float best = -INFINITY;
    uint32_t bi = 0xffffffffu;
    int bad = 0;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = logits[i];
        if (!isfinite(v)) bad = 1;
        else if (bi == 0xffffffffu || v > best) { best = v; bi = i; }
    }
    bad = __syncthreads_or(bad);
    block_best(best, bi, rv, ri);
    if (threadIdx.x == 0) {
        part_v[blockIdx.x] = best;
        part_i[blockIdx.x] = bad ? 0xfffffffeu : bi;
        __threadfence();
        last = atomicAdd(arrivals, 1u) == gridDim.x - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    best = -INFINITY;
    bi = 0xffffffffu;
    bad = 0;
    for (uint32_t b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
        const uint32_t oi = __ldcg(part_i + b);
        if (oi == 0xfffffffeu) bad = 1;
        else better(best, bi, __ldcg(part_v + b), oi);
    }
    bad = __syncthreads_or(bad);
    block_best(best, bi, rv, ri);
    if (threadIdx.x == 0) {
        *arrivals = 0u;
        if (bad) atomicOr(status, kStatusDecoderNonFinite);
        const uint32_t p = *pos_p;
        if (p + 1 < seq_cap) seq[p + 1] = bad || bi == 0xffffffffu ? 0u : bi;
    }
}

__global__ void advance_kernel(uint32_t* pos) { *pos += 1u; }

// A launch that may start while the previous kernel in the stream finishes
// (programmatic dependent launch); the kernel waits for it with
// griddepcontrol.wait before reading its results.
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kernel)(Params...), uint32_t grid, uint32_t block, size_t smem, cudaStream_t s,
                             Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

template <uint32_t T>
cudaError_t launch_embed(const void* table, uint32_t cols, const uint32_t* seq, const uint32_t* pos, float* out,
                         cudaStream_t s) {
    embed_kernel<T><<<1, 256, 0, s>>>(static_cast<const uint8_t*>(table), cols, seq, pos, out);
    return cudaGetLastError();
}

void set_error(char* destination, size_t capacity, const char* message) noexcept {
    if (!destination || capacity == 0) return;
    const size_t n = std::min(capacity - 1, std::strlen(message));
    std::memcpy(destination, message, n);
    destination[n] = '\0';
}

uint64_t align256(uint64_t v) { return (v + 255u) & ~uint64_t(255); }

bool decoder_type(uint32_t t) { return t == kF32 || t == kQ8_0 || t == kQ4_K || t == kQ5_K || t == kQ6_K; }

}  // namespace

// ---------------------------------------------------------------------------
class Decoder {
public:
    explicit Decoder(const pokit_cuda_decoder_config& c) : cfg_(c) {
        const size_t d = c.head_dim;
        hybrid_ = c.arch == POKIT_CUDA_ARCH_QWEN35MOE;
        if (c.arch > POKIT_CUDA_ARCH_QWEN35MOE || c.layers == 0 || c.hidden == 0 || c.hidden % 256 || c.vocab == 0 ||
            c.vocab > 0xffffffffu || c.q_heads == 0 || c.kv_heads == 0 || c.q_heads % c.kv_heads || d == 0 ||
            d % 32 || d > kAttendMaxDim || c.context == 0 || c.context > (1u << 24) || c.eos_token >= c.vocab ||
            !(c.rope_theta > 0.0f) || !(c.rms_epsilon > 0.0f) || (c.q_heads * d) % 256)
            throw std::invalid_argument("invalid decoder configuration");
        if (!decoder_type(c.attn_type) || c.attn_type == kF32 || !decoder_type(c.embed_type) ||
            !decoder_type(c.output_type))
            throw std::invalid_argument("unsupported decoder tensor type");
        rh_ = d / 2;
        if (hybrid_) {
            // Qwen35Index::load_config and Qwen35Runner::Impl checks
            // (src/qwen35_index.cpp:205-220, src/qwen35_runner.cpp:425-434).
            uint64_t sections = 0;
            for (uint32_t v : c.rope_sections) sections += v;
            if (c.rotary_dim == 0 || c.rotary_dim % 2 || c.rotary_dim > d || sections == 0 ||
                sections > c.rotary_dim / 2 || c.full_attention_interval == 0 ||
                c.full_attention_interval > c.layers || c.ssm_conv_kernel == 0 || c.ssm_conv_kernel > 64 ||
                c.ssm_state_size == 0 || c.ssm_state_size % 32 || c.ssm_state_size > 256 || c.ssm_group_count == 0 ||
                c.ssm_time_step_rank == 0 || c.ssm_time_step_rank % c.ssm_group_count ||
                c.ssm_inner_size % c.ssm_time_step_rank || c.ssm_inner_size % 256 ||
                c.ssm_inner_size / c.ssm_time_step_rank > 256 || !(c.expert_weights_scale >= 0.0f) ||
                (c.shared_inter && !decoder_type(c.shared_type)))
                throw std::invalid_argument("invalid Qwen3.5 hybrid configuration");
            rh_ = c.rotary_dim / 2;
            kw_ = c.ssm_group_count * c.ssm_state_size;
            vw_ = c.ssm_inner_size;
            hv_ = c.ssm_time_step_rank;
            conv_ch_ = 2 * kw_ + vw_;
        }
        window_ = c.kv_window ? c.kv_window : std::min<size_t>(c.context, 512);
        if (window_ > c.context || window_ > kMaxWindow) throw std::invalid_argument("invalid KV window");
        qd_ = c.q_heads * d;
        kd_ = c.kv_heads * d;
        qrows_ = hybrid_ ? 2 * qd_ : qd_;
        pokit_cuda_moe_config mc{};
        mc.device = c.device;
        mc.layers = c.layers;
        mc.hidden = c.hidden;
        mc.inter = c.expert_inter;
        mc.experts = c.experts;
        mc.top_k = c.top_k;
        mc.flavour = hybrid_ ? POKIT_CUDA_MOE_QWEN35 : POKIT_CUDA_MOE_QWEN3;
        mc.normalize_top_k = c.normalize_top_k;
        mc.expert_weights_scale = hybrid_ ? c.expert_weights_scale : 1.0f;
        mc.rms_epsilon = c.rms_epsilon;
        mc.gate_type = mc.up_type = mc.down_type = c.expert_type;
        mc.layer_down_types = hybrid_ ? c.layer_down_types : nullptr;
        mc.shared_inter = hybrid_ ? c.shared_inter : 0;
        mc.shared_gate_type = mc.shared_up_type = mc.shared_down_type = hybrid_ && c.shared_inter ? c.shared_type : kQ8_0;
        char err[512];
        const pokit_cuda_status st = pokit_cuda_moe_create(&mc, &moe_, err, sizeof err);
        if (st == POKIT_CUDA_STATUS_INVALID_ARGUMENT) throw std::invalid_argument(err);
        if (st != POKIT_CUDA_STATUS_OK) throw std::runtime_error(err);
        int prev = 0;
        check(cudaGetDevice(&prev), "cudaGetDevice");
        check(cudaSetDevice(c.device), "cudaSetDevice");
        try {
            allocate();
        } catch (...) {
            cudaSetDevice(prev);
            release();
            throw;
        }
        cudaSetDevice(prev);
    }

    ~Decoder() { release(); }
    Decoder(const Decoder&) = delete;
    Decoder& operator=(const Decoder&) = delete;

    std::mutex& mutex() { return mutex_; }
    pokit_cuda_moe* moe() { return moe_; }

    // Layer l is full attention (Qwen3.5Config::is_full_attention_layer,
    // src/qwen35_index.cpp:230-233); every Qwen3-MoE layer is.
    bool attention_layer(size_t l) const { return !hybrid_ || (l + 1) % cfg_.full_attention_interval == 0; }

    uint64_t tensor_bytes(size_t layer, uint32_t t) const {
        const uint64_t H = cfg_.hidden, d = cfg_.head_dim;
        switch (t) {
            case POKIT_CUDA_DEC_TOKEN_EMBD: return cfg_.vocab * row_bytes(cfg_.embed_type, H);
            case POKIT_CUDA_DEC_OUTPUT_NORM: return H * 4;
            case POKIT_CUDA_DEC_OUTPUT: return cfg_.vocab * row_bytes(cfg_.output_type, H);
            default: break;
        }
        if (layer >= cfg_.layers) return 0;
        if (t == POKIT_CUDA_DEC_ATTN_NORM) return H * 4;
        const uint64_t rb = row_bytes(cfg_.attn_type, H);
        if (attention_layer(layer)) {
            switch (t) {
                case POKIT_CUDA_DEC_ATTN_Q: return qrows_ * rb;
                case POKIT_CUDA_DEC_ATTN_Q_NORM: return d * 4;
                case POKIT_CUDA_DEC_ATTN_K: return kd_ * rb;
                case POKIT_CUDA_DEC_ATTN_K_NORM: return d * 4;
                case POKIT_CUDA_DEC_ATTN_V: return kd_ * rb;
                case POKIT_CUDA_DEC_ATTN_OUTPUT: return H * row_bytes(cfg_.attn_type, qd_);
                default: return 0;
            }
        }
        switch (t) {
            case POKIT_CUDA_DEC_SSM_QKV: return conv_ch_ * rb;
            case POKIT_CUDA_DEC_SSM_GATE: return vw_ * rb;
            case POKIT_CUDA_DEC_SSM_ALPHA: case POKIT_CUDA_DEC_SSM_BETA: return hv_ * rb;
            case POKIT_CUDA_DEC_SSM_CONV1D: return conv_ch_ * cfg_.ssm_conv_kernel * 4;
            case POKIT_CUDA_DEC_SSM_A: case POKIT_CUDA_DEC_SSM_DT_BIAS: return hv_ * 4;
            case POKIT_CUDA_DEC_SSM_NORM: return (vw_ / hv_) * 4;
            case POKIT_CUDA_DEC_SSM_OUT: return H * row_bytes(cfg_.attn_type, vw_);
            default: return 0;
        }
    }

    void upload(size_t layer, uint32_t t, const void* host, size_t bytes) {
        ensure_ok();
        uint8_t* dst = tensor_ptr(layer, t);
        if (!dst) throw std::invalid_argument("tensor does not exist in this configuration");
        if (!host || bytes != tensor_bytes(layer, t)) throw std::invalid_argument("tensor byte size does not match");
        Scope scope(cfg_.device);
        guard(cudaMemcpy(dst, host, bytes, cudaMemcpyHostToDevice), "upload");
    }

    void synthesize(size_t layer, uint32_t t, uint64_t seed, uint64_t stream_id) {
        ensure_ok();
        uint8_t* dst = tensor_ptr(layer, t);
        const uint32_t type = tensor_type(t);
        if (!dst || type == kF32) throw std::invalid_argument("only quantised decoder tensors can be synthesised");
        Scope scope(cfg_.device);
        guard(launch_synth_blocks(type, seed, stream_id, tensor_bytes(layer, t) / block_bytes(type), dst, stream_),
              "synthesize");
        guard(cudaStreamSynchronize(stream_), "synthesize");
    }

    void reset() {
        ensure_ok();
        Scope scope(cfg_.device);
        clear_state();
        guard(cudaStreamSynchronize(stream_), "reset");
        next_position_ = 0;
    }

    // Qwen3MoeRunner::forward_token: the token at `position` (the next one),
    // logits out (may be null).
    void forward_token(uint32_t token, uint64_t position, float* logits) {
        ensure_ok();
        if (token >= cfg_.vocab) throw std::out_of_range("token id exceeds model vocabulary");
        if (position != next_position_ || position >= cfg_.context)
            throw std::invalid_argument("token position is not the next position in this decode state");
        Scope scope(cfg_.device);
        *pinned_ids_ = token;
        guard(cudaMemcpyAsync(seq_ + position, pinned_ids_, 4, cudaMemcpyHostToDevice, stream_), "token");
        step(true);
        ++next_position_;
        if (logits) guard(cudaMemcpyAsync(logits, logits_, cfg_.vocab * 4, cudaMemcpyDeviceToHost, stream_), "logits");
        sync_and_check();
    }

    // Qwen3MoeRunner::generate_tokens with greedy sampling (temperature 0):
    // resets the state, prefills the prompt (logits for its last token only),
    // then samples up to max_new tokens, stopping after the end token.
    void generate(const uint32_t* prompt, size_t n, size_t max_new, uint32_t* out, size_t* n_out,
                  pokit_cuda_generation_stats* stats) {
        ensure_ok();
        if (!prompt || n == 0) throw std::invalid_argument("generation prompt must contain at least one token");
        if (n > cfg_.context || max_new > cfg_.context - n)
            throw std::length_error("prompt and generation length exceed model context");
        if (max_new && (!out || !n_out)) throw std::invalid_argument("output buffers are required");
        for (size_t i = 0; i < n; ++i)
            if (prompt[i] >= cfg_.vocab) throw std::out_of_range("token id exceeds model vocabulary");
        Scope scope(cfg_.device);
        if (stats) *stats = {};
        if (n_out) *n_out = 0;
        const auto t0 = std::chrono::steady_clock::now();
        clear_state();
        next_position_ = 0;
        for (size_t i = 0; i < n;) {
            const size_t m = std::min(n - i, kPinnedIds);
            std::memcpy(pinned_ids_, prompt + i, m * 4);
            guard(cudaMemcpyAsync(seq_ + i, pinned_ids_, m * 4, cudaMemcpyHostToDevice, stream_), "prompt");
            guard(cudaStreamSynchronize(stream_), "prompt");
            i += m;
        }
        for (size_t i = 0; i < n; ++i) step(i + 1 == n);
        next_position_ = n;
        sync_and_check();
        const auto t1 = std::chrono::steady_clock::now();
        // Token i (i >= 1) is sampled by the forward of token i - 1; token 0 by
        // the last prompt step.  The forwards of a chunk run back to back on the
        // device and the host reads the chunk's tokens once, to find the end
        // token.  Forwards past the end token are harmless while the KV ring has
        // not wrapped (they write slots no later position reads before it is
        // rewritten) and no layer is recurrent; otherwise one token per round
        // trip.
        size_t produced = 0, forwarded = 0;
        bool ended = false;
        while (produced < max_new && !ended) {
            // A recurrent (DeltaNet) state would absorb forwards past the end
            // token: the hybrid forwards exactly the reference's tokens.
            const bool wrapped = hybrid_ || n + produced + 16 >= window_;
            const size_t chunk = wrapped ? 1 : std::min<size_t>(max_new - produced, 16);
            const size_t last = produced + chunk - 1;
            for (; forwarded < last; ++forwarded) step(true);
            guard(cudaMemcpyAsync(pinned_ids_, seq_ + n + produced, chunk * 4, cudaMemcpyDeviceToHost, stream_),
                  "tokens");
            sync_and_check();
            for (size_t i = 0; i < chunk && !ended; ++i) {
                out[produced] = pinned_ids_[i];
                ++produced;
                if (pinned_ids_[i] == cfg_.eos_token) ended = true;
            }
        }
        // The reference forwards every generated token but the last one.
        next_position_ = n + (produced ? produced - 1 : 0);
        // Forwards past the end token left the device position ahead: align it
        // (and drop their attention words, whose tags the next forwards reuse).
        *pinned_ids_ = static_cast<uint32_t>(next_position_);
        guard(cudaMemcpyAsync(pos_, pinned_ids_, 4, cudaMemcpyHostToDevice, stream_), "position");
        if (attn_ll_) guard(cudaMemsetAsync(attn_ll_, 0, attn_words_ * 8, stream_), "position");
        guard(cudaStreamSynchronize(stream_), "position");
        const auto t2 = std::chrono::steady_clock::now();
        *n_out = produced;
        if (stats) {
            stats->prefill_time_ns = static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count());
            stats->decode_time_ns = static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(t2 - t1).count());
            stats->generated_tokens = produced;
        }
    }

    // Enqueues `steps` token steps with logits on `s` (device-resident
    // sequence: each step's token is the previous step's argmax).  For
    // benchmarks: the caller synchronises.
    void run_steps(size_t steps, cudaStream_t s) {
        ensure_ok();
        if (next_position_ + steps >= cfg_.context) throw std::length_error("steps exceed model context");
        Scope scope(cfg_.device);
        for (size_t i = 0; i < steps; ++i) step(true, s ? s : stream_);
        next_position_ += steps;
    }

    size_t position() const { return next_position_; }
    uint64_t launches_per_step() const { return launches_per_step_; }
    int step_graphs() const { return (graphs_[0] ? 1 : 0) + (graphs_[1] ? 1 : 0); }
    const std::string& capture_error() const { return capture_error_; }

private:
    static constexpr size_t kPinnedIds = 4096;

    struct Scope {
        explicit Scope(int device) {
            cudaGetDevice(&prev);
            if (prev != device) cudaSetDevice(device);
            dev = device;
        }
        ~Scope() {
            if (prev != dev) cudaSetDevice(prev);
        }
        int prev = 0, dev = 0;
    };

    static void check(cudaError_t e, const char* what) {
        if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
    void guard(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return;
        if (e == cudaErrorInvalidValue) throw std::invalid_argument(std::string(what) + ": unsupported shape or argument");
        failed_ = true;
        failure_ = std::string(what) + ": " + cudaGetErrorString(e);
        throw std::runtime_error(failure_);
    }
    void ensure_ok() const {
        if (failed_) throw std::runtime_error("CUDA decoder failed earlier: " + failure_);
    }

    uint32_t tensor_type(uint32_t t) const {
        switch (t) {
            case POKIT_CUDA_DEC_TOKEN_EMBD: return cfg_.embed_type;
            case POKIT_CUDA_DEC_OUTPUT: return cfg_.output_type;
            case POKIT_CUDA_DEC_ATTN_Q: case POKIT_CUDA_DEC_ATTN_K: case POKIT_CUDA_DEC_ATTN_V:
            case POKIT_CUDA_DEC_ATTN_OUTPUT: case POKIT_CUDA_DEC_SSM_QKV: case POKIT_CUDA_DEC_SSM_GATE:
            case POKIT_CUDA_DEC_SSM_ALPHA: case POKIT_CUDA_DEC_SSM_BETA: case POKIT_CUDA_DEC_SSM_OUT:
                return cfg_.attn_type;
            default: return kF32;
        }
    }

    uint8_t* tensor_ptr(size_t layer, uint32_t t) const {
        if (t >= kTensors || tensor_bytes(layer, t) == 0) return nullptr;
        if (t <= POKIT_CUDA_DEC_OUTPUT) return pool_ + global_off_[t];
        return pool_ + off_[layer * kTensors + t];
    }

    void allocate() {
        // Pool: embedding, output norm, LM head, then per layer attn_norm and
        // the projections of one normed input as contiguous rows (one
        // matvec): attention layers [q | k | v], o, q_norm, k_norm; DeltaNet
        // layers [qkv | gate | alpha | beta], ssm_out, conv1d, ssm_a, dt_bias,
        // ssm_norm.
        uint64_t off = 0;
        for (uint32_t t = 0; t <= POKIT_CUDA_DEC_OUTPUT; ++t) {
            global_off_[t] = off;
            off += align256(tensor_bytes(0, t));
        }
        off_.assign(cfg_.layers * kTensors, 0);
        for (size_t l = 0; l < cfg_.layers; ++l) {
            const auto place = [&](uint32_t t, bool pad) {
                off_[l * kTensors + t] = off;
                off += pad ? align256(tensor_bytes(l, t)) : tensor_bytes(l, t);
            };
            place(POKIT_CUDA_DEC_ATTN_NORM, true);
            if (attention_layer(l)) {
                place(POKIT_CUDA_DEC_ATTN_Q, false);
                place(POKIT_CUDA_DEC_ATTN_K, false);
                place(POKIT_CUDA_DEC_ATTN_V, true);
                place(POKIT_CUDA_DEC_ATTN_OUTPUT, true);
                place(POKIT_CUDA_DEC_ATTN_Q_NORM, true);
                place(POKIT_CUDA_DEC_ATTN_K_NORM, true);
            } else {
                place(POKIT_CUDA_DEC_SSM_QKV, false);
                place(POKIT_CUDA_DEC_SSM_GATE, false);
                place(POKIT_CUDA_DEC_SSM_ALPHA, false);
                place(POKIT_CUDA_DEC_SSM_BETA, true);
                place(POKIT_CUDA_DEC_SSM_OUT, true);
                place(POKIT_CUDA_DEC_SSM_CONV1D, true);
                place(POKIT_CUDA_DEC_SSM_A, true);
                place(POKIT_CUDA_DEC_SSM_DT_BIAS, true);
                place(POKIT_CUDA_DEC_SSM_NORM, true);
            }
        }
        check(cudaMalloc(&pool_, off), "cudaMalloc(decoder pool)");
        check(cudaMemset(pool_, 0, off), "cudaMemset(decoder pool)");
        const uint64_t kv = static_cast<uint64_t>(cfg_.layers) * window_ * kd_ * sizeof(__half);
        check(cudaMalloc(&kcache_, kv), "cudaMalloc(K cache)");
        check(cudaMalloc(&vcache_, kv), "cudaMalloc(V cache)");
        // Convolution and recurrent states of the DeltaNet layers.
        if (hybrid_) {
            const uint64_t conv = align256(conv_ch_ * (cfg_.ssm_conv_kernel - 1) * 4);
            const uint64_t rec = align256(hv_ * cfg_.ssm_state_size * (vw_ / hv_) * 4);
            ssm_off_.assign(cfg_.layers, 0);
            uint64_t so = 0;
            for (size_t l = 0; l < cfg_.layers; ++l)
                if (!attention_layer(l)) {
                    ssm_off_[l] = so;
                    so += conv + rec;
                }
            ssm_conv_bytes_ = conv;
            ssm_bytes_ = so;
            if (so) {
                check(cudaMalloc(&ssm_, so), "cudaMalloc(DeltaNet states)");
                check(cudaMemset(ssm_, 0, so), "cudaMemset(DeltaNet states)");
            }
        }
        // RoPE tables [context][rotary half], the reference's float arithmetic:
        // angle = position * theta^(-pair / half) (qwen3_moe_runner.cpp:141-156);
        // Qwen3.5 text positions leave the pairs of the fourth MRoPE section at
        // position 0 (prepare_rope, qwen35_runner.cpp:69-92).
        const size_t half = rh_;
        uint64_t section_total = 0, three = 0;
        if (hybrid_) {
            for (uint32_t v : cfg_.rope_sections) section_total += v;
            three = uint64_t(cfg_.rope_sections[0]) + cfg_.rope_sections[1] + cfg_.rope_sections[2];
        }
        std::vector<float> cs(cfg_.context * half), sn(cfg_.context * half);
        for (size_t p = 0; p < cfg_.context; ++p)
            for (size_t i = 0; i < half; ++i) {
                const bool extra = hybrid_ && (i % section_total) >= three;
                const float at = extra ? 0.0f : static_cast<float>(p);
                const float angle = at * std::pow(cfg_.rope_theta, -static_cast<float>(i) / static_cast<float>(half));
                cs[p * half + i] = std::cos(angle);
                sn[p * half + i] = std::sin(angle);
            }
        check(cudaMalloc(&rope_, cs.size() * 8), "cudaMalloc(rope)");
        check(cudaMemcpy(rope_, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope");
        check(cudaMemcpy(rope_ + cs.size(), sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "rope");
        const uint64_t H = cfg_.hidden;
        const uint64_t proj = std::max<uint64_t>(qrows_ + 2 * kd_, hybrid_ ? conv_ch_ + vw_ + 2 * hv_ : 0);
        const uint64_t mix = std::max<uint64_t>(qd_, vw_);
        const uint64_t fl = align256(H * 4) * 2 + align256(proj * 4) + align256(mix * 4) + align256(cfg_.vocab * 4);
        check(cudaMalloc(&work_, fl), "cudaMalloc(decoder work)");
        uint8_t* w = static_cast<uint8_t*>(work_);
        hidden_ = reinterpret_cast<float*>(w); w += align256(H * 4);
        xn_ = reinterpret_cast<float*>(w); w += align256(H * 4);
        qkv_ = reinterpret_cast<float*>(w); w += align256(proj * 4);
        att_ = reinterpret_cast<float*>(w); w += align256(mix * 4);
        logits_ = reinterpret_cast<float*>(w);
        const size_t seq_words = cfg_.context + 1 + 32 + 32 + 32 + 2 * kArgmaxCtas;
        check(cudaMalloc(&seq_, seq_words * 4), "cudaMalloc(sequence)");
        check(cudaMemset(seq_, 0, seq_words * 4), "cudaMemset(sequence)");
        pos_ = seq_ + cfg_.context + 1 + 32;
        status_ = pos_ + 32;
        arrivals_ = status_ + 32;
        part_i_ = arrivals_ + 32;
        part_v_ = reinterpret_cast<float*>(part_i_ + kArgmaxCtas);
        check(cudaMallocHost(&pinned_ids_, kPinnedIds * 4), "cudaMallocHost");
        check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaStreamCreateWithFlags(&capture_stream_, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaEventCreateWithFlags(&join_, cudaEventDisableTiming), "cudaEventCreate");
        check(cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(attend_smem_bytes())), "attend smem");
        plan_attn_block();
        plan_delta_block();
    }

    // DeltaNet layers run as one cooperative launch each (pokit_deltablock.cu)
    // when the projections are Q4_K and the heads 128 wide
    // (POKIT_CUDA_FUSED_DELTANET=0 keeps the four-kernel path).
    void plan_delta_block() {
        const char* env = std::getenv("POKIT_CUDA_FUSED_DELTANET");
        if (!hybrid_ || (env && env[0] == '0') || cfg_.attn_type != kQ4_K || hv_ == 0) return;
        DeltaBlockShape d{};
        d.hidden = static_cast<uint32_t>(cfg_.hidden);
        d.rows_in = static_cast<uint32_t>(conv_ch_ + vw_ + 2 * hv_);
        d.key_heads = static_cast<uint32_t>(cfg_.ssm_group_count);
        d.value_heads = static_cast<uint32_t>(hv_);
        d.key_dim = static_cast<uint32_t>(cfg_.ssm_state_size);
        d.value_dim = static_cast<uint32_t>(vw_ / hv_);
        d.conv_kernel = static_cast<uint32_t>(cfg_.ssm_conv_kernel);
        d.norm_eps = cfg_.rms_epsilon;
        d.eps = cfg_.rms_epsilon;
        if (2 * cfg_.ssm_group_count * cfg_.ssm_state_size + vw_ != conv_ch_ || vw_ % hv_) return;
        uint32_t grid = 0, smem = 0;
        if (!delta_block_plan(d, &grid, &smem)) return;
        check(cudaMalloc(&delta_scratch_, sizeof(float) * 4 * hv_), "cudaMalloc(DeltaNet scratch)");
        delta_shape_ = d;
        delta_grid_ = grid;
        delta_smem_ = smem;
        // The DeltaNet layer and its MoE block as one launch when the MoE
        // blocks take the Qwen3.5 chain kernel (POKIT_CUDA_FUSED_DELTA_MOE=0
        // keeps two launches per layer).
        const char* both = std::getenv("POKIT_CUDA_FUSED_DELTA_MOE");
        delta_moe_ = !(both && both[0] == '0') && moe_delta_layer_fits(moe_, d);
    }

    size_t attend_smem_bytes() const {
        return (attend_scratch_floats(static_cast<uint32_t>(cfg_.head_dim), kAttendThreads / 32) + window_) * 4;
    }

    // The fused attention block serves Q4_K projections when every CTA owns
    // a Q/K/V row block, the output-projection units and query heads fit the
    // grid, and one CTA per SM fits (POKIT_CUDA_FUSED_ATTN=0 turns it off).
    void plan_attn_block() {
        const char* env = std::getenv("POKIT_CUDA_FUSED_ATTN");
        if (env && env[0] == '0') return;
        int sms = 0;
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg_.device), "SM count");
        const uint32_t rows = static_cast<uint32_t>(qrows_ + 2 * kd_), H = static_cast<uint32_t>(cfg_.hidden);
        const uint32_t grid = static_cast<uint32_t>(sms);
        if (cfg_.attn_type != kQ4_K || rows % 16 || qd_ % 256 || rows / 16 < grid || H / 16 > grid ||
            cfg_.q_heads > grid)
            return;
        if (qd_ / 256 > kAttnBlockWarps * kAttnMaxOutPerWarp || H / 256 > 2 * kAttnBlockWarps || cfg_.layers > 255)
            return;
        const AttnBlockLayout c = attn_block_layout(H, rows, static_cast<uint32_t>(qd_),
                                                    static_cast<uint32_t>(cfg_.head_dim), static_cast<uint32_t>(rh_),
                                                    static_cast<uint32_t>(window_), grid, kAttnBlockWarps);
        if (c.total > 200u * 1024u) return;
        if (cudaFuncSetAttribute(attn_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(c.total)) != cudaSuccess) {
            cudaGetLastError();
            return;
        }
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_block_kernel, kAttnBlockThreads, c.total) !=
                cudaSuccess || per_sm < 1) {
            cudaGetLastError();
            return;
        }
        attn_words_ = rows + qd_ + cfg_.hidden;
        check(cudaMalloc(&attn_ll_, attn_words_ * 8), "cudaMalloc(attention words)");
        check(cudaMemset(attn_ll_, 0, attn_words_ * 8), "cudaMemset(attention words)");
        attn_grid_ = grid;
        attn_smem_ = c.total;
        // A hybrid decoder's attention layer and its MoE block run as one
        // launch when the Qwen3.5 chain kernel fits the attention phase
        // (POKIT_CUDA_FUSED_ATTN_MOE=0 keeps two launches per layer).
        const char* both = std::getenv("POKIT_CUDA_FUSED_ATTN_MOE");
        attn_moe_ = !(both && both[0] == '0');
        plan_layer_chain();
    }

    // The whole layer loop as one chain launch (attention phase + MoE block
    // per layer) when every layer is a full-attention layer whose tensors sit
    // at one stride and the MoE handle's layers take the chain kernel
    // (POKIT_CUDA_FUSED_LAYERS=0 turns it off).
    void plan_layer_chain() {
        const char* env = std::getenv("POKIT_CUDA_FUSED_LAYERS");
        if ((env && env[0] == '0') || hybrid_) return;
        ChainAttnDesc d{};
        const uint32_t ts[5] = {POKIT_CUDA_DEC_ATTN_Q, POKIT_CUDA_DEC_ATTN_OUTPUT, POKIT_CUDA_DEC_ATTN_NORM,
                                POKIT_CUDA_DEC_ATTN_Q_NORM, POKIT_CUDA_DEC_ATTN_K_NORM};
        const uint64_t stride = cfg_.layers > 1 ? off_[kTensors + ts[0]] - off_[ts[0]] : 0;
        for (size_t l = 0; l < cfg_.layers; ++l)
            for (uint32_t t : ts)
                if (off_[l * kTensors + t] != off_[t] + l * stride) return;
        d.wqkv = tensor_ptr(0, POKIT_CUDA_DEC_ATTN_Q);
        d.wo = tensor_ptr(0, POKIT_CUDA_DEC_ATTN_OUTPUT);
        d.attn_norm = reinterpret_cast<const float*>(tensor_ptr(0, POKIT_CUDA_DEC_ATTN_NORM));
        d.q_norm = reinterpret_cast<const float*>(tensor_ptr(0, POKIT_CUDA_DEC_ATTN_Q_NORM));
        d.k_norm = reinterpret_cast<const float*>(tensor_ptr(0, POKIT_CUDA_DEC_ATTN_K_NORM));
        d.w_stride = stride;
        d.rope_cos = rope_;
        d.rope_sin = rope_ + cfg_.context * rh_;
        d.kc = kcache_;
        d.vc = vcache_;
        d.kv_stride = static_cast<uint64_t>(window_) * kd_;
        d.pos = pos_;
        d.q_heads = static_cast<uint32_t>(cfg_.q_heads);
        d.kv_heads = static_cast<uint32_t>(cfg_.kv_heads);
        d.head_dim = static_cast<uint32_t>(cfg_.head_dim);
        d.q_stride = d.head_dim;
        d.gated = 0;
        d.rotary_half = static_cast<uint32_t>(rh_);
        d.window = static_cast<uint32_t>(window_);
        d.eps = cfg_.rms_epsilon;
        d.scale = 1.0f / std::sqrt(static_cast<float>(cfg_.head_dim));
        d.rows = static_cast<uint32_t>(qrows_ + 2 * kd_);
        d.qkv_words = attn_ll_;
        d.att_words = attn_ll_ + d.rows;
        d.hidden_words = attn_ll_ + d.rows + qd_;
        d.status = status_ + 2;
        d.layers_total = static_cast<uint32_t>(cfg_.layers);
        if (!moe_attention_chain_fits(moe_, d)) return;
        layer_chain_ = d;
        fused_layers_ = true;
    }

    // The attention block's arguments for layer l (ash_ holds this step's shape).
    AttnBlockArgs attn_args(size_t l) const {
        AttnBlockArgs a{};
        const auto F = [&](uint32_t t) { return reinterpret_cast<const float*>(tensor_ptr(l, t)); };
        const uint64_t kv_off = static_cast<uint64_t>(l) * window_ * kd_;
        const uint32_t rows = static_cast<uint32_t>(qrows_ + 2 * kd_);
        a.wqkv = tensor_ptr(l, POKIT_CUDA_DEC_ATTN_Q);
        a.wo = tensor_ptr(l, POKIT_CUDA_DEC_ATTN_OUTPUT);
        a.attn_norm = F(POKIT_CUDA_DEC_ATTN_NORM);
        a.q_norm = F(POKIT_CUDA_DEC_ATTN_Q_NORM);
        a.k_norm = F(POKIT_CUDA_DEC_ATTN_K_NORM);
        a.rope_cos = rope_;
        a.rope_sin = rope_ + cfg_.context * rh_;
        a.kc = kcache_ + kv_off;
        a.vc = vcache_ + kv_off;
        a.pos_p = pos_;
        a.sh = ash_;
        a.hidden = hidden_;
        a.qkv_ll = attn_ll_;
        a.att_ll = attn_ll_ + rows;
        a.status = status_ + 2;
        a.H = static_cast<uint32_t>(cfg_.hidden);
        a.rows = rows;
        a.qd = static_cast<uint32_t>(qd_);
        a.layer = static_cast<uint32_t>(l);
        a.layers = static_cast<uint32_t>(cfg_.layers);
        a.eps = cfg_.rms_epsilon;
        return a;
    }

    cudaError_t launch_attn_block(const AttnBlockArgs& a, cudaStream_t s) {
        cudaLaunchConfig_t lc{};
        lc.gridDim = dim3(attn_grid_);
        lc.blockDim = dim3(kAttnBlockThreads);
        lc.dynamicSmemBytes = attn_smem_;
        lc.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
        return cudaLaunchKernelEx(&lc, attn_block_kernel, a);
    }

    // Position 0, zero DeltaNet states and attention words (the KV ring
    // needs no clearing: attention reads only positions written since).
    void clear_state() {
        guard(cudaMemsetAsync(pos_, 0, 4, stream_), "reset");
        if (ssm_) guard(cudaMemsetAsync(ssm_, 0, ssm_bytes_, stream_), "reset");
        // The attention words' tags repeat with the positions of a new sequence.
        if (attn_ll_) guard(cudaMemsetAsync(attn_ll_, 0, attn_words_ * 8, stream_), "reset");
    }

    void release() {
        for (auto& g : graphs_) if (g) cudaGraphExecDestroy(g);
        if (join_) cudaEventDestroy(join_);
        if (capture_stream_) cudaStreamDestroy(capture_stream_);
        if (stream_) cudaStreamDestroy(stream_);
        if (pinned_ids_) cudaFreeHost(pinned_ids_);
        if (seq_) cudaFree(seq_);
        if (delta_scratch_) cudaFree(delta_scratch_);
        if (work_) cudaFree(work_);
        if (rope_) cudaFree(rope_);
        if (vcache_) cudaFree(vcache_);
        if (kcache_) cudaFree(kcache_);
        if (ssm_) cudaFree(ssm_);
        if (attn_ll_) cudaFree(attn_ll_);
        if (pool_) cudaFree(pool_);
        if (moe_) pokit_cuda_moe_destroy(moe_);
        moe_ = nullptr;
    }

    cudaError_t embed(cudaStream_t s) {
        const void* t = pool_ + global_off_[POKIT_CUDA_DEC_TOKEN_EMBD];
        const uint32_t H = static_cast<uint32_t>(cfg_.hidden);
        switch (cfg_.embed_type) {
            case kF32: return launch_embed<kF32>(t, H, seq_, pos_, hidden_, s);
            case kQ8_0: return launch_embed<kQ8_0>(t, H, seq_, pos_, hidden_, s);
            case kQ4_K: return launch_embed<kQ4_K>(t, H, seq_, pos_, hidden_, s);
            case kQ5_K: return launch_embed<kQ5_K>(t, H, seq_, pos_, hidden_, s);
            default: return launch_embed<kQ6_K>(t, H, seq_, pos_, hidden_, s);
        }
    }

    // The launches of one token step on `s`.
    cudaError_t enqueue(bool logits, cudaStream_t s, uint64_t* launches) {
        const uint32_t H = static_cast<uint32_t>(cfg_.hidden), d = static_cast<uint32_t>(cfg_.head_dim);
        const uint32_t qh = static_cast<uint32_t>(cfg_.q_heads), kvh = static_cast<uint32_t>(cfg_.kv_heads);
        const uint32_t win = static_cast<uint32_t>(window_);
        const float eps = cfg_.rms_epsilon, scale = 1.0f / std::sqrt(static_cast<float>(d));
        AttendShape ash{};
        ash.qh = qh;
        ash.kvh = kvh;
        ash.d = d;
        ash.q_stride = hybrid_ ? 2u * d : d;
        ash.gated = hybrid_ ? 1u : 0u;
        ash.rh = static_cast<uint32_t>(rh_);
        ash.window = win;
        ash.eps = eps;
        ash.scale = scale;
        ash_ = ash;
        pokit_cuda_delta_net_shape dsh{};
        dsh.key_heads = cfg_.ssm_group_count;
        dsh.value_heads = hv_;
        dsh.key_dim = cfg_.ssm_state_size;
        dsh.value_dim = hv_ ? vw_ / hv_ : 0;
        dsh.conv_kernel = cfg_.ssm_conv_kernel;
        dsh.rms_epsilon = eps;
        uint64_t n = 0;
        cudaError_t e = embed(s);
        ++n;
        if (fused_layers_ && e == cudaSuccess) {
            std::string err;
            pokit_cuda_moe_stats before{}, after{};
            pokit_cuda_moe_get_stats(moe_, &before);
            e = moe_decode_layers_attention(moe_, 0, cfg_.layers, hidden_, layer_chain_, s, &err);
            if (e != cudaSuccess) {
                moe_error_ = err;
                return e;
            }
            pokit_cuda_moe_get_stats(moe_, &after);
            n += after.kernel_launches - before.kernel_launches;
        }
        for (size_t l = 0; l < cfg_.layers && e == cudaSuccess && !fused_layers_; ++l) {
            const auto P = [&](uint32_t t) { return tensor_ptr(l, t); };
            const auto F = [&](uint32_t t) { return reinterpret_cast<const float*>(tensor_ptr(l, t)); };
            if (attention_layer(l) && attn_grid_) {
                const AttnBlockArgs a = attn_args(l);
                if (attn_moe_ && moe_attention_layer_fits(moe_, &a, sizeof a)) {
                    // The attention block and the layer's MoE block in one launch.
                    std::string err;
                    e = moe_decode_layer_attention(moe_, l, hidden_, &a, sizeof a, s, &err);
                    if (e != cudaSuccess) {
                        moe_error_ = err;
                        return e;
                    }
                    n += 1;
                    continue;
                }
                e = launch_attn_block(a, s);
                ++n;
            } else if (attention_layer(l)) {
                const uint64_t kv_off = static_cast<uint64_t>(l) * window_ * kd_;
                e = launch_linear_normed(cfg_.attn_type, P(POKIT_CUDA_DEC_ATTN_Q), static_cast<uint32_t>(qrows_ + 2 * kd_),
                                         H, hidden_, F(POKIT_CUDA_DEC_ATTN_NORM), eps, qkv_, s, pdl_);
                if (e != cudaSuccess) break;
                const float* qn = F(POKIT_CUDA_DEC_ATTN_Q_NORM);
                const float* kn = F(POKIT_CUDA_DEC_ATTN_K_NORM);
                const float* rc = rope_;
                const float* rs = rope_ + cfg_.context * rh_;
                if (pdl_) {
                    e = launch_dependent(attend_kernel, qh, kAttendThreads, attend_smem_bytes(), s, qkv_, qn, kn, rc, rs,
                                         kcache_ + kv_off, vcache_ + kv_off, pos_, ash, att_);
                    if (e != cudaSuccess) break;
                } else {
                    attend_kernel<<<qh, kAttendThreads, attend_smem_bytes(), s>>>(qkv_, qn, kn, rc, rs, kcache_ + kv_off,
                                                                      vcache_ + kv_off, pos_, ash, att_);
                }
                e = launch_linear(cfg_.attn_type, P(POKIT_CUDA_DEC_ATTN_OUTPUT), H, static_cast<uint32_t>(qd_), att_,
                                  hidden_, s, false, true, pdl_);
                n += 3;
            } else if (delta_grid_) {
                // Gated DeltaNet (qwen35_runner.cpp:582-656) in one launch.
                uint8_t* st = ssm_ + ssm_off_[l];
                DeltaBlockTensors t{};
                t.w_in = P(POKIT_CUDA_DEC_SSM_QKV);
                t.w_out = P(POKIT_CUDA_DEC_SSM_OUT);
                t.attn_norm = F(POKIT_CUDA_DEC_ATTN_NORM);
                t.conv_w = F(POKIT_CUDA_DEC_SSM_CONV1D);
                t.conv_state = reinterpret_cast<float*>(st);
                t.ssm_a = F(POKIT_CUDA_DEC_SSM_A);
                t.dt_bias = F(POKIT_CUDA_DEC_SSM_DT_BIAS);
                t.ssm_norm = F(POKIT_CUDA_DEC_SSM_NORM);
                t.state = reinterpret_cast<float*>(st + ssm_conv_bytes_);
                t.hidden = hidden_;
                t.proj = qkv_;
                t.att = att_;
                t.ms_part = delta_scratch_;
                t.counters = status_ + 16;
                t.timeout = status_ + 2;
                t.gates_bad = status_ + 1;
                if (delta_moe_) {
                    std::string err;
                    e = moe_decode_layer_delta(moe_, l, hidden_, delta_shape_, t, s, &err);
                    if (e != cudaSuccess) {
                        moe_error_ = err;
                        return e;
                    }
                    n += 1;
                    continue;                          // the MoE block ran in the same launch
                }
                e = launch_delta_block(delta_shape_, t, delta_grid_, delta_smem_, s);
                n += 1;
            } else {
                // Gated DeltaNet (qwen35_runner.cpp:582-627): one matvec over
                // [qkv | gate | alpha | beta], the conv1d + delta-rule step, ssm_out.
                e = launch_linear_normed(cfg_.attn_type, P(POKIT_CUDA_DEC_SSM_QKV),
                                         static_cast<uint32_t>(conv_ch_ + vw_ + 2 * hv_), H, hidden_,
                                         F(POKIT_CUDA_DEC_ATTN_NORM), eps, qkv_, s, pdl_);
                if (e != cudaSuccess) break;
                uint8_t* st = ssm_ + ssm_off_[l];
                float* gate = qkv_ + conv_ch_;
                float* alpha = gate + vw_;
                float* beta = alpha + hv_;
                if (!delta_net_shape_valid(dsh)) return cudaErrorInvalidValue;
                e = launch_delta_net_step(dsh, qkv_, gate, alpha, beta, F(POKIT_CUDA_DEC_SSM_CONV1D),
                                          reinterpret_cast<float*>(st), F(POKIT_CUDA_DEC_SSM_A),
                                          F(POKIT_CUDA_DEC_SSM_DT_BIAS), F(POKIT_CUDA_DEC_SSM_NORM),
                                          reinterpret_cast<float*>(st + ssm_conv_bytes_), att_, status_ + 1, s, pdl_);
                if (e != cudaSuccess) break;
                e = launch_linear(cfg_.attn_type, P(POKIT_CUDA_DEC_SSM_OUT), H, static_cast<uint32_t>(vw_), att_,
                                  hidden_, s, false, true, false);
                n += 4;
            }
            if (e != cudaSuccess) break;
            char err[256];
            pokit_cuda_moe_stats before{}, after{};
            pokit_cuda_moe_get_stats(moe_, &before);
            const pokit_cuda_status st = pokit_cuda_moe_decode_layers(moe_, l, 1, hidden_, s, err, sizeof err);
            if (st != POKIT_CUDA_STATUS_OK) {
                moe_error_ = err;
                return st == POKIT_CUDA_STATUS_INVALID_ARGUMENT ? cudaErrorInvalidValue : cudaErrorUnknown;
            }
            pokit_cuda_moe_get_stats(moe_, &after);
            n += after.kernel_launches - before.kernel_launches;
            e = cudaGetLastError();
        }
        if (e != cudaSuccess) return e;
        if (logits) {
            const float* onorm = reinterpret_cast<const float*>(pool_ + global_off_[POKIT_CUDA_DEC_OUTPUT_NORM]);
            const void* ow = pool_ + global_off_[POKIT_CUDA_DEC_OUTPUT];
            e = launch_linear_normed(cfg_.output_type, ow, static_cast<uint32_t>(cfg_.vocab), H, hidden_, onorm, eps,
                                     logits_, s, pdl_);
            if (e == cudaErrorInvalidValue) {        // an F32 or unaligned LM head: norm, then the plain matvec
                rms_norm_kernel<<<1, 1024, 0, s>>>(hidden_, onorm, eps, xn_, H);
                e = launch_linear(cfg_.output_type, ow, static_cast<uint32_t>(cfg_.vocab), H, xn_, logits_, s);
            }
            if (e != cudaSuccess) return e;
            if (pdl_) {
                e = launch_dependent(argmax_kernel, kArgmaxCtas, 256, 0, s, logits_,
                                     static_cast<uint32_t>(cfg_.vocab), part_v_, part_i_, arrivals_, seq_, pos_,
                                     static_cast<uint32_t>(cfg_.context + 1), status_);
                if (e != cudaSuccess) return e;
            } else {
                argmax_kernel<<<kArgmaxCtas, 256, 0, s>>>(logits_, static_cast<uint32_t>(cfg_.vocab), part_v_, part_i_,
                                                          arrivals_, seq_, pos_,
                                                          static_cast<uint32_t>(cfg_.context + 1), status_);
            }
            n += 2;
        }
        advance_kernel<<<1, 1, 0, s>>>(pos_);
        ++n;
        if (launches) *launches = n;
        return cudaGetLastError();
    }

    // One token step: a CUDA graph replay after the variant has run once
    // eagerly (which also sets every kernel attribute); eager launches if the
    // capture is refused.
    void step(bool logits, cudaStream_t s = nullptr) {
        cudaStream_t st = s ? s : stream_;
        const int v = logits ? 1 : 0;
        if (!graphs_[v] && (eager_runs_[v] == 0 || no_graphs_)) {
            uint64_t n = 0;
            const cudaError_t e = enqueue(logits, st, &n);
            if (e != cudaSuccess) fail_enqueue(e);
            ++eager_runs_[v];
            launches_per_step_ = n;
            return;
        }
        if (!graphs_[v]) {
            cudaGraph_t g = nullptr;
            guard(cudaStreamBeginCapture(capture_stream_, cudaStreamCaptureModeThreadLocal), "capture");
            uint64_t n = 0;
            const cudaError_t e = enqueue(logits, capture_stream_, &n);
            const cudaError_t end = cudaStreamEndCapture(capture_stream_, &g);
            cudaGraphExec_t exec = nullptr;
            cudaError_t inst = cudaErrorUnknown;
            if (e == cudaSuccess && end == cudaSuccess) inst = cudaGraphInstantiate(&exec, g, 0);
            if (inst == cudaSuccess) {
                graphs_[v] = exec;
            } else {
                // Capture refused: eager launches from now on (the reason is kept).
                no_graphs_ = true;
                capture_error_ = std::string(cudaGetErrorString(e != cudaSuccess ? e : end != cudaSuccess ? end : inst)) +
                                 (moe_error_.empty() ? "" : " (MoE block: " + moe_error_ + ")");
                moe_error_.clear();
                cudaGetLastError();
            }
            if (g) cudaGraphDestroy(g);
            if (!graphs_[v]) {
                const cudaError_t e2 = enqueue(logits, st, &n);
                if (e2 != cudaSuccess) fail_enqueue(e2);
                return;
            }
        }
        guard(cudaGraphLaunch(graphs_[v], st), "step graph");
    }

    void fail_enqueue(cudaError_t e) {
        if (!moe_error_.empty()) {
            const std::string m = "MoE block: " + moe_error_;
            moe_error_.clear();
            if (e == cudaErrorInvalidValue) throw std::invalid_argument(m);
            failed_ = true;
            failure_ = m;
            throw std::runtime_error(m);
        }
        guard(e, "decoder step");
    }

    void sync_and_check() {
        guard(cudaStreamSynchronize(stream_), "synchronize");
        guard(cudaMemcpyAsync(pinned_ids_ + kPinnedIds - 3, status_, 12, cudaMemcpyDeviceToHost, stream_), "status");
        guard(cudaStreamSynchronize(stream_), "status");
        const uint32_t st = pinned_ids_[kPinnedIds - 3], gates = pinned_ids_[kPinnedIds - 2];
        if (pinned_ids_[kPinnedIds - 1]) {
            // A bounded wait of the attention or DeltaNet block gave up: its
            // counters no longer match (sticky, like a CUDA error).
            failed_ = true;
            failure_ = "a fused attention or DeltaNet block abandoned its work after a bounded device-side wait "
                       "timed out";
            throw std::runtime_error(failure_);
        }
        char err[256];
        if (pokit_cuda_moe_synchronize(moe_, stream_, err, sizeof err) != POKIT_CUDA_STATUS_OK) {
            next_position_ = 0;
            cudaMemsetAsync(pos_, 0, 4, stream_);
            throw std::runtime_error(std::string("MoE block: ") + err);
        }
        if ((st & kStatusDecoderNonFinite) || gates) {
            cudaMemsetAsync(status_, 0, 8, stream_);
            cudaMemsetAsync(pos_, 0, 4, stream_);
            if (ssm_) cudaMemsetAsync(ssm_, 0, ssm_bytes_, stream_);
            if (attn_ll_) cudaMemsetAsync(attn_ll_, 0, attn_words_ * 8, stream_);
            cudaStreamSynchronize(stream_);
            next_position_ = 0;           // the reference resets its state and rethrows
            throw std::runtime_error(gates ? "invalid Gated DeltaNet decay or beta (gated_delta_net.cpp)"
                                           : "model produced non-finite logits");
        }
    }

    static constexpr uint32_t kTensors = POKIT_CUDA_DEC_SSM_OUT + 1;
    pokit_cuda_decoder_config cfg_;
    bool hybrid_ = false;
    size_t window_ = 0, qd_ = 0, kd_ = 0, qrows_ = 0, rh_ = 0;
    size_t kw_ = 0, vw_ = 0, hv_ = 0, conv_ch_ = 0;   // DeltaNet key width, value width, value heads, channels
    pokit_cuda_moe* moe_ = nullptr;
    uint8_t* pool_ = nullptr;
    uint64_t global_off_[3] = {};
    std::vector<uint64_t> off_;      // [layer][tensor] pool offsets
    uint8_t* ssm_ = nullptr;         // per DeltaNet layer: conv state, then recurrent state
    std::vector<uint64_t> ssm_off_;
    uint64_t ssm_conv_bytes_ = 0, ssm_bytes_ = 0;
    __half* kcache_ = nullptr;
    __half* vcache_ = nullptr;
    float* rope_ = nullptr;          // [context][half] cos, then [context][half] sin
    void* work_ = nullptr;
    float *hidden_ = nullptr, *xn_ = nullptr, *qkv_ = nullptr, *att_ = nullptr, *logits_ = nullptr;
    uint32_t *seq_ = nullptr, *pos_ = nullptr, *status_ = nullptr, *arrivals_ = nullptr, *part_i_ = nullptr;
    float* part_v_ = nullptr;
    uint32_t* pinned_ids_ = nullptr;
    cudaStream_t stream_ = nullptr, capture_stream_ = nullptr;
    cudaEvent_t join_ = nullptr;
    cudaGraphExec_t graphs_[2] = {nullptr, nullptr};
    int eager_runs_[2] = {0, 0};
    bool no_graphs_ = false;
    // Programmatic dependent launches between the attention-side kernels
    // (POKIT_CUDA_PDL=0 turns them off).
    bool pdl_ = [] {
        const char* v = std::getenv("POKIT_CUDA_PDL");
        return !(v && v[0] == '0');
    }();
    DeltaBlockShape delta_shape_{};           // the one-launch DeltaNet layer (delta_grid_ > 0)
    uint32_t delta_grid_ = 0, delta_smem_ = 0;
    bool delta_moe_ = false;                  // a DeltaNet layer and its MoE block in one launch
    bool attn_moe_ = false;                   // an attention layer and its MoE block in one launch
    float* delta_scratch_ = nullptr;
    unsigned long long* attn_ll_ = nullptr;   // fused attention: Q/K/V words, output words, hidden words
    uint64_t attn_words_ = 0;
    bool fused_layers_ = false;               // the layer loop as one chain launch
    ChainAttnDesc layer_chain_{};
    uint32_t attn_grid_ = 0;                   // 0: the three-kernel attention path
    size_t attn_smem_ = 0;
    AttendShape ash_{};
    uint64_t launches_per_step_ = 0;
    size_t next_position_ = 0;
    std::string moe_error_;
    std::string capture_error_;
    std::mutex mutex_;
    bool failed_ = false;
    std::string failure_;
};

}  // namespace pokit

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
struct pokit_cuda_decoder {
    explicit pokit_cuda_decoder(const pokit_cuda_decoder_config& c) : impl(c) {}
    pokit::Decoder impl;
};

namespace {
template <typename F>
pokit_cuda_status dguarded(char* err, size_t cap, F&& body) noexcept {
    try {
        body();
        pokit::set_error(err, cap, "");
        return POKIT_CUDA_STATUS_OK;
    } catch (const std::invalid_argument& e) {
        pokit::set_error(err, cap, e.what());
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    } catch (const std::out_of_range& e) {
        pokit::set_error(err, cap, e.what());
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    } catch (const std::length_error& e) {
        pokit::set_error(err, cap, e.what());
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        pokit::set_error(err, cap, e.what());
        return POKIT_CUDA_STATUS_RUNTIME_ERROR;
    } catch (...) {
        pokit::set_error(err, cap, "unknown decoder failure");
        return POKIT_CUDA_STATUS_INTERNAL_ERROR;
    }
}
}  // namespace

extern "C" {

pokit_cuda_status pokit_cuda_decoder_create(const pokit_cuda_decoder_config* config, pokit_cuda_decoder** out,
                                            char* error_buffer, size_t error_capacity) {
    if (out) *out = nullptr;
    return dguarded(error_buffer, error_capacity, [&] {
        if (!config || !out) throw std::invalid_argument("configuration and output handle are required");
        *out = new pokit_cuda_decoder(*config);
    });
}

void pokit_cuda_decoder_destroy(pokit_cuda_decoder* decoder) { delete decoder; }

pokit_cuda_moe* pokit_cuda_decoder_moe(pokit_cuda_decoder* decoder) { return decoder ? decoder->impl.moe() : nullptr; }

size_t pokit_cuda_decoder_tensor_bytes(const pokit_cuda_decoder* decoder, size_t layer, uint32_t tensor) {
    return decoder ? decoder->impl.tensor_bytes(layer, tensor) : 0;
}

pokit_cuda_status pokit_cuda_decoder_upload_tensor(pokit_cuda_decoder* decoder, size_t layer, uint32_t tensor,
                                                   const void* host_bytes, size_t bytes, char* error_buffer,
                                                   size_t error_capacity) {
    return dguarded(error_buffer, error_capacity, [&] {
        if (!decoder) throw std::invalid_argument("decoder handle is required");
        std::lock_guard<std::mutex> lock(decoder->impl.mutex());
        decoder->impl.upload(layer, tensor, host_bytes, bytes);
    });
}

pokit_cuda_status pokit_cuda_decoder_synthesize_tensor(pokit_cuda_decoder* decoder, size_t layer, uint32_t tensor,
                                                       uint64_t seed, uint64_t stream_id, char* error_buffer,
                                                       size_t error_capacity) {
    return dguarded(error_buffer, error_capacity, [&] {
        if (!decoder) throw std::invalid_argument("decoder handle is required");
        std::lock_guard<std::mutex> lock(decoder->impl.mutex());
        decoder->impl.synthesize(layer, tensor, seed, stream_id);
    });
}

pokit_cuda_status pokit_cuda_decoder_forward_token(pokit_cuda_decoder* decoder, uint32_t token, uint64_t position,
                                                   float* logits_host, char* error_buffer, size_t error_capacity) {
    return dguarded(error_buffer, error_capacity, [&] {
        if (!decoder) throw std::invalid_argument("decoder handle is required");
        std::lock_guard<std::mutex> lock(decoder->impl.mutex());
        decoder->impl.forward_token(token, position, logits_host);
    });
}

pokit_cuda_status pokit_cuda_decoder_generate_tokens(pokit_cuda_decoder* decoder, const uint32_t* prompt,
                                                     size_t prompt_tokens, size_t max_new_tokens,
                                                     uint32_t* tokens_out, size_t* generated,
                                                     pokit_cuda_generation_stats* stats, char* error_buffer,
                                                     size_t error_capacity) {
    return dguarded(error_buffer, error_capacity, [&] {
        if (!decoder) throw std::invalid_argument("decoder handle is required");
        std::lock_guard<std::mutex> lock(decoder->impl.mutex());
        decoder->impl.generate(prompt, prompt_tokens, max_new_tokens, tokens_out, generated, stats);
    });
}

pokit_cuda_status pokit_cuda_decoder_run_steps(pokit_cuda_decoder* decoder, size_t steps, void* stream,
                                               char* error_buffer, size_t error_capacity) {
    return dguarded(error_buffer, error_capacity, [&] {
        if (!decoder) throw std::invalid_argument("decoder handle is required");
        std::lock_guard<std::mutex> lock(decoder->impl.mutex());
        decoder->impl.run_steps(steps, static_cast<cudaStream_t>(stream));
    });
}

pokit_cuda_status pokit_cuda_decoder_reset(pokit_cuda_decoder* decoder, char* error_buffer, size_t error_capacity) {
    return dguarded(error_buffer, error_capacity, [&] {
        if (!decoder) throw std::invalid_argument("decoder handle is required");
        std::lock_guard<std::mutex> lock(decoder->impl.mutex());
        decoder->impl.reset();
    });
}

uint64_t pokit_cuda_decoder_launches_per_step(const pokit_cuda_decoder* decoder) {
    return decoder ? decoder->impl.launches_per_step() : 0;
}

int pokit_cuda_decoder_step_graphs(const pokit_cuda_decoder* decoder, char* reason_buffer, size_t reason_capacity) {
    if (!decoder) return 0;
    pokit::set_error(reason_buffer, reason_capacity, decoder->impl.capture_error().c_str());
    return decoder->impl.step_graphs();
}

}  // extern "C"
