// pokit_deltanet.cu -- one token of the Qwen3.5 Gated DeltaNet mixer between
// its projections (PokitLMs src/qwen35_runner.cpp:613-656), on sm_100a:
//
//   conv    depthwise causal conv1d step with SiLU over the projected q|k|v
//           channels, in place, state = the last kernel - 1 inputs
//           (causal_depthwise_conv1d_step, src/causal_conv1d.cpp:25-50)
//   gates   log_decay = ssm_a * softplus(alpha + dt_bias), beta = sigmoid(beta)
//           (qwen35_runner.cpp:633-642; softplus :117-121)
//   delta   per value head h (key head h % key_heads): L2-normalised q (times
//           1/sqrt(dk)) and k, state *= exp(log_decay), delta = (v - state k)
//           beta, state += k delta, o = state q
//           (gated_delta_recurrent_step_grouped, src/gated_delta_net.cpp:28-110)
//   norm    y = o / rms(o) * ssm_norm * silu(z) per head
//           (rms_norm_gated, src/rms_norm.cpp:46-74)
//
// The recurrent state (value_heads x value_dim x key_dim F32, 2 MiB for
// configuration 3) is streamed once per token: a warp owns a value row at a
// time, its lanes the key columns (coalesced 512-byte rows), so the state
// update is HBM-bound.  An invalid decay or gate (the reference throws) sets
// bit 0 of the status word and leaves that head's state untouched.
#include "../../include/pokit_cuda.h"
#include "pokit_kernels.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

namespace pokit {
namespace {

constexpr uint32_t kStepThreads = 512;
constexpr uint32_t kMaxDim = 256;

__device__ __forceinline__ float sigmoid_signed(float v) {
    if (v >= 0.0f) return 1.0f / (1.0f + expf(-v));
    const float e = expf(v);
    return e / (1.0f + e);
}

__device__ __forceinline__ float softplus_runner(float v) {
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return log1pf(expf(v));
}

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ float block_sum(float v, float* red) {
    v = warp_sum32(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) r += red[w];
    return r;
}

// Under a programmatic launch the step kernel may start as soon as this one
// does (it reads x only after griddepcontrol.wait); this kernel's own wait
// orders its read of x after the projection that wrote it.
__global__ void delta_conv_kernel(float* __restrict__ x, const float* __restrict__ w, float* __restrict__ state,
                                  uint32_t channels, uint32_t kernel) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) return;
    const uint32_t sl = kernel - 1;
    const float in = x[c];
    float sum = __fmul_rn(in, w[static_cast<uint64_t>(c) * kernel + sl]);
    for (uint32_t t = 0; t < sl; ++t)
        sum = __fadd_rn(sum, __fmul_rn(state[static_cast<uint64_t>(c) * sl + t], w[static_cast<uint64_t>(c) * kernel + t]));
    if (sl) {
        for (uint32_t t = 0; t + 1 < sl; ++t) state[static_cast<uint64_t>(c) * sl + t] = state[static_cast<uint64_t>(c) * sl + t + 1];
        state[static_cast<uint64_t>(c) * sl + sl - 1] = in;
    }
    float s;
    if (sum >= 0.0f) {
        s = sum / (1.0f + expf(-sum));
    } else {
        const float e = expf(sum);
        s = sum * e / (1.0f + e);
    }
    x[c] = s;
}

__global__ void __launch_bounds__(kStepThreads)
delta_step_kernel(const float* __restrict__ x, const float* __restrict__ gate, const float* __restrict__ alpha,
                  const float* __restrict__ beta_raw, const float* __restrict__ a, const float* __restrict__ dt_bias,
                  const float* __restrict__ norm, float* __restrict__ state, float* __restrict__ out,
                  uint32_t* __restrict__ status, uint32_t kh, uint32_t dk, uint32_t dv, float eps) {
    __shared__ float nq[kMaxDim], nk[kMaxDim], o[kMaxDim];
    __shared__ float red[32];
    const uint32_t h = blockIdx.x, t = threadIdx.x, kq = h % kh;
    const int lane = t & 31, warp = t >> 5, warps = kStepThreads / 32;
    const float log_decay = a[h] * softplus_runner(alpha[h] + dt_bias[h]);
    const float b = sigmoid_signed(beta_raw[h]);
    const bool bad = !isfinite(log_decay) || log_decay > 0.0f || !isfinite(b) || b < 0.0f || b > 1.0f;
    const float* q = x + static_cast<uint64_t>(kq) * dk;
    const float* k = x + static_cast<uint64_t>(kh) * dk + static_cast<uint64_t>(kq) * dk;
    const float* v = x + 2ull * kh * dk + static_cast<uint64_t>(h) * dv;
    const float qv = t < dk ? q[t] : 0.0f, kv = t < dk ? k[t] : 0.0f;
    const float sq = block_sum(qv * qv, red);
    const float sk = block_sum(kv * kv, red);
    if (t < dk) {
        nq[t] = __fmul_rn(__fmul_rn(qv, 1.0f / sqrtf(sq + 1.0e-6f)), 1.0f / sqrtf(static_cast<float>(dk)));
        nk[t] = __fmul_rn(kv, 1.0f / sqrtf(sk + 1.0e-6f));
    }
    __syncthreads();
    if (bad) {
        if (t == 0 && status) atomicOr(status, 1u);
        for (uint32_t i = t; i < dv; i += kStepThreads) out[static_cast<uint64_t>(h) * dv + i] = 0.0f;
        return;
    }
    const float decay = expf(log_decay);
    float* S = state + static_cast<uint64_t>(h) * dv * dk;
    const uint32_t per = dk / 32;
    for (uint32_t r = warp; r < dv; r += warps) {
        float* row = S + static_cast<uint64_t>(r) * dk;
        float c[kMaxDim / 32];
        float mem = 0.0f;
#pragma unroll
        for (uint32_t i = 0; i < kMaxDim / 32; ++i)
            if (i < per) {
                c[i] = __fmul_rn(row[lane + 32 * i], decay);
                mem = fmaf(c[i], nk[lane + 32 * i], mem);
            }
        mem = warp_sum32(mem);
        const float delta = __fmul_rn(__fsub_rn(v[r], mem), b);
        float acc = 0.0f;
#pragma unroll
        for (uint32_t i = 0; i < kMaxDim / 32; ++i)
            if (i < per) {
                c[i] = __fadd_rn(c[i], __fmul_rn(nk[lane + 32 * i], delta));
                acc = fmaf(c[i], nq[lane + 32 * i], acc);
                row[lane + 32 * i] = c[i];
            }
        acc = warp_sum32(acc);
        if (lane == 0) o[r] = acc;
    }
    __syncthreads();
    const float ov = t < dv ? o[t] : 0.0f;
    const float ms = block_sum(ov * ov, red);
    if (t < dv) {
        const float scale = 1.0f / sqrtf(ms / static_cast<float>(dv) + eps);
        const float g = gate[static_cast<uint64_t>(h) * dv + t];
        out[static_cast<uint64_t>(h) * dv + t] =
            __fmul_rn(__fmul_rn(__fmul_rn(ov, scale), norm[t]), __fmul_rn(g, sigmoid_signed(g)));
    }
}

// delta_step_kernel for key and value dims up to 128 (configuration 3's
// 128 x 128 heads): each warp holds its value rows of the head's state in
// registers (rows warp, warp + 16, ...; lanes the key columns), loaded before
// griddepcontrol.wait so the 2 MiB stream overlaps the conv kernel ahead of
// it; the arithmetic is delta_step_kernel's.  The projections (x, gate,
// alpha, beta) are written by the kernels this one may overlap, so they are
// read through L2 (ld.global.cg) after the wait, never the read-only path.
constexpr uint32_t kRegRows = 8, kRegCols = 4;          // 16 warps x 8 rows = 128; 32 lanes x 4 = 128

__global__ void __launch_bounds__(kStepThreads)
delta_step_regs_kernel(const float* x, const float* gate, const float* alpha, const float* beta_raw,
                       const float* __restrict__ a,
                       const float* __restrict__ dt_bias, const float* __restrict__ norm, float* __restrict__ state,
                       float* __restrict__ out, uint32_t* __restrict__ status, uint32_t kh, uint32_t dk, uint32_t dv,
                       float eps) {
    __shared__ float nq[kMaxDim], nk[kMaxDim], o[kMaxDim];
    __shared__ float red[32];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t h = blockIdx.x, t = threadIdx.x, kq = h % kh;
    const int lane = t & 31, warp = t >> 5;
    constexpr int warps = kStepThreads / 32;
    float* S = state + static_cast<uint64_t>(h) * dv * dk;
    const uint32_t per = dk / 32;
    float c[kRegRows][kRegCols];
#pragma unroll
    for (uint32_t j = 0; j < kRegRows; ++j) {
        const uint32_t r = warp + warps * j;
#pragma unroll
        for (uint32_t i = 0; i < kRegCols; ++i)
            c[j][i] = (r < dv && i < per) ? __ldcs(S + static_cast<uint64_t>(r) * dk + lane + 32 * i) : 0.0f;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const float log_decay = a[h] * softplus_runner(__ldcg(alpha + h) + dt_bias[h]);
    const float b = sigmoid_signed(__ldcg(beta_raw + h));
    const bool bad = !isfinite(log_decay) || log_decay > 0.0f || !isfinite(b) || b < 0.0f || b > 1.0f;
    const float* q = x + static_cast<uint64_t>(kq) * dk;
    const float* k = x + static_cast<uint64_t>(kh) * dk + static_cast<uint64_t>(kq) * dk;
    const float* v = x + 2ull * kh * dk + static_cast<uint64_t>(h) * dv;
    const float qv = t < dk ? __ldcg(q + t) : 0.0f, kv = t < dk ? __ldcg(k + t) : 0.0f;
    const float sq = block_sum(qv * qv, red);
    const float sk = block_sum(kv * kv, red);
    if (t < dk) {
        nq[t] = __fmul_rn(__fmul_rn(qv, 1.0f / sqrtf(sq + 1.0e-6f)), 1.0f / sqrtf(static_cast<float>(dk)));
        nk[t] = __fmul_rn(kv, 1.0f / sqrtf(sk + 1.0e-6f));
    }
    __syncthreads();
    if (bad) {
        if (t == 0 && status) atomicOr(status, 1u);
        for (uint32_t i = t; i < dv; i += kStepThreads) out[static_cast<uint64_t>(h) * dv + i] = 0.0f;
        return;
    }
    const float decay = expf(log_decay);
    float kk[kRegCols], qq[kRegCols];
#pragma unroll
    for (uint32_t i = 0; i < kRegCols; ++i) {
        kk[i] = i < per ? nk[lane + 32 * i] : 0.0f;
        qq[i] = i < per ? nq[lane + 32 * i] : 0.0f;
    }
    float mem[kRegRows];
#pragma unroll
    for (uint32_t j = 0; j < kRegRows; ++j) {
        mem[j] = 0.0f;
#pragma unroll
        for (uint32_t i = 0; i < kRegCols; ++i)
            if (i < per) {
                c[j][i] = __fmul_rn(c[j][i], decay);
                mem[j] = fmaf(c[j][i], kk[i], mem[j]);
            }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (uint32_t j = 0; j < kRegRows; ++j) mem[j] += __shfl_xor_sync(0xffffffffu, mem[j], off);
    float acc[kRegRows];
#pragma unroll
    for (uint32_t j = 0; j < kRegRows; ++j) {
        const uint32_t r = warp + warps * j;
        acc[j] = 0.0f;
        if (r < dv) {
            const float delta = __fmul_rn(__fsub_rn(__ldcg(v + r), mem[j]), b);
#pragma unroll
            for (uint32_t i = 0; i < kRegCols; ++i)
                if (i < per) {
                    c[j][i] = __fadd_rn(c[j][i], __fmul_rn(kk[i], delta));
                    acc[j] = fmaf(c[j][i], qq[i], acc[j]);
                    __stcs(S + static_cast<uint64_t>(r) * dk + lane + 32 * i, c[j][i]);
                }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (uint32_t j = 0; j < kRegRows; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
    if (lane == 0)
#pragma unroll
        for (uint32_t j = 0; j < kRegRows; ++j) {
            const uint32_t r = warp + warps * j;
            if (r < dv) o[r] = acc[j];
        }
    __syncthreads();
    const float ov = t < dv ? o[t] : 0.0f;
    const float ms = block_sum(ov * ov, red);
    if (t < dv) {
        const float scale = 1.0f / sqrtf(ms / static_cast<float>(dv) + eps);
        const float g = __ldcg(gate + static_cast<uint64_t>(h) * dv + t);
        out[static_cast<uint64_t>(h) * dv + t] =
            __fmul_rn(__fmul_rn(__fmul_rn(ov, scale), norm[t]), __fmul_rn(g, sigmoid_signed(g)));
    }
}

void set_error(char* destination, size_t capacity, const char* message) noexcept {
    if (!destination || capacity == 0) return;
    const size_t n = std::min(capacity - 1, std::strlen(message));
    std::memcpy(destination, message, n);
    destination[n] = '\0';
}

template <typename... Params, typename... Args>
cudaError_t launch_maybe_dependent(void (*kernel)(Params...), uint32_t grid, uint32_t block, cudaStream_t s, bool pdl,
                                   Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

}  // namespace

bool delta_net_shape_valid(const pokit_cuda_delta_net_shape& s) {
    return s.key_heads != 0 && s.value_heads != 0 && s.value_heads % s.key_heads == 0 && s.key_dim != 0 &&
           s.key_dim % 32 == 0 && s.key_dim <= kMaxDim && s.value_dim != 0 && s.value_dim <= kMaxDim &&
           s.conv_kernel != 0 && s.conv_kernel <= 64 && s.rms_epsilon > 0.0f && s.value_heads <= 65535;
}

cudaError_t launch_delta_net_step(const pokit_cuda_delta_net_shape& s, float* projected, const float* gate,
                                  const float* alpha, const float* beta, const float* conv_weights, float* conv_state,
                                  const float* ssm_a, const float* dt_bias, const float* ssm_norm,
                                  float* recurrent_state, float* output, uint32_t* status, cudaStream_t st, bool pdl) {
    const uint32_t channels = static_cast<uint32_t>(2 * s.key_heads * s.key_dim + s.value_heads * s.value_dim);
    cudaError_t e = launch_maybe_dependent(delta_conv_kernel, (channels + 255) / 256, 256u, st, pdl, projected,
                                           conv_weights, conv_state, channels, static_cast<uint32_t>(s.conv_kernel));
    if (e != cudaSuccess) return e;
    const bool regs = s.key_dim <= 32 * kRegCols && s.value_dim <= (kStepThreads / 32) * kRegRows;
    return launch_maybe_dependent(regs ? delta_step_regs_kernel : delta_step_kernel,
                                  static_cast<uint32_t>(s.value_heads), kStepThreads, st, pdl,
                                  static_cast<const float*>(projected), gate, alpha, beta, ssm_a, dt_bias, ssm_norm,
                                  recurrent_state, output, status, static_cast<uint32_t>(s.key_heads),
                                  static_cast<uint32_t>(s.key_dim), static_cast<uint32_t>(s.value_dim), s.rms_epsilon);
}

}  // namespace pokit

extern "C" pokit_cuda_status pokit_cuda_delta_net_step(
    const pokit_cuda_delta_net_shape* shape, float* projected, const float* gate, const float* alpha,
    const float* beta, const float* conv_weights, float* conv_state, const float* ssm_a, const float* dt_bias,
    const float* ssm_norm, float* recurrent_state, float* output, uint32_t* status, void* stream,
    char* error_buffer, size_t error_capacity) {
    using pokit::set_error;
    if (!shape || !projected || !gate || !alpha || !beta || !conv_weights || !ssm_a || !dt_bias || !ssm_norm ||
        !recurrent_state || !output || (shape->conv_kernel > 1 && !conv_state)) {
        set_error(error_buffer, error_capacity, "shape, tensors, states and output are required");
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const pokit_cuda_delta_net_shape& s = *shape;
    if (!pokit::delta_net_shape_valid(s)) {
        set_error(error_buffer, error_capacity, "invalid DeltaNet shape");
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const cudaError_t e = pokit::launch_delta_net_step(s, projected, gate, alpha, beta, conv_weights, conv_state, ssm_a,
                                                       dt_bias, ssm_norm, recurrent_state, output, status,
                                                       static_cast<cudaStream_t>(stream), false);
    if (e != cudaSuccess) {
        set_error(error_buffer, error_capacity, cudaGetErrorString(e));
        return POKIT_CUDA_STATUS_RUNTIME_ERROR;
    }
    set_error(error_buffer, error_capacity, "");
    return POKIT_CUDA_STATUS_OK;
}
