// pokit_backend.cpp -- C++ host layer of the B200 MoE expert backend and the
// extern "C" entry points declared in include/pokit_cuda.h.
//
//   MoeBackend     HBM-resident expert pool (one allocation for every layer's
//                  router, gate/up/down expert tensors, norms and shared
//                  expert) + the per-block launch sequence + CUDA-graph decode
//                  chain.  Replaces ExpertStore's LRU (PokitLMs
//                  src/expert_store.cpp:81-141): every expert is resident, so
//                  a lookup is an address computation on the device.
//   LinearBackend  TensorLinearBackend::try_linear with host spans and a
//                  device cache of weight payloads (the Vulkan backend's
//                  model cache, src/vulkan_linear.cpp:516-563).
//
// Errors are C++ exceptions inside and status codes at the C boundary, as in
// PokitLMs src/c_api.cpp:92-101.  CUDA failures are sticky per handle, as the
// Vulkan backend's `failed` flag (src/vulkan_linear.cpp:636, 731-735).
#include "../../include/pokit_cuda.h"
#include "pokit_kernels.h"
#include "pokit_types.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <list>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace pokit {
namespace {

struct RouterFailure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    if (e == cudaErrorInvalidValue)
        throw std::invalid_argument(std::string(what) + ": unsupported shape or argument");
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

uint64_t align256(uint64_t v) { return (v + 255u) & ~uint64_t(255); }

bool type_supported(uint32_t t) {
    return t == kF32 || t == kQ8_0 || t == kQ4_K || t == kQ5_K || t == kQ6_K;
}

bool quant_supported(uint32_t t) { return t == kQ8_0 || t == kQ4_K || t == kQ5_K || t == kQ6_K; }

class DeviceScope {
public:
    explicit DeviceScope(int device) {
        check(cudaGetDevice(&previous_), "cudaGetDevice");
        if (previous_ != device) check(cudaSetDevice(device), "cudaSetDevice");
        device_ = device;
    }
    ~DeviceScope() {
        if (previous_ != device_) cudaSetDevice(previous_);
    }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;

private:
    int previous_ = 0;
    int device_ = 0;
};

uint64_t now_ns() {
    return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
        std::chrono::steady_clock::now().time_since_epoch()).count());
}

}  // namespace

// ---------------------------------------------------------------------------
class MoeBackend {
public:
    explicit MoeBackend(const pokit_cuda_moe_config& c) : cfg_(c) {
        if (c.layers == 0 || c.hidden == 0 || c.hidden % 256 || c.inter == 0 || c.inter % 256 ||
            c.experts == 0 || c.experts > 1024 || c.top_k == 0 || c.top_k > c.experts ||
            c.top_k > 64 || c.flavour > 1)
            throw std::invalid_argument("invalid MoE configuration");
        if (!quant_supported(c.gate_type) || !quant_supported(c.up_type) ||
            !quant_supported(c.down_type))
            throw std::invalid_argument("unsupported expert tensor type");
        if (c.expert_count && (c.expert_first >= c.experts || c.expert_count > c.experts - c.expert_first))
            throw std::invalid_argument("expert shard out of range");
        if (c.expert_count && c.expert_count < c.experts && c.shared_inter)
            throw std::invalid_argument("an expert shard cannot hold the shared expert");
        if (c.shared_inter) {
            if (c.flavour != POKIT_CUDA_MOE_QWEN35 || c.shared_inter % 256 ||
                !quant_supported(c.shared_gate_type) || !quant_supported(c.shared_up_type) ||
                !quant_supported(c.shared_down_type))
                throw std::invalid_argument("invalid shared expert configuration");
        }
        device_ = c.device;
        expert_first_ = c.expert_count ? c.expert_first : 0;
        expert_local_ = c.expert_count ? c.expert_count : c.experts;
        DeviceScope scope(device_);
        layer_down_.assign(c.layers, c.down_type);
        if (c.layer_down_types) {
            for (size_t l = 0; l < c.layers; ++l) {
                if (!quant_supported(c.layer_down_types[l]))
                    throw std::invalid_argument("unsupported per-layer down type");
                layer_down_[l] = c.layer_down_types[l];
            }
        }
        // Pool layout: per layer, every tensor at a 256-byte boundary.
        offsets_.resize(c.layers);
        uint64_t off = 0;
        for (size_t l = 0; l < c.layers; ++l) {
            for (uint32_t t = 0; t < 9; ++t) {
                const uint64_t b = tensor_bytes(l, t);
                offsets_[l][t] = b ? off : UINT64_MAX;
                off += align256(b);
            }
        }
        pool_bytes_ = off;
        check(cudaMalloc(&pool_, pool_bytes_), "cudaMalloc(expert pool)");
        check(cudaMemset(pool_, 0, pool_bytes_), "cudaMemset(expert pool)");
        check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaStreamCreateWithFlags(&capture_stream_, cudaStreamNonBlocking), "cudaStreamCreate");

        resident_.assign(c.layers, 0u);
        devs_.resize(c.layers);
        for (size_t l = 0; l < c.layers; ++l) devs_[l] = make_layer_dev(l);
        scratch_bytes_ = moe_scratch_bytes(devs_[0]);
        for (size_t l = 1; l < c.layers; ++l)
            scratch_bytes_ = std::max<uint64_t>(scratch_bytes_, moe_scratch_bytes(devs_[l]));
        check(cudaMalloc(&scratch_, scratch_bytes_), "cudaMalloc(scratch)");
        check(cudaMemset(scratch_, 0, scratch_bytes_), "cudaMemset(scratch)");
        S_ = moe_scratch_carve(devs_[0], scratch_);
        if (!sharded())
            for (size_t l = 0; l < c.layers; ++l) check(prepare_moe_block(devs_[l]), "prepare MoE kernels");
        check(cudaMalloc(&devs_dev_, sizeof(MoeLayerDev) * c.layers), "cudaMalloc(layer table)");
        check(cudaMemcpy(devs_dev_, devs_.data(), sizeof(MoeLayerDev) * c.layers,
                         cudaMemcpyHostToDevice), "upload layer table");
        // The decode chain runs as a CUDA graph of per-block kernels (a graph
        // kernel boundary costs ~0.6 us on B200, a 148-CTA software grid
        // barrier ~1.3 us).  POKIT_CUDA_DECODE=persistent selects the single
        // cooperative kernel with three grid barriers per layer instead.
        // Tensor-core layers of one shape run the persistent chain kernel (one
        // cooperative launch per call, phases handed off through counters);
        // POKIT_CUDA_DECODE=graph keeps the per-block kernel graph for them.
        const char* mode = std::getenv("POKIT_CUDA_DECODE");
        const std::string want = mode ? mode : "";
        const bool want_persistent = want == "persistent";
        decode_grid_ = want_persistent ? moe_decode_grid(devs_[0]) : 0u;
        std::vector<Chain35Maps> chain35_maps;
        if (!sharded() && !want_persistent && want != "graph" &&
            moe_chain_plan(devs_.data(), static_cast<uint32_t>(c.layers), &chain_plan_)) {
            const uint64_t cb = moe_chain_scratch_bytes(devs_[0]);
            check(cudaMalloc(&chain_scratch_, cb), "cudaMalloc(chain scratch)");
            check(cudaMemset(chain_scratch_, 0, cb), "cudaMemset(chain scratch)");
            C_ = moe_chain_scratch_carve(devs_[0], chain_scratch_);
            chain_ok_ = true;
        } else if (!sharded() && !want_persistent && want != "graph" &&
                   moe_chain35_plan(devs_.data(), static_cast<uint32_t>(c.layers), &chain35_plan_, &chain35_maps)) {
            // Qwen3.5-MoE blocks (shared expert, per-layer down types): their chain kernel.
            check(cudaMalloc(&chain35_maps_, sizeof(Chain35Maps) * chain35_maps.size()), "cudaMalloc(tensor maps)");
            check(cudaMemcpy(chain35_maps_, chain35_maps.data(), sizeof(Chain35Maps) * chain35_maps.size(),
                             cudaMemcpyHostToDevice),
                  "cudaMemcpy(tensor maps)");
            const uint64_t cb = moe_chain_scratch_bytes(devs_[0]);
            check(cudaMalloc(&chain_scratch_, cb), "cudaMalloc(chain scratch)");
            check(cudaMemset(chain_scratch_, 0, cb), "cudaMemset(chain scratch)");
            C_ = moe_chain_scratch_carve(devs_[0], chain_scratch_);
            chain35_ok_ = true;
        }
        check(cudaMalloc(&io_, align256(c.hidden * 4) * 2), "cudaMalloc(io)");
        check(cudaMallocHost(&pinned_, align256(c.hidden * 4) * 2 + 4096), "cudaMallocHost");
    }

    ~MoeBackend() {
        for (void* p : ex_opened_) cudaIpcCloseMemHandle(p);
        if (ex_region_) cudaFree(ex_region_);
        if (ex_words_) cudaFree(ex_words_);
        for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second.first);
        if (batch_pinned_) cudaFreeHost(batch_pinned_);
        if (batch_io_) cudaFree(batch_io_);
        if (batch_scratch_) cudaFree(batch_scratch_);
        if (pinned_) cudaFreeHost(pinned_);
        if (io_) cudaFree(io_);
        if (scratch_) cudaFree(scratch_);
        if (chain_scratch_) cudaFree(chain_scratch_);
        if (devs_dev_) cudaFree(devs_dev_);
        if (chain35_maps_) cudaFree(chain35_maps_);
        if (pool_) cudaFree(pool_);
        if (capture_stream_) cudaStreamDestroy(capture_stream_);
        if (stream_) cudaStreamDestroy(stream_);
    }

    MoeBackend(const MoeBackend&) = delete;
    MoeBackend& operator=(const MoeBackend&) = delete;

    std::mutex& mutex() { return mutex_; }

    uint64_t tensor_bytes(size_t layer, uint32_t t) const {
        const uint64_t H = cfg_.hidden, I = cfg_.inter, E = cfg_.experts, SI = cfg_.shared_inter;
        if (layer >= cfg_.layers) return 0;
        switch (t) {
            case POKIT_CUDA_MOE_ROUTER: return E * H * 4;
            case POKIT_CUDA_MOE_GATE: return expert_local_ * I * row_bytes(cfg_.gate_type, H);
            case POKIT_CUDA_MOE_UP: return expert_local_ * I * row_bytes(cfg_.up_type, H);
            case POKIT_CUDA_MOE_DOWN: return expert_local_ * H * row_bytes(layer_down_[layer], I);
            case POKIT_CUDA_MOE_FFN_NORM: return H * 4;
            case POKIT_CUDA_MOE_SHARED_ROUTER: return SI ? H * 4 : 0;
            case POKIT_CUDA_MOE_SHARED_GATE: return SI ? SI * row_bytes(cfg_.shared_gate_type, H) : 0;
            case POKIT_CUDA_MOE_SHARED_UP: return SI ? SI * row_bytes(cfg_.shared_up_type, H) : 0;
            case POKIT_CUDA_MOE_SHARED_DOWN: return SI ? H * row_bytes(cfg_.shared_down_type, SI) : 0;
            default: return 0;
        }
    }

    uint32_t tensor_type(size_t layer, uint32_t t) const {
        switch (t) {
            case POKIT_CUDA_MOE_GATE: return cfg_.gate_type;
            case POKIT_CUDA_MOE_UP: return cfg_.up_type;
            case POKIT_CUDA_MOE_DOWN: return layer_down_[layer];
            case POKIT_CUDA_MOE_SHARED_GATE: return cfg_.shared_gate_type;
            case POKIT_CUDA_MOE_SHARED_UP: return cfg_.shared_up_type;
            case POKIT_CUDA_MOE_SHARED_DOWN: return cfg_.shared_down_type;
            default: return kF32;
        }
    }

    uint8_t* tensor_ptr(size_t layer, uint32_t t) const {
        if (layer >= cfg_.layers || t > 8 || offsets_[layer][t] == UINT64_MAX) return nullptr;
        return pool_ + offsets_[layer][t];
    }

    void upload_tensor(size_t layer, uint32_t t, const void* host, size_t bytes) {
        ensure_ok();
        if (layer >= cfg_.layers || t > 8) throw std::invalid_argument("layer or tensor out of range");
        const uint64_t want = tensor_bytes(layer, t);
        if (want == 0) throw std::invalid_argument("tensor does not exist in this configuration");
        if (!host || bytes != want) throw std::invalid_argument("tensor byte size does not match configuration");
        DeviceScope scope(device_);
        const uint64_t t0 = now_ns();
        guard(cudaMemcpy(tensor_ptr(layer, t), host, bytes, cudaMemcpyHostToDevice), "upload");
        read_time_ns_ += now_ns() - t0;
        bytes_read_ += bytes;
        read_operations_ += 1;
        mark_resident(layer, t);
    }

    void synthesize_tensor(size_t layer, uint32_t t, uint64_t seed, uint64_t stream_id) {
        ensure_ok();
        if (layer >= cfg_.layers || t > 8) throw std::invalid_argument("layer or tensor out of range");
        const uint64_t bytes = tensor_bytes(layer, t);
        const uint32_t type = tensor_type(layer, t);
        if (bytes == 0 || !quant_supported(type))
            throw std::invalid_argument("only quantised expert tensors can be synthesised");
        DeviceScope scope(device_);
        // A shard holds blocks [first * per_expert, ...) of the whole tensor's
        // stream, so every shard sees the same weights as one whole pool.
        const bool expert_tensor =
            t == POKIT_CUDA_MOE_GATE || t == POKIT_CUDA_MOE_UP || t == POKIT_CUDA_MOE_DOWN;
        const uint64_t nblocks = bytes / block_bytes(type);
        const uint64_t first_block = expert_tensor ? expert_first_ * (nblocks / expert_local_) : 0;
        guard(launch_synth_blocks(type, seed, stream_id, nblocks, tensor_ptr(layer, t), stream_, first_block),
              "synthesize");
        guard(cudaStreamSynchronize(stream_), "synthesize");
        kernel_launches_ += 1;
        mark_resident(layer, t);
    }

    void expert_view(size_t layer, uint32_t matrix, size_t expert, const void** ptr, size_t* bytes) const {
        if (layer >= cfg_.layers || expert < expert_first_ || expert >= expert_first_ + expert_local_ ||
            (matrix != POKIT_CUDA_MOE_GATE && matrix != POKIT_CUDA_MOE_UP && matrix != POKIT_CUDA_MOE_DOWN))
            throw std::invalid_argument("expert view out of range (or not held by this shard)");
        const uint64_t slice = tensor_bytes(layer, matrix) / expert_local_;
        *ptr = tensor_ptr(layer, matrix) + (expert - expert_first_) * slice;
        *bytes = slice;
        ++hits_;
    }

    void forward(size_t layer, const float* x, float* out, uint32_t* ids, float* w, cudaStream_t s) {
        ensure_ok();
        refuse_sharded();
        if (layer >= cfg_.layers) throw std::invalid_argument("layer out of range");
        if (!x || !out) throw std::invalid_argument("input and output are required");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        uint32_t n = 0;
        guard(launch_moe_block(devs_[layer], S_, x, nullptr, out, nullptr, nullptr, st, &n), "moe block");
        kernel_launches_ += n;
        if (ids) guard(cudaMemcpyAsync(ids, S_.ids, cfg_.top_k * 4, cudaMemcpyDeviceToDevice, st), "ids");
        if (w) guard(cudaMemcpyAsync(w, S_.weights, cfg_.top_k * 4, cudaMemcpyDeviceToDevice, st), "weights");
        forward_calls_ += 1;
        hits_ += cfg_.top_k;
    }

    // A batch of tokens through one MoE block: the grouped-expert tensor-core
    // path when the layer allows it (Q4_K experts, no shared expert), else
    // one block launch sequence per token (F32 input, layer router only).
    void forward_batch(size_t layer, const void* x, uint32_t x_type, size_t tokens, const float* logits,
                       float* out, uint32_t* ids, float* w, cudaStream_t s) {
        ensure_ok();
        if (layer >= cfg_.layers) throw std::invalid_argument("layer out of range");
        if (!x || !out) throw std::invalid_argument("input and output are required");
        if (tokens == 0 || tokens > kMaxBatchTokens) throw std::invalid_argument("tokens must be 1..65536");
        if (x_type > POKIT_CUDA_INPUT_BF16) throw std::invalid_argument("unknown input type");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        const MoeLayerDev& L = devs_[layer];
        const uint32_t T = static_cast<uint32_t>(tokens), k = static_cast<uint32_t>(cfg_.top_k);
        if (moe_batch_grouped(L)) {
            ensure_batch_scratch(L, T);
            uint32_t n = 0;
            guard(launch_moe_batch(L, B_, x, x_type, T, logits, out, ids, w, S_.status, st, &n, nullptr,
                                   ex_connected_ ? &ex_ : nullptr),
                  "grouped MoE batch");
            kernel_launches_ += n;
        } else {
            refuse_sharded();
            if (ex_connected_) throw std::invalid_argument("the peer-memory exchange needs the grouped path");
            if (x_type != POKIT_CUDA_INPUT_F32)
                throw std::invalid_argument("BF16 input needs the grouped path (Q4_K experts, no shared expert)");
            if (logits) throw std::invalid_argument("caller logits need the grouped path (Q4_K experts, no shared expert)");
            const float* xf = static_cast<const float*>(x);
            for (uint32_t t = 0; t < T; ++t) {
                uint32_t n = 0;
                guard(launch_moe_block(L, S_, xf + size_t(t) * cfg_.hidden, nullptr, out + size_t(t) * cfg_.hidden,
                                       nullptr, nullptr, st, &n),
                      "moe block");
                kernel_launches_ += n;
                if (ids) guard(cudaMemcpyAsync(ids + size_t(t) * k, S_.ids, k * 4, cudaMemcpyDeviceToDevice, st), "ids");
                if (w) guard(cudaMemcpyAsync(w + size_t(t) * k, S_.weights, k * 4, cudaMemcpyDeviceToDevice, st),
                             "weights");
            }
        }
        forward_calls_ += tokens;
        hits_ += tokens * cfg_.top_k;
    }

    // Measurement: the batched forward on device buffers `repetitions` times
    // with an event between its kernels; stage_us[i] receives the average
    // device time of stage i (grouped path only).  Returns the stage count.
    size_t time_batch(size_t layer, const void* x, uint32_t x_type, size_t tokens, const float* logits,
                      float* out, uint32_t reps, float* stage_us, size_t capacity, cudaStream_t s) {
        ensure_ok();
        if (layer >= cfg_.layers) throw std::invalid_argument("layer out of range");
        if (!x || !out || !stage_us || reps == 0) throw std::invalid_argument("buffers and repetitions required");
        if (tokens == 0 || tokens > kMaxBatchTokens) throw std::invalid_argument("tokens must be 1..65536");
        const MoeLayerDev& L = devs_[layer];
        if (!moe_batch_grouped(L)) throw std::invalid_argument("the layer does not use the grouped path");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        const uint32_t T = static_cast<uint32_t>(tokens);
        ensure_batch_scratch(L, T);
        const size_t stages = logits ? 7 : 8;
        if (capacity < stages) throw std::invalid_argument("stage_us needs room for 8 stages");
        std::vector<cudaEvent_t> ev(stages + 1);
        for (auto& e : ev) guard(cudaEventCreate(&e), "event");
        std::vector<double> sum(stages, 0.0);
        for (uint32_t r = 0; r < reps; ++r) {
            uint32_t n = 0;
            guard(launch_moe_batch(L, B_, x, x_type, T, logits, out, nullptr, nullptr, S_.status, st, &n, ev.data()),
                  "grouped MoE batch");
            kernel_launches_ += n;
            guard(cudaEventSynchronize(ev[stages]), "timing");
            for (size_t i = 0; i < stages; ++i) {
                float ms = 0.f;
                guard(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]), "timing");
                sum[i] += ms * 1e3;
            }
        }
        for (auto& e : ev) cudaEventDestroy(e);
        for (size_t i = 0; i < stages; ++i) stage_us[i] = static_cast<float>(sum[i] / reps);
        return stages;
    }

    // Host-span batch: copies the inputs through pinned staging, runs, copies
    // the outputs back and synchronises.
    void forward_batch_host(size_t layer, const void* x, uint32_t x_type, size_t tokens, const float* logits,
                            float* out, uint32_t* ids, float* w) {
        ensure_ok();
        if (!x || !out) throw std::invalid_argument("input and output are required");
        if (tokens == 0 || tokens > kMaxBatchTokens) throw std::invalid_argument("tokens must be 1..65536");
        if (x_type > POKIT_CUDA_INPUT_BF16) throw std::invalid_argument("unknown input type");
        DeviceScope scope(device_);
        const size_t H = cfg_.hidden, E = cfg_.experts, k = cfg_.top_k;
        const size_t xb = tokens * H * (x_type == POKIT_CUDA_INPUT_BF16 ? 2 : 4), lb = logits ? tokens * E * 4 : 0;
        const size_t ob = tokens * H * 4, rb = tokens * k * 4;
        const size_t need = align256(xb) + align256(lb) + align256(ob) + 2 * align256(rb);
        ensure_batch_io(need);
        uint8_t* d = static_cast<uint8_t*>(batch_io_);
        uint8_t* h = static_cast<uint8_t*>(batch_pinned_);
        const size_t ox = 0, ol = align256(xb), oo = ol + align256(lb), oi = oo + align256(ob), ow = oi + align256(rb);
        std::memcpy(h + ox, x, xb);
        if (logits) std::memcpy(h + ol, logits, lb);
        guard(cudaMemcpyAsync(d + ox, h + ox, logits ? ol + lb : xb, cudaMemcpyHostToDevice, stream_), "h2d");
        forward_batch(layer, d + ox, x_type, tokens, logits ? reinterpret_cast<const float*>(d + ol) : nullptr,
                      reinterpret_cast<float*>(d + oo), reinterpret_cast<uint32_t*>(d + oi),
                      reinterpret_cast<float*>(d + ow), stream_);
        guard(cudaMemcpyAsync(h + oo, d + oo, ow + rb - oo, cudaMemcpyDeviceToHost, stream_), "d2h");
        synchronize(stream_);
        std::memcpy(out, h + oo, ob);
        if (ids) std::memcpy(ids, h + oi, rb);
        if (w) std::memcpy(w, h + ow, rb);
    }

    // Average device time of one launch of a tensor-core kernel over the
    // layers [first, first + count), launched back to back.
    float time_kernel(uint32_t which, size_t first, size_t count, uint32_t reps, float* work, cudaStream_t s) {
        ensure_ok();
        refuse_sharded();
        if (count == 0 || first + count > cfg_.layers) throw std::invalid_argument("layer range out of bounds");
        if (!work) throw std::invalid_argument("a device buffer of hidden floats is required");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        float us = 0.0f;
        const cudaError_t e = time_moe_kernel(devs_.data() + first, static_cast<uint32_t>(count), S_, which, reps,
                                              work, st, &us);
        if (e == cudaErrorNotSupported) throw std::invalid_argument("the layers do not use the tensor-core path");
        guard(e, "kernel timing");
        kernel_launches_ += reps + 4;
        return us;
    }

    void forward_host(size_t layer, const float* x, float* out, uint32_t* ids, float* w) {
        ensure_ok();
        if (!x || !out) throw std::invalid_argument("input and output are required");
        DeviceScope scope(device_);
        float* dx = static_cast<float*>(io_);
        float* dy = reinterpret_cast<float*>(static_cast<uint8_t*>(io_) + align256(cfg_.hidden * 4));
        float* h_out = static_cast<float*>(pinned_);
        uint8_t* h_tail = static_cast<uint8_t*>(pinned_) + align256(cfg_.hidden * 4) * 2;
        float* h_in = reinterpret_cast<float*>(static_cast<uint8_t*>(pinned_) + align256(cfg_.hidden * 4));
        std::memcpy(h_in, x, cfg_.hidden * 4);
        guard(cudaMemcpyAsync(dx, h_in, cfg_.hidden * 4, cudaMemcpyHostToDevice, stream_), "h2d");
        forward(layer, dx, dy, nullptr, nullptr, stream_);
        guard(cudaMemcpyAsync(h_out, dy, cfg_.hidden * 4, cudaMemcpyDeviceToHost, stream_), "d2h");
        guard(cudaMemcpyAsync(h_tail, S_.ids, cfg_.top_k * 4, cudaMemcpyDeviceToHost, stream_), "d2h");
        guard(cudaMemcpyAsync(h_tail + 1024, S_.weights, cfg_.top_k * 4, cudaMemcpyDeviceToHost, stream_), "d2h");
        synchronize_host_call();
        std::memcpy(out, h_out, cfg_.hidden * 4);
        if (ids) std::memcpy(ids, h_tail, cfg_.top_k * 4);
        if (w) std::memcpy(w, h_tail + 1024, cfg_.top_k * 4);
    }

    void decode_layers(size_t first, size_t count, float* hidden, cudaStream_t s) {
        ensure_ok();
        refuse_sharded();
        if (count == 0 || first >= cfg_.layers || count > cfg_.layers - first)
            throw std::invalid_argument("layer range out of bounds");
        if (!hidden) throw std::invalid_argument("hidden state is required");
        for (size_t l = first; l < first + count; ++l)
            if (!resident_complete(l)) throw std::invalid_argument("layer weights were not uploaded");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        if (decode_grid_) {
            guard(launch_moe_decode(devs_dev_, devs_[first], static_cast<uint32_t>(first),
                                    static_cast<uint32_t>(count), S_, hidden, barrier_count_,
                                    decode_grid_, st), "decode kernel");
            barrier_count_ += static_cast<uint32_t>(count) * moe_barriers_per_layer() * decode_grid_;
            forward_calls_ += count;
            hits_ += count * cfg_.top_k;
            kernel_launches_ += 1;
            return;
        }
        if (chain35_ok_) {
            guard(launch_moe_chain35(chain35_plan_, devs_dev_, chain35_maps_, static_cast<uint32_t>(first),
                                     static_cast<uint32_t>(count), S_, C_, hidden, st),
                  "decode chain kernel");
            forward_calls_ += count;
            hits_ += count * cfg_.top_k;
            kernel_launches_ += 1;
            return;
        }
        if (chain_ok_) {
            guard(launch_moe_chain(chain_plan_, devs_dev_, static_cast<uint32_t>(first), static_cast<uint32_t>(count),
                                   S_, C_, hidden, st), "decode chain kernel");
            forward_calls_ += count;
            hits_ += count * cfg_.top_k;
            kernel_launches_ += 1;
            return;
        }
        // Inside the caller's stream capture (a decoder's token-step graph)
        // the blocks' kernels join that capture directly: a graph launch
        // cannot be captured.
        cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
        guard(cudaStreamIsCapturing(st, &capturing), "capture status");
        if (capturing == cudaStreamCaptureStatusActive) {
            uint32_t launches = 0;
            for (size_t l = first; l < first + count; ++l) {
                const MoeLayerDev* prev = l > first ? &devs_[l - 1] : nullptr;
                const MoeLayerDev* next = l + 1 < first + count ? &devs_[l + 1] : nullptr;
                uint32_t n = 0;
                guard(launch_moe_block(devs_[l], S_, nullptr, hidden, nullptr, prev, next, st, &n), "block launch");
                launches += n;
            }
            forward_calls_ += count;
            hits_ += count * cfg_.top_k;
            kernel_launches_ += launches;
            return;
        }
        const auto key = std::make_tuple(first, count, hidden);
        auto it = graphs_.find(key);
        if (it == graphs_.end()) {
            cudaGraph_t graph = nullptr;
            guard(cudaStreamBeginCapture(capture_stream_, cudaStreamCaptureModeThreadLocal), "capture");
            cudaError_t e = cudaSuccess;
            uint32_t launches = 0;
            for (size_t l = first; l < first + count && e == cudaSuccess; ++l) {
                const MoeLayerDev* prev = l > first ? &devs_[l - 1] : nullptr;
                const MoeLayerDev* next = l + 1 < first + count ? &devs_[l + 1] : nullptr;
                uint32_t n = 0;
                e = launch_moe_block(devs_[l], S_, nullptr, hidden, nullptr, prev, next, capture_stream_, &n);
                launches += n;
            }
            const cudaError_t end = cudaStreamEndCapture(capture_stream_, &graph);
            if (e != cudaSuccess) { if (graph) cudaGraphDestroy(graph); guard(e, "capture launch"); }
            guard(end, "end capture");
            cudaGraphExec_t exec = nullptr;
            const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            guard(inst, "instantiate");
            it = graphs_.emplace(key, std::make_pair(exec, launches)).first;
        }
        guard(cudaGraphLaunch(it->second.first, st), "graph launch");
        forward_calls_ += count;
        hits_ += count * cfg_.top_k;
        kernel_launches_ += it->second.second;
    }

    // Measurement: one decode_layers call through the chain kernel with its
    // per-phase stamps written to `stamps` (device, count * grid * 16 words).
    uint32_t trace_decode(size_t first, size_t count, float* hidden, unsigned long long* stamps, size_t capacity,
                          cudaStream_t s) {
        ensure_ok();
        if (!chain_ok_ && !chain35_ok_) throw std::invalid_argument("the layers do not run a persistent chain kernel");
        if (count == 0 || first >= cfg_.layers || count > cfg_.layers - first || !hidden || !stamps)
            throw std::invalid_argument("layer range, hidden state and stamp buffer are required");
        const uint32_t grid = chain_ok_ ? chain_plan_.grid : chain35_plan_.grid;
        if (capacity < count * grid * kChainTraceStamps)
            throw std::invalid_argument("stamp buffer too small (count x grid x 16 words)");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        if (chain_ok_)
            guard(launch_moe_chain(chain_plan_, devs_dev_, static_cast<uint32_t>(first), static_cast<uint32_t>(count),
                                   S_, C_, hidden, st, stamps), "decode chain kernel");
        else
            guard(launch_moe_chain35(chain35_plan_, devs_dev_, chain35_maps_, static_cast<uint32_t>(first),
                                     static_cast<uint32_t>(count), S_, C_, hidden, st, stamps), "decode chain kernel");
        kernel_launches_ += 1;
        return grid;
    }

    // A decoder's Gated DeltaNet layer and this MoE block in one chain launch.
    bool delta_layer_fits(const DeltaBlockShape& d) const {
        return chain35_ok_ && !failed_ && moe_chain35_delta_fits(chain35_plan_, d);
    }
    void decode_layer_delta(size_t layer, float* hidden, const DeltaBlockShape& d, const DeltaBlockTensors& t,
                            cudaStream_t s) {
        ensure_ok();
        if (!chain35_ok_) throw std::invalid_argument("the layers do not run the Qwen3.5-MoE chain kernel");
        if (layer >= cfg_.layers || !hidden) throw std::invalid_argument("layer and hidden state are required");
        if (!resident_complete(layer)) throw std::invalid_argument("layer weights were not uploaded");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        guard(launch_moe_chain35(chain35_plan_, devs_dev_, chain35_maps_, static_cast<uint32_t>(layer), 1u, S_, C_,
                                 hidden, st, nullptr, &d, &t),
              "decode chain kernel");
        forward_calls_ += 1;
        hits_ += cfg_.top_k;
        kernel_launches_ += 1;
    }

    bool attention_layer_fits(const void* args, size_t bytes) const {
        return chain35_ok_ && !failed_ && moe_chain35_attention_fits(chain35_plan_, args, bytes);
    }
    void decode_layer_attention(size_t layer, float* hidden, const void* args, size_t bytes, cudaStream_t s) {
        ensure_ok();
        if (!chain35_ok_) throw std::invalid_argument("the layers do not run the Qwen3.5-MoE chain kernel");
        if (layer >= cfg_.layers || !hidden) throw std::invalid_argument("layer and hidden state are required");
        if (!resident_complete(layer)) throw std::invalid_argument("layer weights were not uploaded");
        DeviceScope scope(device_);
        cudaStream_t st = s ? s : stream_;
        guard(launch_moe_chain35(chain35_plan_, devs_dev_, chain35_maps_, static_cast<uint32_t>(layer), 1u, S_, C_,
                                 hidden, st, nullptr, nullptr, nullptr, args, bytes),
              "decode chain kernel");
        forward_calls_ += 1;
        hits_ += cfg_.top_k;
        kernel_launches_ += 1;
    }

    // A decoder's layer loop: its attention blocks and these MoE blocks in
    // one chain launch (false when the layers do not take the chain kernel or
    // the attention phase does not fit it).
    bool attention_chain_fits(const ChainAttnDesc& att) const {
        return chain_ok_ && !failed_ && chain_attention_smem(chain_plan_, att) <=
                                             chain_plan_.smem - chain_tile_offset(chain_plan_);
    }
    void decode_layers_attention(size_t first, size_t count, float* hidden, const ChainAttnDesc& att,
                                 cudaStream_t s) {
        ensure_ok();
        if (!chain_ok_) throw std::invalid_argument("the layers do not run the persistent chain kernel");
        if (count == 0 || first >= cfg_.layers || count > cfg_.layers - first || !hidden)
            throw std::invalid_argument("layer range and hidden state are required");
        for (size_t l = first; l < first + count; ++l)
            if (!resident_complete(l)) throw std::invalid_argument("layer weights were not uploaded");
        DeviceScope scope(device_);
        guard(launch_moe_chain(chain_plan_, devs_dev_, static_cast<uint32_t>(first), static_cast<uint32_t>(count), S_,
                               C_, hidden, s ? s : stream_, nullptr, &att), "decode chain kernel with attention");
        forward_calls_ += count;
        hits_ += count * cfg_.top_k;
        kernel_launches_ += 1;
    }

    void decode_layers_host(size_t first, size_t count, const float* in, float* out) {
        ensure_ok();
        if (!in || !out) throw std::invalid_argument("hidden buffers are required");
        DeviceScope scope(device_);
        float* dh = static_cast<float*>(io_);
        float* h_out = static_cast<float*>(pinned_);
        // The input through pinned memory: an asynchronous copy instead of a
        // staged pageable one.
        float* h_in = reinterpret_cast<float*>(static_cast<uint8_t*>(pinned_) + align256(cfg_.hidden * 4));
        std::memcpy(h_in, in, cfg_.hidden * 4);
        guard(cudaMemcpyAsync(dh, h_in, cfg_.hidden * 4, cudaMemcpyHostToDevice, stream_), "h2d");
        decode_layers(first, count, dh, stream_);
        guard(cudaMemcpyAsync(h_out, dh, cfg_.hidden * 4, cudaMemcpyDeviceToHost, stream_), "d2h");
        synchronize_host_call();
        std::memcpy(out, h_out, cfg_.hidden * 4);
    }

    void synchronize(cudaStream_t s) {
        ensure_ok();
        DeviceScope scope(device_);
        guard(cudaStreamSynchronize(s ? s : stream_), "synchronize");
        uint32_t status = 0;
        guard(cudaMemcpy(&status, S_.status, 4, cudaMemcpyDeviceToHost), "status");
        raise_status(status);
    }

    // The host-buffer entries: the status word rides the same stream as the
    // results, into pinned memory, so a call waits on its stream once.
    void synchronize_host_call() {
        uint32_t* h_status = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(pinned_) +
                                                         align256(cfg_.hidden * 4) * 2 + 2048);
        guard(cudaMemcpyAsync(h_status, S_.status, 4, cudaMemcpyDeviceToHost, stream_), "status");
        guard(cudaStreamSynchronize(stream_), "synchronize");
        raise_status(*h_status);
    }

    void raise_status(uint32_t status) {
        if (status & kStatusWaitTimeout) {
            // A grid barrier gave up: the launch was abandoned and the barrier
            // counter no longer matches the host's count.  Sticky, like a CUDA error.
            failed_ = true;
            failure_ = "a kernel abandoned its work after a bounded device-side wait timed out";
            throw std::runtime_error(failure_);
        }
        if (status) {
            guard(cudaMemset(S_.status, 0, 4), "status reset");
            if (status & kStatusNonFiniteLogits)
                throw RouterFailure("expert router produced non-finite logits");
            throw RouterFailure("expert router softmax is invalid");
        }
    }

    pokit_cuda_moe_stats stats() const {
        pokit_cuda_moe_stats s{};
        s.capacity_bytes = pool_bytes_;
        s.resident_bytes = resident_bytes_;
        s.bytes_read = bytes_read_;
        s.read_operations = read_operations_;
        s.read_time_ns = read_time_ns_;
        s.hits = hits_;
        s.misses = 0;
        s.forward_calls = forward_calls_;
        s.kernel_launches = kernel_launches_;
        return s;
    }

    // Expert-parallel exchange over peer memory: this rank's region (partial
    // outputs of every rank, flags), exported for the other processes.
    void exchange_create(size_t world, size_t rank, size_t max_tokens, void* handle_out) {
        ensure_ok();
        if (ex_region_) throw std::invalid_argument("the exchange is already created");
        if (world < 1 || world > kMaxExchangeRanks || rank >= world || max_tokens == 0 || max_tokens > kMaxBatchTokens ||
            !handle_out)
            throw std::invalid_argument("exchange needs 1..8 ranks, rank < world, 1..65536 tokens and a handle buffer");
        DeviceScope scope(device_);
        const uint64_t bytes = ep_exchange_bytes(static_cast<uint32_t>(world), static_cast<uint32_t>(max_tokens),
                                                 static_cast<uint32_t>(cfg_.hidden));
        guard(cudaMalloc(&ex_region_, bytes), "cudaMalloc(exchange)");
        guard(cudaMemset(ex_region_, 0, bytes), "exchange");
        guard(cudaMalloc(reinterpret_cast<void**>(&ex_words_), 256), "cudaMalloc(exchange counters)");
        guard(cudaMemset(ex_words_, 0, 256), "exchange");
        cudaIpcMemHandle_t h{};
        guard(cudaIpcGetMemHandle(&h, ex_region_), "cudaIpcGetMemHandle");
        static_assert(sizeof(h) == POKIT_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
        std::memcpy(handle_out, &h, sizeof(h));
        ex_ = EpExchange{};
        ex_.world = static_cast<uint32_t>(world);
        ex_.rank = static_cast<uint32_t>(rank);
        ex_.max_tokens = static_cast<uint32_t>(max_tokens);
        ex_.hidden = static_cast<uint32_t>(cfg_.hidden);
        ex_.epoch = ex_words_;
        ex_.arrive = ex_words_ + 32;
    }

    // Maps the other ranks' regions (handles in rank order) and routes the
    // batched forward through the exchange.
    void exchange_connect(const void* handles) {
        ensure_ok();
        if (!ex_region_) throw std::invalid_argument("create the exchange first");
        if (ex_connected_) throw std::invalid_argument("the exchange is already connected");
        if (!handles) throw std::invalid_argument("the ranks' IPC handles are required");
        DeviceScope scope(device_);
        guard(cudaDeviceSynchronize(), "exchange");
        for (uint32_t r = 0; r < ex_.world; ++r) {
            if (r == ex_.rank) {
                ex_.peers[r] = static_cast<uint8_t*>(ex_region_);
                continue;
            }
            cudaIpcMemHandle_t h{};
            std::memcpy(&h, static_cast<const uint8_t*>(handles) + r * sizeof(h), sizeof(h));
            void* p = nullptr;
            guard(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
            ex_opened_.push_back(p);
            ex_.peers[r] = static_cast<uint8_t*>(p);
        }
        ex_connected_ = true;
    }

    // Unmaps the other ranks' regions (after this rank's work on them is done)
    // and returns forward_batch to the local combine.  Every rank disconnects
    // before any rank destroys its handle: an exported region must not be
    // freed while another process still maps it.  Works on a failed handle.
    void exchange_disconnect() {
        DeviceScope scope(device_);
        cudaStreamSynchronize(stream_);
        for (void* p : ex_opened_) cudaIpcCloseMemHandle(p);
        ex_opened_.clear();
        for (auto& p : ex_.peers) p = nullptr;
        ex_connected_ = false;
    }

private:
    static constexpr size_t kMaxBatchTokens = 65536;

    void ensure_batch_scratch(const MoeLayerDev& L, uint32_t tokens) {
        if (batch_scratch_ && tokens <= B_.max_tokens) return;
        uint32_t cap = std::max<uint32_t>(tokens, 64u);
        if (batch_scratch_) {
            guard(cudaStreamSynchronize(stream_), "batch scratch");
            cudaFree(batch_scratch_);
            batch_scratch_ = nullptr;
        }
        guard(cudaMalloc(&batch_scratch_, moe_batch_scratch_bytes(L, cap)), "cudaMalloc(batch scratch)");
        B_ = moe_batch_scratch_carve(L, cap, batch_scratch_);
    }

    void ensure_batch_io(size_t bytes) {
        if (bytes <= batch_io_bytes_) return;
        if (batch_io_) cudaFree(batch_io_);
        if (batch_pinned_) cudaFreeHost(batch_pinned_);
        batch_io_ = nullptr;
        batch_pinned_ = nullptr;
        batch_io_bytes_ = 0;
        guard(cudaMalloc(&batch_io_, bytes), "cudaMalloc(batch io)");
        guard(cudaMallocHost(&batch_pinned_, bytes), "cudaMallocHost(batch io)");
        batch_io_bytes_ = bytes;
    }

    MoeLayerDev make_layer_dev(size_t l) const {
        MoeLayerDev L;
        L.hidden = static_cast<uint32_t>(cfg_.hidden);
        L.inter = static_cast<uint32_t>(cfg_.inter);
        L.experts = static_cast<uint32_t>(cfg_.experts);
        L.expert_first = static_cast<uint32_t>(expert_first_);
        L.expert_local = static_cast<uint32_t>(expert_local_);
        L.top_k = static_cast<uint32_t>(cfg_.top_k);
        L.flavour = cfg_.flavour;
        L.normalize = cfg_.normalize_top_k ? 1u : 0u;
        L.expert_weights_scale = cfg_.flavour == POKIT_CUDA_MOE_QWEN35 ? cfg_.expert_weights_scale : 1.0f;
        L.rms_eps = cfg_.rms_epsilon > 0.0f ? cfg_.rms_epsilon : 1e-6f;
        L.router = reinterpret_cast<const float*>(tensor_ptr(l, POKIT_CUDA_MOE_ROUTER));
        L.gate_type = cfg_.gate_type;
        L.up_type = cfg_.up_type;
        L.down_type = layer_down_[l];
        L.gate = tensor_ptr(l, POKIT_CUDA_MOE_GATE);
        L.up = tensor_ptr(l, POKIT_CUDA_MOE_UP);
        L.down = tensor_ptr(l, POKIT_CUDA_MOE_DOWN);
        L.gate_slice = tensor_bytes(l, POKIT_CUDA_MOE_GATE) / expert_local_;
        L.up_slice = tensor_bytes(l, POKIT_CUDA_MOE_UP) / expert_local_;
        L.down_slice = tensor_bytes(l, POKIT_CUDA_MOE_DOWN) / expert_local_;
        L.ffn_norm = reinterpret_cast<const float*>(tensor_ptr(l, POKIT_CUDA_MOE_FFN_NORM));
        if (cfg_.shared_inter) {
            L.shared_inter = static_cast<uint32_t>(cfg_.shared_inter);
            L.shared_router = reinterpret_cast<const float*>(tensor_ptr(l, POKIT_CUDA_MOE_SHARED_ROUTER));
            L.shared_gate_type = cfg_.shared_gate_type;
            L.shared_up_type = cfg_.shared_up_type;
            L.shared_down_type = cfg_.shared_down_type;
            L.shared_gate = tensor_ptr(l, POKIT_CUDA_MOE_SHARED_GATE);
            L.shared_up = tensor_ptr(l, POKIT_CUDA_MOE_SHARED_UP);
            L.shared_down = tensor_ptr(l, POKIT_CUDA_MOE_SHARED_DOWN);
        }
        return L;
    }

    void mark_resident(size_t layer, uint32_t t) {
        if (!(resident_[layer] & (1u << t))) {
            resident_[layer] |= 1u << t;
            resident_bytes_ += tensor_bytes(layer, t);
        }
    }

    // Every tensor this configuration defines for `layer` has been written.
    bool resident_complete(size_t layer) const {
        uint32_t need = 0;
        for (uint32_t t = 0; t < 9; ++t)
            if (tensor_bytes(layer, t)) need |= 1u << t;
        return (resident_[layer] & need) == need;
    }

    bool sharded() const { return expert_local_ != cfg_.experts; }
    void refuse_sharded() const {
        if (sharded())
            throw std::invalid_argument("an expert-shard handle serves pokit_cuda_moe_forward_batch (grouped path) only");
    }

    void ensure_ok() const {
        if (failed_) throw std::runtime_error("CUDA MoE backend failed earlier: " + failure_);
    }

    void guard(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return;
        if (e == cudaErrorInvalidValue)
            throw std::invalid_argument(std::string(what) + ": unsupported shape or argument");
        failed_ = true;
        failure_ = std::string(what) + ": " + cudaGetErrorString(e);
        throw std::runtime_error(failure_);
    }

    pokit_cuda_moe_config cfg_;
    int device_ = 0;
    size_t expert_first_ = 0, expert_local_ = 0;   // experts this handle holds
    std::vector<uint32_t> layer_down_;
    std::vector<std::array<uint64_t, 9>> offsets_;
    uint8_t* pool_ = nullptr;
    uint64_t pool_bytes_ = 0;
    std::vector<MoeLayerDev> devs_;
    void* scratch_ = nullptr;
    MoeLayerDev* devs_dev_ = nullptr;
    uint32_t decode_grid_ = 0;
    uint32_t barrier_count_ = 0;
    bool chain_ok_ = false;              // decode_layers runs moe_chain_kernel
    ChainPlan chain_plan_{};
    bool chain35_ok_ = false;            // decode_layers runs moe_chain35_kernel (Qwen3.5-MoE blocks)
    Chain35Plan chain35_plan_{};
    Chain35Maps* chain35_maps_ = nullptr;   // device table of the chain's per-layer tensor maps
    void* chain_scratch_ = nullptr;
    ChainScratch C_;
    uint64_t scratch_bytes_ = 0;
    MoeScratch S_;
    void* batch_scratch_ = nullptr;   // grouped-path scratch, grown on demand
    MoeBatchScratch B_;
    void* ex_region_ = nullptr;          // this rank's exchange region (exported)
    uint32_t* ex_words_ = nullptr;       // call number and arrival counter of the exchange kernel
    std::vector<void*> ex_opened_;       // the other ranks' regions, mapped here
    EpExchange ex_{};
    bool ex_connected_ = false;
    void* batch_io_ = nullptr;        // host-span batch staging (device, pinned host)
    void* batch_pinned_ = nullptr;
    size_t batch_io_bytes_ = 0;
    void* io_ = nullptr;
    void* pinned_ = nullptr;
    cudaStream_t stream_ = nullptr;
    cudaStream_t capture_stream_ = nullptr;
    // (first, count, hidden) -> (graph, kernels it launches)
    std::map<std::tuple<size_t, size_t, float*>, std::pair<cudaGraphExec_t, uint32_t>> graphs_;
    std::vector<uint32_t> resident_;   // per layer: bit t = tensor t written
    std::mutex mutex_;
    bool failed_ = false;
    std::string failure_;
    uint64_t resident_bytes_ = 0, bytes_read_ = 0, read_operations_ = 0, read_time_ns_ = 0;
    mutable uint64_t hits_ = 0;
    uint64_t forward_calls_ = 0, kernel_launches_ = 0;
};

// ---------------------------------------------------------------------------
class LinearBackend {
public:
    explicit LinearBackend(int device) : device_(device) {
        int count = 0;
        check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (device < 0 || device >= count) throw std::invalid_argument("CUDA device out of range");
        DeviceScope scope(device_);
        check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaEventCreate(&start_), "cudaEventCreate");
        check(cudaEventCreate(&stop_), "cudaEventCreate");
    }
    ~LinearBackend() {
        for (auto& kv : cache_) cudaFree(kv.second.dev);
        if (stage_) cudaFree(stage_);
        if (io_) cudaFree(io_);
        if (start_) cudaEventDestroy(start_);
        if (stop_) cudaEventDestroy(stop_);
        if (stream_) cudaStreamDestroy(stream_);
    }
    LinearBackend(const LinearBackend&) = delete;
    LinearBackend& operator=(const LinearBackend&) = delete;

    // key == nullptr: the payload is streamed to the device on every call
    // (the Vulkan backend does the same for readers without a model file,
    // vulkan_linear.cpp:516-563, 705-714); a host address says nothing about
    // the bytes behind it once the caller frees and reuses the buffer.
    // key != nullptr: the caller names the matrix by a stable identity (the
    // tensor's GGUF file offset, say) and its payload stays in HBM under that
    // key, least recently used entries evicted beyond the cache capacity.
    bool try_linear(uint32_t type, const void* w, size_t w_bytes, size_t rows, size_t cols,
                    const float* x, float* y, const uint64_t* key) {
        std::lock_guard<std::mutex> lock(mutex_);
        if (failed_) throw std::runtime_error("CUDA linear backend failed earlier: " + failure_);
        if (!type_supported(type)) return false;
        if (!x || !y || rows == 0 || cols == 0 || cols % block_elems(type) || rows > UINT32_MAX ||
            cols > UINT32_MAX)
            throw std::invalid_argument("GGUF matrix dimensions do not match linear input/output");
        if (w_bytes != rows * row_bytes(type, cols))
            throw std::invalid_argument("weight byte size does not match dimensions");
        if (!w && !(key && cache_.count(*key)))
            throw std::invalid_argument("weights are required (the key holds no cached payload)");
        DeviceScope scope(device_);
        ++stats_.linear_calls;
        const void* dw = key ? cached_weights(*key, type, w, w_bytes, rows, cols) : streamed_weights(w, w_bytes);
        const size_t need = align256(cols * 4) + align256(rows * 4);
        if (need > io_bytes_) {
            if (io_) cudaFree(io_);
            io_ = nullptr;
            io_bytes_ = 0;
            guard(cudaMalloc(&io_, need), "cudaMalloc(io)");
            io_bytes_ = need;
        }
        float* dx = static_cast<float*>(io_);
        float* dy = reinterpret_cast<float*>(static_cast<uint8_t*>(io_) + align256(cols * 4));
        guard(cudaMemcpyAsync(dx, x, cols * 4, cudaMemcpyHostToDevice, stream_), "h2d");
        guard(cudaEventRecord(start_, stream_), "event");
        guard(launch_linear(type, dw, static_cast<uint32_t>(rows), static_cast<uint32_t>(cols), dx,
                            dy, stream_), "linear");
        guard(cudaEventRecord(stop_, stream_), "event");
        guard(cudaMemcpyAsync(y, dy, rows * 4, cudaMemcpyDeviceToHost, stream_), "d2h");
        guard(cudaStreamSynchronize(stream_), "synchronize");
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, start_, stop_);
        stats_.gpu_time_ns += static_cast<uint64_t>(ms * 1.0e6f);
        stats_.weight_bytes += w_bytes;
        ++stats_.dispatches;
        switch (type) {
            case kQ4_K: ++stats_.q4_k_dispatches; break;
            case kQ5_K: ++stats_.q5_k_dispatches; break;
            case kQ6_K: ++stats_.q6_k_dispatches; break;
            case kQ8_0: ++stats_.q8_0_dispatches; break;
            default: ++stats_.other_dispatches; break;
        }
        return true;
    }

    void set_cache_capacity(uint64_t bytes) {
        std::lock_guard<std::mutex> lock(mutex_);
        DeviceScope scope(device_);
        capacity_ = bytes;
        evict_to(capacity_);
    }

    bool is_cached(uint64_t key) const {
        std::lock_guard<std::mutex> lock(mutex_);
        return cache_.count(key) != 0;
    }

    bool forget(uint64_t key) {
        std::lock_guard<std::mutex> lock(mutex_);
        DeviceScope scope(device_);
        const auto it = cache_.find(key);
        if (it == cache_.end()) return false;
        drop(it);
        return true;
    }

    pokit_cuda_linear_stats stats() const {
        std::lock_guard<std::mutex> lock(mutex_);
        return stats_;
    }

private:
    struct Entry {
        void* dev = nullptr;
        uint32_t type = 0;
        size_t bytes = 0, rows = 0, cols = 0;
        std::list<uint64_t>::iterator lru;
    };

    void guard(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return;
        if (e == cudaErrorInvalidValue)
            throw std::invalid_argument(std::string(what) + ": unsupported shape or argument");
        failed_ = true;
        failure_ = std::string(what) + ": " + cudaGetErrorString(e);
        throw std::runtime_error(failure_);
    }

    // One reusable device buffer, refilled from the host payload every call.
    const void* streamed_weights(const void* w, size_t bytes) {
        if (bytes > stage_bytes_) {
            if (stage_) cudaFree(stage_);
            stage_ = nullptr;
            stage_bytes_ = 0;
            guard(cudaMalloc(&stage_, bytes), "cudaMalloc(weight staging)");
            stage_bytes_ = bytes;
        }
        guard(cudaMemcpyAsync(stage_, w, bytes, cudaMemcpyHostToDevice, stream_), "weights h2d");
        return stage_;
    }

    const void* cached_weights(uint64_t key, uint32_t type, const void* w, size_t bytes, size_t rows,
                               size_t cols) {
        auto it = cache_.find(key);
        if (it != cache_.end()) {
            const Entry& e = it->second;
            if (e.type != type || e.bytes != bytes || e.rows != rows || e.cols != cols)
                throw std::invalid_argument("weight key was cached for a matrix of another type or shape");
            lru_.splice(lru_.begin(), lru_, e.lru);
            return e.dev;
        }
        if (bytes > capacity_) return streamed_weights(w, bytes);     // never fits: stream it
        evict_to(capacity_ - bytes);
        const uint64_t t0 = now_ns();
        Entry e;
        e.type = type;
        e.bytes = bytes;
        e.rows = rows;
        e.cols = cols;
        guard(cudaMalloc(&e.dev, bytes), "cudaMalloc(weights)");
        const cudaError_t ce = cudaMemcpy(e.dev, w, bytes, cudaMemcpyHostToDevice);
        if (ce != cudaSuccess) cudaFree(e.dev);
        guard(ce, "upload");
        lru_.push_front(key);
        e.lru = lru_.begin();
        cache_.emplace(key, e);
        resident_ += bytes;
        stats_.model_cache_capacity_bytes = resident_;
        stats_.model_cache_uploaded_bytes += bytes;
        stats_.model_cache_upload_time_ns += now_ns() - t0;
        return e.dev;
    }

    void drop(std::map<uint64_t, Entry>::iterator it) {
        cudaFree(it->second.dev);
        resident_ -= it->second.bytes;
        lru_.erase(it->second.lru);
        cache_.erase(it);
        stats_.model_cache_capacity_bytes = resident_;
    }

    void evict_to(uint64_t limit) {
        while (resident_ > limit && !lru_.empty()) drop(cache_.find(lru_.back()));
    }

    int device_;
    cudaStream_t stream_ = nullptr;
    cudaEvent_t start_ = nullptr, stop_ = nullptr;
    std::map<uint64_t, Entry> cache_;
    std::list<uint64_t> lru_;                       // most recently used first
    uint64_t resident_ = 0;
    uint64_t capacity_ = uint64_t(16) << 30;        // bytes of cached payloads
    void* stage_ = nullptr;
    size_t stage_bytes_ = 0;
    void* io_ = nullptr;
    size_t io_bytes_ = 0;
    mutable std::mutex mutex_;
    bool failed_ = false;
    std::string failure_;
    pokit_cuda_linear_stats stats_{};
};

}  // namespace pokit

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
struct pokit_cuda_moe {
    explicit pokit_cuda_moe(const pokit_cuda_moe_config& c) : impl(c) {}
    pokit::MoeBackend impl;
};

namespace pokit {

bool moe_attention_layer_fits(const pokit_cuda_moe* moe, const void* args, size_t bytes) {
    return moe && moe->impl.attention_layer_fits(args, bytes);
}

cudaError_t moe_decode_layer_attention(pokit_cuda_moe* moe, size_t layer, float* hidden, const void* args,
                                       size_t bytes, cudaStream_t stream, std::string* error) {
    if (!moe) return cudaErrorInvalidValue;
    try {
        moe->impl.decode_layer_attention(layer, hidden, args, bytes, stream);
        return cudaSuccess;
    } catch (const std::invalid_argument& e) {
        if (error) *error = e.what();
        return cudaErrorInvalidValue;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return cudaErrorUnknown;
    }
}

bool moe_delta_layer_fits(const pokit_cuda_moe* moe, const DeltaBlockShape& d) {
    return moe && moe->impl.delta_layer_fits(d);
}

cudaError_t moe_decode_layer_delta(pokit_cuda_moe* moe, size_t layer, float* hidden, const DeltaBlockShape& d,
                                   const DeltaBlockTensors& t, cudaStream_t stream, std::string* error) {
    if (!moe) return cudaErrorInvalidValue;
    try {
        moe->impl.decode_layer_delta(layer, hidden, d, t, stream);
        return cudaSuccess;
    } catch (const std::invalid_argument& e) {
        if (error) *error = e.what();
        return cudaErrorInvalidValue;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return cudaErrorUnknown;
    }
}

bool moe_attention_chain_fits(const pokit_cuda_moe* moe, const ChainAttnDesc& att) {
    return moe && moe->impl.attention_chain_fits(att);
}

cudaError_t moe_decode_layers_attention(pokit_cuda_moe* moe, size_t first, size_t count, float* hidden,
                                        const ChainAttnDesc& att, cudaStream_t stream, std::string* error) {
    if (!moe) return cudaErrorInvalidValue;
    try {
        moe->impl.decode_layers_attention(first, count, hidden, att, stream);
        return cudaSuccess;
    } catch (const std::invalid_argument& e) {
        if (error) *error = e.what();
        return cudaErrorInvalidValue;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return cudaErrorUnknown;
    }
}

}  // namespace pokit

struct pokit_cuda_linear_backend {
    explicit pokit_cuda_linear_backend(int device) : impl(device) {}
    pokit::LinearBackend impl;
};

namespace {

void set_error(char* destination, size_t capacity, const char* message) noexcept {
    if (!destination || capacity == 0) return;
    const size_t n = std::min(capacity - 1, std::strlen(message));
    std::memcpy(destination, message, n);
    destination[n] = '\0';
}

template <typename F>
pokit_cuda_status guarded(char* err, size_t cap, F&& body) noexcept {
    try {
        body();
        set_error(err, cap, "");
        return POKIT_CUDA_STATUS_OK;
    } catch (const std::invalid_argument& e) {
        set_error(err, cap, e.what());
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        set_error(err, cap, e.what());
        return POKIT_CUDA_STATUS_RUNTIME_ERROR;
    } catch (...) {
        set_error(err, cap, "unknown CUDA backend failure");
        return POKIT_CUDA_STATUS_INTERNAL_ERROR;
    }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

const char* pokit_cuda_version(void) { return "0.1.0"; }

pokit_cuda_status pokit_cuda_linear(uint32_t ggml_type, const void* weights, size_t rows,
                                    size_t cols, const float* input, float* output, void* stream,
                                    char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!pokit::type_supported(ggml_type)) throw std::invalid_argument("unsupported GGML type");
        if (!weights || !input || !output || rows == 0 || cols == 0 ||
            cols % pokit::block_elems(ggml_type) || rows > UINT32_MAX || cols > UINT32_MAX)
            throw std::invalid_argument("invalid linear dimensions");
        pokit::check(pokit::launch_linear(ggml_type, weights, static_cast<uint32_t>(rows),
                                          static_cast<uint32_t>(cols), input, output,
                                          as_stream(stream)), "linear");
    });
}

pokit_cuda_status pokit_cuda_dequantize_rows(uint32_t ggml_type, const void* encoded, size_t rows,
                                             size_t cols, float* output, void* stream,
                                             char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!pokit::type_supported(ggml_type)) throw std::invalid_argument("unsupported GGML type");
        if (!encoded || !output || rows == 0 || cols == 0 || cols % pokit::block_elems(ggml_type) ||
            cols % 32 || rows > UINT32_MAX || cols > UINT32_MAX)
            throw std::invalid_argument("invalid row dimensions");
        pokit::check(pokit::launch_dequantize(ggml_type, encoded, static_cast<uint32_t>(rows),
                                              static_cast<uint32_t>(cols), output, as_stream(stream)),
                     "dequantize");
    });
}

pokit_cuda_status pokit_cuda_route_experts(const float* logits, size_t n, size_t top_k,
                                           uint32_t flavour, int normalize,
                                           float expert_weights_scale, uint32_t* ids_out,
                                           float* weights_out, uint32_t* status_out, void* stream,
                                           char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!logits || !ids_out || !weights_out || n == 0 || n > 1024 || top_k == 0 ||
            top_k > n || top_k > 64 || flavour > 1)
            throw std::invalid_argument("invalid expert top-k");
        pokit::check(pokit::launch_route_experts(logits, static_cast<uint32_t>(n),
                                                 static_cast<uint32_t>(top_k), flavour,
                                                 normalize ? 1u : 0u, expert_weights_scale, ids_out,
                                                 weights_out, status_out, as_stream(stream)),
                     "route");
    });
}

pokit_cuda_status pokit_cuda_synthesize_blocks(uint32_t ggml_type, uint64_t seed, uint64_t stream_id,
                                               size_t nblocks, void* dst, void* stream,
                                               char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!dst || !pokit::quant_supported(ggml_type))
            throw std::invalid_argument("synthesis needs a quantised type and a destination");
        pokit::check(pokit::launch_synth_blocks(ggml_type, seed, stream_id, nblocks, dst,
                                                as_stream(stream)), "synthesize");
    });
}

pokit_cuda_status pokit_cuda_linear_backend_create(int device, pokit_cuda_linear_backend** out,
                                                   char* error_buffer, size_t error_capacity) {
    if (out) *out = nullptr;
    return guarded(error_buffer, error_capacity, [&] {
        if (!out) throw std::invalid_argument("output handle is required");
        *out = new pokit_cuda_linear_backend(device);
    });
}

void pokit_cuda_linear_backend_destroy(pokit_cuda_linear_backend* backend) { delete backend; }

pokit_cuda_status pokit_cuda_linear_backend_try_linear(
    pokit_cuda_linear_backend* backend, uint32_t ggml_type, const void* weights_host,
    size_t weights_bytes, size_t rows, size_t cols, const float* input_host, float* output_host,
    int* handled, char* error_buffer, size_t error_capacity) {
    if (handled) *handled = 0;
    return guarded(error_buffer, error_capacity, [&] {
        if (!backend || !handled) throw std::invalid_argument("backend and handled flag are required");
        *handled = backend->impl.try_linear(ggml_type, weights_host, weights_bytes, rows, cols,
                                            input_host, output_host, nullptr) ? 1 : 0;
    });
}

pokit_cuda_status pokit_cuda_linear_backend_try_linear_cached(
    pokit_cuda_linear_backend* backend, uint64_t weights_key, uint32_t ggml_type, const void* weights_host,
    size_t weights_bytes, size_t rows, size_t cols, const float* input_host, float* output_host,
    int* handled, char* error_buffer, size_t error_capacity) {
    if (handled) *handled = 0;
    return guarded(error_buffer, error_capacity, [&] {
        if (!backend || !handled) throw std::invalid_argument("backend and handled flag are required");
        *handled = backend->impl.try_linear(ggml_type, weights_host, weights_bytes, rows, cols,
                                            input_host, output_host, &weights_key) ? 1 : 0;
    });
}

int pokit_cuda_linear_backend_is_cached(const pokit_cuda_linear_backend* backend, uint64_t weights_key) {
    if (!backend) return 0;
    try {
        return backend->impl.is_cached(weights_key) ? 1 : 0;
    } catch (...) {
        return 0;
    }
}

pokit_cuda_status pokit_cuda_linear_backend_set_cache_capacity(pokit_cuda_linear_backend* backend,
                                                               uint64_t capacity_bytes, char* error_buffer,
                                                               size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!backend) throw std::invalid_argument("backend is required");
        backend->impl.set_cache_capacity(capacity_bytes);
    });
}

pokit_cuda_status pokit_cuda_linear_backend_forget(pokit_cuda_linear_backend* backend, uint64_t weights_key,
                                                   int* was_cached, char* error_buffer, size_t error_capacity) {
    if (was_cached) *was_cached = 0;
    return guarded(error_buffer, error_capacity, [&] {
        if (!backend) throw std::invalid_argument("backend is required");
        const bool hit = backend->impl.forget(weights_key);
        if (was_cached) *was_cached = hit ? 1 : 0;
    });
}

pokit_cuda_status pokit_cuda_linear_backend_get_stats(const pokit_cuda_linear_backend* backend,
                                                      pokit_cuda_linear_stats* out_stats) {
    if (!backend || !out_stats) return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    try {
        *out_stats = backend->impl.stats();
        return POKIT_CUDA_STATUS_OK;
    } catch (...) {
        return POKIT_CUDA_STATUS_INTERNAL_ERROR;
    }
}

pokit_cuda_status pokit_cuda_moe_create(const pokit_cuda_moe_config* config, pokit_cuda_moe** out_moe,
                                        char* error_buffer, size_t error_capacity) {
    if (out_moe) *out_moe = nullptr;
    return guarded(error_buffer, error_capacity, [&] {
        if (!config || !out_moe) throw std::invalid_argument("configuration and output handle are required");
        *out_moe = new pokit_cuda_moe(*config);
    });
}

void pokit_cuda_moe_destroy(pokit_cuda_moe* moe) { delete moe; }

pokit_cuda_status pokit_cuda_moe_upload_tensor(pokit_cuda_moe* moe, size_t layer, uint32_t tensor,
                                               const void* host_bytes, size_t bytes,
                                               char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.upload_tensor(layer, tensor, host_bytes, bytes);
    });
}

pokit_cuda_status pokit_cuda_moe_upload_layer(pokit_cuda_moe* moe, size_t layer,
                                              const pokit_cuda_moe_layer_host* t,
                                              char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe || !t) throw std::invalid_argument("MoE handle and tensors are required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        const void* ptrs[9] = {t->router, t->gate, t->up, t->down, t->ffn_norm,
                               t->shared_router, t->shared_gate, t->shared_up, t->shared_down};
        for (uint32_t i = 0; i < 9; ++i) {
            if (!ptrs[i]) continue;
            moe->impl.upload_tensor(layer, i, ptrs[i], moe->impl.tensor_bytes(layer, i));
        }
    });
}

pokit_cuda_status pokit_cuda_moe_synthesize_tensor(pokit_cuda_moe* moe, size_t layer, uint32_t tensor,
                                                   uint64_t seed, uint64_t stream_id,
                                                   char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.synthesize_tensor(layer, tensor, seed, stream_id);
    });
}

pokit_cuda_status pokit_cuda_moe_expert_view(const pokit_cuda_moe* moe, size_t layer, uint32_t matrix,
                                             size_t expert, const void** device_ptr, size_t* bytes) {
    if (!moe || !device_ptr || !bytes) return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    try {
        moe->impl.expert_view(layer, matrix, expert, device_ptr, bytes);
        return POKIT_CUDA_STATUS_OK;
    } catch (const std::invalid_argument&) {
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    } catch (...) {
        return POKIT_CUDA_STATUS_INTERNAL_ERROR;
    }
}

pokit_cuda_status pokit_cuda_moe_forward(pokit_cuda_moe* moe, size_t layer, const float* input,
                                         float* output, uint32_t* route_ids, float* route_weights,
                                         void* stream, char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.forward(layer, input, output, route_ids, route_weights, as_stream(stream));
    });
}

pokit_cuda_status pokit_cuda_moe_forward_batch(pokit_cuda_moe* moe, size_t layer, const void* input,
                                               uint32_t input_type, size_t tokens, const float* router_logits,
                                               float* output, uint32_t* route_ids, float* route_weights,
                                               void* stream, char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.forward_batch(layer, input, input_type, tokens, router_logits, output, route_ids, route_weights,
                                as_stream(stream));
    });
}

pokit_cuda_status pokit_cuda_moe_exchange_create(pokit_cuda_moe* moe, size_t world, size_t rank, size_t max_tokens,
                                                 void* ipc_handle_out, char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.exchange_create(world, rank, max_tokens, ipc_handle_out);
    });
}

pokit_cuda_status pokit_cuda_moe_exchange_connect(pokit_cuda_moe* moe, const void* ipc_handles, char* error_buffer,
                                                  size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.exchange_connect(ipc_handles);
    });
}

pokit_cuda_status pokit_cuda_moe_exchange_disconnect(pokit_cuda_moe* moe, char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.exchange_disconnect();
    });
}

pokit_cuda_status pokit_cuda_moe_time_batch(pokit_cuda_moe* moe, size_t layer, const void* input,
                                            uint32_t input_type, size_t tokens, const float* router_logits,
                                            float* output, uint32_t repetitions, float* stage_us,
                                            size_t stage_capacity, size_t* stages, void* stream,
                                            char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe || !stages) throw std::invalid_argument("handle and stages are required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        *stages = moe->impl.time_batch(layer, input, input_type, tokens, router_logits, output, repetitions, stage_us,
                                       stage_capacity, as_stream(stream));
    });
}

pokit_cuda_status pokit_cuda_moe_forward_batch_host(pokit_cuda_moe* moe, size_t layer, const void* input_host,
                                                    uint32_t input_type, size_t tokens,
                                                    const float* router_logits_host, float* output_host,
                                                    uint32_t* route_ids_host, float* route_weights_host,
                                                    char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.forward_batch_host(layer, input_host, input_type, tokens, router_logits_host, output_host,
                                     route_ids_host, route_weights_host);
    });
}

pokit_cuda_status pokit_cuda_moe_time_kernel(pokit_cuda_moe* moe, uint32_t kernel, size_t first_layer,
                                              size_t layer_count, uint32_t repetitions, float* work,
                                              void* stream, float* average_us, char* error_buffer,
                                              size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe || !average_us) throw std::invalid_argument("handle and average_us are required");
        if (kernel > 1 || repetitions == 0) throw std::invalid_argument("kernel must be 0 or 1, repetitions > 0");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        *average_us = moe->impl.time_kernel(kernel, first_layer, layer_count, repetitions, work, as_stream(stream));
    });
}

pokit_cuda_status pokit_cuda_moe_forward_host(pokit_cuda_moe* moe, size_t layer, const float* input_host,
                                              float* output_host, uint32_t* route_ids_host,
                                              float* route_weights_host, char* error_buffer,
                                              size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.forward_host(layer, input_host, output_host, route_ids_host, route_weights_host);
    });
}

pokit_cuda_status pokit_cuda_moe_decode_layers(pokit_cuda_moe* moe, size_t first, size_t count,
                                               float* hidden, void* stream, char* error_buffer,
                                               size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.decode_layers(first, count, hidden, as_stream(stream));
    });
}

pokit_cuda_status pokit_cuda_moe_decode_layers_host(pokit_cuda_moe* moe, size_t first, size_t count,
                                                    const float* hidden_in, float* hidden_out,
                                                    char* error_buffer, size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.decode_layers_host(first, count, hidden_in, hidden_out);
    });
}

pokit_cuda_status pokit_cuda_moe_trace_decode(pokit_cuda_moe* moe, size_t first, size_t count, float* hidden,
                                              uint64_t* stamps, size_t stamp_capacity, uint32_t* grid, void* stream,
                                              char* error_buffer, size_t error_capacity) {
    if (grid) *grid = 0;
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        const uint32_t g = moe->impl.trace_decode(first, count, hidden,
                                                  reinterpret_cast<unsigned long long*>(stamps), stamp_capacity,
                                                  as_stream(stream));
        if (grid) *grid = g;
    });
}

pokit_cuda_status pokit_cuda_moe_synchronize(pokit_cuda_moe* moe, void* stream, char* error_buffer,
                                             size_t error_capacity) {
    return guarded(error_buffer, error_capacity, [&] {
        if (!moe) throw std::invalid_argument("MoE handle is required");
        std::lock_guard<std::mutex> lock(moe->impl.mutex());
        moe->impl.synchronize(as_stream(stream));
    });
}

pokit_cuda_status pokit_cuda_moe_get_stats(const pokit_cuda_moe* moe, pokit_cuda_moe_stats* out_stats) {
    if (!moe || !out_stats) return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    *out_stats = moe->impl.stats();
    return POKIT_CUDA_STATUS_OK;
}

size_t pokit_cuda_moe_tensor_bytes(const pokit_cuda_moe* moe, size_t layer, uint32_t tensor) {
    return moe ? static_cast<size_t>(moe->impl.tensor_bytes(layer, tensor)) : 0;
}

}  // extern "C"
