// pokit_static_scratch.cu -- one MoE block that allocates no device memory.
//
// Some callers of this library cannot call cudaMalloc: a host framework that
// reserves all of the GPU's memory up front for its own pool (an inference
// server, a runtime embedding the library as a plugin) leaves nothing for the
// library to allocate, and a latency-critical thread may not make a call that
// can synchronise the whole device.  pokit_cuda_moe_forward_static_scratch
// serves them: the caller passes the block's weights, input and outputs as
// device pointers it already owns, and the router partials, routes and
// activations live in a fixed array compiled into the library.
//
// The array below is allocated by the CUDA module loader on every GPU that
// loads the library and is held until the process exits.  Every call shares
// it and it keeps the previous call's contents: the status word is cleared at
// the start of each call, everything else is fully rewritten before it is
// read.  Two calls whose work overlaps on the GPU (different streams, or
// different host threads, without ordering between them) race on the array.
#include "../../include/pokit_cuda.h"
#include "pokit_kernels.h"
#include "pokit_types.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace {

// Maximum scratch one block may use (POKIT_CUDA_STATIC_SCRATCH_BYTES).
constexpr size_t kStaticScratchBytes = POKIT_CUDA_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

// The array's device address for the current device.  In host code the symbol
// names a host-side stand-in, not device memory, so the address must come from
// cudaGetSymbolAddress with the owning device current; it is looked up on the
// first call on each device and cached.
void* scratch_for_current_device() {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (device < 0 || device >= kMaxDevices) throw std::runtime_error("CUDA device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[device]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p)
            throw std::runtime_error(std::string("cudaGetSymbolAddress(static scratch): ") +
                                     cudaGetErrorString(e));
        g_scratch_address[device] = p;
    }
    return g_scratch_address[device];
}

void check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    if (e == cudaErrorInvalidValue)
        throw std::invalid_argument(std::string(what) + ": unsupported shape or argument");
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

bool quant_type(uint32_t t) {
    return t == pokit::kQ8_0 || t == pokit::kQ4_K || t == pokit::kQ5_K || t == pokit::kQ6_K;
}

pokit::MoeLayerDev to_layer(const pokit_cuda_moe_block_device& b) {
    if (b.hidden == 0 || b.hidden % 256 || b.inter == 0 || b.inter % 256 || b.experts == 0 ||
        b.experts > 1024 || b.top_k == 0 || b.top_k > b.experts || b.top_k > 64 ||
        b.flavour > 1 || b.hidden > 0xffffffffu || b.inter > 0xffffffffu)
        throw std::invalid_argument("invalid MoE block shape");
    if (!b.router || !b.gate || !b.up || !b.down)
        throw std::invalid_argument("router, gate, up and down tensors are required");
    if (!quant_type(b.gate_type) || !quant_type(b.up_type) || !quant_type(b.down_type))
        throw std::invalid_argument("unsupported expert tensor type");
    // Every kernel reads the weights and the routers' rows with 16-byte loads
    // (TMA boxes, float4), so a misaligned tensor is refused here rather than
    // faulting on the GPU.
    const auto a16 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!a16(b.gate) || !a16(b.up) || !a16(b.down) || !a16(b.shared_gate) || !a16(b.shared_up) ||
        !a16(b.shared_down) || !a16(b.router) || !a16(b.shared_router))
        throw std::invalid_argument("expert tensors and routers must be 16-byte aligned");
    pokit::MoeLayerDev L;
    L.hidden = static_cast<uint32_t>(b.hidden);
    L.inter = static_cast<uint32_t>(b.inter);
    L.experts = static_cast<uint32_t>(b.experts);
    L.top_k = static_cast<uint32_t>(b.top_k);
    L.flavour = b.flavour;
    L.normalize = b.normalize_top_k ? 1u : 0u;
    L.expert_weights_scale = b.flavour == POKIT_CUDA_MOE_QWEN35 ? b.expert_weights_scale : 1.0f;
    L.router = b.router;
    L.gate_type = b.gate_type;
    L.up_type = b.up_type;
    L.down_type = b.down_type;
    L.gate = static_cast<const uint8_t*>(b.gate);
    L.up = static_cast<const uint8_t*>(b.up);
    L.down = static_cast<const uint8_t*>(b.down);
    L.gate_slice = b.inter * pokit::row_bytes(b.gate_type, b.hidden);
    L.up_slice = b.inter * pokit::row_bytes(b.up_type, b.hidden);
    L.down_slice = b.hidden * pokit::row_bytes(b.down_type, b.inter);
    if (b.shared_inter) {
        if (b.flavour != POKIT_CUDA_MOE_QWEN35 || b.shared_inter % 256 || !b.shared_router ||
            !b.shared_gate || !b.shared_up || !b.shared_down || !quant_type(b.shared_gate_type) ||
            !quant_type(b.shared_up_type) || !quant_type(b.shared_down_type))
            throw std::invalid_argument("invalid shared expert");
        L.shared_inter = static_cast<uint32_t>(b.shared_inter);
        L.shared_router = b.shared_router;
        L.shared_gate_type = b.shared_gate_type;
        L.shared_up_type = b.shared_up_type;
        L.shared_down_type = b.shared_down_type;
        L.shared_gate = static_cast<const uint8_t*>(b.shared_gate);
        L.shared_up = static_cast<const uint8_t*>(b.shared_up);
        L.shared_down = static_cast<const uint8_t*>(b.shared_down);
    }
    return L;
}

void set_error(char* destination, size_t capacity, const char* message) noexcept {
    if (!destination || capacity == 0) return;
    const size_t n = std::min(capacity - 1, std::strlen(message));
    std::memcpy(destination, message, n);
    destination[n] = '\0';
}

}  // namespace

extern "C" pokit_cuda_status pokit_cuda_moe_forward_static_scratch(
    const pokit_cuda_moe_block_device* block, const float* input, float* output,
    uint32_t* route_ids, float* route_weights, void* stream, char* error_buffer,
    size_t error_capacity) {
    try {
        if (!block || !input || !output) throw std::invalid_argument("block, input and output are required");
        const pokit::MoeLayerDev L = to_layer(*block);
        // As many activation replicas as fit (at least one).
        uint32_t rep = pokit::kActReplicas;
        while (rep > 1 && pokit::moe_scratch_bytes(L, rep) > kStaticScratchBytes) rep /= 2;
        const uint64_t need = pokit::moe_scratch_bytes(L, rep);
        if (need > kStaticScratchBytes)
            throw std::invalid_argument("MoE block needs " + std::to_string(need) +
                                        " bytes of scratch, above the static scratch limit of " +
                                        std::to_string(kStaticScratchBytes) + " bytes");
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        void* base = scratch_for_current_device();
        const pokit::MoeScratch S = pokit::moe_scratch_carve(L, base, rep);
        check(pokit::prepare_moe_block(L), "prepare MoE kernels");
        // The router accumulators, the counters and the status word end the
        // carve: one clear covers them.
        const size_t tail = static_cast<size_t>(reinterpret_cast<const uint8_t*>(S.status) + sizeof(uint32_t) -
                                                reinterpret_cast<const uint8_t*>(S.racc));
        check(cudaMemsetAsync(S.racc, 0, tail, st), "clear accumulators, counters and status");
        check(pokit::launch_moe_block(L, S, input, nullptr, output, nullptr, nullptr, st, nullptr), "MoE block");
        if (route_ids)
            check(cudaMemcpyAsync(route_ids, S.ids, L.top_k * sizeof(uint32_t),
                                  cudaMemcpyDeviceToDevice, st), "route ids");
        if (route_weights)
            check(cudaMemcpyAsync(route_weights, S.weights, L.top_k * sizeof(float),
                                  cudaMemcpyDeviceToDevice, st), "route weights");
        // The status word comes back on the caller's stream, which is the only
        // thing this call waits for (no legacy-stream copy, no device-wide sync).
        uint32_t status = 0;
        check(cudaMemcpyAsync(&status, S.status, sizeof status, cudaMemcpyDeviceToHost, st), "status");
        check(cudaStreamSynchronize(st), "synchronize");
        if (status & pokit::kStatusNonFiniteLogits)
            throw std::runtime_error("expert router produced non-finite logits");
        if (status) throw std::runtime_error("expert router softmax is invalid");
        set_error(error_buffer, error_capacity, "");
        return POKIT_CUDA_STATUS_OK;
    } catch (const std::invalid_argument& e) {
        set_error(error_buffer, error_capacity, e.what());
        return POKIT_CUDA_STATUS_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        set_error(error_buffer, error_capacity, e.what());
        return POKIT_CUDA_STATUS_RUNTIME_ERROR;
    } catch (...) {
        set_error(error_buffer, error_capacity, "unknown static-scratch MoE failure");
        return POKIT_CUDA_STATUS_INTERNAL_ERROR;
    }
}
