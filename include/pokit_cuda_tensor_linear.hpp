// pokit_cuda_tensor_linear.hpp -- the B200 backend behind PokitLMs'
// per-matrix seam, model::TensorLinearBackend
// (include/pokitlms/model/tensor_linear.hpp:11-18), beside
// gpu::VulkanLinearBackend (include/pokitlms/gpu/vulkan_linear.hpp:69-84).
//
// Header-only; compiles inside a PokitLMs tree (its include/ on the path) and
// links libpokit_cuda.so.  Install it as the Vulkan backend is installed:
// Qwen35Runner::set_linear_backend (qwen35_runner.hpp:90-91) or
// TensorLinearScratch::backend (tensor_linear.hpp:25).
//
// Weights: a reader backed by the model file names its matrix by the
// tensor's GGUF file offset, and the payload stays in HBM under that key
// (the Vulkan backend's whole-model cache, vulkan_linear.cpp:516-563); one
// backend serves one model file.  An in-memory reader (a routed expert's
// slice, tensor_reader.cpp:75-94) has no stable identity, so its payload is
// streamed to the device on every call, as the Vulkan backend streams it
// through its windows (vulkan_linear.cpp:705-714).
//
// Contract of try_linear: false for types the CUDA kernels do not serve (the
// caller's CPU path runs); a failure throws and never leaves partial output
// (tensor_linear.hpp:14-15).
#pragma once

#include "pokit_cuda.h"
#include "pokitlms/model/tensor_linear.hpp"

#include <cstddef>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

namespace pokitlms::gpu {

class CudaLinearBackend final : public model::TensorLinearBackend {
public:
    explicit CudaLinearBackend(int device = 0) {
        char err[512];
        if (pokit_cuda_linear_backend_create(device, &handle_, err, sizeof err) != POKIT_CUDA_STATUS_OK)
            throw std::runtime_error(std::string("CUDA linear backend: ") + err);
    }
    ~CudaLinearBackend() override { pokit_cuda_linear_backend_destroy(handle_); }
    CudaLinearBackend(const CudaLinearBackend&) = delete;
    CudaLinearBackend& operator=(const CudaLinearBackend&) = delete;

    bool try_linear(const model::TensorReader& weights, std::span<const float> input,
                    std::span<float> output) override {
        const model::TensorInfo& info = weights.tensor();
        const std::size_t bytes = static_cast<std::size_t>(weights.row_count()) * weights.row_bytes();
        int handled = 0;
        char err[512];
        pokit_cuda_status st;
        if (weights.model_file()) {
            // Read the file only when HBM does not hold the matrix yet.
            std::vector<std::byte> payload;
            if (!pokit_cuda_linear_backend_is_cached(handle_, info.file_offset)) payload = weights.read_all();
            st = pokit_cuda_linear_backend_try_linear_cached(
                handle_, info.file_offset, info.type, payload.empty() ? nullptr : payload.data(), bytes,
                output.size(), input.size(), input.data(), output.data(), &handled, err, sizeof err);
        } else {
            const std::vector<std::byte> payload = weights.read_all();
            st = pokit_cuda_linear_backend_try_linear(handle_, info.type, payload.data(), payload.size(),
                                                      output.size(), input.size(), input.data(),
                                                      output.data(), &handled, err, sizeof err);
        }
        if (st != POKIT_CUDA_STATUS_OK) throw std::runtime_error(std::string("CUDA linear backend: ") + err);
        return handled != 0;
    }

    [[nodiscard]] pokit_cuda_linear_stats stats() const {
        pokit_cuda_linear_stats s{};
        pokit_cuda_linear_backend_get_stats(handle_, &s);
        return s;
    }

private:
    pokit_cuda_linear_backend* handle_{};
};

}  // namespace pokitlms::gpu
