// ref_shim.cpp -- extern "C" shim over the PokitLMs reference's own C++ kernels.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified sources (src/quantized_linear.cpp, src/linear.cpp,
// src/tensor_linear.cpp, src/tensor_reader.cpp, src/model_file.cpp,
// src/rms_norm.cpp) into oracle/_ref/libpokit_ref.so.  It is used to (1) pin
// the C restatement in oracle/pokit_oracle.c, (2) generate the golden
// fixtures under tests/golden/, and (3) time the reference's CPU path in
// bench.py's reference arm.  The product library never loads it.
//
// The reference's routing functions (route_experts, select_experts) live in
// anonymous namespaces of the runners and cannot be linked, so the MoE block
// below calls the restated routing from pokit_oracle.c; every matrix product
// goes through the reference's own model::tensor_linear (row executor
// included), exactly as the runner's MoE block does
// (src/qwen3_moe_runner.cpp:643-692, src/qwen35_runner.cpp:691-763).
#include "pokitlms/model/tensor_linear.hpp"
#include "pokitlms/model/tensor_reader.hpp"
#include "pokitlms/ops/linear.hpp"
#include "pokitlms/ops/quantized_linear.hpp"
#include "pokitlms/ops/rms_norm.hpp"
#include "pokitlms/ops/causal_conv1d.hpp"
#include "pokitlms/ops/gated_delta_net.hpp"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <vector>

extern "C" {
int po_route_qwen3(const float* logits, size_t n, size_t k, int normalize, uint32_t* ids,
                   float* probs);
int po_route_qwen35(const float* logits, size_t n, size_t k, int normalize, uint32_t* ids,
                    float* probs);
float po_sigmoid(float v);
}

namespace {

using pokitlms::model::TensorInfo;
using pokitlms::model::TensorReader;

std::size_t row_bytes(std::uint32_t type, std::size_t cols) {
    switch (type) {
        case 0: return cols * 4;
        case 8: return cols / 32 * 34;
        case 12: return cols / 256 * 144;
        case 13: return cols / 256 * 176;
        case 14: return cols / 256 * 210;
        default: throw std::invalid_argument("unsupported GGML type");
    }
}

// An in-memory reader over a [rows, cols] matrix, the same construction the
// reference's runners use for expert slices (TensorReader(TensorInfo, payload),
// src/tensor_reader.cpp:75-94).
TensorReader make_reader(std::uint32_t type, std::size_t cols, std::size_t rows,
                         const void* bytes) {
    const auto size = row_bytes(type, cols) * rows;
    auto payload = std::make_shared<std::vector<std::byte>>(size);
    std::memcpy(payload->data(), bytes, size);
    TensorInfo info;
    info.name = "shim";
    info.dimensions = {cols, rows};
    info.type = type;
    info.payload_size = size;
    return TensorReader(info, payload);
}

template <typename F>
int guarded(F&& body) {
    try {
        body();
        return 0;
    } catch (const std::invalid_argument&) {
        return 1;
    } catch (const std::exception&) {
        return 2;
    } catch (...) {
        return 4;
    }
}

struct MoeLayer {
    std::size_t hidden{}, inter{}, experts{}, top_k{};
    int flavour{}, normalize{};
    float expert_weights_scale{1.0F};
    std::unique_ptr<TensorReader> router;
    std::vector<TensorReader> gate, up, down;
    std::size_t shared_inter{};
    std::unique_ptr<TensorReader> shared_router, shared_gate, shared_up, shared_down;
    std::vector<float> logits, g, u, a, y;
    pokitlms::model::TensorLinearScratch scratch;
};

}  // namespace

extern "C" {

// Same field order as po_moe_layer in pokit_oracle.c.
struct pr_moe_desc {
    size_t hidden, inter, experts, top_k;
    int flavour, normalize;
    float expert_weights_scale;
    const float* router;
    uint32_t gate_type, up_type, down_type;
    const void* gate;
    const void* up;
    const void* down;
    size_t shared_inter;
    const float* shared_router;
    uint32_t shared_gate_type, shared_up_type, shared_down_type;
    const void* shared_gate;
    const void* shared_up;
    const void* shared_down;
};

// Direct per-format kernel call (no row executor):
// linear_q8_0/q4_k/q5_k/q6_k (include/pokitlms/ops/quantized_linear.hpp:23-53)
// or linear() for F32 (include/pokitlms/ops/linear.hpp:10-14).
int pr_linear(uint32_t type, const float* x, size_t cols, const void* w, size_t rows, float* y) {
    return guarded([&] {
        std::span<const float> input(x, cols);
        std::span<float> output(y, rows);
        std::span<const std::byte> weights(static_cast<const std::byte*>(w),
                                           row_bytes(type, cols) * rows);
        switch (type) {
            case 0:
                pokitlms::linear(input, std::span<const float>(static_cast<const float*>(w),
                                                                cols * rows), {}, output);
                break;
            case 8: pokitlms::linear_q8_0(input, weights, rows, {}, output); break;
            case 12: pokitlms::linear_q4_k(input, weights, rows, {}, output); break;
            case 13: pokitlms::linear_q5_k(input, weights, rows, {}, output); break;
            case 14: pokitlms::linear_q6_k(input, weights, rows, {}, output); break;
            default: throw std::invalid_argument("unsupported GGML type");
        }
    });
}

// Through the reference's dispatch seam, model::tensor_linear
// (src/tensor_linear.cpp:196-227): multi-threaded row executor for >=256 rows.
int pr_tensor_linear(uint32_t type, const float* x, size_t cols, const void* w, size_t rows,
                     float* y) {
    return guarded([&] {
        auto reader = make_reader(type, cols, rows, w);
        pokitlms::model::tensor_linear(reader, std::span<const float>(x, cols),
                                       std::span<float>(y, rows));
    });
}

// dequantize_quantized_row, include/pokitlms/ops/quantized_linear.hpp:11-13.
int pr_dequantize_row(uint32_t type, const void* encoded, size_t elements, float* out) {
    return guarded([&] {
        pokitlms::dequantize_quantized_row(
            type, std::span<const std::byte>(static_cast<const std::byte*>(encoded),
                                             row_bytes(type, elements)),
            std::span<float>(out, elements));
    });
}

// rms_norm, include/pokitlms/ops/rms_norm.hpp.
int pr_rms_norm(const float* x, const float* w, size_t n, float eps, float* y) {
    return guarded([&] {
        pokitlms::rms_norm(std::span<const float>(x, n), std::span<const float>(w, n),
                           std::span<float>(y, n), eps);
    });
}

void* pr_moe_create(const pr_moe_desc* d) {
    try {
        auto L = std::make_unique<MoeLayer>();
        L->hidden = d->hidden;
        L->inter = d->inter;
        L->experts = d->experts;
        L->top_k = d->top_k;
        L->flavour = d->flavour;
        L->normalize = d->normalize;
        L->expert_weights_scale = d->expert_weights_scale;
        L->router = std::make_unique<TensorReader>(make_reader(0, d->hidden, d->experts, d->router));
        const auto gs = row_bytes(d->gate_type, d->hidden) * d->inter;
        const auto us = row_bytes(d->up_type, d->hidden) * d->inter;
        const auto ds = row_bytes(d->down_type, d->inter) * d->hidden;
        for (std::size_t e = 0; e < d->experts; ++e) {
            L->gate.push_back(make_reader(d->gate_type, d->hidden, d->inter,
                                          static_cast<const std::byte*>(d->gate) + e * gs));
            L->up.push_back(make_reader(d->up_type, d->hidden, d->inter,
                                        static_cast<const std::byte*>(d->up) + e * us));
            L->down.push_back(make_reader(d->down_type, d->inter, d->hidden,
                                          static_cast<const std::byte*>(d->down) + e * ds));
        }
        if (d->flavour == 1 && d->shared_inter && d->shared_router) {
            L->shared_inter = d->shared_inter;
            L->shared_router = std::make_unique<TensorReader>(
                make_reader(0, d->hidden, 1, d->shared_router));
            L->shared_gate = std::make_unique<TensorReader>(
                make_reader(d->shared_gate_type, d->hidden, d->shared_inter, d->shared_gate));
            L->shared_up = std::make_unique<TensorReader>(
                make_reader(d->shared_up_type, d->hidden, d->shared_inter, d->shared_up));
            L->shared_down = std::make_unique<TensorReader>(
                make_reader(d->shared_down_type, d->shared_inter, d->hidden, d->shared_down));
        }
        const auto width = std::max(d->inter, d->shared_inter);
        L->logits.resize(d->experts);
        L->g.resize(width);
        L->u.resize(width);
        L->a.resize(width);
        L->y.resize(d->hidden);
        return L.release();
    } catch (...) {
        return nullptr;
    }
}

void pr_moe_destroy(void* handle) { delete static_cast<MoeLayer*>(handle); }

// One MoE block with the reference's kernels and executor.  `out` gets the
// MoE contribution (the runner then adds it to the residual stream).
int pr_moe_forward(void* handle, const float* x, float* out, uint32_t* ids, float* probs) {
    auto* L = static_cast<MoeLayer*>(handle);
    if (!L) return 1;
    return guarded([&] {
        using pokitlms::model::tensor_linear;
        const auto H = L->hidden, I = L->inter;
        std::span<const float> input(x, H);
        tensor_linear(*L->router, input, L->logits, 0, &L->scratch);
        const int st = L->flavour == 0
            ? po_route_qwen3(L->logits.data(), L->experts, L->top_k, L->normalize, ids, probs)
            : po_route_qwen35(L->logits.data(), L->experts, L->top_k, L->normalize, ids, probs);
        if (st == 2) throw std::runtime_error("expert router produced non-finite logits");
        if (st) throw std::invalid_argument("invalid expert top-k");
        std::span<float> result(out, H);
        std::fill(result.begin(), result.end(), 0.0F);
        auto g = std::span<float>(L->g).first(I);
        auto u = std::span<float>(L->u).first(I);
        auto a = std::span<float>(L->a).first(I);
        for (std::size_t r = 0; r < L->top_k; ++r) {
            const auto e = ids[r];
            tensor_linear(L->gate[e], input, g, 0, &L->scratch);
            tensor_linear(L->up[e], input, u, 0, &L->scratch);
            for (std::size_t i = 0; i < I; ++i) {
                a[i] = L->flavour == 0 ? (g[i] / (1.0F + std::exp(-g[i]))) * u[i]
                                       : (g[i] * po_sigmoid(g[i])) * u[i];
            }
            tensor_linear(L->down[e], a, L->y, 0, &L->scratch);
            const float scale = L->flavour == 0 ? probs[r] : probs[r] * L->expert_weights_scale;
            for (std::size_t i = 0; i < H; ++i) result[i] += scale * L->y[i];
        }
        if (L->shared_router) {
            const auto SI = L->shared_inter;
            float gate_value = 0.0F;
            tensor_linear(*L->shared_router, input, std::span<float>(&gate_value, 1), 0,
                          &L->scratch);
            auto sg = std::span<float>(L->g).first(SI);
            auto su = std::span<float>(L->u).first(SI);
            auto sa = std::span<float>(L->a).first(SI);
            tensor_linear(*L->shared_gate, input, sg, 0, &L->scratch);
            tensor_linear(*L->shared_up, input, su, 0, &L->scratch);
            for (std::size_t i = 0; i < SI; ++i) sa[i] = (sg[i] * po_sigmoid(sg[i])) * su[i];
            tensor_linear(*L->shared_down, sa, L->y, 0, &L->scratch);
            const float shared_scale = po_sigmoid(gate_value);
            for (std::size_t i = 0; i < H; ++i) result[i] = result[i] + shared_scale * L->y[i];
        }
    });
}

}  // extern "C"

// The reference's own Gated DeltaNet pieces (src/causal_conv1d.cpp,
// src/gated_delta_net.cpp, src/rms_norm.cpp), for pinning the restatement.
extern "C" int ref_causal_conv1d_step(const float* input, const float* weights, size_t channels, size_t kernel,
                                      float* state, float* output) {
    try {
        pokitlms::causal_depthwise_conv1d_step(input, weights, channels, kernel, state, output);
        return 0;
    } catch (...) {
        return 1;
    }
}

extern "C" int ref_gated_delta_step(const float* query, const float* key, const float* value,
                                    const float* log_decay, const float* beta, size_t key_heads,
                                    size_t value_heads, size_t dk, size_t dv, float* state, float* output) {
    try {
        pokitlms::GatedDeltaNetScratch scratch;
        pokitlms::gated_delta_recurrent_step_grouped(query, key, value, log_decay, beta, key_heads, value_heads,
                                                     dk, dv, state, output, scratch);
        return 0;
    } catch (...) {
        return 1;
    }
}

extern "C" int ref_rms_norm_gated(const float* x, const float* w, const float* gate, size_t rows, size_t width,
                                  float eps, float* y) {
    try {
        pokitlms::rms_norm_gated(std::span<const float>(x, rows * width), std::span<const float>(w, width),
                                 std::span<const float>(gate, rows * width), std::span<float>(y, rows * width),
                                 rows, eps);
        return 0;
    } catch (...) {
        return 1;
    }
}
