/*
 * pokit_oracle.c -- CPU restatement of the PokitLMs MoE expert path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * backend: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load it.  The product library (pokitlms_b200/libpokit_cuda.so) never
 * links, loads or calls it, and has no CPU fallback.
 *
 * Parity is pinned two ways:
 *   - against the reference's own known-answer blocks (regression_test.cpp
 *     Q5_K cases) and the golden vectors under tests/golden/, which were
 *     produced by the reference's own C++ sources compiled into oracle/_ref;
 *   - bit-for-bit against oracle/_ref on seeded random blocks (CPU tests).
 *
 * Every function follows the reference's arithmetic order exactly (scalar x86
 * path: decode a block to FP32, then a sequential FP32 dot per block, summed
 * block by block), so results are bit-identical to the reference when both
 * are compiled without FMA contraction.  Each function cites the file:line of
 * the reference (paths relative to the PokitLMs project root) it restates.
 *
 * GGML type ids used here: 0 = F32, 8 = Q8_0, 12 = Q4_K, 13 = Q5_K, 14 = Q6_K.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define PO_OK 0
#define PO_INVALID 1
#define PO_RUNTIME 2

/* IEEE binary16 -> binary32, exact, subnormals included.
 * Restates half_to_float, src/quantized_linear.cpp:18-39. */
float po_half_to_float(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    uint32_t exponent = (bits >> 10) & 0x1fu;
    uint32_t mantissa = bits & 0x03ffu;
    uint32_t result;
    if (exponent == 0) {
        if (mantissa == 0) {
            result = sign;
        } else {
            int e = -14;
            while ((mantissa & 0x0400u) == 0) {
                mantissa <<= 1;
                --e;
            }
            mantissa &= 0x03ffu;
            result = sign | ((uint32_t)(e + 127) << 23) | (mantissa << 13);
        }
    } else if (exponent == 0x1fu) {
        result = sign | 0x7f800000u | (mantissa << 13);
    } else {
        result = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    float out;
    memcpy(&out, &result, sizeof(out));
    return out;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Q4_K/Q5_K 6-bit scale/min unpack for sub-block j of 8.
 * Restates the scale_min lambda, src/quantized_linear.cpp:176-188 (and 292-304). */
static void k_scale_min(const uint8_t* packed, int j, uint8_t* scale, uint8_t* minimum) {
    if (j < 4) {
        *scale = packed[j] & 63u;
        *minimum = packed[j + 4] & 63u;
    } else {
        *scale = (uint8_t)((packed[j + 4] & 0x0fu) | ((packed[j - 4] >> 6) << 4));
        *minimum = (uint8_t)((packed[j + 4] >> 4) | ((packed[j] >> 6) << 4));
    }
}

/* Q4_K superblock (144 B: fp16 d, fp16 dmin, 12 B scales, 128 B nibbles) -> 256 floats.
 * Restates decode_q4_k, src/quantized_linear.cpp:166-205. */
void po_decode_q4_k(const uint8_t* block, float* values) {
    const float d = po_half_to_float(rd16(block));
    const float dmin = po_half_to_float(rd16(block + 2));
    const uint8_t* packed = block + 4;
    const uint8_t* q = block + 16;
    int out = 0;
    for (int chunk = 0; chunk < 4; ++chunk) {
        uint8_t s0, m0, s1, m1;
        k_scale_min(packed, 2 * chunk, &s0, &m0);
        k_scale_min(packed, 2 * chunk + 1, &s1, &m1);
        const float ds0 = d * s0, dm0 = dmin * m0;
        const float ds1 = d * s1, dm1 = dmin * m1;
        for (int i = 0; i < 32; ++i) values[out++] = ds0 * (float)(q[i] & 0x0fu) - dm0;
        for (int i = 0; i < 32; ++i) values[out++] = ds1 * (float)(q[i] >> 4) - dm1;
        q += 32;
    }
}

/* Q5_K superblock (176 B: d, dmin, scales[12], qh[32], qs[128]) -> 256 floats.
 * Restates decode_q5_k, src/quantized_linear.cpp:286-328. */
void po_decode_q5_k(const uint8_t* block, float* values) {
    const float d = po_half_to_float(rd16(block));
    const float dmin = po_half_to_float(rd16(block + 2));
    const uint8_t* packed = block + 4;
    const uint8_t* high = block + 16;
    const uint8_t* q = block + 48;
    int out = 0, is = 0;
    uint8_t mask1 = 1, mask2 = 2;
    for (int chunk = 0; chunk < 4; ++chunk) {
        uint8_t s0, m0, s1, m1;
        k_scale_min(packed, is++, &s0, &m0);
        k_scale_min(packed, is++, &s1, &m1);
        const float ds0 = d * s0, dm0 = dmin * m0;
        const float ds1 = d * s1, dm1 = dmin * m1;
        for (int i = 0; i < 32; ++i) {
            const unsigned v = (q[i] & 0x0fu) + ((high[i] & mask1) ? 16u : 0u);
            values[out++] = ds0 * (float)v - dm0;
        }
        for (int i = 0; i < 32; ++i) {
            const unsigned v = (q[i] >> 4) + ((high[i] & mask2) ? 16u : 0u);
            values[out++] = ds1 * (float)v - dm1;
        }
        q += 32;
        mask1 = (uint8_t)(mask1 << 2);
        mask2 = (uint8_t)(mask2 << 2);
    }
}

/* Q6_K superblock (210 B: ql[128], qh[64], int8 scales[16], fp16 d) -> 256 floats.
 * Restates decode_q6_k, src/quantized_linear.cpp:330-358.  The reference
 * evaluates d * s * q left to right as float * int8 (promoted) * int. */
void po_decode_q6_k(const uint8_t* block, float* values) {
    const uint8_t* low = block;
    const uint8_t* high = block + 128;
    const int8_t* scales = (const int8_t*)(block + 192);
    const float d = po_half_to_float(rd16(block + 208));
    for (int half = 0; half < 2; ++half) {
        const int base = half * 128;
        for (int lane = 0; lane < 32; ++lane) {
            const int is = lane / 16;
            const uint8_t lo0 = low[lane], lo1 = low[lane + 32], hi = high[lane];
            const int q0 = (int)((lo0 & 0x0fu) | ((hi & 0x03u) << 4)) - 32;
            const int q1 = (int)((lo1 & 0x0fu) | (((hi >> 2) & 0x03u) << 4)) - 32;
            const int q2 = (int)((lo0 >> 4) | (((hi >> 4) & 0x03u) << 4)) - 32;
            const int q3 = (int)((lo1 >> 4) | (((hi >> 6) & 0x03u) << 4)) - 32;
            const int8_t s0 = scales[half * 8 + is];
            const int8_t s1 = scales[half * 8 + is + 2];
            const int8_t s2 = scales[half * 8 + is + 4];
            const int8_t s3 = scales[half * 8 + is + 6];
            values[base + lane] = d * (float)s0 * (float)q0;
            values[base + lane + 32] = d * (float)s1 * (float)q1;
            values[base + lane + 64] = d * (float)s2 * (float)q2;
            values[base + lane + 96] = d * (float)s3 * (float)q3;
        }
        low += 64;
        high += 32;
    }
}

/* Q8_0 block (34 B: fp16 d, int8 q[32]) -> 32 floats, d * q.
 * Restates dequantize_quantized_row for type 8, src/quantized_linear.cpp:430-451
 * (scale_i8_f32, src/simd_kernels.hpp:67-86 scalar path: scale * q). */
void po_decode_q8_0(const uint8_t* block, float* values) {
    const float d = po_half_to_float(rd16(block));
    const int8_t* q = (const int8_t*)(block + 2);
    for (int i = 0; i < 32; ++i) values[i] = d * (float)q[i];
}

/* Sequential FP32 dot, scalar (non-AArch64) path of dot_f32,
 * src/simd_kernels.hpp:12-24. */
float po_dot_f32(const float* lhs, const float* rhs, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += lhs[i] * rhs[i];
    return sum;
}

/* Sequential int8 x FP32 dot, scalar path of dot_i8_f32, src/simd_kernels.hpp:26-48. */
static float po_dot_i8_f32(const float* lhs, const int8_t* q, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += (float)q[i] * lhs[i];
    return sum;
}

/* Block geometry of a supported GGML type (src/model/gguf_reader.cpp type_layout, :21-57). */
int po_type_layout(uint32_t type, size_t* block_elements, size_t* block_bytes) {
    switch (type) {
        case 0: *block_elements = 1; *block_bytes = 4; return PO_OK;
        case 8: *block_elements = 32; *block_bytes = 34; return PO_OK;
        case 12: *block_elements = 256; *block_bytes = 144; return PO_OK;
        case 13: *block_elements = 256; *block_bytes = 176; return PO_OK;
        case 14: *block_elements = 256; *block_bytes = 210; return PO_OK;
        default: return PO_INVALID;
    }
}

/* Decodes `elements` weights of one row.  Restates dequantize_quantized_row,
 * src/quantized_linear.cpp:427-493, for F32/Q8_0/Q4_K/Q5_K/Q6_K. */
int po_dequantize_row(uint32_t type, const void* encoded, size_t elements, float* out) {
    size_t be, bb;
    if (po_type_layout(type, &be, &bb) != PO_OK || elements == 0 || elements % be != 0)
        return PO_INVALID;
    const uint8_t* p = (const uint8_t*)encoded;
    if (type == 0) {
        memcpy(out, p, elements * sizeof(float));
        return PO_OK;
    }
    for (size_t b = 0; b < elements / be; ++b) {
        const uint8_t* blk = p + b * bb;
        float* dst = out + b * be;
        switch (type) {
            case 8: po_decode_q8_0(blk, dst); break;
            case 12: po_decode_q4_k(blk, dst); break;
            case 13: po_decode_q5_k(blk, dst); break;
            default: po_decode_q6_k(blk, dst); break;
        }
    }
    return PO_OK;
}

/* y[rows] = W[rows, cols] . x[cols], W row-major in its GGML block encoding.
 *  F32:  linear(), src/linear.cpp:26-30 (0 + dot_f32(weight_row, input)).
 *  Q8_0: linear_quantized<false>, src/quantized_linear.cpp:405-421
 *        (sum += d * dot_i8_f32(x_block, q) per 32-block).
 *  K:    linear_k<256, bytes>, src/quantized_linear.cpp:374-384
 *        (decode a block, sum += dot_f32(decoded, x_block)). */
int po_linear(uint32_t type, const float* x, size_t cols, const void* weights, size_t rows,
              float* y) {
    size_t be, bb;
    if (po_type_layout(type, &be, &bb) != PO_OK || cols == 0 || rows == 0 || cols % be != 0)
        return PO_INVALID;
    const uint8_t* w = (const uint8_t*)weights;
    if (type == 0) {
        const float* wf = (const float*)weights;
        for (size_t r = 0; r < rows; ++r) y[r] = 0.0f + po_dot_f32(wf + r * cols, x, cols);
        return PO_OK;
    }
    const size_t bpr = cols / be;
    float decoded[256];
    for (size_t r = 0; r < rows; ++r) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; ++b) {
            const uint8_t* blk = w + (r * bpr + b) * bb;
            if (type == 8) {
                const float d = po_half_to_float(rd16(blk));
                sum += d * po_dot_i8_f32(x + b * 32, (const int8_t*)(blk + 2), 32);
            } else {
                if (type == 12) po_decode_q4_k(blk, decoded);
                else if (type == 13) po_decode_q5_k(blk, decoded);
                else po_decode_q6_k(blk, decoded);
                sum += po_dot_f32(decoded, x + b * 256, 256);
            }
        }
        y[r] = sum;
    }
    return PO_OK;
}

/* Ordering used by both routers: higher logit first, ties to the lower id.
 * src/qwen3_moe_runner.cpp:283-287, src/qwen35_runner.cpp:154-157. */
static int route_before(float la, size_t ia, float lb, size_t ib) {
    return la > lb || (la == lb && ia < ib);
}

/* Insertion top-k of the reference (lower_bound insert, pop_back when full):
 * src/qwen3_moe_runner.cpp:279-293.  Writes ids in rank order. */
static void top_k_insert(const float* logits, size_t n, size_t k, uint32_t* ids) {
    size_t count = 0;
    for (size_t id = 0; id < n; ++id) {
        /* lower_bound: first position whose element is not "before" the candidate */
        size_t where = 0;
        while (where < count && route_before(logits[ids[where]], ids[where], logits[id], id)) ++where;
        if (count < k) {
            for (size_t j = count; j > where; --j) ids[j] = ids[j - 1];
            ids[where] = (uint32_t)id;
            ++count;
        } else if (where < count) {
            for (size_t j = count - 1; j > where; --j) ids[j] = ids[j - 1];
            ids[where] = (uint32_t)id;
        }
    }
}

static int all_finite(const float* v, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(v[i])) return 0;
    return 1;
}

/* Qwen3-MoE routing: full softmax with an FP64 denominator, top-k by insertion,
 * probability exp(l - max) / denominator, optional renormalisation over the
 * selected set.  Restates route_experts, src/qwen3_moe_runner.cpp:267-305.
 * Returns PO_RUNTIME for non-finite logits (the reference throws). */
int po_route_qwen3(const float* logits, size_t n, size_t k, int normalize, uint32_t* ids,
                   float* probs) {
    if (k == 0 || k > n) return PO_INVALID;
    if (!all_finite(logits, n)) return PO_RUNTIME;
    float maximum = logits[0];
    for (size_t i = 1; i < n; ++i)
        if (logits[i] > maximum) maximum = logits[i];
    double denominator = 0.0;
    for (size_t i = 0; i < n; ++i) denominator += exp((double)(logits[i] - maximum));
    top_k_insert(logits, n, k, ids);
    float selected_sum = 0.0f;
    for (size_t i = 0; i < k; ++i) {
        probs[i] = (float)(exp((double)(logits[ids[i]] - maximum)) / denominator);
        selected_sum += probs[i];
    }
    if (normalize)
        for (size_t i = 0; i < k; ++i) probs[i] /= selected_sum;
    return PO_OK;
}

/* Qwen3.5-MoE routing: FP32 softmax over all logits, top-k by insertion,
 * optional renormalisation.  Restates select_experts,
 * src/qwen35_runner.cpp:131-173. */
int po_route_qwen35(const float* logits, size_t n, size_t k, int normalize, uint32_t* ids,
                    float* probs) {
    if (k == 0 || k > n) return PO_INVALID;
    float maximum = logits[0];
    for (size_t i = 1; i < n; ++i)
        if (logits[i] > maximum) maximum = logits[i];
    if (!isfinite(maximum) || !all_finite(logits, n)) return PO_RUNTIME;
    float denominator = 0.0f;
    for (size_t i = 0; i < n; ++i) denominator += expf(logits[i] - maximum);
    if (!isfinite(denominator) || denominator <= 0.0f) return PO_RUNTIME;
    top_k_insert(logits, n, k, ids);
    for (size_t i = 0; i < k; ++i) probs[i] = expf(logits[ids[i]] - maximum) / denominator;
    if (normalize) {
        float sum = 0.0f;
        for (size_t i = 0; i < k; ++i) sum += probs[i];
        if (!isfinite(sum) || sum <= 0.0f) return PO_RUNTIME;
        for (size_t i = 0; i < k; ++i) probs[i] /= sum;
    }
    return PO_OK;
}

/* SiLU as written in the Qwen3-MoE block, src/qwen3_moe_runner.cpp:683. */
static float silu_qwen3(float g) { return g / (1.0f + expf(-g)); }

/* sigmoid / silu of the Qwen3.5 runner, src/qwen35_runner.cpp:111-123. */
float po_sigmoid(float v) {
    if (v >= 0.0f) return 1.0f / (1.0f + expf(-v));
    const float e = expf(v);
    return e / (1.0f + e);
}
static float silu_qwen35(float g) { return g * po_sigmoid(g); }

/* One MoE FFN block for one token.
 *
 * flavour 0 = Qwen3-MoE block, src/qwen3_moe_runner.cpp:643-692
 *   logits = W_r . x (F32), route_experts, per route: g = W_g . x, u = W_u . x,
 *   a = g / (1 + exp(-g)) * u, y = W_d . a, out += p * y.
 * flavour 1 = Qwen3.5-MoE block, src/qwen35_runner.cpp:691-763
 *   select_experts, silu(g) * u, out += (p * expert_weights_scale) * y, then
 *   the shared expert: out = out + sigmoid(w_s . x) * down_s(silu(gate_s x) * up_s x).
 *
 * Expert tensors are the GGUF [H, I, E] / [I, H, E] payloads: expert e's slice
 * starts at e * slice_bytes (split_expert_tensor, src/expert_store.cpp:17-36).
 * `out` receives the MoE contribution (no residual).  ids/probs (k entries)
 * receive the routes in rank order.  act_scratch needs 3 * inter floats and
 * y_scratch `hidden` floats. */
typedef struct po_moe_layer {
    size_t hidden, inter, experts, top_k;
    int flavour, normalize;
    float expert_weights_scale;
    const float* router;          /* F32 [experts, hidden] */
    uint32_t gate_type, up_type, down_type;
    const void* gate;             /* experts slices of [inter rows, hidden cols] */
    const void* up;
    const void* down;             /* experts slices of [hidden rows, inter cols] */
    /* shared expert (flavour 1 only; may be NULL) */
    size_t shared_inter;
    const float* shared_router;   /* F32 [hidden] */
    uint32_t shared_gate_type, shared_up_type, shared_down_type;
    const void* shared_gate;
    const void* shared_up;
    const void* shared_down;
} po_moe_layer;

static size_t row_bytes_of(uint32_t type, size_t cols) {
    size_t be, bb;
    if (po_type_layout(type, &be, &bb) != PO_OK) return 0;
    return cols / be * bb;
}

static int moe_body(const po_moe_layer* L, const float* x, float* out, uint32_t* ids, float* probs,
                    float* logits, float* act_scratch, float* y_scratch, int run_router);

int po_moe_forward(const po_moe_layer* L, const float* x, float* out, uint32_t* ids, float* probs,
                   float* logits, float* act_scratch, float* y_scratch) {
    return moe_body(L, x, out, ids, probs, logits, act_scratch, y_scratch, 1);
}

/* po_moe_forward with the router logits given (`logits`, experts entries)
 * instead of computed from L->router: the routes, experts and combine are
 * the same.  Serves batched-token checks whose logits are inputs. */
int po_moe_forward_routed(const po_moe_layer* L, const float* x, const float* logits, float* out,
                          uint32_t* ids, float* probs, float* act_scratch, float* y_scratch) {
    return moe_body(L, x, out, ids, probs, (float*)logits, act_scratch, y_scratch, 0);
}

static int moe_body(const po_moe_layer* L, const float* x, float* out, uint32_t* ids, float* probs,
                    float* logits, float* act_scratch, float* y_scratch, int run_router) {
    if (!L || !x || !out || L->top_k == 0 || L->top_k > L->experts) return PO_INVALID;
    const size_t H = L->hidden, I = L->inter;
    int st = run_router ? po_linear(0, x, H, L->router, L->experts, logits) : PO_OK;
    if (st) return st;
    st = L->flavour == 0 ? po_route_qwen3(logits, L->experts, L->top_k, L->normalize, ids, probs)
                         : po_route_qwen35(logits, L->experts, L->top_k, L->normalize, ids, probs);
    if (st) return st;
    const size_t gate_slice = row_bytes_of(L->gate_type, H) * I;
    const size_t up_slice = row_bytes_of(L->up_type, H) * I;
    const size_t down_slice = row_bytes_of(L->down_type, I) * H;
    float* g = act_scratch;
    float* u = act_scratch + I;
    float* a = act_scratch + 2 * I;
    for (size_t i = 0; i < H; ++i) out[i] = 0.0f;
    for (size_t r = 0; r < L->top_k; ++r) {
        const size_t e = ids[r];
        st = po_linear(L->gate_type, x, H, (const uint8_t*)L->gate + e * gate_slice, I, g);
        if (!st) st = po_linear(L->up_type, x, H, (const uint8_t*)L->up + e * up_slice, I, u);
        if (st) return st;
        for (size_t i = 0; i < I; ++i)
            a[i] = L->flavour == 0 ? silu_qwen3(g[i]) * u[i] : silu_qwen35(g[i]) * u[i];
        st = po_linear(L->down_type, a, I, (const uint8_t*)L->down + e * down_slice, H, y_scratch);
        if (st) return st;
        const float scale = L->flavour == 0 ? probs[r] : probs[r] * L->expert_weights_scale;
        for (size_t i = 0; i < H; ++i) out[i] += scale * y_scratch[i];
    }
    if (L->flavour == 1 && L->shared_inter && L->shared_router) {
        const size_t SI = L->shared_inter;
        float gate_value = 0.0f;
        st = po_linear(0, x, H, L->shared_router, 1, &gate_value);
        if (!st) st = po_linear(L->shared_gate_type, x, H, L->shared_gate, SI, g);
        if (!st) st = po_linear(L->shared_up_type, x, H, L->shared_up, SI, u);
        if (st) return st;
        for (size_t i = 0; i < SI; ++i) a[i] = silu_qwen35(g[i]) * u[i];
        st = po_linear(L->shared_down_type, a, SI, L->shared_down, H, y_scratch);
        if (st) return st;
        const float shared_scale = po_sigmoid(gate_value);
        for (size_t i = 0; i < H; ++i) out[i] = out[i] + shared_scale * y_scratch[i];
    }
    return PO_OK;
}

/* RMS norm y = x * (1 / sqrt(mean(x^2) + eps)) * w.  Restates rms_norm,
 * src/rms_norm.cpp:9-27 with rms_scale_f32, src/simd_kernels.hpp:109-122. */
void po_rms_norm(const float* x, const float* w, size_t n, float eps, float* y) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += x[i] * x[i];
    const float scale = 1.0f / sqrtf(sum / (float)n + eps);
    for (size_t i = 0; i < n; ++i) y[i] = x[i] * scale * w[i];
}

/* ---------------------------------------------------------------------------
 * Qwen3.5 Gated DeltaNet mixer, one token (the pieces between its
 * projections, src/qwen35_runner.cpp:613-656).
 * ------------------------------------------------------------------------- */

/* softplus of the runner, src/qwen35_runner.cpp:117-121. */
float po_softplus(float v) {
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return log1pf(expf(v));
}

/* Depthwise causal convolution step with SiLU, restating
 * causal_depthwise_conv1d_step, src/causal_conv1d.cpp:25-50: input and
 * output may alias; state holds the last kernel - 1 inputs per channel. */
void po_causal_conv1d_step(const float* input, const float* weights, size_t channels, size_t kernel,
                           float* state, float* output) {
    const size_t sl = kernel - 1;
    for (size_t c = 0; c < channels; ++c) {
        const size_t wo = c * kernel, so = c * sl;
        float sum = input[c] * weights[wo + sl];
        for (size_t t = 0; t < sl; ++t) sum += state[so + t] * weights[wo + t];
        if (sl) {
            for (size_t t = 0; t + 1 < sl; ++t) state[so + t] = state[so + t + 1];
            state[so + sl - 1] = input[c];
        }
        /* silu with the sign branch, src/causal_conv1d.cpp:17-21 */
        float s;
        if (sum >= 0.0f) s = sum / (1.0f + expf(-sum));
        else {
            const float e = expf(sum);
            s = sum * e / (1.0f + e);
        }
        output[c] = s;
    }
}

/* The per-head decay and update gate of the mixer, src/qwen35_runner.cpp:633-642:
 * log_decay = a * softplus(alpha + dt_bias), beta = sigmoid(beta_raw). */
void po_delta_gates(const float* a, const float* dt_bias, const float* alpha, const float* beta_raw,
                    size_t heads, float* log_decay, float* beta) {
    for (size_t h = 0; h < heads; ++h) {
        log_decay[h] = a[h] * po_softplus(alpha[h] + dt_bias[h]);
        beta[h] = po_sigmoid(beta_raw[h]);
    }
}

/* Restates gated_delta_recurrent_step_grouped, src/gated_delta_net.cpp:28-110:
 * L2-normalised q (times 1/sqrt(dk)) and k per key head, value head h uses key
 * head h % key_heads; state[h][v][k] decays, then delta = (v - state.k) * beta,
 * state += k delta, out = state.q.  Returns 1 (nothing changed) for an invalid
 * decay or gate, where the reference throws. */
int po_gated_delta_step(const float* query, const float* key, const float* value, const float* log_decay,
                        const float* beta, size_t key_heads, size_t value_heads, size_t dk, size_t dv,
                        float* state, float* output) {
    for (size_t h = 0; h < value_heads; ++h)
        if (!isfinite(log_decay[h]) || log_decay[h] > 0.0f || !isfinite(beta[h]) || beta[h] < 0.0f ||
            beta[h] > 1.0f)
            return 1;
    float* nq = (float*)malloc(key_heads * dk * sizeof(float));
    float* nk = (float*)malloc(key_heads * dk * sizeof(float));
    float* delta = (float*)malloc(dv * sizeof(float));
    if (!nq || !nk || !delta) {
        free(nq); free(nk); free(delta);
        return 2;
    }
    const float qs = 1.0f / sqrtf((float)dk);
    for (size_t h = 0; h < key_heads; ++h) {
        float sq = 0.0f, sk = 0.0f;
        for (size_t i = 0; i < dk; ++i) {
            sq += query[h * dk + i] * query[h * dk + i];
            sk += key[h * dk + i] * key[h * dk + i];
        }
        const float iq = 1.0f / sqrtf(sq + 1.0e-6f), ik = 1.0f / sqrtf(sk + 1.0e-6f);
        for (size_t i = 0; i < dk; ++i) {
            nq[h * dk + i] = query[h * dk + i] * iq * qs;
            nk[h * dk + i] = key[h * dk + i] * ik;
        }
    }
    for (size_t h = 0; h < value_heads; ++h) {
        const float* q = nq + (h % key_heads) * dk;
        const float* k = nk + (h % key_heads) * dk;
        float* S = state + h * dv * dk;
        const float decay = expf(log_decay[h]);
        for (size_t i = 0; i < dv * dk; ++i) S[i] *= decay;
        for (size_t v = 0; v < dv; ++v) {
            float mem = 0.0f;
            for (size_t i = 0; i < dk; ++i) mem += S[v * dk + i] * k[i];
            delta[v] = (value[h * dv + v] - mem) * beta[h];
            output[h * dv + v] = 0.0f;
        }
        for (size_t v = 0; v < dv; ++v)
            for (size_t i = 0; i < dk; ++i) {
                float* cell = &S[v * dk + i];
                *cell += k[i] * delta[v];
                output[h * dv + v] += *cell * q[i];
            }
    }
    free(nq); free(nk); free(delta);
    return 0;
}

/* Restates rms_norm_gated, src/rms_norm.cpp:46-74: per row of `width`,
 * y = x * (1 / sqrt(mean(x^2) + eps)) * w * (g * sigmoid(g)). */
void po_rms_norm_gated(const float* x, const float* w, const float* gate, size_t rows, size_t width, float eps,
                       float* y) {
    for (size_t r = 0; r < rows; ++r) {
        const float* xr = x + r * width;
        float sum = 0.0f;
        for (size_t i = 0; i < width; ++i) sum += xr[i] * xr[i];
        const float scale = 1.0f / sqrtf(sum / (float)width + eps);
        for (size_t i = 0; i < width; ++i) {
            const float g = gate[r * width + i];
            const float sg = g >= 0.0f ? 1.0f / (1.0f + expf(-g)) : expf(g) / (1.0f + expf(g));
            y[r * width + i] = xr[i] * scale * w[i] * (g * sg);
        }
    }
}
