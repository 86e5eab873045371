/*
 * pokit_cuda.h -- C ABI of the B200 (sm_100a) backend for the PokitLMs MoE
 * expert path.
 *
 * Conventions follow PokitLMs' own C API (include/pokitlms/pokitlms.h):
 *   - status codes mirror pokitlms_status (pokitlms.h:18-24);
 *   - every call that can fail takes (error_buffer, error_capacity); the text is
 *     truncated and NUL-terminated, and set to "" on success (c_api.cpp:22-27);
 *   - no C++ exception crosses this boundary (c_api.cpp:92-101);
 *   - calls on one handle must be serialised (pokitlms.h:81);
 *   - the library owns every device allocation it makes; callers own their
 *     host buffers and any device buffers they pass in.
 *
 * Pointers documented as "device" must be CUDA device pointers on the handle's
 * device; "host" pointers are ordinary (pageable or pinned) host memory.
 * `stream` is a cudaStream_t (NULL = the handle's own stream, or the legacy
 * default stream for handle-free calls).
 *
 * GGML type ids: 0 = F32, 8 = Q8_0, 12 = Q4_K, 13 = Q5_K, 14 = Q6_K.
 */
#ifndef POKIT_CUDA_H
#define POKIT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define POKIT_CUDA_VERSION_MAJOR 0
#define POKIT_CUDA_VERSION_MINOR 1
#define POKIT_CUDA_VERSION_PATCH 0

/* Mirrors pokitlms_status (include/pokitlms/pokitlms.h:18-24). */
typedef enum pokit_cuda_status {
    POKIT_CUDA_STATUS_OK = 0,
    POKIT_CUDA_STATUS_INVALID_ARGUMENT = 1,
    POKIT_CUDA_STATUS_RUNTIME_ERROR = 2,
    POKIT_CUDA_STATUS_BUFFER_TOO_SMALL = 3,
    POKIT_CUDA_STATUS_INTERNAL_ERROR = 4
} pokit_cuda_status;

/* Library version string; replaces pokitlms_version (pokitlms.h:14) for this backend. */
const char* pokit_cuda_version(void);

/* ------------------------------------------------------------------------ */
/* Per-matrix kernels on device memory                                      */
/* ------------------------------------------------------------------------ */

/* output[rows] = W[rows, cols] . input[cols] with W in its GGUF block encoding
 * (row-major, row r at r * row_bytes).  FP32 input, FP32 accumulation.
 * Replaces linear_q8_0 / linear_q4_k / linear_q5_k / linear_q6_k
 * (include/pokitlms/ops/quantized_linear.hpp:23-53) and linear() for F32
 * (include/pokitlms/ops/linear.hpp:10-14), without the bias term.
 * All pointers are device pointers; asynchronous on `stream`. */
pokit_cuda_status pokit_cuda_linear(uint32_t ggml_type, const void* weights, size_t rows,
                                    size_t cols, const float* input, float* output,
                                    void* stream, char* error_buffer, size_t error_capacity);

/* Decodes rows x cols GGUF-encoded weights to FP32 (output row-major), bit-identical
 * to dequantize_quantized_row (include/pokitlms/ops/quantized_linear.hpp:11-13).
 * Device pointers; asynchronous on `stream`. */
pokit_cuda_status pokit_cuda_dequantize_rows(uint32_t ggml_type, const void* encoded,
                                             size_t rows, size_t cols, float* output,
                                             void* stream, char* error_buffer,
                                             size_t error_capacity);

/* Softmax top-k routing of `n` device logits, on device.
 * flavour 0 = Qwen3-MoE route_experts (src/qwen3_moe_runner.cpp:267-305, FP64
 * denominator); flavour 1 = Qwen3.5 select_experts (src/qwen35_runner.cpp:131-173,
 * FP32) with weights multiplied by expert_weights_scale.  Ties go to the lower
 * id.  ids_out/weights_out: device arrays of top_k entries.  status_out (device
 * uint32, may be NULL) is OR-ed with 1 for non-finite logits and 2 for an
 * invalid softmax, where the reference throws. */
pokit_cuda_status pokit_cuda_route_experts(const float* logits, size_t n, size_t top_k,
                                           uint32_t flavour, int normalize,
                                           float expert_weights_scale, uint32_t* ids_out,
                                           float* weights_out, uint32_t* status_out,
                                           void* stream, char* error_buffer,
                                           size_t error_capacity);

/* Fills `nblocks` GGUF blocks of `ggml_type` at device address `dst` with the
 * library's seeded synthetic generator (the same bytes as
 * pokitlms_b200.synth.synth_blocks on the host).  Benchmark/test utility: no
 * counterpart in the reference. */
pokit_cuda_status pokit_cuda_synthesize_blocks(uint32_t ggml_type, uint64_t seed,
                                               uint64_t stream_id, size_t nblocks, void* dst,
                                               void* stream, char* error_buffer,
                                               size_t error_capacity);

/* ------------------------------------------------------------------------ */
/* TensorLinearBackend seam with host spans                                 */
/* ------------------------------------------------------------------------ */

/* Device counterpart of model::TensorLinearBackend
 * (include/pokitlms/model/tensor_linear.hpp:11-18) and sibling of
 * gpu::VulkanLinearBackend (include/pokitlms/gpu/vulkan_linear.hpp:69-84).
 * Plain try_linear streams the weight payload to the device on every call, as
 * the Vulkan backend does for readers without a model file
 * (vulkan_linear.cpp:516-563, 705-714): a host address is not an identity once
 * the caller frees and reuses its buffer.  try_linear_cached keeps payloads in
 * HBM under a key the caller chooses (the tensor's GGUF file offset, say: the
 * Vulkan backend's whole-model device cache), least recently used first out
 * beyond the cache capacity (default 16 GiB). */
typedef struct pokit_cuda_linear_backend pokit_cuda_linear_backend;

/* Mirrors the fields of VulkanLinearStats (vulkan_linear.hpp:41-67) that apply. */
typedef struct pokit_cuda_linear_stats {
    uint64_t linear_calls;
    uint64_t dispatches;
    uint64_t q4_k_dispatches;
    uint64_t q5_k_dispatches;
    uint64_t q6_k_dispatches;
    uint64_t q8_0_dispatches;
    uint64_t other_dispatches;
    uint64_t weight_bytes;            /* bytes streamed by the kernels */
    uint64_t gpu_time_ns;             /* CUDA-event time of the kernels */
    uint64_t model_cache_capacity_bytes;  /* bytes held in HBM by try_linear_cached now */
    uint64_t model_cache_uploaded_bytes;
    uint64_t model_cache_upload_time_ns;
} pokit_cuda_linear_stats;

pokit_cuda_status pokit_cuda_linear_backend_create(int device, pokit_cuda_linear_backend** out,
                                                   char* error_buffer, size_t error_capacity);
void pokit_cuda_linear_backend_destroy(pokit_cuda_linear_backend* backend);

/* try_linear (tensor_linear.hpp:16-17): output[rows] = W . input, host spans.
 * *handled = 1 when the type is supported (F32/Q8_0/Q4_K/Q5_K/Q6_K) and the
 * result was written; 0 for other types (the caller's CPU path then runs, as
 * with the Vulkan backend).  Execution failures return RUNTIME_ERROR and leave
 * the backend failed (sticky, like vulkan_linear.cpp:636, 731-735). */
pokit_cuda_status pokit_cuda_linear_backend_try_linear(
    pokit_cuda_linear_backend* backend, uint32_t ggml_type, const void* weights_host,
    size_t weights_bytes, size_t rows, size_t cols, const float* input_host,
    float* output_host, int* handled, char* error_buffer, size_t error_capacity);

/* try_linear with the payload cached in HBM under weights_key: the first call
 * with a key uploads the payload, later calls with that key use the device
 * copy and do not read weights_host (which may then be NULL; weights_bytes
 * must still give the payload's size).  A key reused for a matrix of
 * another type or shape is INVALID_ARGUMENT; a payload larger than the cache
 * capacity is streamed instead.  The caller must forget (or never reuse) a key
 * whose bytes change. */
pokit_cuda_status pokit_cuda_linear_backend_try_linear_cached(
    pokit_cuda_linear_backend* backend, uint64_t weights_key, uint32_t ggml_type,
    const void* weights_host, size_t weights_bytes, size_t rows, size_t cols,
    const float* input_host, float* output_host, int* handled, char* error_buffer,
    size_t error_capacity);

/* 1 when a payload is cached under weights_key, else 0 (also for a NULL backend). */
int pokit_cuda_linear_backend_is_cached(const pokit_cuda_linear_backend* backend, uint64_t weights_key);

/* Bytes of payload try_linear_cached may keep in HBM (evicts down to it now). */
pokit_cuda_status pokit_cuda_linear_backend_set_cache_capacity(pokit_cuda_linear_backend* backend,
                                                               uint64_t capacity_bytes,
                                                               char* error_buffer,
                                                               size_t error_capacity);

/* Drops the payload cached under weights_key; *was_cached (may be NULL) = 1 if
 * there was one. */
pokit_cuda_status pokit_cuda_linear_backend_forget(pokit_cuda_linear_backend* backend,
                                                   uint64_t weights_key, int* was_cached,
                                                   char* error_buffer, size_t error_capacity);

pokit_cuda_status pokit_cuda_linear_backend_get_stats(const pokit_cuda_linear_backend* backend,
                                                      pokit_cuda_linear_stats* out_stats);

/* ------------------------------------------------------------------------ */
/* MoE FFN block with an HBM-resident expert pool                          */
/* ------------------------------------------------------------------------ */

typedef struct pokit_cuda_moe pokit_cuda_moe;

typedef enum pokit_cuda_moe_flavour {
    POKIT_CUDA_MOE_QWEN3 = 0,   /* src/qwen3_moe_runner.cpp:643-692 */
    POKIT_CUDA_MOE_QWEN35 = 1   /* src/qwen35_runner.cpp:691-763 (shared expert) */
} pokit_cuda_moe_flavour;

/* Tensor selector for per-tensor upload/synthesis/views. */
typedef enum pokit_cuda_moe_tensor {
    POKIT_CUDA_MOE_ROUTER = 0,        /* F32 [experts, hidden]  (ffn_gate_inp) */
    POKIT_CUDA_MOE_GATE = 1,          /* [hidden, inter, experts] (ffn_gate_exps) */
    POKIT_CUDA_MOE_UP = 2,            /* [hidden, inter, experts] (ffn_up_exps) */
    POKIT_CUDA_MOE_DOWN = 3,          /* [inter, hidden, experts] (ffn_down_exps) */
    POKIT_CUDA_MOE_FFN_NORM = 4,      /* F32 [hidden] (ffn_norm), decode chain only */
    POKIT_CUDA_MOE_SHARED_ROUTER = 5, /* F32 [hidden] (ffn_gate_inp_shexp) */
    POKIT_CUDA_MOE_SHARED_GATE = 6,   /* [hidden, shared_inter] (ffn_gate_shexp) */
    POKIT_CUDA_MOE_SHARED_UP = 7,     /* [hidden, shared_inter] (ffn_up_shexp) */
    POKIT_CUDA_MOE_SHARED_DOWN = 8    /* [shared_inter, hidden] (ffn_down_shexp) */
} pokit_cuda_moe_tensor;

typedef struct pokit_cuda_moe_config {
    int device;                       /* CUDA device ordinal */
    size_t layers;                    /* MoE blocks held by the pool */
    size_t hidden;                    /* embedding_length, multiple of 256 */
    size_t inter;                     /* expert_feed_forward_length, multiple of 256 */
    size_t experts;                   /* expert_count (<= 1024) */
    size_t top_k;                     /* experts_per_token (<= 64) */
    uint32_t flavour;                 /* pokit_cuda_moe_flavour */
    int normalize_top_k;              /* expert_weights_norm */
    float expert_weights_scale;       /* Qwen3.5 expert_weights_scale (1 for Qwen3) */
    float rms_epsilon;                /* layer_norm_rms_epsilon for the decode chain */
    uint32_t gate_type, up_type, down_type;
    const uint32_t* layer_down_types; /* optional [layers] override of down_type */
    size_t shared_inter;              /* 0 = no shared expert */
    uint32_t shared_gate_type, shared_up_type, shared_down_type;
    /* Expert parallelism: the handle holds experts [expert_first,
     * expert_first + expert_count) of every layer (expert_count 0 = all).
     * The router stays whole; a sharded handle serves the batched forward
     * only and returns the contribution of its experts (the partial sums of
     * all shards add up to the block's output). */
    size_t expert_first;
    size_t expert_count;
} pokit_cuda_moe_config;

/* Host payloads of one layer in GGUF layout.  NULL entries are skipped. */
typedef struct pokit_cuda_moe_layer_host {
    const float* router;
    const void* gate;
    const void* up;
    const void* down;
    const float* ffn_norm;
    const float* shared_router;
    const void* shared_gate;
    const void* shared_up;
    const void* shared_down;
} pokit_cuda_moe_layer_host;

/* First seven fields mirror pokitlms_expert_cache_stats (pokitlms.h:36-44):
 * the pool holds every expert, so hits count every routed lookup and misses
 * stay 0.  bytes_read/read_operations/read_time_ns count host->HBM uploads. */
typedef struct pokit_cuda_moe_stats {
    size_t capacity_bytes;
    size_t resident_bytes;
    uint64_t bytes_read;
    uint64_t read_operations;
    uint64_t read_time_ns;
    uint64_t hits;
    uint64_t misses;
    uint64_t forward_calls;           /* MoE blocks executed */
    uint64_t kernel_launches;         /* this library's kernels launched */
} pokit_cuda_moe_stats;

/* Creates a handle and reserves the expert pool for config->layers blocks in
 * one HBM allocation (replaces the per-layer ExpertStores built in
 * Qwen3MoeRunner::Impl::Impl, src/qwen3_moe_runner.cpp:481-523). */
pokit_cuda_status pokit_cuda_moe_create(const pokit_cuda_moe_config* config,
                                        pokit_cuda_moe** out_moe, char* error_buffer,
                                        size_t error_capacity);
void pokit_cuda_moe_destroy(pokit_cuda_moe* moe);

/* Uploads one tensor of `layer` from host memory; bytes must equal the
 * tensor's GGUF payload size.  Expert tensors are the whole [.., .., experts]
 * payload; expert e is the contiguous slice at e * payload/experts
 * (split_expert_tensor, src/expert_store.cpp:17-36).  Synchronous. */
pokit_cuda_status pokit_cuda_moe_upload_tensor(pokit_cuda_moe* moe, size_t layer,
                                               uint32_t tensor, const void* host_bytes,
                                               size_t bytes, char* error_buffer,
                                               size_t error_capacity);

/* Uploads every non-NULL tensor of `layer`.  Synchronous. */
pokit_cuda_status pokit_cuda_moe_upload_layer(pokit_cuda_moe* moe, size_t layer,
                                              const pokit_cuda_moe_layer_host* tensors,
                                              char* error_buffer, size_t error_capacity);

/* Fills a quantised tensor of `layer` on the device with the synthetic block
 * generator (seed, stream_id).  Benchmark utility; no counterpart in the reference. */
pokit_cuda_status pokit_cuda_moe_synthesize_tensor(pokit_cuda_moe* moe, size_t layer,
                                                   uint32_t tensor, uint64_t seed,
                                                   uint64_t stream_id, char* error_buffer,
                                                   size_t error_capacity);

/* Device view of one expert slice (replaces ExpertStore::get,
 * include/pokitlms/storage/expert_store.hpp:39): matrix is
 * POKIT_CUDA_MOE_GATE/UP/DOWN; writes the slice's device address and size. */
pokit_cuda_status pokit_cuda_moe_expert_view(const pokit_cuda_moe* moe, size_t layer,
                                             uint32_t matrix, size_t expert,
                                             const void** device_ptr, size_t* bytes);

/* One MoE block on device pointers -- the layer-level seam the runners' MoE
 * blocks call (src/qwen3_moe_runner.cpp:645-691, src/qwen35_runner.cpp:691-763):
 * output[hidden] = sum_k w_k * down_k(silu(gate_k x) * up_k x) (+ shared expert),
 * without the residual.  route_ids/route_weights (device, top_k entries each,
 * may be NULL) receive the chosen experts in rank order and their combine
 * weights.  Asynchronous: a router failure (non-finite logits) is reported by
 * the next pokit_cuda_moe_synchronize or *_host call. */
pokit_cuda_status pokit_cuda_moe_forward(pokit_cuda_moe* moe, size_t layer, const float* input,
                                         float* output, uint32_t* route_ids,
                                         float* route_weights, void* stream,
                                         char* error_buffer, size_t error_capacity);

/* Activation element type of a batched forward's input rows. */
typedef enum pokit_cuda_input_type {
    POKIT_CUDA_INPUT_F32 = 0,
    POKIT_CUDA_INPUT_BF16 = 1
} pokit_cuda_input_type;

/* A batch of `tokens` (1..65536) rows through one MoE block on device
 * pointers: output[t] = MoE(input[t]) for each row independently, the same
 * block as pokit_cuda_moe_forward (the reference runs a prompt's tokens one
 * forward_into call at a time, src/qwen3_moe_runner.cpp:785-790).
 * input: [tokens][hidden] of input_type.  router_logits (may be NULL):
 * [tokens][experts] F32 logits to route by instead of the layer's router.
 * route_ids / route_weights (may be NULL): [tokens][top_k].
 * Layers with Q4_K gate/up/down experts and no shared expert run the
 * grouped-expert tensor-core GEMM (tokens sorted by expert, one GEMM tile per
 * <= 64 tokens of an expert); other layers run the single-token block per row
 * and then require F32 input and router_logits == NULL.  Asynchronous. */
pokit_cuda_status pokit_cuda_moe_forward_batch(pokit_cuda_moe* moe, size_t layer, const void* input,
                                               uint32_t input_type, size_t tokens,
                                               const float* router_logits, float* output,
                                               uint32_t* route_ids, float* route_weights, void* stream,
                                               char* error_buffer, size_t error_capacity);

/* Expert parallelism over peer memory (no counterpart in the reference, which
 * runs on one device; the north star shards the experts over the GPUs of one
 * box).  One process per GPU, each with an expert-shard handle
 * (expert_first / expert_count) of the same model, calling
 * pokit_cuda_moe_forward_batch on the same rows in the same order.  After
 * pokit_cuda_moe_exchange_create on every rank (it returns this rank's
 * POKIT_CUDA_IPC_HANDLE_BYTES-byte CUDA IPC handle) and
 * pokit_cuda_moe_exchange_connect with all ranks' handles in rank order, a
 * grouped-path forward_batch of <= max_tokens rows returns the whole block's
 * output on every rank: its last kernel stores the shard's partial sums into
 * every rank's region over NVLink, raises a flag there, waits for the other
 * ranks' flags (at most ~1 s, then a sticky RUNTIME_ERROR) and adds the
 * ranks' partials in rank order.  Every rank must make the same forward_batch
 * calls (as with a collective); pokit_cuda_moe_time_batch stays local. */
#define POKIT_CUDA_IPC_HANDLE_BYTES 64
pokit_cuda_status pokit_cuda_moe_exchange_create(pokit_cuda_moe* moe, size_t world, size_t rank,
                                                 size_t max_tokens, void* ipc_handle_out,
                                                 char* error_buffer, size_t error_capacity);
pokit_cuda_status pokit_cuda_moe_exchange_connect(pokit_cuda_moe* moe, const void* ipc_handles,
                                                  char* error_buffer, size_t error_capacity);
/* Unmaps the other ranks' regions (waiting for this handle's work first) and
 * returns forward_batch to this rank's partial output.  Call it on every rank
 * before any rank destroys its handle: a rank's region must not be freed
 * while another process still maps it.  Allowed on a failed handle. */
pokit_cuda_status pokit_cuda_moe_exchange_disconnect(pokit_cuda_moe* moe, char* error_buffer,
                                                     size_t error_capacity);

/* Measurement hook for benchmarks (no counterpart in the reference): runs the
 * grouped-path batched forward `repetitions` times on device buffers with an
 * event between its kernels and writes the average device time (us) of each
 * stage to stage_us: [router,] route, group, pack activations, gate/up GEMM,
 * pack intermediate, down GEMM, combine (*stages = 8, or 7 when router_logits
 * is given).  INVALID_ARGUMENT for layers off the grouped path. */
pokit_cuda_status pokit_cuda_moe_time_batch(pokit_cuda_moe* moe, size_t layer, const void* input,
                                            uint32_t input_type, size_t tokens,
                                            const float* router_logits, float* output,
                                            uint32_t repetitions, float* stage_us,
                                            size_t stage_capacity, size_t* stages, void* stream,
                                            char* error_buffer, size_t error_capacity);

/* Host-span variant of pokit_cuda_moe_forward_batch: copies in, runs, copies
 * out and synchronises (RUNTIME_ERROR for non-finite router logits). */
pokit_cuda_status pokit_cuda_moe_forward_batch_host(pokit_cuda_moe* moe, size_t layer,
                                                    const void* input_host, uint32_t input_type,
                                                    size_t tokens, const float* router_logits_host,
                                                    float* output_host, uint32_t* route_ids_host,
                                                    float* route_weights_host, char* error_buffer,
                                                    size_t error_capacity);

/* Measurement hook for benchmarks: the average device time (microseconds) of
 * one launch of a tensor-core path kernel (kernel 0: the Q4_K gate/up matvec,
 * 1: the down matvec and combine), launched `repetitions` times back to back
 * over layers [first_layer, first_layer + layer_count) cyclically, as in a
 * decode chain (replayed from a CUDA graph, timed with CUDA events).  The routes are those of one forward of first_layer on the
 * contents of `work` (device, hidden floats), which also receives outputs.
 * INVALID_ARGUMENT when a layer does not use the tensor-core path. */
pokit_cuda_status pokit_cuda_moe_time_kernel(pokit_cuda_moe* moe, uint32_t kernel, size_t first_layer,
                                             size_t layer_count, uint32_t repetitions, float* work,
                                             void* stream, float* average_us, char* error_buffer,
                                             size_t error_capacity);

/* Host-span variant of pokit_cuda_moe_forward: copies in, runs, copies out and
 * synchronises; returns RUNTIME_ERROR (nothing written to output) when the
 * router produced non-finite logits, as the reference throws. */
pokit_cuda_status pokit_cuda_moe_forward_host(pokit_cuda_moe* moe, size_t layer,
                                              const float* input_host, float* output_host,
                                              uint32_t* route_ids_host,
                                              float* route_weights_host, char* error_buffer,
                                              size_t error_capacity);

/* Decode chain over layers [first, first + count) on a device hidden state:
 * hidden += MoE_l(rms_norm(hidden, ffn_norm_l)) per layer (the FFN half of
 * src/qwen3_moe_runner.cpp:643-692).  Captured once into a CUDA graph per
 * (first, count, hidden) and replayed.  Asynchronous. */
pokit_cuda_status pokit_cuda_moe_decode_layers(pokit_cuda_moe* moe, size_t first, size_t count,
                                               float* hidden, void* stream,
                                               char* error_buffer, size_t error_capacity);

/* Host-span decode chain: copies hidden_in (host) to the device, runs the
 * chain, copies the result to hidden_out (host) and synchronises. */
pokit_cuda_status pokit_cuda_moe_decode_layers_host(pokit_cuda_moe* moe, size_t first,
                                                    size_t count, const float* hidden_in,
                                                    float* hidden_out, char* error_buffer,
                                                    size_t error_capacity);

/* Measurement hook (no counterpart in the reference): one
 * pokit_cuda_moe_decode_layers call through the persistent decode-chain
 * kernel, which also writes per-phase stamps to `stamps` (device, count x
 * grid x 16 words: for layer l and CTA c at (l * grid + c) * 16 + i the
 * globaltimer (ns) and at + 8 + i the SM clock (cycles), i = route wait
 * done, routes and x records ready, gate/up products done, act published, act
 * wait done, down records built, down products combined, router partials
 * published).  *grid receives the
 * kernel's CTA count.  INVALID_ARGUMENT when the layers do not run the chain
 * kernel.  Asynchronous. */
pokit_cuda_status pokit_cuda_moe_trace_decode(pokit_cuda_moe* moe, size_t first, size_t count, float* hidden,
                                              uint64_t* stamps, size_t stamp_capacity, uint32_t* grid,
                                              void* stream, char* error_buffer, size_t error_capacity);

/* Waits for the handle's work and reports (then clears) any device-side router
 * failure; a CUDA error is sticky and fails every later call. */
pokit_cuda_status pokit_cuda_moe_synchronize(pokit_cuda_moe* moe, void* stream,
                                             char* error_buffer, size_t error_capacity);

pokit_cuda_status pokit_cuda_moe_get_stats(const pokit_cuda_moe* moe,
                                           pokit_cuda_moe_stats* out_stats);

/* Bytes of one tensor's payload for this handle's configuration (0 if the
 * tensor does not exist in this configuration). */
size_t pokit_cuda_moe_tensor_bytes(const pokit_cuda_moe* moe, size_t layer, uint32_t tensor);

/* ------------------------------------------------------------------------ */
/* The whole Qwen3-MoE decoder of one sequence                              */
/* ------------------------------------------------------------------------ */

/* Replaces Qwen3MoeRunner (include/pokitlms/model/qwen3_moe_runner.hpp:56-101)
 * for greedy decoding on one GPU: token embedding, per layer RMSNorm -> Q/K/V
 * projections -> per-head Q/K RMSNorm -> rotate-half RoPE -> FP16 ring KV cache
 * -> GQA attention -> output projection + residual -> the MoE block, then the
 * final RMSNorm, the LM head and the argmax (src/qwen3_moe_runner.cpp:580-704,
 * 751-821).  Every weight is resident in HBM; the MoE tensors (router,
 * ffn_norm, experts) live in the handle returned by pokit_cuda_decoder_moe and
 * are uploaded or synthesised with the pokit_cuda_moe_* calls.
 *
 * With arch = POKIT_CUDA_ARCH_QWEN35MOE the same handle replaces Qwen35Runner
 * (include/pokitlms/model/qwen35_runner.hpp:56-100) for the Qwen3.5-MoE hybrid
 * (src/qwen35_runner.cpp:538-777): layer l is full attention when
 * (l + 1) % full_attention_interval == 0 (gated query: sigmoid(gate) times the
 * attention output, partial MRoPE over rotary_dim dimensions), otherwise a
 * Gated DeltaNet layer (attn_qkv / attn_gate / ssm_alpha / ssm_beta
 * projections, causal conv1d, the gated delta rule, gated RMSNorm, ssm_out);
 * the MoE blocks carry the sigmoid-gated shared expert. */
typedef struct pokit_cuda_decoder pokit_cuda_decoder;

typedef enum pokit_cuda_decoder_arch {
    POKIT_CUDA_ARCH_QWEN3MOE = 0,     /* general.architecture "qwen3moe" */
    POKIT_CUDA_ARCH_QWEN35MOE = 1     /* general.architecture "qwen35moe" */
} pokit_cuda_decoder_arch;

typedef struct pokit_cuda_decoder_config {
    int device;
    size_t layers;                    /* block_count */
    size_t hidden;                    /* embedding_length, multiple of 256 */
    size_t vocab;                     /* tokenizer vocabulary size */
    size_t q_heads, kv_heads;         /* attention.head_count(_kv) */
    size_t head_dim;                  /* key_length = value_length = rope dimension */
    size_t experts, top_k, expert_inter;
    size_t context;                   /* context_length: positions 0 .. context - 1 */
    size_t kv_window;                 /* KV ring capacity; 0 = min(context, 512), the reference's default */
    float rms_epsilon;                /* attention.layer_norm_rms_epsilon */
    float rope_theta;                 /* rope.freq_base */
    int normalize_top_k;              /* expert_weights_norm */
    uint32_t eos_token;               /* tokenizer.ggml.eos_token_id: generation stops after it */
    uint32_t attn_type;               /* GGML type of attn_q/k/v/output */
    uint32_t expert_type;             /* GGML type of the routed experts */
    uint32_t embed_type;              /* GGML type of token_embd */
    uint32_t output_type;             /* GGML type of output (the LM head) */
    /* Qwen3.5-MoE hybrid (arch = POKIT_CUDA_ARCH_QWEN35MOE); zero for qwen3moe. */
    uint32_t arch;                    /* pokit_cuda_decoder_arch */
    size_t rotary_dim;                /* rope.dimension_count: even, <= head_dim */
    uint32_t rope_sections[4];        /* rope.dimension_sections (text positions) */
    size_t full_attention_interval;   /* full_attention_interval */
    size_t ssm_conv_kernel;           /* ssm.conv_kernel */
    size_t ssm_state_size;            /* ssm.state_size: linear key head dimension */
    size_t ssm_group_count;           /* ssm.group_count: linear key heads */
    size_t ssm_time_step_rank;        /* ssm.time_step_rank: linear value heads */
    size_t ssm_inner_size;            /* ssm.inner_size: value heads x value head dimension */
    float expert_weights_scale;       /* expert_weights_scale */
    size_t shared_inter;              /* expert_shared_feed_forward_length */
    uint32_t shared_type;             /* GGML type of the shared expert tensors */
    const uint32_t* layer_down_types; /* optional [layers] routed down types (NULL: expert_type) */
} pokit_cuda_decoder_config;

/* Decoder tensors outside the MoE blocks (GGUF names in comments). */
typedef enum pokit_cuda_decoder_tensor {
    POKIT_CUDA_DEC_TOKEN_EMBD = 0,    /* token_embd.weight   [hidden, vocab] */
    POKIT_CUDA_DEC_OUTPUT_NORM = 1,   /* output_norm.weight  F32 [hidden] */
    POKIT_CUDA_DEC_OUTPUT = 2,        /* output.weight       [hidden, vocab] */
    POKIT_CUDA_DEC_ATTN_NORM = 3,     /* blk.L.attn_norm.weight   F32 [hidden] */
    POKIT_CUDA_DEC_ATTN_Q = 4,        /* blk.L.attn_q.weight      [hidden, q_heads * head_dim] */
    POKIT_CUDA_DEC_ATTN_Q_NORM = 5,   /* blk.L.attn_q_norm.weight F32 [head_dim] */
    POKIT_CUDA_DEC_ATTN_K = 6,        /* blk.L.attn_k.weight      [hidden, kv_heads * head_dim] */
    POKIT_CUDA_DEC_ATTN_K_NORM = 7,   /* blk.L.attn_k_norm.weight F32 [head_dim] */
    POKIT_CUDA_DEC_ATTN_V = 8,        /* blk.L.attn_v.weight      [hidden, kv_heads * head_dim] */
    POKIT_CUDA_DEC_ATTN_OUTPUT = 9,   /* blk.L.attn_output.weight [q_heads * head_dim, hidden] */
    /* Qwen3.5: attn_q is [hidden, q_heads * head_dim * 2] (per head: query,
     * then gate); the tensors below exist on Gated DeltaNet layers only. */
    POKIT_CUDA_DEC_SSM_QKV = 10,      /* blk.L.attn_qkv.weight  [hidden, 2 * key width + ssm_inner_size] */
    POKIT_CUDA_DEC_SSM_GATE = 11,     /* blk.L.attn_gate.weight [hidden, ssm_inner_size] */
    POKIT_CUDA_DEC_SSM_ALPHA = 12,    /* blk.L.ssm_alpha.weight [hidden, ssm_time_step_rank] */
    POKIT_CUDA_DEC_SSM_BETA = 13,     /* blk.L.ssm_beta.weight  [hidden, ssm_time_step_rank] */
    POKIT_CUDA_DEC_SSM_CONV1D = 14,   /* blk.L.ssm_conv1d.weight F32 [conv_kernel, channels] */
    POKIT_CUDA_DEC_SSM_A = 15,        /* blk.L.ssm_a             F32 [ssm_time_step_rank] */
    POKIT_CUDA_DEC_SSM_DT_BIAS = 16,  /* blk.L.ssm_dt.bias       F32 [ssm_time_step_rank] */
    POKIT_CUDA_DEC_SSM_NORM = 17,     /* blk.L.ssm_norm.weight   F32 [value head dimension] */
    POKIT_CUDA_DEC_SSM_OUT = 18       /* blk.L.ssm_out.weight    [ssm_inner_size, hidden] */
} pokit_cuda_decoder_tensor;

/* Mirrors GenerationStats (qwen3_moe_runner.hpp:33-37). */
typedef struct pokit_cuda_generation_stats {
    uint64_t prefill_time_ns;
    uint64_t decode_time_ns;
    size_t generated_tokens;
} pokit_cuda_generation_stats;

pokit_cuda_status pokit_cuda_decoder_create(const pokit_cuda_decoder_config* config,
                                            pokit_cuda_decoder** out_decoder, char* error_buffer,
                                            size_t error_capacity);
void pokit_cuda_decoder_destroy(pokit_cuda_decoder* decoder);

/* The decoder's MoE blocks (owned by the decoder; do not destroy). */
pokit_cuda_moe* pokit_cuda_decoder_moe(pokit_cuda_decoder* decoder);

/* Bytes of one decoder tensor (layer ignored for the first three). */
size_t pokit_cuda_decoder_tensor_bytes(const pokit_cuda_decoder* decoder, size_t layer, uint32_t tensor);

/* Host payload in GGUF layout, bytes = pokit_cuda_decoder_tensor_bytes.  Synchronous. */
pokit_cuda_status pokit_cuda_decoder_upload_tensor(pokit_cuda_decoder* decoder, size_t layer, uint32_t tensor,
                                                   const void* host_bytes, size_t bytes, char* error_buffer,
                                                   size_t error_capacity);

/* Fills a quantised decoder tensor with the seeded synthetic block generator
 * (pokitlms_b200.gguf writes the same bytes into a GGUF).  Benchmark utility. */
pokit_cuda_status pokit_cuda_decoder_synthesize_tensor(pokit_cuda_decoder* decoder, size_t layer, uint32_t tensor,
                                                       uint64_t seed, uint64_t stream_id, char* error_buffer,
                                                       size_t error_capacity);

/* Qwen3MoeRunner::forward_token: consumes `token` at `position` (must be the
 * next position) and, when logits_host is not NULL, writes vocab F32 logits.
 * A non-finite logit returns RUNTIME_ERROR and resets the state, as the
 * reference throws and resets. */
pokit_cuda_status pokit_cuda_decoder_forward_token(pokit_cuda_decoder* decoder, uint32_t token, uint64_t position,
                                                   float* logits_host, char* error_buffer, size_t error_capacity);

/* Qwen3MoeRunner::generate_tokens with greedy sampling: resets the state,
 * prefills the prompt, then writes up to max_new_tokens ids to tokens_out
 * (*generated of them; the end token is included when generated). */
pokit_cuda_status pokit_cuda_decoder_generate_tokens(pokit_cuda_decoder* decoder, const uint32_t* prompt,
                                                     size_t prompt_tokens, size_t max_new_tokens,
                                                     uint32_t* tokens_out, size_t* generated,
                                                     pokit_cuda_generation_stats* stats, char* error_buffer,
                                                     size_t error_capacity);

/* Measurement hook (no counterpart in the reference): enqueues `steps` greedy
 * token steps on `stream` (each step's token is the previous step's argmax,
 * all on the device) after the current position.  Asynchronous. */
pokit_cuda_status pokit_cuda_decoder_run_steps(pokit_cuda_decoder* decoder, size_t steps, void* stream,
                                               char* error_buffer, size_t error_capacity);

/* Clears the decode state (position 0, empty KV cache, zero convolution and
 * recurrent states). */
pokit_cuda_status pokit_cuda_decoder_reset(pokit_cuda_decoder* decoder, char* error_buffer, size_t error_capacity);

/* Kernels one token step with logits launches (measurement). */
uint64_t pokit_cuda_decoder_launches_per_step(const pokit_cuda_decoder* decoder);

/* How many of the two token-step variants (with and without logits) replay
 * as CUDA graphs (measurement); when a capture was refused, reason_buffer (may
 * be NULL) receives why and the steps run as plain launches. */
int pokit_cuda_decoder_step_graphs(const pokit_cuda_decoder* decoder, char* reason_buffer, size_t reason_capacity);

/* ------------------------------------------------------------------------ */
/* Qwen3.5 Gated DeltaNet mixer (configuration 3's linear-attention layers)  */
/* ------------------------------------------------------------------------ */

typedef struct pokit_cuda_delta_net_shape {
    size_t key_heads;                 /* ssm.group_count */
    size_t value_heads;               /* ssm.time_step_rank (a multiple of key_heads) */
    size_t key_dim;                   /* ssm.state_size: multiple of 32, <= 256 */
    size_t value_dim;                 /* ssm.inner_size / value_heads: <= 256 */
    size_t conv_kernel;               /* ssm.conv_kernel */
    float rms_epsilon;
} pokit_cuda_delta_net_shape;

/* One token of the mixer between its projections (src/qwen35_runner.cpp:613-656):
 * the causal conv1d step with SiLU over `projected` (the linear_qkv output,
 * [2 key_heads key_dim + value_heads value_dim], convolved in place; replaces
 * causal_depthwise_conv1d_step, src/causal_conv1d.cpp:25-50), the decay and
 * update gates from the linear_alpha / linear_beta outputs (log_decay = ssm_a *
 * softplus(alpha + dt_bias), beta = sigmoid(beta); :633-642), the gated
 * delta-rule step on recurrent_state ([value_heads][value_dim][key_dim] F32,
 * updated in place; replaces gated_delta_recurrent_step_grouped,
 * src/gated_delta_net.cpp:28-110) and the gated RMSNorm with the linear_gate
 * output `gate` and ssm_norm (replaces rms_norm_gated, src/rms_norm.cpp:46-74);
 * `output` [value_heads value_dim] is the linear_output projection's input.
 * conv_weights [channels][conv_kernel], conv_state [channels][conv_kernel - 1]
 * (in place).  All device pointers; asynchronous on `stream`.  An invalid decay
 * or gate (the reference throws) OR-s 1 into *status (device, may be NULL),
 * leaves that head's state untouched and writes zeros. */
pokit_cuda_status pokit_cuda_delta_net_step(const pokit_cuda_delta_net_shape* shape, float* projected,
                                            const float* gate, const float* alpha, const float* beta,
                                            const float* conv_weights, float* conv_state, const float* ssm_a,
                                            const float* dt_bias, const float* ssm_norm, float* recurrent_state,
                                            float* output, uint32_t* status, void* stream, char* error_buffer,
                                            size_t error_capacity);

/* ------------------------------------------------------------------------ */
/* One MoE block without any device allocation                              */
/* ------------------------------------------------------------------------ */

/* Size of the scratch array compiled into the library for
 * pokit_cuda_moe_forward_static_scratch (router partials, routes,
 * activations of one block). */
#define POKIT_CUDA_STATIC_SCRATCH_BYTES (256u * 1024u)

/* One MoE block's tensors in device memory the caller owns (GGUF layouts as
 * for pokit_cuda_moe_upload_tensor; shared_* only for the Qwen3.5 flavour).
 * Expert tensors and routers start on 16-byte boundaries (as cudaMalloc
 * returns them; the kernels read them with 16-byte loads); others are rejected
 * with INVALID_ARGUMENT before any GPU work. */
typedef struct pokit_cuda_moe_block_device {
    size_t hidden, inter, experts, top_k;
    uint32_t flavour;                 /* pokit_cuda_moe_flavour */
    int normalize_top_k;
    float expert_weights_scale;
    const float* router;              /* F32 [experts, hidden] */
    uint32_t gate_type, up_type, down_type;
    const void* gate;                 /* [hidden, inter, experts] */
    const void* up;
    const void* down;                 /* [inter, hidden, experts] */
    size_t shared_inter;              /* 0 = no shared expert */
    const float* shared_router;
    uint32_t shared_gate_type, shared_up_type, shared_down_type;
    const void* shared_gate;
    const void* shared_up;
    const void* shared_down;
} pokit_cuda_moe_block_device;

/* No counterpart in the reference.  The same MoE block as
 * pokit_cuda_moe_forward (same kernels, same results), for callers that cannot
 * allocate device memory: a host that hands all of the GPU's memory to its own
 * pool leaves nothing for cudaMalloc, and a latency-critical thread may not
 * make a call that can synchronise the device.  No handle is needed and
 * nothing is allocated: the caller passes the block's tensors, the input and
 * the outputs as device pointers it owns, and the block's scratch is a fixed
 * POKIT_CUDA_STATIC_SCRATCH_BYTES array compiled into the library, which every
 * GPU that loads the library holds until the process exits.  A block whose
 * scratch would not fit is rejected with INVALID_ARGUMENT before any GPU work.
 * The first call on a device looks up that device's copy of the array
 * (cudaGetSymbolAddress, with the device current); make that first call
 * before any stream capture.  Every call shares the array and it keeps the
 * previous call's contents (the status word is cleared at the start of each
 * call); calls whose work overlaps on the GPU race on it.  Runs on `stream`
 * (a cudaStream_t; NULL = the legacy default stream) and waits for that stream
 * only (the status word is read back on it); returns
 * RUNTIME_ERROR when the router produced non-finite logits, as the reference
 * throws.  route_ids/route_weights (device, top_k entries) may be NULL. */
pokit_cuda_status pokit_cuda_moe_forward_static_scratch(
    const pokit_cuda_moe_block_device* block, const float* input, float* output,
    uint32_t* route_ids, float* route_weights, void* stream, char* error_buffer,
    size_t error_capacity);

#ifdef __cplusplus
}
#endif

#endif /* POKIT_CUDA_H */
