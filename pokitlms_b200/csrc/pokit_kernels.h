// pokit_kernels.h -- internal launcher API between the C++ host layer and the
// sm_100a kernels.  Not part of the public C ABI (include/pokit_cuda.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

struct pokit_cuda_delta_net_shape;   // include/pokit_cuda.h

namespace pokit {

int device_sm_count();

// y[rows] = W[rows, cols] . x for a GGUF-encoded W (F32, Q8_0, Q4_K, Q5_K, Q6_K);
// with accumulate, y[rows] += W . x.  pdl: launched as a programmatic
// dependent of the previous kernel in the stream (the quantised row kernel
// requests its first weight rows before waiting for it).
cudaError_t launch_linear(uint32_t type, const void* w, uint32_t rows, uint32_t cols,
                          const float* x, float* y, cudaStream_t stream,
                          bool force_generic = false, bool accumulate = false, bool pdl = false);

// y[rows] = W . rms_norm(x, norm_w) (every CTA normalises x as it stages it);
// quantised W with 16-byte aligned rows of at most 4 KiB, else cudaErrorInvalidValue.
cudaError_t launch_linear_normed(uint32_t type, const void* w, uint32_t rows, uint32_t cols, const float* x,
                                 const float* norm_w, float eps, float* y, cudaStream_t stream, bool pdl = false);

// out[rows, cols] = decoded weights, bit-identical to the reference decoders.
cudaError_t launch_dequantize(uint32_t type, const void* w, uint32_t rows, uint32_t cols,
                              float* out, cudaStream_t stream);

// Softmax top-k routing of `rows` device logits vectors of E entries (one CTA
// per row): ids/weights receive k entries per row.  With splits > 1 a row is
// the sum of `splits` partial rows (partial s of row r at (s * rows + r) * E).
// pdl: launched as a programmatic dependent of the previous kernel in the
// stream (the kernel waits for it before reading the logits).
cudaError_t launch_route_experts(const float* logits, uint32_t E, uint32_t k, uint32_t flavour,
                                 uint32_t normalize, float ew_scale, uint32_t* ids, float* weights,
                                 uint32_t* status, cudaStream_t stream, uint32_t rows = 1, uint32_t splits = 1,
                                 bool pdl = false);

// TMA tensor map over a Q4_K expert tensor: (byte column, row, expert), boxes
// of one superblock (144 bytes) by box_rows rows; cached per argument set.
bool encode_expert_map(CUtensorMap* map, const uint8_t* base, uint64_t row_bytes, uint64_t rows,
                       uint64_t experts, uint64_t slice, uint32_t box_rows);

// Fills blocks [first_block, first_block + nblocks) of the counter-based
// synthetic stream (seed, stream_id) of GGUF `type` into dst; see
// pokitlms_b200/synth.py.
cudaError_t launch_synth_blocks(uint32_t type, uint64_t seed, uint64_t stream_id,
                                uint64_t nblocks, void* dst, cudaStream_t stream, uint64_t first_block = 0);

// Everything one MoE FFN block needs on the device.
struct MoeLayerDev {
    uint32_t hidden = 0, inter = 0, experts = 0, top_k = 0;
    // Experts held by this device: [expert_first, expert_first + expert_local);
    // gate/up/down hold expert_local slices (expert e at e - expert_first).
    uint32_t expert_first = 0, expert_local = 0;
    uint32_t flavour = 0;        // 0 = Qwen3-MoE block, 1 = Qwen3.5-MoE block
    uint32_t normalize = 1;      // renormalise the selected probabilities
    float expert_weights_scale = 1.0f;
    const float* router = nullptr;            // F32 [experts, hidden]
    uint32_t gate_type = 0, up_type = 0, down_type = 0;
    const uint8_t* gate = nullptr;            // experts x [inter rows, hidden cols]
    const uint8_t* up = nullptr;
    const uint8_t* down = nullptr;            // experts x [hidden rows, inter cols]
    uint64_t gate_slice = 0, up_slice = 0, down_slice = 0;   // bytes per expert
    const float* ffn_norm = nullptr;          // F32 [hidden], decode chain only
    float rms_eps = 1e-6f;
    // Qwen3.5 shared expert (absent when shared_inter == 0).
    uint32_t shared_inter = 0;
    const float* shared_router = nullptr;     // F32 [hidden]
    uint32_t shared_gate_type = 0, shared_up_type = 0, shared_down_type = 0;
    const uint8_t* shared_gate = nullptr;
    const uint8_t* shared_up = nullptr;
    const uint8_t* shared_down = nullptr;
};

// Scratch used by one in-flight MoE block (device memory owned by the caller).
struct MoeScratch {
    float* x = nullptr;            // [hidden] normalised input
    float* partial = nullptr;      // [(experts + 1) * splits] router partial dots
    float* logits = nullptr;       // [experts]
    uint32_t* ids = nullptr;       // [top_k]
    float* weights = nullptr;      // [top_k + 1] combine weights (last = shared gate)
    float* act = nullptr;          // [(top_k + 1) * max(inter, shared_inter)]
    // Tensor-core path: router dots summed exactly in carry-save fixed point
    // [experts][8 limbs],
    // per-chunk sums of squares [hidden / 16], the out-of-range flag, x'
    // fragment records, the rms scale and the routing-tail counter (racc, rbad
    // and route_count are zero between launches).
    // The activations written in `rep` replicas [rep][top_k * inter] so the
    // down kernel's CTAs spread their reads (CTA b reads copy b % rep).
    uint32_t rep = 1;
    float* actr = nullptr;
    unsigned long long* racc = nullptr;
    float* rsq = nullptr;
    uint32_t* rbad = nullptr;
    uint32_t* xrec = nullptr;
    float* scale = nullptr;
    uint32_t* route_count = nullptr;
    uint32_t* counter = nullptr;   // last-block hand-off counter (must start at 0)
    uint32_t* status = nullptr;    // sticky StatusBits
};

// Scratch sizing helper (bytes) for `rep` activation replicas, shared by the
// allocator and the no-alloc path.
constexpr uint32_t kActReplicas = 8;
uint64_t moe_scratch_bytes(const MoeLayerDev& L, uint32_t rep = kActReplicas);
// Carves `base` (256-byte aligned, moe_scratch_bytes(L, rep) long) into a MoeScratch.
MoeScratch moe_scratch_carve(const MoeLayerDev& L, void* base, uint32_t rep = kActReplicas);

// Validates the block's shapes and raises the kernels' shared-memory limits
// without launching anything; call once per configuration before capturing
// launch_moe_block into a CUDA graph.
cudaError_t prepare_moe_block(const MoeLayerDev& L);

// One MoE block: routes `x_in` (already normalised) or, when `hidden` is
// non-null, rms_norm(hidden, ffn_norm); writes the routed (+ shared) MoE
// output to `moe_out`, or adds it into `hidden` when moe_out is null.
// In a decode chain `prev` and `next` (may be null) are the neighbouring
// blocks: a block may take its router partials from `prev`'s last kernel and
// produce `next`'s (or warm L2 with `next`'s router).  `launches` (may be
// null) receives the number of kernels launched.
// `marks` (may be null; one more entry than kernels launched) receives an
// event record before the first kernel and after each kernel.
cudaError_t launch_moe_block(const MoeLayerDev& L, const MoeScratch& S, const float* x_in,
                             float* hidden, float* moe_out, const MoeLayerDev* prev,
                             const MoeLayerDev* next, cudaStream_t stream, uint32_t* launches,
                             cudaEvent_t* marks = nullptr);

// Measurement: the average device time (us) of one launch of a tensor-core
// path kernel (which = 0 gate/up, 1 down), launched `reps` times back to back
// over layers[0 .. count) cyclically, with the routes of one forward of
// layers[0] (x and the output in `out`, hidden floats).
cudaError_t time_moe_kernel(const MoeLayerDev* layers, uint32_t count, const MoeScratch& S, uint32_t which,
                            uint32_t reps, float* out, cudaStream_t stream, float* avg_us);

// ---------------------------------------------------------------------------
// Batched tokens (prefill / batched decode): the grouped-expert path.
// ---------------------------------------------------------------------------
// Device scratch of one batched forward for up to `max_tokens` tokens.
struct MoeBatchScratch {
    uint32_t max_tokens = 0;
    uint32_t max_tiles = 0;      // tile list capacity
    uint32_t max_padded = 0;     // padded token-slot capacity
    float* logits = nullptr;     // [tokens][experts] when the router runs here
    uint32_t* ids = nullptr;     // [tokens][top_k] routes in rank order
    float* weights = nullptr;    // [tokens][top_k] combine weights
    uint32_t* rank = nullptr;    // [pairs] position of a (token, rank) pair within its expert
    uint32_t* plan = nullptr;    // [4]: tiles, padded slots, large tiles, skinny tiles
    uint32_t* tile_order = nullptr;  // [max_tiles] large tiles, then skinny tiles (<= 8 tokens)
    uint32_t* tile_expert = nullptr, *tile_first = nullptr, *tile_n = nullptr, *tile_pad0 = nullptr;
    uint32_t* slot_pair = nullptr;   // [pairs] expert-sorted slot -> pair (token * top_k + rank)
    uint8_t* b_gate_up = nullptr;    // packed fp16 activations + scales per tile (gate/up operand)
    float* act = nullptr;            // [padded][inter] silu(gate) * up
    uint8_t* b_down = nullptr;       // packed fp16 hi/lo activations + scales (down operand)
    float* pair_out = nullptr;       // [pairs][hidden] weighted expert outputs
};

// The grouped path serves this layer (Q4_K gate/up/down, no shared expert,
// hidden and inter multiples of 256, TMA-aligned expert tensors).
bool moe_batch_grouped(const MoeLayerDev& L);
uint64_t moe_batch_scratch_bytes(const MoeLayerDev& L, uint32_t max_tokens);
MoeBatchScratch moe_batch_scratch_carve(const MoeLayerDev& L, uint32_t max_tokens, void* base);

// Expert-parallel exchange over peer memory (one process per GPU, the same
// rows on every rank).  Every rank owns one exchange region, mapped into the
// others' address spaces: [2 parities][world][max_tokens][hidden] F32 partial
// outputs, then [2 parities][world] uint32 flags.  peers[r] is rank r's region
// as seen from this GPU (peers[rank] the local one); epoch and arrive are two
// local device words (zero at set-up).
constexpr uint32_t kMaxExchangeRanks = 8;
struct EpExchange {
    uint32_t world = 0, rank = 0, max_tokens = 0, hidden = 0;
    uint8_t* peers[kMaxExchangeRanks] = {};
    uint32_t* epoch = nullptr;
    uint32_t* arrive = nullptr;
};
// Bytes of one rank's exchange region.
uint64_t ep_exchange_bytes(uint32_t world, uint32_t max_tokens, uint32_t hidden);

// out[t] = MoE(x[t]) for `tokens` rows of x (F32, or BF16 when x_bf16), each
// routed independently: by `logits` ([tokens][experts] F32 on the device)
// when given, else by the layer's router.  ids/weights (may be null) receive
// the routes.  `status` collects the sticky StatusBits.  With `ex`, the
// combine kernel also exchanges the shard's partial outputs with the other
// ranks over peer memory and writes their sum (every rank the same values).
cudaError_t launch_moe_batch(const MoeLayerDev& L, const MoeBatchScratch& S, const void* x, uint32_t x_bf16,
                             uint32_t tokens, const float* logits, float* out, uint32_t* ids, float* weights,
                             uint32_t* status, cudaStream_t stream, uint32_t* launches,
                             cudaEvent_t* marks = nullptr, const EpExchange* ex = nullptr);
// Stages (kernels) of one launch_moe_batch: 8, or 7 when logits are given.
// marks (one more than stages) receive an event before the first and after
// each kernel.

// ---------------------------------------------------------------------------
// Persistent decode chain on the tensor-core path (one cooperative launch per
// token; see moe_chain_kernel in pokit_moe.cu).
// ---------------------------------------------------------------------------
constexpr uint32_t kChainCounterStride = 64;   // uint32 words between the counters (256 B)
struct ChainScratch {
    unsigned long long* racc = nullptr;   // [layer % 3][experts][8 limbs] router accumulators
    float* rsq = nullptr;                 // [layer % 2][hidden / 16] per-chunk sums of squares
    uint32_t* rbad = nullptr;             // [layer % 3] non-finite partial flags
    float* xrep = nullptr;                // [kChainXReplicas][hidden] x' = ffn_norm * hidden of the next layer
    unsigned long long* act = nullptr;    // [kChainXReplicas][top_k][inter] (layer tag << 32 | activation bits)
    uint32_t* counters = nullptr;         // route, (unused), exit counters and the layer sequence
                                          // number, kChainCounterStride apart
};
constexpr uint32_t kChainXReplicas = 8;
// Bytes of the chain scratch (must be zero before the first launch; every
// launch leaves the accumulators and counters at zero and advances the
// sequence number by its layer count).
uint64_t moe_chain_scratch_bytes(const MoeLayerDev& shape);
ChainScratch moe_chain_scratch_carve(const MoeLayerDev& shape, void* base);

// What one launch needs besides the per-call arguments: the 4-D TMA maps over
// every layer's gate/up/down tensors, the common shape and the grid.
struct ChainPlan {
    CUtensorMap tm_gate, tm_up, tm_down;
    MoeLayerDev shape;
    uint64_t stride = 0;                  // bytes between consecutive layers' tensors
    uint32_t layers = 0, grid = 0, smem = 0;
};
// Builds the plan for layers[0 .. n) (host copies of the device table) when
// every layer takes the tensor-core path with one shape, their expert tensors
// sit at one constant stride per layer, and the chain fits the device's SMs;
// returns false (and leaves the plan unused) otherwise.
bool moe_chain_plan(const MoeLayerDev* layers, uint32_t n, ChainPlan* plan);
// hidden += MoE_l(rms_norm(hidden, ffn_norm_l)) for l in [first, first + count)
// in one cooperative launch.
// trace (may be null): [count][grid][16] stamps per layer and CTA, 8
// globaltimer readings (ns) then the same 8 points in clock64 cycles: route
// wait done, routes and x records ready, gate/up products done, act
// published, act wait done, down records built, down products combined,
// router partials published.
constexpr uint32_t kChainTraceStamps = 16;
// A decoder's attention blocks run inside the chain: before layer l's MoE
// block, rms_norm(attn_norm_l) -> the Q4_K [q (| gate) | k | v] matvec ->
// attention over layer l's FP16 ring -> the Q4_K output projection into the
// residual (the attention phase of pokit_attention.cuh), with every per-layer
// tensor `w_stride` bytes after the previous layer's and the rings
// `kv_stride` halves apart.  Words exchange hidden rows, Q/K/V rows and the
// attention output between CTAs (tags from the device position).
struct ChainAttnDesc {
    const uint8_t* wqkv = nullptr;        // layer 0's tensors
    const uint8_t* wo = nullptr;
    const float* attn_norm = nullptr;
    const float* q_norm = nullptr;
    const float* k_norm = nullptr;
    uint64_t w_stride = 0;
    const float* rope_cos = nullptr;      // [context][rotary half]
    const float* rope_sin = nullptr;
    void* kc = nullptr;                   // layer 0's rings (__half)
    void* vc = nullptr;
    uint64_t kv_stride = 0;
    const uint32_t* pos = nullptr;        // the decoder's device position
    uint32_t q_heads = 0, kv_heads = 0, head_dim = 0, q_stride = 0, gated = 0, rotary_half = 0, window = 0;
    float eps = 0.0f, scale = 0.0f;
    unsigned long long* qkv_words = nullptr;   // [rows]
    unsigned long long* att_words = nullptr;   // [q_heads * head_dim]
    unsigned long long* hidden_words = nullptr;  // [hidden]
    uint32_t* status = nullptr;           // attention timeout flag
    uint32_t rows = 0, layers_total = 0;
};
// The decode chain for Qwen3.5-MoE blocks (Q4_K gate/up, any K-quant or Q8_0
// down per layer, the Q8_0 shared expert with its sigmoid gate), per-layer
// pointers read from the device table.
// The Gated DeltaNet mixer step (conv1d, gates, delta rule, gated norm) of
// pokit_cuda_delta_net_step, its two kernels launched as programmatic
// dependents when `pdl` (each waits for its predecessor before reading its
// outputs, and loads only its own states before that).
bool delta_net_shape_valid(const pokit_cuda_delta_net_shape& s);
cudaError_t launch_delta_net_step(const pokit_cuda_delta_net_shape& s, float* projected, const float* gate,
                                  const float* alpha, const float* beta, const float* conv_weights, float* conv_state,
                                  const float* ssm_a, const float* dt_bias, const float* ssm_norm,
                                  float* recurrent_state, float* output, uint32_t* status, cudaStream_t st, bool pdl);

// A Gated DeltaNet layer's mixer, from the attention norm to ssm_out's
// residual add, in one cooperative launch (pokit_deltablock.cu): Q4_K
// in-projection [q|k|v|z|alpha|beta] and ssm_out, 128-wide key and value heads.
struct DeltaBlockShape {
    uint32_t hidden = 0, rows_in = 0, key_heads = 0, value_heads = 0, key_dim = 0, value_dim = 0, conv_kernel = 0;
    float norm_eps = 0.0f, eps = 0.0f;
};
struct DeltaBlockTensors {
    const void* w_in = nullptr;        // Q4_K [rows_in][hidden]
    const void* w_out = nullptr;       // Q4_K [hidden][value_heads * value_dim]
    const float* attn_norm = nullptr;
    const float* conv_w = nullptr;
    float* conv_state = nullptr;
    const float* ssm_a = nullptr;
    const float* dt_bias = nullptr;
    const float* ssm_norm = nullptr;
    float* state = nullptr;            // [value_heads][value_dim][key_dim]
    float* hidden = nullptr;           // the residual, in and out
    float* proj = nullptr;             // [rows_in] scratch
    float* att = nullptr;              // [value_heads * value_dim] scratch
    float* ms_part = nullptr;          // [value_heads * 4] scratch
    uint32_t* counters = nullptr;      // [2], zero between launches
    uint32_t* timeout = nullptr;       // set when a bounded device-side wait gave up
    uint32_t* gates_bad = nullptr;     // bit 0: an invalid decay or beta
};
bool delta_block_plan(const DeltaBlockShape& s, uint32_t* grid, uint32_t* smem);
cudaError_t launch_delta_block(const DeltaBlockShape& s, const DeltaBlockTensors& t, uint32_t grid, uint32_t smem,
                               cudaStream_t stream);

struct Chain35Plan {
    MoeLayerDev shape;
    uint32_t layers = 0, grid = 0, smem = 0, rb_down_max = 0;
};
// A layer's tensor maps for the chain's gate/up boxes: (8-byte column, row,
// expert) views of the routed Q4_K gate and up, boxes of 16 rows by two
// superblocks; (8-byte column, row) views of the shared expert's Q8_0 gate
// and up, boxes of 8 rows by half a row.  Kept in device memory, a table per
// layer.
struct Chain35Maps {
    CUtensorMap gate, up, shared_gate, shared_up;
};
// Plans the chain for `n` layers and encodes each layer's maps into `maps`.
bool moe_chain35_plan(const MoeLayerDev* layers, uint32_t n, Chain35Plan* plan, std::vector<Chain35Maps>* maps);
// With `delta` (count 1): the layer's Gated DeltaNet mixer (delta_block's
// phases) runs first in the same launch, leaving each D unit's residual rows
// in its own CTA.
// With `att_args` (an AttnBlockArgs of pokit_attention.cuh, `att_bytes` its
// size; count 1): the layer's attention block runs first instead.
cudaError_t launch_moe_chain35(const Chain35Plan& plan, const MoeLayerDev* layers_dev, const Chain35Maps* maps_dev,
                               uint32_t first, uint32_t count, const MoeScratch& S, const ChainScratch& C,
                               float* hidden, cudaStream_t stream, unsigned long long* trace = nullptr,
                               const DeltaBlockShape* delta_shape = nullptr, const DeltaBlockTensors* delta = nullptr,
                               const void* att_args = nullptr, size_t att_bytes = 0);
bool moe_chain35_delta_fits(const Chain35Plan& plan, const DeltaBlockShape& d);
bool moe_chain35_attention_fits(const Chain35Plan& plan, const void* att_args, size_t bytes);
// Bytes of shared memory the attention phase needs, and where the chain's
// tile region (which it runs in) starts.
uint32_t chain_attention_smem(const ChainPlan& plan, const ChainAttnDesc& att);
uint32_t chain_tile_offset(const ChainPlan& plan);
cudaError_t launch_moe_chain(const ChainPlan& plan, const MoeLayerDev* layers_dev, uint32_t first, uint32_t count,
                             const MoeScratch& S, const ChainScratch& C, float* hidden, cudaStream_t stream,
                             unsigned long long* trace = nullptr, const ChainAttnDesc* attention = nullptr);
}  // namespace pokit
struct pokit_cuda_moe;
namespace pokit {
// A MoE handle's decode chain with a decoder's attention blocks (pokit_backend.cpp).
bool moe_attention_chain_fits(const pokit_cuda_moe* moe, const ChainAttnDesc& att);
// A Qwen3.5 decoder's DeltaNet layer `layer` and the handle's MoE block of
// that layer in one launch (moe_chain35_kernel with the mixer ahead).
bool moe_delta_layer_fits(const pokit_cuda_moe* moe, const DeltaBlockShape& d);
// The same for an attention layer (`args`: an AttnBlockArgs, `bytes` its size).
bool moe_attention_layer_fits(const pokit_cuda_moe* moe, const void* args, size_t bytes);
cudaError_t moe_decode_layer_attention(pokit_cuda_moe* moe, size_t layer, float* hidden, const void* args,
                                       size_t bytes, cudaStream_t stream, std::string* error);
cudaError_t moe_decode_layer_delta(pokit_cuda_moe* moe, size_t layer, float* hidden, const DeltaBlockShape& d,
                                   const DeltaBlockTensors& t, cudaStream_t stream, std::string* error);
cudaError_t moe_decode_layers_attention(pokit_cuda_moe* moe, size_t first, size_t count, float* hidden,
                                        const ChainAttnDesc& att, cudaStream_t stream, std::string* error);

// Grid-wide barriers one layer of launch_moe_decode performs.
uint32_t moe_barriers_per_layer();

// CTAs of the persistent decode kernel for this shape (all co-resident), or 0
// if the shape cannot run it.
uint32_t moe_decode_grid(const MoeLayerDev& shape);

// One token through layers [first, first + count) of the device array
// `layers_dev` in a single cooperative launch: hidden += MoE_l(rms_norm(hidden)).
// `barrier_base` is the value of S.counter when the launch starts; the launch
// adds count * moe_barriers_per_layer() * grid to it.
cudaError_t launch_moe_decode(const MoeLayerDev* layers_dev, const MoeLayerDev& shape,
                              uint32_t first, uint32_t count, const MoeScratch& S, float* hidden,
                              uint32_t barrier_base, uint32_t grid, cudaStream_t stream);

}  // namespace pokit
