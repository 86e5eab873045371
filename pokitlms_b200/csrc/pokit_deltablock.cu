// pokit_deltablock.cu -- one decode token through a Gated DeltaNet layer's
// mixer in a single cooperative launch (PokitLMs src/qwen35_runner.cpp:582-656
// from the attention norm to ssm_out's residual add), on sm_100a.  The same
// arithmetic as the four-kernel path (the Q4_K in-projection, delta_conv_kernel,
// delta_step_regs_kernel, the Q4_K ssm_out projection with accumulate), with
// two grid barriers instead of three kernel boundaries:
//
//   phase 1  every CTA: x' = rms_norm(hidden) * attn_norm as fragment records;
//            its 16-row tiles of the in-projection [q|k|v|z|alpha|beta]
//            (tile t on CTA t % grid, rows bulk-copied at kernel start) on the
//            integer tensor path (q4k_mma_superblock); a projected row in the
//            conv channels goes straight through its causal conv1d + SiLU step
//            (the CTA that computes a channel owns its conv state)
//   barrier
//   phase 2  four CTAs per value head, 32 rows each: those rows of the head's
//            recurrent state (bulk-copied into shared memory at kernel start)
//            through the delta rule, as delta_step_regs_kernel; the raw
//            outputs o to global memory
//   barrier
//   phase 3  CTA c < hidden / 16: the gated RMS norm of every head's o (as
//            delta_step_regs_kernel forms it), then rows [16c, 16c + 16) of
//            ssm_out (tile copied once phase 1 is done with the tile space),
//            added into the residual
//
// The 16-row weight tiles sit in shared memory at a row pitch of row bytes +
// 32, so the 8-byte fragment reads of rows g = 0..7 fall on distinct banks.
// Every wait is bounded: a barrier or copy that gives up sets status[0] and
// the CTA returns (the caller treats the layer state as lost).
#include "pokit_deltablock.cuh"

#include <cuda_runtime.h>

namespace pokit {
namespace {

__global__ void __launch_bounds__(kDbThreads, 1) delta_block_kernel(const __grid_constant__ DeltaBlockArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t last_sh;
    const int tid = threadIdx.x;
    const uint32_t G = gridDim.x;
    const bool ok = delta_layer_run(a, smem);
    if (!ok) return;
    // The last CTA out leaves the counters at zero.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        last_sh = atomicAdd(a.counters + 1, 1u) == G - 1u ? 1u : 0u;
    }
    __syncthreads();
    if (last_sh && tid == 0) {
        a.counters[0] = 0u;
        a.counters[1] = 0u;
        __threadfence();
    }
}

}  // namespace

bool delta_block_plan(const DeltaBlockShape& s, uint32_t* grid, uint32_t* smem) {
    if (s.key_dim != kDbHeadDim || s.value_dim != kDbHeadDim || s.hidden % 256u || s.hidden / 16u == 0 ||
        s.conv_kernel == 0 || s.conv_kernel > kDbMaxConv || s.key_heads == 0 || s.value_heads % s.key_heads ||
        (s.value_heads * kDbHeadDim) % 256u || s.rows_in % 16u)
        return false;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return false;
    const uint32_t G = static_cast<uint32_t>(sms);
    const DbLayout L = db_layout(s.hidden, s.value_heads * kDbHeadDim);
    if ((s.rows_in / 16u + G - 1u) / G > kDbMaxTiles || s.value_heads * kDbSplit > G || s.hidden / 16u > G ||
        L.total > 227u * 1024u)
        return false;
    if (cudaFuncSetAttribute(delta_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(L.total)) != cudaSuccess)
        return false;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, delta_block_kernel, kDbThreads, L.total) !=
            cudaSuccess ||
        per_sm < 1)
        return false;
    *grid = G;
    *smem = L.total;
    return true;
}

cudaError_t launch_delta_block(const DeltaBlockShape& s, const DeltaBlockTensors& t, uint32_t grid, uint32_t smem,
                               cudaStream_t stream) {
    const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!a16(t.w_in) || !a16(t.w_out) || !a16(t.state) || !t.counters || !t.timeout || !t.gates_bad || !t.proj ||
        !t.att || !t.hidden || !t.ms_part)
        return cudaErrorInvalidValue;
    const DeltaBlockArgs a = make_delta_args(s, t);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kDbThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, delta_block_kernel, a);
}

}  // namespace pokit
