// pokit_linear.cu -- per-matrix GGUF matvec and row dequantisation on sm_100a.
//
// Device side of the TensorLinearBackend seam (PokitLMs
// include/pokitlms/model/tensor_linear.hpp:11-18): y[rows] = W[rows, cols] . x
// with W in its GGUF block encoding, FP32 x and FP32 accumulation, plus the
// row decoder behind dequantize_quantized_row (quantized_linear.hpp:11-13).
#include "pokit_kernels.h"
#include "pokit_mma.cuh"
#include "pokit_quant.cuh"

#include <map>
#include <mutex>

namespace pokit {
namespace {

constexpr int kLinearThreads = 256;

// F32: one warp per row, 128-bit loads straight from global.
__global__ void __launch_bounds__(kLinearThreads)
linear_f32_kernel(const float* __restrict__ w, uint32_t rows, uint32_t cols,
                  const float* __restrict__ x, float* __restrict__ y, int accumulate) {
    const int lane = threadIdx.x & 31;
    const uint32_t warps_total = gridDim.x * (blockDim.x >> 5);
    for (uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
         row += warps_total) {
        const float* rp = w + static_cast<uint64_t>(row) * cols;
        float acc = 0.0f;
        if ((cols & 3u) == 0 && (reinterpret_cast<uint64_t>(rp) & 15u) == 0) {
            for (uint32_t i = lane * 4u; i < cols; i += 128u) {
                const uint4 v = ldg_stream128(rp + i);
                const float4 xv = *reinterpret_cast<const float4*>(x + i);
                acc = fmaf(__uint_as_float(v.x), xv.x, acc);
                acc = fmaf(__uint_as_float(v.y), xv.y, acc);
                acc = fmaf(__uint_as_float(v.z), xv.z, acc);
                acc = fmaf(__uint_as_float(v.w), xv.w, acc);
            }
        } else {
            for (uint32_t i = lane; i < cols; i += 32u) acc = fmaf(__ldg(rp + i), x[i], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[row] = accumulate ? y[row] + acc : acc;
    }
}

// Quantised rows of 16-byte multiples (every K-quant row, Q8_0 rows of 128
// multiples): x in shared memory, one warp per row at a time, the warp's next
// row loaded into registers (16-byte streaming loads) while the current one,
// staged in shared memory, is dotted four weights per lane and step
// (lane_row_dot4: byte-parallel decode, one scale per four weights).  The
// grid is a few CTAs per SM so x is read once per CTA, not once per row.
constexpr uint32_t kRowsMaxUnits = 8;          // 16-byte units per lane: rows up to 4 KiB

template <uint32_t T>
__global__ void __launch_bounds__(kLinearThreads)
linear_rows_kernel(const uint8_t* __restrict__ w, uint32_t rows, uint32_t cols, const float* __restrict__ x,
                   float* __restrict__ y, int accumulate, const float* __restrict__ norm_w, float norm_eps) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    float* xs = reinterpret_cast<float*>(smem_raw);
    const uint32_t rb = static_cast<uint32_t>(row_bytes(T, cols)), units = rb / 16u;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint8_t* buf0 = smem_raw + cols * 4u + warp * 2u * rb;
    uint8_t* buf1 = buf0 + rb;
    const uint32_t nw = gridDim.x * (blockDim.x >> 5);
    uint32_t row = blockIdx.x * (blockDim.x >> 5) + warp;
    uint4 v[kRowsMaxUnits];
    const auto load = [&](uint32_t r) {
        const uint4* src = reinterpret_cast<const uint4*>(w + static_cast<uint64_t>(r) * rb);
#pragma unroll
        for (uint32_t j = 0; j < kRowsMaxUnits; ++j) {
            const uint32_t u = lane + 32u * j;
            if (u < units) v[j] = ldg_stream128(src + u);
        }
    };
    // The weights do not depend on the previous kernel: the warp's first row
    // is requested before waiting for it (a programmatic dependent launch
    // starts this grid while its predecessor finishes; a no-op otherwise).
    if (row < rows) load(row);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        for (uint32_t i = threadIdx.x * 4u; i < cols; i += blockDim.x * 4u)
            *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(x + i);
    } else {
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) xs[i] = x[i];
    }
    __syncthreads();
    if (norm_w) {
        // x = rms_norm(x, norm_w) first (src/rms_norm.cpp:9-27), in every CTA.
        __shared__ float red[kLinearThreads / 32];
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) ss = fmaf(xs[i], xs[i], ss);
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float total = 0.0f;
        for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) total += red[i];
        const float scale = 1.0f / sqrtf(total / static_cast<float>(cols) + norm_eps);
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], scale), norm_w[i]);
        __syncthreads();
    }
    if (row >= rows) return;
    const auto store = [&](uint8_t* dst) {
#pragma unroll
        for (uint32_t j = 0; j < kRowsMaxUnits; ++j) {
            const uint32_t u = lane + 32u * j;
            if (u < units) reinterpret_cast<uint4*>(dst)[u] = v[j];
        }
    };
    store(buf0);
    __syncwarp();
    bool cur0 = true;
    for (; row < rows; row += nw) {
        const uint32_t next = row + nw;
        if (next < rows) load(next);
        float acc = lane_row_dot4<T>(cur0 ? buf0 : buf1, cols, xs, lane);
        acc = warp_sum(acc);
        if (lane == 0) y[row] = accumulate ? y[row] + acc : acc;
        if (next < rows) store(cur0 ? buf1 : buf0);
        __syncwarp();
        cur0 = !cur0;
    }
}

// Any quantised type: one warp per row, row staged in shared memory, lanes
// take 32-weight groups.  x sits in shared memory in plain order.
template <uint32_t T>
__global__ void __launch_bounds__(kLinearThreads)
linear_generic_kernel(const uint8_t* __restrict__ w, uint32_t rows, uint32_t cols,
                      const float* __restrict__ x, float* __restrict__ y, int accumulate) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    float* xs = reinterpret_cast<float*>(smem_raw);
    const uint32_t rbytes = static_cast<uint32_t>(row_bytes(T, cols));
    const uint32_t stage = (rbytes + 15u) & ~15u;
    uint8_t* stage_base = smem_raw + static_cast<uint64_t>(cols) * 4u;
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint8_t* my_row = stage_base + warp * stage;
    const uint32_t warps_total = gridDim.x * (blockDim.x >> 5);
    const int groups = static_cast<int>(cols >> 5);
    for (uint32_t row = blockIdx.x * (blockDim.x >> 5) + warp; row < rows; row += warps_total) {
        warp_stage_row(w + static_cast<uint64_t>(row) * rbytes, rbytes, my_row, lane);
        __syncwarp();
        float acc = 0.0f;
        for (int g = lane; g < groups; g += 32) acc += group_dot<T>(my_row, g, xs);
        acc = warp_sum(acc);
        if (lane == 0) y[row] = accumulate ? y[row] + acc : acc;
        __syncwarp();
    }
}

template <uint32_t T>
__global__ void __launch_bounds__(kLinearThreads)
dequantize_kernel(const uint8_t* __restrict__ w, uint32_t rows, uint32_t cols,
                  float* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const uint32_t rbytes = static_cast<uint32_t>(row_bytes(T, cols));
    const uint32_t stage = (rbytes + 15u) & ~15u;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint8_t* my_row = smem_raw + warp * stage;
    const uint32_t warps_total = gridDim.x * (blockDim.x >> 5);
    const int groups = static_cast<int>(cols >> 5);
    for (uint32_t row = blockIdx.x * (blockDim.x >> 5) + warp; row < rows; row += warps_total) {
        warp_stage_row(w + static_cast<uint64_t>(row) * rbytes, rbytes, my_row, lane);
        __syncwarp();
        for (int g = lane; g < groups; g += 32)
            group_decode<T>(my_row, g, out + static_cast<uint64_t>(row) * cols + g * 32);
        __syncwarp();
    }
}

int sm_count_cached() {
    static int count = 0;
    if (count == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
        if (count <= 0) count = 148;
    }
    return count;
}

// Raises a kernel's dynamic shared-memory limit once per (kernel, device);
// the attribute is per device, and later launches skip the call.
template <typename K>
cudaError_t set_smem(K kernel, size_t bytes) {
    if (bytes <= 48u * 1024u) return cudaSuccess;
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> granted;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    size_t& have = granted[{reinterpret_cast<const void*>(kernel), dev}];
    if (bytes <= have) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) have = bytes;
    return e;
}

template <uint32_t T>
cudaError_t launch_generic(const void* w, uint32_t rows, uint32_t cols, const float* x, float* y,
                           cudaStream_t stream, bool accumulate) {
    const size_t stage = (row_bytes(T, cols) + 15u) & ~size_t(15);
    const size_t smem = static_cast<size_t>(cols) * 4u + stage * (kLinearThreads / 32);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    cudaError_t e = set_smem(linear_generic_kernel<T>, smem);
    if (e != cudaSuccess) return e;
    const uint32_t warps = kLinearThreads / 32;
    uint32_t grid = (rows + warps - 1) / warps;
    const uint32_t cap = static_cast<uint32_t>(sm_count_cached()) * 4u;
    if (grid > cap) grid = cap;
    linear_generic_kernel<T><<<grid, kLinearThreads, smem, stream>>>(
        static_cast<const uint8_t*>(w), rows, cols, x, y, accumulate ? 1 : 0);
    return cudaGetLastError();
}

// The row kernel serves the matrix: 16-byte aligned rows of at most 4 KiB.
template <uint32_t T>
bool rows_kernel_fits(const void* w, uint32_t cols) {
    const uint64_t rb = row_bytes(T, cols);
    if ((reinterpret_cast<uint64_t>(w) & 15u) || (rb & 15u) || rb > 16u * 32u * kRowsMaxUnits) return false;
    if (T == kQ8_0 && (cols & 127u)) return false;
    return static_cast<uint64_t>(cols) * 4u + 2u * rb * (kLinearThreads / 32) <= 200u * 1024u;
}

template <uint32_t T>
cudaError_t launch_rows(const void* w, uint32_t rows, uint32_t cols, const float* x, float* y, cudaStream_t stream,
                        bool accumulate, const float* norm_w = nullptr, float norm_eps = 0.0f, bool pdl = false) {
    const size_t smem = static_cast<size_t>(cols) * 4u + 2u * row_bytes(T, cols) * (kLinearThreads / 32);
    cudaError_t e = set_smem(linear_rows_kernel<T>, smem);
    if (e != cudaSuccess) return e;
    const uint32_t warps = kLinearThreads / 32;
    uint32_t grid = (rows + warps - 1) / warps;
    const uint32_t cap = static_cast<uint32_t>(sm_count_cached()) * 4u;
    if (grid > cap) grid = cap;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLinearThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, linear_rows_kernel<T>, static_cast<const uint8_t*>(w), rows, cols, x, y,
                              accumulate ? 1 : 0, norm_w, norm_eps);
}

// ---------------------------------------------------------------------------
// Q4_K matvec on the integer tensor path (mma.sync m16n8k32, u8 weights x
// int8 pieces of x, q4k_mma_superblock): CTA c owns rows [16c, 16c + 16) and
// its warp w the superblocks w, w + 8, ... of those rows.  Each warp copies
// its 16-row x 144-byte superblock tiles with bulk copies (lanes 0..15, one
// row each) before waiting on the previous kernel (the weights do not depend
// on it), builds the x records of its own superblocks (after the fused RMS
// norm, when given), multiplies, and the CTA adds the eight warps' partial
// rows in warp order.  Rows past `rows` in the last block are neither copied
// nor written.
constexpr uint32_t kMmaLinWarps = 8;
constexpr uint32_t kMmaLinMaxPer = 4;           // superblocks per warp: cols <= 8192

__global__ void __launch_bounds__(kMmaLinWarps * 32)
linear_q4k_mma_kernel(const uint8_t* __restrict__ w, uint32_t rows, uint32_t cols, const float* __restrict__ x,
                      float* __restrict__ y, int accumulate, const float* __restrict__ norm_w, float norm_eps) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar[kMmaLinWarps];
    __shared__ float red[kMmaLinWarps];
    __shared__ float part[kMmaLinWarps][16];
    const uint32_t nsb = cols / 256u, per = (nsb + kMmaLinWarps - 1) / kMmaLinWarps;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2;
    const uint32_t row0 = blockIdx.x * 16u, nrows = min(16u, rows - row0);
    const uint64_t rb = static_cast<uint64_t>(nsb) * 144u;
    const uint32_t mine = static_cast<uint32_t>(warp) < nsb ? (nsb - warp + kMmaLinWarps - 1) / kMmaLinWarps : 0u;
    uint8_t* tiles = smem + static_cast<uint32_t>(warp) * per * kBoxBytes;
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + kMmaLinWarps * per * kBoxBytes) + warp * per * kFragWords;
    if (lane == 0) {
        mbar_init(&bar[warp], 1);
        mbar_fence_init();
    }
    __syncwarp();
    if (mine) {
        if (lane == 0) mbar_expect_tx(&bar[warp], mine * nrows * 144u);
        __syncwarp();
        if (static_cast<uint32_t>(lane) < nrows)
            for (uint32_t i = 0; i < mine; ++i)
                bulk_copy_g2s(tiles + i * kBoxBytes + lane * 144u,
                              w + static_cast<uint64_t>(row0 + lane) * rb + (warp + kMmaLinWarps * i) * 144u, 144u,
                              &bar[warp]);
    }
    grid_dep_launch();
    grid_dep_wait();
    float scale = 1.0f;
    if (norm_w) {
        // x = rms_norm(x, norm_w) first (src/rms_norm.cpp:9-27).
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float total = 0.0f;
        for (uint32_t i = 0; i < kMmaLinWarps; ++i) total += red[i];
        scale = 1.0f / sqrtf(total / static_cast<float>(cols) + norm_eps);
    }
    for (uint32_t i = 0; i < mine; ++i) {
        const uint32_t sb = warp + kMmaLinWarps * i;
        float* stage = reinterpret_cast<float*>(recs + i * kFragWords);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t c = sb * 256u + 32u * j + lane;
            v[j] = norm_w ? __fmul_rn(__fmul_rn(x[c], scale), norm_w[c]) : x[c];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) stage[32 * j + lane] = v[j];
        __syncwarp();
        q4k_frag_superblock(stage, recs + i * kFragWords, lane);
        __syncwarp();
    }
    float acc0 = 0.0f, acc1 = 0.0f;
    if (mine) {
        // The copies land well within the bound; if not, wait once more:
        // shared memory a copy may still write is never given up.
        if (!mbar_wait(&bar[warp], 0)) {
            mbar_wait(&bar[warp], 0);
            acc0 = acc1 = __int_as_float(0x7fc00000);
        }
        for (uint32_t i = 0; i < mine; ++i) {
            const uint8_t* t = tiles + i * kBoxBytes;
            q4k_mma_superblock(t + g * 144u, t + (g + 8) * 144u, recs + i * kFragWords, acc0, acc1);
        }
    }
    acc0 = quad_sum(acc0);
    acc1 = quad_sum(acc1);
    if ((lane & 3) == 0) {
        part[warp][g] = acc0;
        part[warp][g + 8] = acc1;
    }
    __syncthreads();
    if (threadIdx.x < nrows) {
        float v = part[0][threadIdx.x];
        for (uint32_t i = 1; i < kMmaLinWarps; ++i) v += part[i][threadIdx.x];
        const uint32_t r = row0 + threadIdx.x;
        y[r] = accumulate ? y[r] + v : v;
    }
}

// Q6_K y = W x on the integer tensor path (q6k_mma_superblock): a persistent
// grid.  CTA c builds the x records once (after the fused RMS norm, when
// given; warp w the superblocks w, w + 8, ...) and then takes the 16-row tiles
// c, c + grid, ...: a tile's rows are bulk-copied (one copy per row; a row of
// 2048k columns is a multiple of 16 bytes) into one of two buffers at a row
// pitch of row bytes + 16, the next tile's copies in flight while the current
// one is multiplied; warp w multiplies superblocks w, w + 8, ... of the 16
// rows and the CTA adds the warps' partial rows in warp order.
constexpr uint32_t kQ6MmaWarps = 8;
constexpr uint32_t kQ6MmaMaxSb = 32;            // cols <= 8192

__host__ __device__ inline uint32_t q6mma_pitch(uint32_t cols) { return (cols / 256u) * 210u + 16u; }
__host__ __device__ inline uint32_t q6mma_smem(uint32_t cols) {
    return 2u * 16u * q6mma_pitch(cols) + (cols / 256u) * kFragWords * 4u;
}

__global__ void __launch_bounds__(kQ6MmaWarps * 32)
linear_q6k_mma_kernel(const uint8_t* __restrict__ w, uint32_t rows, uint32_t cols, const float* x, float* y,
                      int accumulate, const float* __restrict__ norm_w, float norm_eps) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar[2];
    __shared__ float red[kQ6MmaWarps];
    __shared__ float part[kQ6MmaWarps][16];
    const uint32_t nsb = cols / 256u, rb = nsb * 210u, pitch = q6mma_pitch(cols);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2;
    const uint32_t ntiles = (rows + 15u) / 16u, G = gridDim.x;
    uint8_t* const buf0 = smem;
    uint8_t* const buf1 = smem + 16u * pitch;
    uint32_t* recs = reinterpret_cast<uint32_t*>(smem + 32u * pitch);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    const auto issue = [&](uint32_t t, uint32_t b) {
        const uint32_t row0 = t * 16u, nr = min(16u, rows - row0);
        if (warp == 0) {
            if (lane == 0) mbar_expect_tx(&bar[b], nr * rb);
            __syncwarp();
            if (static_cast<uint32_t>(lane) < nr)
                bulk_copy_g2s((b ? buf1 : buf0) + lane * pitch, w + static_cast<uint64_t>(row0 + lane) * rb, rb,
                              &bar[b]);
        }
    };
    // The weights do not depend on the previous kernel: the first tile is
    // requested before waiting for it (programmatic dependent launch).
    if (blockIdx.x < ntiles) issue(blockIdx.x, 0);
    grid_dep_launch();
    grid_dep_wait();
    float scale = 1.0f;
    if (norm_w) {
        // x = rms_norm(x, norm_w) first (src/rms_norm.cpp:9-27).
        float ss = 0.0f;
        for (uint32_t i = tid; i < cols; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float total = 0.0f;
        for (uint32_t i = 0; i < kQ6MmaWarps; ++i) total += red[i];
        scale = 1.0f / sqrtf(total / static_cast<float>(cols) + norm_eps);
    }
    for (uint32_t q = warp; q < nsb; q += kQ6MmaWarps) {
        float* stage = reinterpret_cast<float*>(recs + q * kFragWords);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t c = q * 256u + 32u * j + lane;
            v[j] = norm_w ? __fmul_rn(__fmul_rn(x[c], scale), norm_w[c]) : x[c];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) stage[32 * j + lane] = v[j];
        __syncwarp();
        q4k_frag_superblock(stage, recs + q * kFragWords, lane);
        __syncwarp();
    }
    __syncthreads();
    uint32_t it = 0;
    for (uint32_t t = blockIdx.x; t < ntiles; t += G, ++it) {
        const uint32_t b = it & 1u, ph = (it >> 1) & 1u;
        if (t + G < ntiles) issue(t + G, b ^ 1u);
        float acc0 = 0.0f, acc1 = 0.0f;
        // The copies land well within the bound; if not, wait once more:
        // shared memory a copy may still write is never given up.
        if (!mbar_wait(&bar[b], ph)) {
            mbar_wait(&bar[b], ph);
            acc0 = acc1 = __int_as_float(0x7fc00000);
        }
        const uint8_t* tile = b ? buf1 : buf0;
        for (uint32_t q = warp; q < nsb; q += kQ6MmaWarps)
            q6k_mma_superblock(tile + g * pitch + q * 210u, tile + (g + 8) * pitch + q * 210u, recs + q * kFragWords,
                               acc0, acc1);
        acc0 = quad_sum(acc0);
        acc1 = quad_sum(acc1);
        if ((lane & 3) == 0) {
            part[warp][g] = acc0;
            part[warp][g + 8] = acc1;
        }
        __syncthreads();
        const uint32_t row0 = t * 16u, nr = min(16u, rows - row0);
        if (static_cast<uint32_t>(tid) < nr) {
            float v = part[0][tid];
            for (uint32_t i = 1; i < kQ6MmaWarps; ++i) v += part[i][tid];
            const uint32_t r = row0 + tid;
            y[r] = accumulate ? y[r] + v : v;
        }
        // This buffer's generic reads come before its next bulk copies.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
    }
}

bool q6k_mma_linear_fits(const void* w, uint32_t cols) {
    return (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && cols % 2048u == 0 && cols / 256u <= kQ6MmaMaxSb &&
           q6mma_smem(cols) <= 200u * 1024u;
}

cudaError_t launch_q6k_mma(const void* w, uint32_t rows, uint32_t cols, const float* x, float* y,
                           cudaStream_t stream, bool accumulate, const float* norm_w, float norm_eps, bool pdl) {
    const size_t smem = q6mma_smem(cols);
    cudaError_t e = set_smem(linear_q6k_mma_kernel, smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, linear_q6k_mma_kernel, kQ6MmaWarps * 32, smem);
    if (e != cudaSuccess) return e;
    const uint32_t ntiles = (rows + 15u) / 16u;
    uint32_t grid = static_cast<uint32_t>(sm_count_cached()) * static_cast<uint32_t>(per_sm < 1 ? 1 : per_sm);
    if (grid > ntiles) grid = ntiles;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kQ6MmaWarps * 32u);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, linear_q6k_mma_kernel, static_cast<const uint8_t*>(w), rows, cols, x, y,
                              accumulate ? 1 : 0, norm_w, norm_eps);
}

bool mma_linear_fits(const void* w, uint32_t cols) {
    return (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && cols % 256u == 0 &&
           (cols / 256u + kMmaLinWarps - 1) / kMmaLinWarps <= kMmaLinMaxPer;
}

cudaError_t launch_q4k_mma(const void* w, uint32_t rows, uint32_t cols, const float* x, float* y,
                           cudaStream_t stream, bool accumulate, const float* norm_w, float norm_eps, bool pdl) {
    const uint32_t per = (cols / 256u + kMmaLinWarps - 1) / kMmaLinWarps;
    const size_t smem = static_cast<size_t>(kMmaLinWarps) * per * (kBoxBytes + kFragWords * 4u);
    cudaError_t e = set_smem(linear_q4k_mma_kernel, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((rows + 15u) / 16u);
    cfg.blockDim = dim3(kMmaLinWarps * 32u);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, linear_q4k_mma_kernel, static_cast<const uint8_t*>(w), rows, cols, x, y,
                              accumulate ? 1 : 0, norm_w, norm_eps);
}

template <uint32_t T>
cudaError_t launch_quant(const void* w, uint32_t rows, uint32_t cols, const float* x, float* y, cudaStream_t stream,
                         bool force_generic, bool accumulate, bool pdl) {
    if constexpr (T == kQ4_K)
        if (!force_generic && mma_linear_fits(w, cols))
            return launch_q4k_mma(w, rows, cols, x, y, stream, accumulate, nullptr, 0.0f, pdl);
    if constexpr (T == kQ6_K)
        if (!force_generic && q6k_mma_linear_fits(w, cols))
            return launch_q6k_mma(w, rows, cols, x, y, stream, accumulate, nullptr, 0.0f, pdl);
    if (!force_generic && rows_kernel_fits<T>(w, cols))
        return launch_rows<T>(w, rows, cols, x, y, stream, accumulate, nullptr, 0.0f, pdl);
    return launch_generic<T>(w, rows, cols, x, y, stream, accumulate);
}

template <uint32_t T>
cudaError_t launch_dequant(const void* w, uint32_t rows, uint32_t cols, float* out,
                           cudaStream_t stream) {
    const size_t stage = (row_bytes(T, cols) + 15u) & ~size_t(15);
    const size_t smem = stage * (kLinearThreads / 32);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    cudaError_t e = set_smem(dequantize_kernel<T>, smem);
    if (e != cudaSuccess) return e;
    const uint32_t warps = kLinearThreads / 32;
    uint32_t grid = (rows + warps - 1) / warps;
    const uint32_t cap = static_cast<uint32_t>(sm_count_cached()) * 4u;
    if (grid > cap) grid = cap;
    dequantize_kernel<T><<<grid, kLinearThreads, smem, stream>>>(
        static_cast<const uint8_t*>(w), rows, cols, out);
    return cudaGetLastError();
}

}  // namespace

int device_sm_count() { return sm_count_cached(); }

cudaError_t launch_linear(uint32_t type, const void* w, uint32_t rows, uint32_t cols,
                          const float* x, float* y, cudaStream_t stream, bool force_generic, bool accumulate,
                          bool pdl) {
    if (rows == 0 || cols == 0) return cudaErrorInvalidValue;
    switch (type) {
        case kF32: {
            const uint32_t warps = kLinearThreads / 32;
            uint32_t grid = (rows + warps - 1) / warps;
            const uint32_t cap = static_cast<uint32_t>(sm_count_cached()) * 8u;
            if (grid > cap) grid = cap;
            linear_f32_kernel<<<grid, kLinearThreads, 0, stream>>>(
                static_cast<const float*>(w), rows, cols, x, y, accumulate ? 1 : 0);
            return cudaGetLastError();
        }
        case kQ4_K: return launch_quant<kQ4_K>(w, rows, cols, x, y, stream, force_generic, accumulate, pdl);
        case kQ5_K: return launch_quant<kQ5_K>(w, rows, cols, x, y, stream, force_generic, accumulate, pdl);
        case kQ6_K: return launch_quant<kQ6_K>(w, rows, cols, x, y, stream, force_generic, accumulate, pdl);
        case kQ8_0: return launch_quant<kQ8_0>(w, rows, cols, x, y, stream, force_generic, accumulate, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_linear_normed(uint32_t type, const void* w, uint32_t rows, uint32_t cols, const float* x,
                                 const float* norm_w, float eps, float* y, cudaStream_t stream, bool pdl) {
    if (rows == 0 || cols == 0 || !norm_w) return cudaErrorInvalidValue;
    switch (type) {
        case kQ4_K:
            if (mma_linear_fits(w, cols)) return launch_q4k_mma(w, rows, cols, x, y, stream, false, norm_w, eps, pdl);
            if (!rows_kernel_fits<kQ4_K>(w, cols)) return cudaErrorInvalidValue;
            return launch_rows<kQ4_K>(w, rows, cols, x, y, stream, false, norm_w, eps, pdl);
        case kQ5_K:
            if (!rows_kernel_fits<kQ5_K>(w, cols)) return cudaErrorInvalidValue;
            return launch_rows<kQ5_K>(w, rows, cols, x, y, stream, false, norm_w, eps, pdl);
        case kQ6_K:
            if (q6k_mma_linear_fits(w, cols)) return launch_q6k_mma(w, rows, cols, x, y, stream, false, norm_w, eps, pdl);
            if (!rows_kernel_fits<kQ6_K>(w, cols)) return cudaErrorInvalidValue;
            return launch_rows<kQ6_K>(w, rows, cols, x, y, stream, false, norm_w, eps, pdl);
        case kQ8_0:
            if (!rows_kernel_fits<kQ8_0>(w, cols)) return cudaErrorInvalidValue;
            return launch_rows<kQ8_0>(w, rows, cols, x, y, stream, false, norm_w, eps, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_dequantize(uint32_t type, const void* w, uint32_t rows, uint32_t cols,
                              float* out, cudaStream_t stream) {
    if (rows == 0 || cols == 0) return cudaErrorInvalidValue;
    switch (type) {
        case kF32: return launch_dequant<kF32>(w, rows, cols, out, stream);
        case kQ8_0: return launch_dequant<kQ8_0>(w, rows, cols, out, stream);
        case kQ4_K: return launch_dequant<kQ4_K>(w, rows, cols, out, stream);
        case kQ5_K: return launch_dequant<kQ5_K>(w, rows, cols, out, stream);
        case kQ6_K: return launch_dequant<kQ6_K>(w, rows, cols, out, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace pokit
