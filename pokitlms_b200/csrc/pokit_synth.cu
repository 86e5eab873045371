// pokit_synth.cu -- on-device fill of synthetic GGUF blocks.
//
// Benchmark inputs at full model scale (tens of GB of expert weights) are
// generated where they live instead of being pushed over PCIe.  The byte
// stream is a counter-based function of (seed, stream_id, byte offset), so the
// host implementation in pokitlms_b200/synth.py reproduces any block exactly:
//
//   key        = mix64(seed * G + stream_id * C + K0)
//   word(i)    = mix64(key + (i + 1) * G)            (i = byte_offset / 8)
//   byte(o)    = (word(o / 8) >> 8 * (o % 8)) & 0xff
//   then the fp16 scale fields of every block are overwritten with
//   half_rn(1e-3f + f32(u24) * 2^-24 * 9e-3f), u24 = word'(j) >> 40 from the
//   stream key' = mix64(key ^ S), j = 2 * block + field
// (mix64 = the SplitMix64 finaliser).  Q4_K/Q5_K: d, dmin at bytes 0 and 2;
// Q6_K: d at byte 208; Q8_0: d at byte 0.  All other bytes (6-bit scales and
// mins, nibbles, high bits, int8 quants) stay uniformly random.
#include "pokit_kernels.h"
#include "pokit_common.cuh"

namespace pokit {
namespace {

constexpr uint64_t kG = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kC = 0xD1B54A32D192ED03ull;
constexpr uint64_t kK0 = 0x8CB92BA72F3D8DD7ull;
constexpr uint64_t kS = 0x5851F42D4C957F2Dull;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint16_t scale_half(uint64_t skey, uint64_t j) {
    const uint64_t w = mix64(skey + (j + 1) * kG);
    const float t = static_cast<float>(static_cast<uint32_t>(w >> 40)) * 0x1p-24f;  // exact
    const float v = __fadd_rn(1e-3f, __fmul_rn(t, 9e-3f));
    return __half_as_ushort(__float2half_rn(v));
}

// One thread per 8-byte word of the stream covering bytes [start, start +
// nbytes); dst receives those bytes (dst[0] = stream byte `start`).
__global__ void synth_kernel(uint32_t type, uint64_t key, uint64_t skey, uint64_t start, uint64_t nbytes,
                             uint8_t* __restrict__ dst) {
    const uint32_t B = block_bytes(type);
    const uint64_t w_first = start / 8, w_end = (start + nbytes + 7) / 8;
    for (uint64_t i = w_first + blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < w_end;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        uint64_t w = mix64(key + (i + 1) * kG);
        const uint64_t o0 = i * 8;
        // Patch the fp16 scale bytes that fall inside this word.
        for (int b = 0; b < 8; ++b) {
            const uint64_t o = o0 + b;
            const uint64_t blk = o / B;
            const uint32_t off = static_cast<uint32_t>(o - blk * B);
            int field = -1, hi = 0;
            if (type == kQ4_K || type == kQ5_K) {
                if (off < 4) { field = off >> 1; hi = off & 1; }
            } else if (type == kQ6_K) {
                if (off >= 208) { field = 0; hi = off & 1; }
            } else if (type == kQ8_0) {
                if (off < 2) { field = 0; hi = off & 1; }
            }
            if (field >= 0) {
                const uint16_t h = scale_half(skey, 2 * blk + field);
                const uint64_t byte = hi ? (h >> 8) : (h & 0xffu);
                w = (w & ~(0xffull << (8 * b))) | (byte << (8 * b));
            }
        }
        if (o0 >= start && o0 + 8 <= start + nbytes && (reinterpret_cast<uint64_t>(dst + (o0 - start)) & 7u) == 0) {
            *reinterpret_cast<uint64_t*>(dst + (o0 - start)) = w;
        } else {
            for (int b = 0; b < 8; ++b) {
                const uint64_t o = o0 + b;
                if (o >= start && o < start + nbytes) dst[o - start] = static_cast<uint8_t>(w >> (8 * b));
            }
        }
    }
}

}  // namespace

cudaError_t launch_synth_blocks(uint32_t type, uint64_t seed, uint64_t stream_id,
                                uint64_t nblocks, void* dst, cudaStream_t stream, uint64_t first_block) {
    if (type != kQ4_K && type != kQ5_K && type != kQ6_K && type != kQ8_0) return cudaErrorInvalidValue;
    if (nblocks == 0) return cudaSuccess;
    const uint64_t key = [&] {
        uint64_t z = seed * kG + stream_id * kC + kK0;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }();
    uint64_t skey = key ^ kS;
    skey = (skey ^ (skey >> 30)) * 0xBF58476D1CE4E5B9ull;
    skey = (skey ^ (skey >> 27)) * 0x94D049BB133111EBull;
    skey = skey ^ (skey >> 31);
    const uint64_t nbytes = nblocks * block_bytes(type), start = first_block * block_bytes(type);
    const uint64_t nwords = (start + nbytes + 7) / 8 - start / 8;
    uint64_t grid = (nwords + 255) / 256;
    const uint64_t cap = static_cast<uint64_t>(device_sm_count()) * 32u;
    if (grid > cap) grid = cap;
    synth_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(type, key, skey, start, nbytes,
                                                                   static_cast<uint8_t*>(dst));
    return cudaGetLastError();
}

}  // namespace pokit
