// pokit_types.h -- GGML block geometry and device status bits, usable from
// both host C++ and device code.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define POKIT_HD __host__ __device__
#else
#define POKIT_HD
#endif

namespace pokit {

// GGML type ids (GGUF tensor directory, PokitLMs src/gguf_reader.cpp:21-57).
enum GgmlType : uint32_t {
    kF32 = 0,
    kQ8_0 = 8,
    kQ4_K = 12,
    kQ5_K = 13,
    kQ6_K = 14,
};

// Bytes per GGML block and weights per block for the supported types.
POKIT_HD constexpr uint32_t block_bytes(uint32_t t) {
    return t == kF32 ? 4u : t == kQ8_0 ? 34u : t == kQ4_K ? 144u : t == kQ5_K ? 176u
         : t == kQ6_K ? 210u : 0u;
}
POKIT_HD constexpr uint32_t block_elems(uint32_t t) {
    return t == kF32 ? 1u : t == kQ8_0 ? 32u : (t == kQ4_K || t == kQ5_K || t == kQ6_K) ? 256u : 0u;
}
POKIT_HD constexpr uint64_t row_bytes(uint32_t t, uint64_t cols) {
    return block_elems(t) ? cols / block_elems(t) * block_bytes(t) : 0;
}

// Device status word bits (sticky until the host reads and clears them).
enum StatusBits : uint32_t {
    kStatusNonFiniteLogits = 1u << 0,   // router produced NaN/Inf (the reference throws)
    kStatusBadSoftmax = 1u << 1,        // softmax denominator / selected sum invalid
    kStatusWaitTimeout = 1u << 2,       // a bounded device-side wait gave up
};

}  // namespace pokit
