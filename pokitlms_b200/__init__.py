"""pokitlms_b200 -- B200 (sm_100a) CUDA backend for the PokitLMs MoE expert path.

The product is libpokit_cuda.so (C ABI in include/pokit_cuda.h); this package
builds it (pokitlms_b200.build), binds it (pokitlms_b200._lib), mirrors the
reference's backend seams over it (pokitlms_b200.backend) and generates the
seeded synthetic inputs the benchmarks use (pokitlms_b200.synth).
"""
from ._lib import (F32, Q4_K, Q5_K, Q6_K, Q8_0, ROUTER, GATE, UP, DOWN, FFN_NORM, SHARED_ROUTER,
                   SHARED_GATE, SHARED_UP, SHARED_DOWN, QWEN3, QWEN35, InvalidArgument,
                   PokitCudaError, row_bytes)

__all__ = ["F32", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "ROUTER", "GATE", "UP", "DOWN", "FFN_NORM",
           "SHARED_ROUTER", "SHARED_GATE", "SHARED_UP", "SHARED_DOWN", "QWEN3", "QWEN35",
           "InvalidArgument", "PokitCudaError", "row_bytes"]
