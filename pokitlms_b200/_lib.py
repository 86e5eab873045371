"""ctypes binding of include/pokit_cuda.h (libpokit_cuda.so).

The shared library is the product: every call below goes straight into the
sm_100a kernels.  There is no CPU fallback; if the library is missing or
cannot be loaded, `lib()` raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libpokit_cuda.so"

F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
BLOCK = {F32: (1, 4), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}

STATUS_OK, STATUS_INVALID_ARGUMENT, STATUS_RUNTIME_ERROR = 0, 1, 2
STATUS_BUFFER_TOO_SMALL, STATUS_INTERNAL_ERROR = 3, 4

(ROUTER, GATE, UP, DOWN, FFN_NORM, SHARED_ROUTER, SHARED_GATE, SHARED_UP,
 SHARED_DOWN) = range(9)
QWEN3, QWEN35 = 0, 1
INPUT_F32, INPUT_BF16 = 0, 1
IPC_HANDLE_BYTES = 64   # POKIT_CUDA_IPC_HANDLE_BYTES


def row_bytes(ggml_type: int, cols: int) -> int:
    elems, nbytes = BLOCK[ggml_type]
    return cols // elems * nbytes


class PokitCudaError(RuntimeError):
    """A non-OK pokit_cuda_status, with the library's error text."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[status {status}] {message}")
        self.status = status
        self.message = message


class InvalidArgument(PokitCudaError, ValueError):
    pass


class MoeConfig(C.Structure):
    _fields_ = [
        ("device", C.c_int),
        ("layers", C.c_size_t),
        ("hidden", C.c_size_t),
        ("inter", C.c_size_t),
        ("experts", C.c_size_t),
        ("top_k", C.c_size_t),
        ("flavour", C.c_uint32),
        ("normalize_top_k", C.c_int),
        ("expert_weights_scale", C.c_float),
        ("rms_epsilon", C.c_float),
        ("gate_type", C.c_uint32),
        ("up_type", C.c_uint32),
        ("down_type", C.c_uint32),
        ("layer_down_types", C.POINTER(C.c_uint32)),
        ("shared_inter", C.c_size_t),
        ("shared_gate_type", C.c_uint32),
        ("shared_up_type", C.c_uint32),
        ("shared_down_type", C.c_uint32),
        ("expert_first", C.c_size_t),
        ("expert_count", C.c_size_t),
    ]


class MoeLayerHost(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "router", "gate", "up", "down", "ffn_norm", "shared_router", "shared_gate",
        "shared_up", "shared_down")]


class MoeStats(C.Structure):
    _fields_ = [
        ("capacity_bytes", C.c_size_t),
        ("resident_bytes", C.c_size_t),
        ("bytes_read", C.c_uint64),
        ("read_operations", C.c_uint64),
        ("read_time_ns", C.c_uint64),
        ("hits", C.c_uint64),
        ("misses", C.c_uint64),
        ("forward_calls", C.c_uint64),
        ("kernel_launches", C.c_uint64),
    ]


class LinearStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "linear_calls", "dispatches", "q4_k_dispatches", "q5_k_dispatches", "q6_k_dispatches",
        "q8_0_dispatches", "other_dispatches", "weight_bytes", "gpu_time_ns",
        "model_cache_capacity_bytes", "model_cache_uploaded_bytes", "model_cache_upload_time_ns")]


class MoeBlockDevice(C.Structure):
    _fields_ = [
        ("hidden", C.c_size_t), ("inter", C.c_size_t), ("experts", C.c_size_t),
        ("top_k", C.c_size_t), ("flavour", C.c_uint32), ("normalize_top_k", C.c_int),
        ("expert_weights_scale", C.c_float), ("router", C.c_void_p),
        ("gate_type", C.c_uint32), ("up_type", C.c_uint32), ("down_type", C.c_uint32),
        ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
        ("shared_inter", C.c_size_t), ("shared_router", C.c_void_p),
        ("shared_gate_type", C.c_uint32), ("shared_up_type", C.c_uint32),
        ("shared_down_type", C.c_uint32), ("shared_gate", C.c_void_p),
        ("shared_up", C.c_void_p), ("shared_down", C.c_void_p),
    ]


class DecoderConfig(C.Structure):
    _fields_ = [
        ("device", C.c_int), ("layers", C.c_size_t), ("hidden", C.c_size_t), ("vocab", C.c_size_t),
        ("q_heads", C.c_size_t), ("kv_heads", C.c_size_t), ("head_dim", C.c_size_t),
        ("experts", C.c_size_t), ("top_k", C.c_size_t), ("expert_inter", C.c_size_t),
        ("context", C.c_size_t), ("kv_window", C.c_size_t), ("rms_epsilon", C.c_float),
        ("rope_theta", C.c_float), ("normalize_top_k", C.c_int), ("eos_token", C.c_uint32),
        ("attn_type", C.c_uint32), ("expert_type", C.c_uint32), ("embed_type", C.c_uint32),
        ("output_type", C.c_uint32),
        # Qwen3.5-MoE hybrid (arch ARCH_QWEN35MOE); zero for qwen3moe.
        ("arch", C.c_uint32), ("rotary_dim", C.c_size_t), ("rope_sections", C.c_uint32 * 4),
        ("full_attention_interval", C.c_size_t), ("ssm_conv_kernel", C.c_size_t),
        ("ssm_state_size", C.c_size_t), ("ssm_group_count", C.c_size_t), ("ssm_time_step_rank", C.c_size_t),
        ("ssm_inner_size", C.c_size_t), ("expert_weights_scale", C.c_float), ("shared_inter", C.c_size_t),
        ("shared_type", C.c_uint32), ("layer_down_types", C.POINTER(C.c_uint32)),
    ]


ARCH_QWEN3MOE, ARCH_QWEN35MOE = 0, 1


class GenerationStats(C.Structure):
    _fields_ = [("prefill_time_ns", C.c_uint64), ("decode_time_ns", C.c_uint64),
                ("generated_tokens", C.c_size_t)]


DEC_TOKEN_EMBD, DEC_OUTPUT_NORM, DEC_OUTPUT = 0, 1, 2
DEC_ATTN_NORM, DEC_ATTN_Q, DEC_ATTN_Q_NORM, DEC_ATTN_K, DEC_ATTN_K_NORM, DEC_ATTN_V, DEC_ATTN_OUTPUT = range(3, 10)
(DEC_SSM_QKV, DEC_SSM_GATE, DEC_SSM_ALPHA, DEC_SSM_BETA, DEC_SSM_CONV1D, DEC_SSM_A, DEC_SSM_DT_BIAS, DEC_SSM_NORM,
 DEC_SSM_OUT) = range(10, 19)

class DeltaNetShape(C.Structure):
    _fields_ = [("key_heads", C.c_size_t), ("value_heads", C.c_size_t), ("key_dim", C.c_size_t),
                ("value_dim", C.c_size_t), ("conv_kernel", C.c_size_t), ("rms_epsilon", C.c_float)]


STATIC_SCRATCH_BYTES = 256 * 1024

_ERR = C.c_char_p
_SZ = C.c_size_t
_VP = C.c_void_p

# name -> (restype, argtypes); every symbol of include/pokit_cuda.h.
SIGNATURES = {
    "pokit_cuda_version": (C.c_char_p, []),
    "pokit_cuda_linear": (C.c_int, [C.c_uint32, _VP, _SZ, _SZ, _VP, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_dequantize_rows": (C.c_int, [C.c_uint32, _VP, _SZ, _SZ, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_route_experts": (C.c_int, [_VP, _SZ, _SZ, C.c_uint32, C.c_int, C.c_float, _VP,
                                           _VP, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_synthesize_blocks": (C.c_int, [C.c_uint32, C.c_uint64, C.c_uint64, _SZ, _VP,
                                               _VP, _ERR, _SZ]),
    "pokit_cuda_linear_backend_create": (C.c_int, [C.c_int, C.POINTER(_VP), _ERR, _SZ]),
    "pokit_cuda_linear_backend_destroy": (None, [_VP]),
    "pokit_cuda_linear_backend_try_linear": (C.c_int, [_VP, C.c_uint32, _VP, _SZ, _SZ, _SZ, _VP,
                                                       _VP, C.POINTER(C.c_int), _ERR, _SZ]),
    "pokit_cuda_linear_backend_try_linear_cached": (C.c_int, [_VP, C.c_uint64, C.c_uint32, _VP, _SZ, _SZ,
                                                              _SZ, _VP, _VP, C.POINTER(C.c_int), _ERR,
                                                              _SZ]),
    "pokit_cuda_linear_backend_is_cached": (C.c_int, [_VP, C.c_uint64]),
    "pokit_cuda_linear_backend_set_cache_capacity": (C.c_int, [_VP, C.c_uint64, _ERR, _SZ]),
    "pokit_cuda_linear_backend_forget": (C.c_int, [_VP, C.c_uint64, C.POINTER(C.c_int), _ERR, _SZ]),
    "pokit_cuda_linear_backend_get_stats": (C.c_int, [_VP, C.POINTER(LinearStats)]),
    "pokit_cuda_moe_create": (C.c_int, [C.POINTER(MoeConfig), C.POINTER(_VP), _ERR, _SZ]),
    "pokit_cuda_moe_destroy": (None, [_VP]),
    "pokit_cuda_moe_upload_tensor": (C.c_int, [_VP, _SZ, C.c_uint32, _VP, _SZ, _ERR, _SZ]),
    "pokit_cuda_moe_upload_layer": (C.c_int, [_VP, _SZ, C.POINTER(MoeLayerHost), _ERR, _SZ]),
    "pokit_cuda_moe_synthesize_tensor": (C.c_int, [_VP, _SZ, C.c_uint32, C.c_uint64, C.c_uint64,
                                                   _ERR, _SZ]),
    "pokit_cuda_moe_expert_view": (C.c_int, [_VP, _SZ, C.c_uint32, _SZ, C.POINTER(_VP),
                                             C.POINTER(_SZ)]),
    "pokit_cuda_moe_forward": (C.c_int, [_VP, _SZ, _VP, _VP, _VP, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_forward_batch": (C.c_int, [_VP, _SZ, _VP, C.c_uint32, _SZ, _VP, _VP, _VP, _VP, _VP,
                                               _ERR, _SZ]),
    "pokit_cuda_moe_exchange_create": (C.c_int, [_VP, _SZ, _SZ, _SZ, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_exchange_connect": (C.c_int, [_VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_exchange_disconnect": (C.c_int, [_VP, _ERR, _SZ]),
    "pokit_cuda_moe_time_batch": (C.c_int, [_VP, _SZ, _VP, C.c_uint32, _SZ, _VP, _VP, C.c_uint32, _VP, _SZ,
                                            C.POINTER(_SZ), _VP, _ERR, _SZ]),
    "pokit_cuda_moe_forward_batch_host": (C.c_int, [_VP, _SZ, _VP, C.c_uint32, _SZ, _VP, _VP, _VP, _VP,
                                                    _ERR, _SZ]),
    "pokit_cuda_moe_time_kernel": (C.c_int, [_VP, C.c_uint32, _SZ, _SZ, C.c_uint32, _VP, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_forward_host": (C.c_int, [_VP, _SZ, _VP, _VP, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_decode_layers": (C.c_int, [_VP, _SZ, _SZ, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_decode_layers_host": (C.c_int, [_VP, _SZ, _SZ, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_synchronize": (C.c_int, [_VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_get_stats": (C.c_int, [_VP, C.POINTER(MoeStats)]),
    "pokit_cuda_moe_tensor_bytes": (C.c_size_t, [_VP, _SZ, C.c_uint32]),
    "pokit_cuda_moe_trace_decode": (C.c_int, [_VP, _SZ, _SZ, _VP, _VP, _SZ, C.POINTER(C.c_uint32), _VP, _ERR,
                                              _SZ]),
    "pokit_cuda_decoder_create": (C.c_int, [C.POINTER(DecoderConfig), C.POINTER(_VP), _ERR, _SZ]),
    "pokit_cuda_decoder_destroy": (None, [_VP]),
    "pokit_cuda_decoder_moe": (_VP, [_VP]),
    "pokit_cuda_decoder_tensor_bytes": (_SZ, [_VP, _SZ, C.c_uint32]),
    "pokit_cuda_decoder_upload_tensor": (C.c_int, [_VP, _SZ, C.c_uint32, _VP, _SZ, _ERR, _SZ]),
    "pokit_cuda_decoder_synthesize_tensor": (C.c_int, [_VP, _SZ, C.c_uint32, C.c_uint64, C.c_uint64, _ERR, _SZ]),
    "pokit_cuda_decoder_forward_token": (C.c_int, [_VP, C.c_uint32, C.c_uint64, _VP, _ERR, _SZ]),
    "pokit_cuda_decoder_generate_tokens": (C.c_int, [_VP, _VP, _SZ, _SZ, _VP, C.POINTER(_SZ),
                                                     C.POINTER(GenerationStats), _ERR, _SZ]),
    "pokit_cuda_decoder_run_steps": (C.c_int, [_VP, _SZ, _VP, _ERR, _SZ]),
    "pokit_cuda_decoder_reset": (C.c_int, [_VP, _ERR, _SZ]),
    "pokit_cuda_decoder_launches_per_step": (C.c_uint64, [_VP]),
    "pokit_cuda_decoder_step_graphs": (C.c_int, [_VP, _ERR, _SZ]),
    "pokit_cuda_delta_net_step": (C.c_int, [C.POINTER(DeltaNetShape), _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
                                            _VP, _VP, _VP, _VP, _VP, _ERR, _SZ]),
    "pokit_cuda_moe_forward_static_scratch": (C.c_int, [C.POINTER(MoeBlockDevice), _VP, _VP, _VP,
                                                        _VP, _VP, _ERR, _SZ]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads libpokit_cuda.so, raising if it has not been built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("POKIT_CUDA_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"{path} is missing: build it with `python -m pokitlms_b200.build` "
                "(the CUDA path has no CPU fallback)")
        handle = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class ErrorBuffer:
    """A (char*, capacity) pair for the C ABI's error reporting."""

    def __init__(self, capacity: int = 512):
        self.buf = C.create_string_buffer(capacity)
        self.cap = capacity

    def args(self):
        return self.buf, self.cap

    def text(self) -> str:
        return self.buf.value.decode(errors="replace")


def check(status: int, err: ErrorBuffer | None = None, what: str = "") -> None:
    if status == STATUS_OK:
        return
    msg = err.text() if err is not None else ""
    if what:
        msg = f"{what}: {msg}" if msg else what
    if status == STATUS_INVALID_ARGUMENT:
        raise InvalidArgument(status, msg)
    raise PokitCudaError(status, msg)


def call(name: str, *args) -> None:
    """Calls an entry point that ends in (error_buffer, error_capacity)."""
    err = ErrorBuffer()
    check(getattr(lib(), name)(*args, *err.args()), err, name)
