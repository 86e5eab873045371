"""Python mirror of the PokitLMs backend seams, over the C ABI.

Names and argument meaning follow the reference:
  * CudaLinearBackend.try_linear  <- model::TensorLinearBackend::try_linear
    (include/pokitlms/model/tensor_linear.hpp:11-18); returns False for an
    unsupported type, raises on execution failure.
  * CudaMoeBackend                <- the runners' MoE block + ExpertStore
    (src/qwen3_moe_runner.cpp:643-692, src/qwen35_runner.cpp:691-763,
    include/pokitlms/storage/expert_store.hpp:26-53), with every expert
    resident in HBM.
  * linear / dequantize_rows / route_experts on device tensors
    <- linear_q4_k & co. (quantized_linear.hpp), route_experts /
    select_experts (runner-internal).

Device buffers are torch CUDA tensors (torch is only the allocator and stream
provider here); all compute runs in libpokit_cuda.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import (BLOCK, F32, GATE, UP, DOWN, QWEN3, QWEN35, InvalidArgument, LinearStats,
                   MoeConfig, MoeLayerHost, MoeStats, PokitCudaError, call, check, lib, row_bytes)


def _ptr(t) -> int | None:
    if t is None:
        return None
    return int(t.data_ptr())


# cudaStreamLegacy: the C ABI reads a NULL stream as "the handle's own
# stream", so torch's legacy default stream (handle 0) is passed explicitly.
_CUDA_STREAM_LEGACY = 0x1


def _stream(stream) -> int:
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    handle = int(getattr(stream, "cuda_stream", stream) or 0)
    return handle if handle else _CUDA_STREAM_LEGACY


def _np_ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def version() -> str:
    return lib().pokit_cuda_version().decode()


def linear(ggml_type: int, weights, rows: int, cols: int, x, y, stream=None) -> None:
    """y[rows] = W[rows, cols] . x on device tensors (W: uint8 GGUF bytes)."""
    call("pokit_cuda_linear", ggml_type, _ptr(weights), rows, cols, _ptr(x), _ptr(y),
         _stream(stream))


def dequantize_rows(ggml_type: int, encoded, rows: int, cols: int, out, stream=None) -> None:
    call("pokit_cuda_dequantize_rows", ggml_type, _ptr(encoded), rows, cols, _ptr(out),
         _stream(stream))


def route_experts(logits, top_k: int, flavour: int, normalize: bool, ids, weights,
                  expert_weights_scale: float = 1.0, status=None, stream=None) -> None:
    call("pokit_cuda_route_experts", _ptr(logits), logits.numel(), top_k, flavour,
         int(normalize), float(expert_weights_scale), _ptr(ids), _ptr(weights), _ptr(status),
         _stream(stream))


def synthesize_blocks(ggml_type: int, seed: int, stream_id: int, nblocks: int, dst,
                      stream=None) -> None:
    call("pokit_cuda_synthesize_blocks", ggml_type, seed, stream_id, nblocks, _ptr(dst),
         _stream(stream))


def delta_net_step(shape: dict, projected, gate, alpha, beta, conv_weights, conv_state, ssm_a, dt_bias, ssm_norm,
                   recurrent_state, output, status=None, stream=None) -> None:
    """One token of the Gated DeltaNet mixer on device tensors (see
    pokit_cuda_delta_net_step); projected, conv_state and recurrent_state are
    updated in place."""
    s = _lib.DeltaNetShape(shape["key_heads"], shape["value_heads"], shape["key_dim"], shape["value_dim"],
                           shape["conv_kernel"], shape["rms_epsilon"])
    call("pokit_cuda_delta_net_step", C.byref(s), _ptr(projected), _ptr(gate), _ptr(alpha), _ptr(beta),
         _ptr(conv_weights), _ptr(conv_state), _ptr(ssm_a), _ptr(dt_bias), _ptr(ssm_norm), _ptr(recurrent_state),
         _ptr(output), _ptr(status), _stream(stream))


class CudaLinearBackend:
    """TensorLinearBackend with host spans; payloads are streamed per call, or
    cached in HBM under a caller-chosen key (try_linear(..., key=...))."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        call("pokit_cuda_linear_backend_create", device, C.byref(h))
        self._h = h

    def try_linear(self, ggml_type: int, weights: np.ndarray, rows: int, cols: int,
                   x: np.ndarray, out: np.ndarray, key: int | None = None) -> bool:
        x = np.ascontiguousarray(x, dtype=np.float32)
        if out.dtype != np.float32 or not out.flags.c_contiguous or out.size != rows:
            raise ValueError("output must be a contiguous float32 array of `rows` elements")
        handled = C.c_int(0)
        if key is None:
            call("pokit_cuda_linear_backend_try_linear", self._h, ggml_type, _np_ptr(weights),
                 weights.nbytes, rows, cols, _np_ptr(x), _np_ptr(out), C.byref(handled))
        else:
            call("pokit_cuda_linear_backend_try_linear_cached", self._h, key, ggml_type,
                 _np_ptr(weights), weights.nbytes, rows, cols, _np_ptr(x), _np_ptr(out),
                 C.byref(handled))
        return bool(handled.value)

    def set_cache_capacity(self, nbytes: int) -> None:
        call("pokit_cuda_linear_backend_set_cache_capacity", self._h, nbytes)

    def forget(self, key: int) -> bool:
        hit = C.c_int(0)
        call("pokit_cuda_linear_backend_forget", self._h, key, C.byref(hit))
        return bool(hit.value)

    def stats(self) -> dict:
        s = LinearStats()
        check(lib().pokit_cuda_linear_backend_get_stats(self._h, C.byref(s)))
        return {n: getattr(s, n) for n, _ in s._fields_}

    def close(self) -> None:
        if self._h:
            lib().pokit_cuda_linear_backend_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaMoeBackend:
    """MoE FFN blocks over an HBM-resident expert pool."""

    def __init__(self, *, layers: int, hidden: int, inter: int, experts: int, top_k: int,
                 flavour: int = QWEN3, normalize_top_k: bool = True,
                 expert_weights_scale: float = 1.0, rms_epsilon: float = 1e-6,
                 gate_type: int = 12, up_type: int = 12, down_type: int = 12,
                 layer_down_types: list[int] | None = None, shared_inter: int = 0,
                 shared_gate_type: int = 8, shared_up_type: int = 8, shared_down_type: int = 8,
                 device: int = 0, expert_first: int = 0, expert_count: int = 0):
        """expert_first / expert_count select an expert shard (count 0 = all
        experts): the handle then holds only those experts' gate/up/down
        slices and its batched forward returns their contribution."""
        self._ldt = None
        if layer_down_types is not None:
            self._ldt = (C.c_uint32 * layers)(*layer_down_types)
        cfg = MoeConfig(device, layers, hidden, inter, experts, top_k, flavour,
                        int(normalize_top_k), expert_weights_scale, rms_epsilon, gate_type,
                        up_type, down_type,
                        C.cast(self._ldt, C.POINTER(C.c_uint32)) if self._ldt else None,
                        shared_inter, shared_gate_type, shared_up_type, shared_down_type,
                        expert_first, expert_count)
        h = C.c_void_p()
        call("pokit_cuda_moe_create", C.byref(cfg), C.byref(h))
        self._h = h
        self.layers, self.hidden, self.inter = layers, hidden, inter
        self.experts, self.top_k, self.flavour = experts, top_k, flavour
        self.shared_inter = shared_inter
        self.expert_first = expert_first if expert_count else 0
        self.expert_count = expert_count if expert_count else experts

    # -- weights ------------------------------------------------------------
    def tensor_bytes(self, layer: int, tensor: int) -> int:
        return int(lib().pokit_cuda_moe_tensor_bytes(self._h, layer, tensor))

    def upload_tensor(self, layer: int, tensor: int, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        call("pokit_cuda_moe_upload_tensor", self._h, layer, tensor, _np_ptr(data), data.nbytes)

    def upload_layer(self, layer: int, *, router=None, gate=None, up=None, down=None,
                     ffn_norm=None, shared_router=None, shared_gate=None, shared_up=None,
                     shared_down=None) -> None:
        arrays = [None if a is None else np.ascontiguousarray(a) for a in (
            router, gate, up, down, ffn_norm, shared_router, shared_gate, shared_up,
            shared_down)]
        host = MoeLayerHost(*[None if a is None else a.ctypes.data for a in arrays])
        call("pokit_cuda_moe_upload_layer", self._h, layer, C.byref(host))

    def synthesize_tensor(self, layer: int, tensor: int, seed: int, stream_id: int) -> None:
        call("pokit_cuda_moe_synthesize_tensor", self._h, layer, tensor, seed, stream_id)

    def expert_view(self, layer: int, matrix: int, expert: int) -> tuple[int, int]:
        p = C.c_void_p()
        n = C.c_size_t()
        check(lib().pokit_cuda_moe_expert_view(self._h, layer, matrix, expert, C.byref(p),
                                               C.byref(n)))
        return int(p.value or 0), int(n.value)

    # -- execution ----------------------------------------------------------
    def forward(self, layer: int, x, out, route_ids=None, route_weights=None, stream=None) -> None:
        call("pokit_cuda_moe_forward", self._h, layer, _ptr(x), _ptr(out), _ptr(route_ids),
             _ptr(route_weights), _stream(stream))

    def forward_batch(self, layer: int, x, out, *, logits=None, route_ids=None, route_weights=None,
                      stream=None) -> None:
        """out[t] = MoE(x[t]) for the rows of a device tensor x ([tokens, hidden],
        float32 or bfloat16); `logits` ([tokens, experts] float32) replaces the
        layer's router when given.  Q4_K layers run the grouped-expert GEMM."""
        import torch
        kind = _lib.INPUT_BF16 if x.dtype == torch.bfloat16 else _lib.INPUT_F32
        if kind == _lib.INPUT_F32 and x.dtype != torch.float32:
            raise InvalidArgument(1, "x must be float32 or bfloat16")
        tokens = x.numel() // self.hidden
        call("pokit_cuda_moe_forward_batch", self._h, layer, _ptr(x), kind, tokens, _ptr(logits), _ptr(out),
             _ptr(route_ids), _ptr(route_weights), _stream(stream))

    def exchange_create(self, world: int, rank: int, max_tokens: int) -> bytes:
        """This rank's part of the peer-memory exchange (pokit_cuda_moe_exchange_create):
        returns its CUDA IPC handle for the other ranks."""
        buf = C.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        call("pokit_cuda_moe_exchange_create", self._h, world, rank, max_tokens, C.cast(buf, C.c_void_p))
        return buf.raw

    def exchange_connect(self, handles: list[bytes]) -> None:
        """Maps the other ranks' regions (handles in rank order); from then on
        forward_batch returns the whole block's output (pokit_cuda_moe_exchange_connect)."""
        raw = b"".join(handles)
        buf = C.create_string_buffer(raw, len(raw))
        call("pokit_cuda_moe_exchange_connect", self._h, C.cast(buf, C.c_void_p))

    def exchange_disconnect(self) -> None:
        """Unmaps the other ranks' regions (pokit_cuda_moe_exchange_disconnect); every
        rank disconnects before any rank closes its handle."""
        call("pokit_cuda_moe_exchange_disconnect", self._h)

    def time_batch(self, layer: int, x, out, *, logits=None, reps: int = 10, stream=None) -> list[float]:
        """Average device time (us) of each kernel of the grouped batched
        forward over `reps` runs: [router,] route, group, pack, gate/up,
        pack, down, combine."""
        import torch
        kind = _lib.INPUT_BF16 if x.dtype == torch.bfloat16 else _lib.INPUT_F32
        tokens = x.numel() // self.hidden
        us = (C.c_float * 8)()
        n = C.c_size_t(0)
        call("pokit_cuda_moe_time_batch", self._h, layer, _ptr(x), kind, tokens, _ptr(logits), _ptr(out), reps,
             C.cast(us, C.c_void_p), 8, C.byref(n), _stream(stream))
        return [float(us[i]) for i in range(n.value)]

    def forward_batch_host(self, layer: int, x: np.ndarray, *, bf16_bits: bool = False,
                           logits: np.ndarray | None = None):
        """Host-array batch: x float32 [tokens, hidden], or uint16 BF16 bit
        patterns when bf16_bits.  Returns (out, ids, weights)."""
        if bf16_bits:
            x = np.ascontiguousarray(x, dtype=np.uint16)
            kind = _lib.INPUT_BF16
        else:
            x = np.ascontiguousarray(x, dtype=np.float32)
            kind = _lib.INPUT_F32
        tokens = x.size // self.hidden
        lg = None if logits is None else np.ascontiguousarray(logits, dtype=np.float32)
        out = np.empty((tokens, self.hidden), dtype=np.float32)
        ids = np.empty((tokens, self.top_k), dtype=np.uint32)
        w = np.empty((tokens, self.top_k), dtype=np.float32)
        call("pokit_cuda_moe_forward_batch_host", self._h, layer, _np_ptr(x), kind, tokens, _np_ptr(lg),
             _np_ptr(out), _np_ptr(ids), _np_ptr(w))
        return out, ids, w

    def time_kernel(self, kernel: int, first: int, count: int, reps: int, work, stream=None) -> float:
        """Average device time (us) of one back-to-back launch of a tensor-core
        kernel (0 gate/up, 1 down) over layers [first, first + count)."""
        us = C.c_float(0.0)
        call("pokit_cuda_moe_time_kernel", self._h, kernel, first, count, reps, _ptr(work), _stream(stream),
             C.cast(C.pointer(us), C.c_void_p))
        return us.value

    def forward_host(self, layer: int, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.hidden, dtype=np.float32)
        ids = np.empty(self.top_k, dtype=np.uint32)
        w = np.empty(self.top_k, dtype=np.float32)
        call("pokit_cuda_moe_forward_host", self._h, layer, _np_ptr(x), _np_ptr(out),
             _np_ptr(ids), _np_ptr(w))
        return out, ids, w

    def decode_layers(self, first: int, count: int, hidden, stream=None) -> None:
        call("pokit_cuda_moe_decode_layers", self._h, first, count, _ptr(hidden), _stream(stream))

    def trace_decode(self, first: int, count: int, hidden, stamps, stream=None) -> int:
        """One decode_layers call through the chain kernel with per-phase
        stamps (torch int64 device tensor of count x grid x 16 entries:
        8 globaltimer readings, then the same 8 points in SM clock cycles);
        returns the grid size."""
        grid = C.c_uint32(0)
        call("pokit_cuda_moe_trace_decode", self._h, first, count, _ptr(hidden), _ptr(stamps), stamps.numel(),
             C.byref(grid), _stream(stream))
        return int(grid.value)

    def decode_layers_host(self, first: int, count: int, hidden_in: np.ndarray,
                           hidden_out: np.ndarray | None = None) -> np.ndarray:
        hidden_in = np.ascontiguousarray(hidden_in, dtype=np.float32)
        if hidden_out is None:
            hidden_out = np.empty(self.hidden, dtype=np.float32)
        call("pokit_cuda_moe_decode_layers_host", self._h, first, count, _np_ptr(hidden_in),
             _np_ptr(hidden_out))
        return hidden_out

    def synchronize(self, stream=None) -> None:
        call("pokit_cuda_moe_synchronize", self._h, None if stream is None else _stream(stream))

    def stats(self) -> dict:
        s = MoeStats()
        check(lib().pokit_cuda_moe_get_stats(self._h, C.byref(s)))
        return {n: getattr(s, n) for n, _ in s._fields_}

    def close(self) -> None:
        if self._h and not getattr(self, "_borrowed", False):
            lib().pokit_cuda_moe_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["CudaLinearBackend", "CudaMoeBackend", "linear", "dequantize_rows", "route_experts",
           "synthesize_blocks", "version", "PokitCudaError", "InvalidArgument", "BLOCK",
           "row_bytes", "F32", "GATE", "UP", "DOWN", "QWEN3", "QWEN35", "_lib"]


class CudaDecoder:
    """The whole decoder of one sequence on the GPU: the reference's
    Qwen3MoeRunner for a gguf.Qwen3MoeShape, or its Qwen35Runner (the
    Qwen3.5-MoE hybrid of Gated DeltaNet and gated full-attention layers) for
    a gguf.Qwen35MoeShape; forward_token, generate_tokens with greedy sampling."""

    def __init__(self, shape, *, device: int = 0, kv_window: int = 0):
        """`shape`: a pokitlms_b200.gguf.Qwen3MoeShape or Qwen35MoeShape (the
        model's hyper-parameters and tensor types)."""
        from . import gguf
        self.hybrid = isinstance(shape, gguf.Qwen35MoeShape)
        cfg = _lib.DecoderConfig(device, shape.layers, shape.hidden, shape.vocab, shape.q_heads, shape.kv_heads,
                                 shape.head_dim, shape.experts, shape.top_k, shape.expert_inter, shape.context,
                                 kv_window, shape.rms_epsilon, shape.rope_theta, 1, shape.eos, shape.attn_type,
                                 shape.expert_type, shape.embed_type, shape.output_type)
        self._ldt = None
        if self.hybrid:
            self._ldt = (C.c_uint32 * shape.layers)(*[shape.down_type(l) for l in range(shape.layers)])
            cfg.arch = _lib.ARCH_QWEN35MOE
            cfg.rotary_dim = shape.rotary_dim
            cfg.rope_sections[:] = list(shape.rope_sections)
            cfg.full_attention_interval = shape.full_attention_interval
            cfg.ssm_conv_kernel = shape.ssm_conv_kernel
            cfg.ssm_state_size = shape.ssm_state_size
            cfg.ssm_group_count = shape.ssm_group_count
            cfg.ssm_time_step_rank = shape.ssm_time_step_rank
            cfg.ssm_inner_size = shape.ssm_inner_size
            cfg.expert_weights_scale = shape.expert_weights_scale
            cfg.shared_inter = shape.shared_inter
            cfg.shared_type = shape.shared_type
            cfg.layer_down_types = C.cast(self._ldt, C.POINTER(C.c_uint32))
        h = C.c_void_p()
        call("pokit_cuda_decoder_create", C.byref(cfg), C.byref(h))
        self._h = h
        self.shape = shape
        moe = CudaMoeBackend.__new__(CudaMoeBackend)
        moe._h = C.c_void_p(lib().pokit_cuda_decoder_moe(h))
        moe._borrowed = True
        moe._ldt = None
        moe.layers, moe.hidden, moe.inter = shape.layers, shape.hidden, shape.expert_inter
        moe.experts, moe.top_k = shape.experts, shape.top_k
        moe.flavour = QWEN35 if self.hybrid else QWEN3
        moe.shared_inter = shape.shared_inter if self.hybrid else 0
        moe.expert_first, moe.expert_count = 0, shape.experts
        self.moe = moe

    def tensor_bytes(self, layer: int, tensor: int) -> int:
        return int(lib().pokit_cuda_decoder_tensor_bytes(self._h, layer, tensor))

    def upload_tensor(self, layer: int, tensor: int, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        call("pokit_cuda_decoder_upload_tensor", self._h, layer, tensor, _np_ptr(data), data.nbytes)

    def synthesize_tensor(self, layer: int, tensor: int, seed: int, stream_id: int) -> None:
        call("pokit_cuda_decoder_synthesize_tensor", self._h, layer, tensor, seed, stream_id)

    def synthesize_model(self) -> None:
        """Every tensor of the synthetic model that pokitlms_b200.gguf writes
        for this shape, generated in HBM from the same seeds (F32 routers,
        norms and DeltaNet parameters uploaded from the host)."""
        from . import gguf, synth
        from ._lib import (DOWN as MD, FFN_NORM, GATE as MG, ROUTER, SHARED_DOWN, SHARED_GATE, SHARED_ROUTER,
                           SHARED_UP, UP as MU)
        s = self.shape
        seed = s.seed
        H, d = s.hidden, s.head_dim
        self.synthesize_tensor(0, _lib.DEC_TOKEN_EMBD, seed, gguf.EMBED_STREAM)
        self.synthesize_tensor(0, _lib.DEC_OUTPUT, seed, gguf.OUTPUT_STREAM)
        self.upload_tensor(0, _lib.DEC_OUTPUT_NORM, np.ones(H, np.float32))
        for l in range(s.layers):
            self.upload_tensor(l, _lib.DEC_ATTN_NORM, np.ones(H, np.float32))
            if not self.hybrid or s.attention_layer(l):
                self.upload_tensor(l, _lib.DEC_ATTN_Q_NORM, np.ones(d, np.float32))
                self.upload_tensor(l, _lib.DEC_ATTN_K_NORM, np.ones(d, np.float32))
                for t, sid in ((_lib.DEC_ATTN_Q, gguf.ATTN_Q), (_lib.DEC_ATTN_K, gguf.ATTN_K),
                               (_lib.DEC_ATTN_V, gguf.ATTN_V), (_lib.DEC_ATTN_OUTPUT, gguf.ATTN_OUTPUT)):
                    self.synthesize_tensor(l, t, seed, synth.stream_id(l, sid))
            else:
                for t, sid in ((_lib.DEC_SSM_QKV, gguf.SSM_QKV), (_lib.DEC_SSM_GATE, gguf.SSM_GATE),
                               (_lib.DEC_SSM_ALPHA, gguf.SSM_ALPHA), (_lib.DEC_SSM_BETA, gguf.SSM_BETA),
                               (_lib.DEC_SSM_OUT, gguf.SSM_OUT)):
                    self.synthesize_tensor(l, t, seed, synth.stream_id(l, sid))
                f = gguf.ssm_f32_tensors(s, l)
                self.upload_tensor(l, _lib.DEC_SSM_CONV1D, f["conv1d"])
                self.upload_tensor(l, _lib.DEC_SSM_A, f["a"])
                self.upload_tensor(l, _lib.DEC_SSM_DT_BIAS, f["dt_bias"])
                self.upload_tensor(l, _lib.DEC_SSM_NORM, f["norm"])
            self.moe.upload_tensor(l, ROUTER, synth.router_weights(s.experts, H, seed, l))
            self.moe.upload_tensor(l, FFN_NORM, np.ones(H, np.float32))
            for t in (MG, MU, MD):
                self.moe.synthesize_tensor(l, t, seed, synth.stream_id(l, t))
            if self.hybrid and s.shared_inter:
                self.moe.upload_tensor(l, SHARED_ROUTER, gguf.shared_router(s, l))
                for t in (SHARED_GATE, SHARED_UP, SHARED_DOWN):
                    self.moe.synthesize_tensor(l, t, seed, synth.stream_id(l, t))

    def forward_token(self, token: int, position: int, logits: bool = True) -> np.ndarray | None:
        out = np.empty(self.shape.vocab, np.float32) if logits else None
        call("pokit_cuda_decoder_forward_token", self._h, token, position, _np_ptr(out))
        return out

    def generate_tokens(self, prompt, max_new: int):
        """(generated ids, stats dict) of greedy decoding after `prompt`."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = C.c_size_t(0)
        st = _lib.GenerationStats()
        call("pokit_cuda_decoder_generate_tokens", self._h, _np_ptr(p), p.size, max_new, _np_ptr(out),
             C.byref(n), C.byref(st))
        return out[:n.value].copy(), {f: getattr(st, f) for f, _ in st._fields_}

    def run_steps(self, steps: int, stream=None) -> None:
        call("pokit_cuda_decoder_run_steps", self._h, steps, _stream(stream))

    def reset(self) -> None:
        call("pokit_cuda_decoder_reset", self._h)

    def launches_per_step(self) -> int:
        return int(lib().pokit_cuda_decoder_launches_per_step(self._h))

    def step_graphs(self) -> tuple[int, str]:
        """(token-step variants replayed as CUDA graphs, why a capture was refused)."""
        buf = C.create_string_buffer(256)
        n = lib().pokit_cuda_decoder_step_graphs(self._h, buf, 256)
        return int(n), buf.value.decode()

    def close(self) -> None:
        if self._h:
            self.moe._h = None
            lib().pokit_cuda_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
