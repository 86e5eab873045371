"""ctypes access to the CPU parity checkers (TEST INFRASTRUCTURE ONLY).

Two libraries, both built by oracle/Makefile:
  * libpokit_oracle.so -- oracle/pokit_oracle.c, a C restatement of the
    reference's MoE expert path (always buildable from this repository);
  * _ref/libpokit_ref.so -- the PokitLMs reference's own C++ kernels and
    dispatch (tensor_linear + row executor) compiled from its sources, plus
    ref_shim.cpp.  Present where it was built (it travels with the tree).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module.  The product library never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_PATH = HERE / "libpokit_oracle.so"
REF_PATH = HERE / "_ref" / "libpokit_ref.so"

F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
BLOCK = {F32: (1, 4), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}


def row_bytes(t: int, cols: int) -> int:
    e, b = BLOCK[t]
    return cols // e * b


class _MoeDesc(C.Structure):
    # Field order of po_moe_layer (pokit_oracle.c) and pr_moe_desc (ref_shim.cpp).
    _fields_ = [
        ("hidden", C.c_size_t), ("inter", C.c_size_t), ("experts", C.c_size_t),
        ("top_k", C.c_size_t), ("flavour", C.c_int), ("normalize", C.c_int),
        ("expert_weights_scale", C.c_float), ("router", C.c_void_p),
        ("gate_type", C.c_uint32), ("up_type", C.c_uint32), ("down_type", C.c_uint32),
        ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
        ("shared_inter", C.c_size_t), ("shared_router", C.c_void_p),
        ("shared_gate_type", C.c_uint32), ("shared_up_type", C.c_uint32),
        ("shared_down_type", C.c_uint32), ("shared_gate", C.c_void_p),
        ("shared_up", C.c_void_p), ("shared_down", C.c_void_p),
    ]


@dataclass
class MoeLayer:
    """One MoE block's tensors in GGUF layout (numpy, host)."""
    hidden: int
    inter: int
    experts: int
    top_k: int
    router: np.ndarray                  # f32 [experts, hidden]
    gate: np.ndarray                    # uint8, experts slices of [inter, hidden]
    up: np.ndarray
    down: np.ndarray                    # uint8, experts slices of [hidden, inter]
    gate_type: int = Q4_K
    up_type: int = Q4_K
    down_type: int = Q4_K
    flavour: int = 0
    normalize: bool = True
    expert_weights_scale: float = 1.0
    shared_inter: int = 0
    shared_router: np.ndarray | None = None
    shared_gate: np.ndarray | None = None
    shared_up: np.ndarray | None = None
    shared_down: np.ndarray | None = None
    shared_gate_type: int = Q8_0
    shared_up_type: int = Q8_0
    shared_down_type: int = Q8_0
    ffn_norm: np.ndarray | None = None
    _keep: list = field(default_factory=list, repr=False)

    def desc(self) -> _MoeDesc:
        arrays = [np.ascontiguousarray(a) if a is not None else None for a in (
            self.router, self.gate, self.up, self.down, self.shared_router, self.shared_gate,
            self.shared_up, self.shared_down)]
        self._keep = arrays
        p = [a.ctypes.data if a is not None else None for a in arrays]
        return _MoeDesc(self.hidden, self.inter, self.experts, self.top_k, self.flavour,
                        int(self.normalize), self.expert_weights_scale, p[0], self.gate_type,
                        self.up_type, self.down_type, p[1], p[2], p[3], self.shared_inter, p[4],
                        self.shared_gate_type, self.shared_up_type, self.shared_down_type,
                        p[5], p[6], p[7])


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def build_port() -> Path:
    if not PORT_PATH.exists() or PORT_PATH.stat().st_mtime < (HERE / "pokit_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return PORT_PATH


class _Lib:
    def __init__(self, path: Path, prefix: str):
        self.dll = C.CDLL(str(path))
        self.prefix = prefix


_port = None
_ref = None


def port() -> C.CDLL:
    """The C restatement (builds it with gcc on first use if needed)."""
    global _port
    if _port is None:
        dll = C.CDLL(str(build_port()))
        V, S, U = C.c_void_p, C.c_size_t, C.c_uint32
        for name, res, args in [
            ("po_linear", C.c_int, [U, V, S, V, S, V]),
            ("po_dequantize_row", C.c_int, [U, V, S, V]),
            ("po_route_qwen3", C.c_int, [V, S, S, C.c_int, V, V]),
            ("po_route_qwen35", C.c_int, [V, S, S, C.c_int, V, V]),
            ("po_moe_forward", C.c_int, [C.POINTER(_MoeDesc), V, V, V, V, V, V, V]),
            ("po_rms_norm", None, [V, V, S, C.c_float, V]),
            ("po_half_to_float", C.c_float, [C.c_uint16]),
            ("po_causal_conv1d_step", None, [V, V, S, S, V, V]),
            ("po_delta_gates", None, [V, V, V, V, S, V, V]),
            ("po_gated_delta_step", C.c_int, [V, V, V, V, V, S, S, S, S, V, V]),
            ("po_rms_norm_gated", None, [V, V, V, S, S, C.c_float, V]),
        ]:
            f = getattr(dll, name)
            f.restype = res
            f.argtypes = args
        _port = dll
    return _port


def ref_available() -> bool:
    return REF_PATH.exists()


def ref() -> C.CDLL:
    """The reference's own kernels (oracle/_ref); raises if not built."""
    global _ref
    if _ref is None:
        if not REF_PATH.exists():
            raise FileNotFoundError(f"{REF_PATH} not built (make -C oracle ref)")
        dll = C.CDLL(str(REF_PATH))
        V, S, U = C.c_void_p, C.c_size_t, C.c_uint32
        for name, res, args in [
            ("pr_linear", C.c_int, [U, V, S, V, S, V]),
            ("pr_tensor_linear", C.c_int, [U, V, S, V, S, V]),
            ("pr_dequantize_row", C.c_int, [U, V, S, V]),
            ("pr_rms_norm", C.c_int, [V, V, S, C.c_float, V]),
            ("pr_moe_create", C.c_void_p, [C.POINTER(_MoeDesc)]),
            ("pr_moe_destroy", None, [V]),
            ("pr_moe_forward", C.c_int, [V, V, V, V, V]),
            ("ref_causal_conv1d_step", C.c_int, [V, V, S, S, V, V]),
            ("ref_gated_delta_step", C.c_int, [V, V, V, V, V, S, S, S, S, V, V]),
            ("ref_rms_norm_gated", C.c_int, [V, V, V, S, S, C.c_float, V]),
        ]:
            f = getattr(dll, name)
            f.restype = res
            f.argtypes = args
        _ref = dll
    return _ref


def _check(st: int, what: str) -> None:
    if st == 1:
        raise ValueError(f"{what}: invalid argument")
    if st:
        raise RuntimeError(f"{what}: status {st}")


# --- C restatement -----------------------------------------------------------

def linear(t: int, x: np.ndarray, w: np.ndarray, rows: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    y = np.empty(rows, dtype=np.float32)
    _check(port().po_linear(t, _fptr(x), x.size, _fptr(w), rows, _fptr(y)), "po_linear")
    return y


def dequantize_row(t: int, enc: np.ndarray, elements: int) -> np.ndarray:
    enc = np.ascontiguousarray(enc)
    out = np.empty(elements, dtype=np.float32)
    _check(port().po_dequantize_row(t, _fptr(enc), elements, _fptr(out)), "po_dequantize_row")
    return out


def route(flavour: int, logits: np.ndarray, k: int, normalize: bool = True):
    """(ids uint32[k], probs f32[k]); raises RuntimeError for non-finite logits."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    ids = np.empty(k, dtype=np.uint32)
    probs = np.empty(k, dtype=np.float32)
    fn = port().po_route_qwen3 if flavour == 0 else port().po_route_qwen35
    _check(fn(_fptr(logits), logits.size, k, int(normalize), _fptr(ids), _fptr(probs)), "route")
    return ids, probs


def moe_forward(layer: MoeLayer, x: np.ndarray):
    """(moe_out f32[hidden], ids, probs, logits) of one MoE block (no residual)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(layer.hidden, dtype=np.float32)
    ids = np.empty(layer.top_k, dtype=np.uint32)
    probs = np.empty(layer.top_k, dtype=np.float32)
    logits = np.empty(layer.experts, dtype=np.float32)
    width = max(layer.inter, layer.shared_inter)
    act = np.empty(3 * width, dtype=np.float32)
    ys = np.empty(layer.hidden, dtype=np.float32)
    d = layer.desc()
    _check(port().po_moe_forward(C.byref(d), _fptr(x), _fptr(out), _fptr(ids), _fptr(probs),
                                 _fptr(logits), _fptr(act), _fptr(ys)), "po_moe_forward")
    return out, ids, probs, logits


def moe_forward_batch(layer: MoeLayer, x: np.ndarray, logits: np.ndarray | None = None):
    """Rows of x ([tokens, hidden] f32) through the block one at a time, as the
    reference's prefill does (src/qwen3_moe_runner.cpp:785-790); routed by the
    given logits ([tokens, experts]) when not None.  Returns (out, ids, probs)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, layer.hidden)
    T = x.shape[0]
    out = np.empty((T, layer.hidden), dtype=np.float32)
    ids = np.empty((T, layer.top_k), dtype=np.uint32)
    probs = np.empty((T, layer.top_k), dtype=np.float32)
    width = max(layer.inter, layer.shared_inter)
    act = np.empty(3 * width, dtype=np.float32)
    ys = np.empty(layer.hidden, dtype=np.float32)
    lg_scratch = np.empty(layer.experts, dtype=np.float32)
    d = layer.desc()
    if logits is not None:
        logits = np.ascontiguousarray(logits, dtype=np.float32).reshape(T, layer.experts)
    for t in range(T):
        row, o, i, p = x[t], out[t], ids[t], probs[t]
        if logits is None:
            st = port().po_moe_forward(C.byref(d), _fptr(row), _fptr(o), _fptr(i), _fptr(p),
                                       _fptr(lg_scratch), _fptr(act), _fptr(ys))
        else:
            st = port().po_moe_forward_routed(C.byref(d), _fptr(row), _fptr(logits[t]), _fptr(o), _fptr(i),
                                              _fptr(p), _fptr(act), _fptr(ys))
        _check(st, "po_moe_forward")
    return out, ids, probs


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    port().po_rms_norm(_fptr(x), _fptr(w), x.size, eps, _fptr(y))
    return y


def decode_layers(layers: list[MoeLayer], hidden: np.ndarray, eps: float) -> np.ndarray:
    """hidden += MoE_l(rms_norm(hidden, ffn_norm_l)) for each layer, in order."""
    h = np.array(hidden, dtype=np.float32, copy=True)
    for L in layers:
        norm = L.ffn_norm if L.ffn_norm is not None else np.ones(L.hidden, dtype=np.float32)
        x = rms_norm(h, norm, eps)
        out, _, _, _ = moe_forward(L, x)
        h = (h + out).astype(np.float32)
    return h


# --- the reference's own kernels (oracle/_ref) --------------------------------

def ref_linear(t: int, x: np.ndarray, w: np.ndarray, rows: int, threaded: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    y = np.empty(rows, dtype=np.float32)
    fn = ref().pr_tensor_linear if threaded else ref().pr_linear
    _check(fn(t, _fptr(x), x.size, _fptr(w), rows, _fptr(y)), "pr_linear")
    return y


def ref_dequantize_row(t: int, enc: np.ndarray, elements: int) -> np.ndarray:
    enc = np.ascontiguousarray(enc)
    out = np.empty(elements, dtype=np.float32)
    _check(ref().pr_dequantize_row(t, _fptr(enc), elements, _fptr(out)), "pr_dequantize_row")
    return out


def ref_rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    _check(ref().pr_rms_norm(_fptr(x), _fptr(w), x.size, eps, _fptr(y)), "pr_rms_norm")
    return y


class RefMoe:
    """A MoE block evaluated by the reference's tensor_linear (multi-threaded
    row executor) and kernels, with the restated routing."""

    def __init__(self, layer: MoeLayer):
        self.layer = layer
        self._desc = layer.desc()
        self.handle = ref().pr_moe_create(C.byref(self._desc))
        if not self.handle:
            raise RuntimeError("pr_moe_create failed")

    def forward(self, x: np.ndarray):
        L = self.layer
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(L.hidden, dtype=np.float32)
        ids = np.empty(L.top_k, dtype=np.uint32)
        probs = np.empty(L.top_k, dtype=np.float32)
        _check(ref().pr_moe_forward(self.handle, _fptr(x), _fptr(out), _fptr(ids), _fptr(probs)),
               "pr_moe_forward")
        return out, ids, probs

    def close(self):
        if self.handle:
            ref().pr_moe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --- Qwen3.5 Gated DeltaNet mixer (src/qwen35_runner.cpp:613-656) ----------------

def delta_net_step(shape: dict, projected, gate, alpha, beta_raw, conv_w, conv_state, a, dt_bias, norm, state,
                   fn_prefix: str = "po"):
    """One token of the DeltaNet mixer between its projections, in place on
    conv_state and state: conv1d + SiLU of the projected q|k|v, the gates,
    the gated delta-rule step and the gated RMSNorm.  Returns (out, conv
    output) F32.  fn_prefix "ref" runs the reference's own conv1d, delta step
    and gated norm (oracle/_ref) instead of the restatement."""
    kh, vh, dk, dv, K = (shape[k] for k in ("key_heads", "value_heads", "key_dim", "value_dim", "conv_kernel"))
    eps = shape["rms_epsilon"]
    P, R = port(), (ref() if fn_prefix == "ref" else None)
    xq = np.array(projected, dtype=np.float32, copy=True)
    conv = (R.ref_causal_conv1d_step if R else P.po_causal_conv1d_step)
    conv(_fptr(xq), _fptr(conv_w), xq.size, K, _fptr(conv_state), _fptr(xq))
    qk = kh * dk
    q, k, v = xq[:qk].copy(), xq[qk:2 * qk].copy(), xq[2 * qk:].copy()
    log_decay = np.empty(vh, np.float32)
    beta = np.empty(vh, np.float32)
    P.po_delta_gates(_fptr(a), _fptr(dt_bias), _fptr(alpha), _fptr(beta_raw), vh, _fptr(log_decay), _fptr(beta))
    out = np.empty(vh * dv, np.float32)
    step = R.ref_gated_delta_step if R else P.po_gated_delta_step
    if step(_fptr(q), _fptr(k), _fptr(v), _fptr(log_decay), _fptr(beta), kh, vh, dk, dv, _fptr(state), _fptr(out)):
        raise ValueError("invalid gated-delta decay or update gate")
    y = np.empty_like(out)
    g = np.ascontiguousarray(gate, dtype=np.float32)
    (R.ref_rms_norm_gated if R else P.po_rms_norm_gated)(_fptr(out), _fptr(norm), _fptr(g), vh, dv, eps, _fptr(y))
    return y, xq
