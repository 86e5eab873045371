"""Seeded synthetic GGUF blocks and activations (host side).

Expert blocks come from a counter-based generator so that the device fill
(pokit_cuda_synthesize_blocks, csrc/pokit_synth.cu) and this numpy version
produce identical bytes for any (seed, stream_id) and any block range:

    key      = mix64(seed * G + stream_id * C + K0)
    word(i)  = mix64(key + (i + 1) * G)                      i = byte_offset // 8
    byte(o)  = (word(o // 8) >> 8 * (o % 8)) & 0xff
    fp16 scale fields := half_rn(1e-3f + f32(u24) * 2^-24 * 9e-3f),
                         u24 = word'(2 * block + field) >> 40, key' = mix64(key ^ S)

so d and dmin are uniform in [1e-3, 1e-2], the 6-bit scales and mins and the
4-bit quants are uniform (every bit is random), as the benchmark
configurations specify.  Router weights (~N(0, 0.02)) and activations
(~N(0, 1)) are F32 draws from numpy's PCG64 with the seed.
"""
from __future__ import annotations

import numpy as np

from ._lib import BLOCK, F32, Q4_K, Q5_K, Q6_K, Q8_0

_G = np.uint64(0x9E3779B97F4A7C15)
_C = np.uint64(0xD1B54A32D192ED03)
_K0 = np.uint64(0x8CB92BA72F3D8DD7)
_S = np.uint64(0x5851F42D4C957F2D)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

# fp16 scale fields per block: (byte offset, field index)
_SCALE_FIELDS = {Q4_K: ((0, 0), (2, 1)), Q5_K: ((0, 0), (2, 1)), Q6_K: ((208, 0),),
                 Q8_0: ((0, 0),)}


def _mix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _key(seed: int, stream_id: int) -> np.uint64:
    with np.errstate(over="ignore"):
        z = (np.array([seed], dtype=np.uint64) * _G
             + np.array([stream_id], dtype=np.uint64) * _C + _K0)
    return _mix64(z)[0]


def _words(key: np.uint64, first: int, count: int) -> np.ndarray:
    idx = np.arange(first + 1, first + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix64(key + idx * _G)


def _scale_halves(skey: np.uint64, first_j: int, count: int) -> np.ndarray:
    w = _words(skey, first_j, count)
    u24 = (w >> np.uint64(40)).astype(np.float32)
    t = u24 * np.float32(2.0 ** -24)                # exact
    v = np.float32(1e-3) + t * np.float32(9e-3)     # two float32 roundings, as on the device
    return v.astype(np.float16)


def synth_blocks(ggml_type: int, nblocks: int, seed: int, stream_id: int,
                 first_block: int = 0) -> np.ndarray:
    """Bytes of blocks [first_block, first_block + nblocks) of the stream, uint8."""
    if ggml_type not in _SCALE_FIELDS:
        raise ValueError("synthetic blocks exist for Q8_0/Q4_K/Q5_K/Q6_K only")
    bb = BLOCK[ggml_type][1]
    start = first_block * bb
    nbytes = nblocks * bb
    w0 = start // 8
    w1 = (start + nbytes + 7) // 8
    key = _key(seed, stream_id)
    raw = _words(key, w0, w1 - w0).view(np.uint8)
    out = raw[start - w0 * 8: start - w0 * 8 + nbytes].copy().reshape(nblocks, bb)
    skey = _mix64(np.array([key ^ _S], dtype=np.uint64))[0]
    fields = _SCALE_FIELDS[ggml_type]
    # field j index = 2 * block + field  (Q6_K / Q8_0 use field 0 only)
    halves = _scale_halves(skey, 2 * first_block, 2 * nblocks).reshape(nblocks, 2)
    for off, field in fields:
        out[:, off:off + 2] = halves[:, field:field + 1].view(np.uint8).reshape(nblocks, 2)
    return out.reshape(-1)


def synth_matrix(ggml_type: int, rows: int, cols: int, seed: int, stream_id: int) -> np.ndarray:
    """A [rows, cols] GGUF-encoded matrix (row-major blocks) as uint8 bytes."""
    elems, _ = BLOCK[ggml_type]
    if cols % elems:
        raise ValueError("cols must be a multiple of the block size")
    return synth_blocks(ggml_type, rows * (cols // elems), seed, stream_id)


def router_weights(experts: int, hidden: int, seed: int, layer: int = 0) -> np.ndarray:
    """F32 [experts, hidden] router ~ N(0, 0.02)."""
    rng = np.random.default_rng([seed, layer, 0x7261])
    return (rng.standard_normal((experts, hidden), dtype=np.float32) * np.float32(0.02))


def activation(hidden: int, seed: int, index: int = 0) -> np.ndarray:
    """F32 [hidden] activation ~ N(0, 1)."""
    rng = np.random.default_rng([seed, index, 0x7861])
    return rng.standard_normal(hidden, dtype=np.float32)


def bf16_round(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(BF16 bit patterns uint16, their F32 values) of x, rounded to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return bits, (bits.astype(np.uint32) << 16).view(np.float32)


def grouped_inputs(tokens: int, experts: int, hidden: int, seed: int = 0, zipf: float = 1.1):
    """A batch for the grouped-expert GEMM: activations ~ N(0, 1) rounded to
    BF16 ([tokens, hidden] as BF16 bits and as F32) and router logits ~ N(0, 1)
    plus a popularity bias -zipf * log(rank) over a seeded ranking of the
    experts (a Zipf(zipf) skew of how often each expert is chosen)."""
    rng = np.random.default_rng([seed, 0x6770])
    bits, xf = bf16_round(rng.standard_normal((tokens, hidden), dtype=np.float32))
    rank = rng.permutation(experts).astype(np.float64) + 1.0
    bias = (-zipf * np.log(rank)).astype(np.float32)
    logits = rng.standard_normal((tokens, experts), dtype=np.float32) + bias[None, :]
    return bits, xf, logits.astype(np.float32)


def stream_id(layer: int, tensor: int) -> int:
    """Stream id of one tensor of one layer (tensor ids as in pokit_cuda_moe_tensor)."""
    return layer * 16 + tensor


__all__ = ["synth_blocks", "synth_matrix", "router_weights", "activation", "bf16_round", "grouped_inputs",
           "stream_id", "F32"]
