"""Synthetic K-quant GGUF models (version 3) for the Qwen3-MoE decoder and
the Qwen3.5-MoE hybrid.

Writes a `qwen3moe` model whose quantised tensors come from the seeded
counter-based generator in pokitlms_b200.synth (so the GPU can synthesise
the very same bytes in HBM without reading the file), F32 routers ~N(0, 0.02)
and F32 norms of 1.0, plus a GPT-2 byte-level tokenizer vocabulary that the
reference's QwenBpeTokenizer accepts.  The reference's own runner
(Qwen3MoeRunner::generate_tokens) then loads the file, which is how its
greedy token ids become the parity target of the CUDA decoder.

File layout (the GGUF v3 container as the reference reads it,
src/gguf_reader.cpp:173-255): magic "GGUF", version 3, tensor count,
metadata count, the metadata key/value pairs, the tensor directory (name,
rank, dimensions with the contiguous one first, GGML type, offset relative
to the data section), padding to `general.alignment`, then every tensor
payload at an aligned offset.  Tensor names and shapes follow the
reference's Qwen3-MoE index (src/qwen3_moe_index.cpp:36-90) and metadata
keys its configuration loader (src/architecture.cpp:59-120); the tokenizer
keys are the ones src/qwen_bpe_tokenizer.cpp:152-246 checks.  The
`qwen35moe` model follows the Qwen3.5 index (src/qwen35_index.cpp:118-357):
Gated DeltaNet layers with every full_attention_interval-th layer full
attention (gated query), and MoE blocks with a sigmoid-gated shared expert;
Qwen35Runner::generate_tokens reads it.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import synth
from ._lib import BLOCK, F32, Q4_K, Q5_K, Q6_K, Q8_0

ALIGNMENT = 32

# Metadata value types of the GGUF format.
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)

# Stream ids of the tensors outside the MoE blocks (per-layer MoE tensors use
# synth.stream_id(layer, tensor) with the pokit_cuda_moe_tensor ids 0..8).
ATTN_Q, ATTN_K, ATTN_V, ATTN_OUTPUT = 9, 10, 11, 12
GLOBAL_LAYER = 1 << 12                # pseudo-layer of the embedding and the LM head
EMBED_STREAM = synth.stream_id(GLOBAL_LAYER, 0)
OUTPUT_STREAM = synth.stream_id(GLOBAL_LAYER, 1)


@dataclass
class Qwen3MoeShape:
    """Benchmark configuration 2's model (Qwen3-30B-A3B-shaped) by default."""
    layers: int = 48
    hidden: int = 2048
    q_heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    expert_inter: int = 768
    vocab: int = 151936
    context: int = 4096
    rms_epsilon: float = 1e-6
    rope_theta: float = 1e6
    attn_type: int = Q4_K
    expert_type: int = Q4_K
    embed_type: int = Q6_K
    output_type: int = Q6_K
    seed: int = 0

    @property
    def eos(self) -> int:
        return self.vocab - 1


def _s(text: str) -> bytes:
    b = text.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    return _s(key) + struct.pack("<I", vtype) + payload


def _u32(key, v):
    return _kv(key, _U32, struct.pack("<I", v))


def _f32(key, v):
    return _kv(key, _F32, struct.pack("<f", v))


def _str(key, v):
    return _kv(key, _STR, _s(v))


def _bool(key, v):
    return _kv(key, _BOOL, struct.pack("<B", 1 if v else 0))


def _str_array(key, values):
    return _kv(key, _ARR, struct.pack("<IQ", _STR, len(values)) + b"".join(_s(v) for v in values))


def _i32_array(key, values):
    return _kv(key, _ARR, struct.pack("<IQ", _I32, len(values)) + np.asarray(values, "<i4").tobytes())


def _u32_array(key, values):
    return _kv(key, _ARR, struct.pack("<IQ", _U32, len(values)) + np.asarray(values, "<u4").tobytes())


def byte_level_symbols() -> list[str]:
    """The 256 base symbols of a GPT-2 byte-level vocabulary: printable bytes
    stand for themselves, the rest map to code points from 256 up in byte order."""
    keep = set(range(0x21, 0x7F)) | set(range(0xA1, 0xAD)) | set(range(0xAE, 0x100))
    out, extra = [], 0x100
    for b in range(256):
        if b in keep:
            out.append(chr(b))
        else:
            out.append(chr(extra))
            extra += 1
    return out


def tokenizer_vocab(vocab: int) -> list[str]:
    """The byte symbols, then unique filler tokens up to `vocab` entries."""
    base = byte_level_symbols()
    if vocab < len(base) + 1:
        raise ValueError("vocabulary must hold the 256 byte tokens and an end token")
    return base + [f"<|tok{i}|>" for i in range(len(base), vocab)]


@dataclass
class _Tensor:
    name: str
    dims: tuple            # GGUF order: contiguous dimension first
    ggml_type: int
    nbytes: int
    fill: object           # callable(first_block, nblocks) -> bytes, or an array


def _quant(ggml_type, rows, cols, seed, stream):
    elems, bb = BLOCK[ggml_type]
    nblocks = rows * (cols // elems)
    return nblocks * bb, (lambda first, n: synth.synth_blocks(ggml_type, n, seed, stream, first_block=first))


def model_tensors(shape: Qwen3MoeShape) -> list[_Tensor]:
    H, s = shape.hidden, shape.seed
    qd, kd = shape.q_heads * shape.head_dim, shape.kv_heads * shape.head_dim
    ones_h = np.ones(H, np.float32)
    ones_d = np.ones(shape.head_dim, np.float32)
    out = []

    def quant(name, dims, t, rows, cols, stream):
        nb, fill = _quant(t, rows, cols, s, stream)
        out.append(_Tensor(name, dims, t, nb, fill))

    def f32(name, dims, arr):
        out.append(_Tensor(name, dims, F32, arr.nbytes, np.ascontiguousarray(arr, np.float32)))

    quant("token_embd.weight", (H, shape.vocab), shape.embed_type, shape.vocab, H, EMBED_STREAM)
    for l in range(shape.layers):
        p = f"blk.{l}."
        f32(p + "attn_norm.weight", (H,), ones_h)
        quant(p + "attn_q.weight", (H, qd), shape.attn_type, qd, H, synth.stream_id(l, ATTN_Q))
        f32(p + "attn_q_norm.weight", (shape.head_dim,), ones_d)
        quant(p + "attn_k.weight", (H, kd), shape.attn_type, kd, H, synth.stream_id(l, ATTN_K))
        f32(p + "attn_k_norm.weight", (shape.head_dim,), ones_d)
        quant(p + "attn_v.weight", (H, kd), shape.attn_type, kd, H, synth.stream_id(l, ATTN_V))
        quant(p + "attn_output.weight", (qd, H), shape.attn_type, H, qd, synth.stream_id(l, ATTN_OUTPUT))
        f32(p + "ffn_norm.weight", (H,), ones_h)
        f32(p + "ffn_gate_inp.weight", (H, shape.experts), synth.router_weights(shape.experts, H, s, l))
        E, I = shape.experts, shape.expert_inter
        quant(p + "ffn_gate_exps.weight", (H, I, E), shape.expert_type, E * I, H, synth.stream_id(l, 1))
        quant(p + "ffn_up_exps.weight", (H, I, E), shape.expert_type, E * I, H, synth.stream_id(l, 2))
        quant(p + "ffn_down_exps.weight", (I, H, E), shape.expert_type, E * H, I, synth.stream_id(l, 3))
    f32("output_norm.weight", (H,), ones_h)
    quant("output.weight", (H, shape.vocab), shape.output_type, shape.vocab, H, OUTPUT_STREAM)
    return out


def metadata(shape: Qwen3MoeShape) -> list[bytes]:
    a = "qwen3moe."
    vocab = tokenizer_vocab(shape.vocab)
    return [
        _str("general.architecture", "qwen3moe"),
        _u32("general.alignment", ALIGNMENT),
        _u32(a + "context_length", shape.context),
        _u32(a + "embedding_length", shape.hidden),
        _u32(a + "block_count", shape.layers),
        _u32(a + "feed_forward_length", shape.expert_inter * shape.top_k),
        _u32(a + "attention.head_count", shape.q_heads),
        _u32(a + "attention.head_count_kv", shape.kv_heads),
        _u32(a + "attention.key_length", shape.head_dim),
        _u32(a + "attention.value_length", shape.head_dim),
        _u32(a + "rope.dimension_count", shape.head_dim),
        _u32(a + "expert_count", shape.experts),
        _u32(a + "expert_used_count", shape.top_k),
        _u32(a + "expert_feed_forward_length", shape.expert_inter),
        _bool(a + "expert_weights_norm", True),
        _f32(a + "attention.layer_norm_rms_epsilon", shape.rms_epsilon),
        _f32(a + "rope.freq_base", shape.rope_theta),
        _str("tokenizer.ggml.model", "gpt2"),
        _str("tokenizer.ggml.pre", "qwen2"),
        _str_array("tokenizer.ggml.tokens", vocab),
        _i32_array("tokenizer.ggml.token_type", [1] * len(vocab)),
        _str_array("tokenizer.ggml.merges", []),
        _u32("tokenizer.ggml.bos_token_id", shape.eos),
        _u32("tokenizer.ggml.eos_token_id", shape.eos),
    ]


def write_qwen3moe(path: str | Path, shape: Qwen3MoeShape, chunk_bytes: int = 64 << 20) -> Path:
    """Writes the synthetic model to `path`, streaming tensors in chunks."""
    return _write(path, model_tensors(shape), metadata(shape), chunk_bytes)


# Stream ids of the Gated DeltaNet projections: a layer is either full
# attention or DeltaNet, so they reuse the attention tensors' ids 9..12.
SSM_QKV, SSM_GATE, SSM_ALPHA, SSM_OUT, SSM_BETA = 9, 10, 11, 12, 13


@dataclass
class Qwen35MoeShape:
    """Benchmark configuration 3's model (Qwen3.5-MoE hybrid) by default: 48
    layers, every fourth full attention (16 query / 2 KV heads of 256, gated
    query, MRoPE over 64 dimensions), the others Gated DeltaNet (16 key heads,
    32 value heads of 128, conv kernel 4); MoE hidden 2048, 512 experts
    top-10, inter 512, a 512-wide Q8_0 shared expert; Q4_K gate/up, Q5_K
    (even layers) / Q6_K (odd layers) down."""
    layers: int = 48
    hidden: int = 2048
    q_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 256
    rotary_dim: int = 64
    rope_sections: tuple = (11, 11, 10, 0)
    full_attention_interval: int = 4
    ssm_conv_kernel: int = 4
    ssm_state_size: int = 128
    ssm_group_count: int = 16
    ssm_time_step_rank: int = 32
    ssm_inner_size: int = 4096
    experts: int = 512
    top_k: int = 10
    expert_inter: int = 512
    shared_inter: int = 512
    expert_weights_scale: float = 1.0
    vocab: int = 151936
    context: int = 4096
    rms_epsilon: float = 1e-6
    rope_theta: float = 1e7
    attn_type: int = Q4_K
    expert_type: int = Q4_K
    down_types: tuple = (Q5_K, Q6_K)      # layer l uses down_types[l % len]
    shared_type: int = Q8_0
    embed_type: int = Q6_K
    output_type: int = Q6_K
    seed: int = 0

    @property
    def eos(self) -> int:
        return self.vocab - 1

    def attention_layer(self, layer: int) -> bool:
        return (layer + 1) % self.full_attention_interval == 0

    def down_type(self, layer: int) -> int:
        return self.down_types[layer % len(self.down_types)]

    @property
    def conv_channels(self) -> int:
        return 2 * self.ssm_group_count * self.ssm_state_size + self.ssm_inner_size


def ssm_f32_tensors(shape: Qwen35MoeShape, layer: int) -> dict:
    """The F32 tensors of one Gated DeltaNet layer: conv1d weights ~ N(0, 0.25)
    ([channels][kernel]), ssm_a = -A with A ~ U[1, 16] (the converter stores
    -exp(A_log)), dt bias ~ N(0, 0.5), ssm_norm = 1."""
    rng = np.random.default_rng([shape.seed, layer, 0x73736D])
    hv = shape.ssm_time_step_rank
    return {
        "conv1d": (rng.standard_normal((shape.conv_channels, shape.ssm_conv_kernel), dtype=np.float32)
                   * np.float32(0.25)),
        "a": -rng.uniform(1.0, 16.0, hv).astype(np.float32),
        "dt_bias": rng.standard_normal(hv, dtype=np.float32) * np.float32(0.5),
        "norm": np.ones(shape.ssm_inner_size // hv, np.float32),
    }


def shared_router(shape, layer: int) -> np.ndarray:
    """F32 [hidden] shared-expert gate ~ N(0, 0.02)."""
    return synth.router_weights(1, shape.hidden, shape.seed, 1000 + layer)[0]


def qwen35_tensors(shape: Qwen35MoeShape) -> list[_Tensor]:
    H, s = shape.hidden, shape.seed
    qd, kd = shape.q_heads * shape.head_dim, shape.kv_heads * shape.head_dim
    ones_h = np.ones(H, np.float32)
    ones_d = np.ones(shape.head_dim, np.float32)
    hv, vw, ch = shape.ssm_time_step_rank, shape.ssm_inner_size, shape.conv_channels
    out = []

    def quant(name, dims, t, rows, cols, stream):
        nb, fill = _quant(t, rows, cols, s, stream)
        out.append(_Tensor(name, dims, t, nb, fill))

    def f32(name, dims, arr):
        out.append(_Tensor(name, dims, F32, arr.nbytes, np.ascontiguousarray(arr, np.float32)))

    quant("token_embd.weight", (H, shape.vocab), shape.embed_type, shape.vocab, H, EMBED_STREAM)
    for l in range(shape.layers):
        p = f"blk.{l}."
        f32(p + "attn_norm.weight", (H,), ones_h)
        f32(p + "post_attention_norm.weight", (H,), ones_h)
        if shape.attention_layer(l):
            quant(p + "attn_q.weight", (H, 2 * qd), shape.attn_type, 2 * qd, H, synth.stream_id(l, ATTN_Q))
            quant(p + "attn_k.weight", (H, kd), shape.attn_type, kd, H, synth.stream_id(l, ATTN_K))
            quant(p + "attn_v.weight", (H, kd), shape.attn_type, kd, H, synth.stream_id(l, ATTN_V))
            f32(p + "attn_q_norm.weight", (shape.head_dim,), ones_d)
            f32(p + "attn_k_norm.weight", (shape.head_dim,), ones_d)
            quant(p + "attn_output.weight", (qd, H), shape.attn_type, H, qd, synth.stream_id(l, ATTN_OUTPUT))
        else:
            f = ssm_f32_tensors(shape, l)
            quant(p + "attn_qkv.weight", (H, ch), shape.attn_type, ch, H, synth.stream_id(l, SSM_QKV))
            quant(p + "attn_gate.weight", (H, vw), shape.attn_type, vw, H, synth.stream_id(l, SSM_GATE))
            f32(p + "ssm_a", (hv,), f["a"])
            quant(p + "ssm_alpha.weight", (H, hv), shape.attn_type, hv, H, synth.stream_id(l, SSM_ALPHA))
            quant(p + "ssm_beta.weight", (H, hv), shape.attn_type, hv, H, synth.stream_id(l, SSM_BETA))
            f32(p + "ssm_conv1d.weight", (shape.ssm_conv_kernel, ch), f["conv1d"])
            f32(p + "ssm_dt.bias", (hv,), f["dt_bias"])
            f32(p + "ssm_norm.weight", (vw // hv,), f["norm"])
            quant(p + "ssm_out.weight", (vw, H), shape.attn_type, H, vw, synth.stream_id(l, SSM_OUT))
        E, I, Is = shape.experts, shape.expert_inter, shape.shared_inter
        f32(p + "ffn_gate_inp.weight", (H, E), synth.router_weights(E, H, s, l))
        quant(p + "ffn_gate_exps.weight", (H, I, E), shape.expert_type, E * I, H, synth.stream_id(l, 1))
        quant(p + "ffn_up_exps.weight", (H, I, E), shape.expert_type, E * I, H, synth.stream_id(l, 2))
        quant(p + "ffn_down_exps.weight", (I, H, E), shape.down_type(l), E * H, I, synth.stream_id(l, 3))
        f32(p + "ffn_gate_inp_shexp.weight", (H,), shared_router(shape, l))
        quant(p + "ffn_gate_shexp.weight", (H, Is), shape.shared_type, Is, H, synth.stream_id(l, 6))
        quant(p + "ffn_up_shexp.weight", (H, Is), shape.shared_type, Is, H, synth.stream_id(l, 7))
        quant(p + "ffn_down_shexp.weight", (Is, H), shape.shared_type, H, Is, synth.stream_id(l, 8))
    f32("output_norm.weight", (H,), ones_h)
    quant("output.weight", (H, shape.vocab), shape.output_type, shape.vocab, H, OUTPUT_STREAM)
    return out


def qwen35_metadata(shape: Qwen35MoeShape) -> list[bytes]:
    a = "qwen35moe."
    vocab = tokenizer_vocab(shape.vocab)
    return [
        _str("general.architecture", "qwen35moe"),
        _u32("general.alignment", ALIGNMENT),
        _u32(a + "context_length", shape.context),
        _u32(a + "embedding_length", shape.hidden),
        _u32(a + "block_count", shape.layers),
        _u32(a + "expert_count", shape.experts),
        _u32(a + "expert_used_count", shape.top_k),
        _u32(a + "expert_feed_forward_length", shape.expert_inter),
        _u32(a + "expert_shared_feed_forward_length", shape.shared_inter),
        _bool(a + "expert_weights_norm", True),
        _f32(a + "expert_weights_scale", shape.expert_weights_scale),
        _u32(a + "attention.head_count", shape.q_heads),
        _u32(a + "attention.head_count_kv", shape.kv_heads),
        _u32(a + "attention.key_length", shape.head_dim),
        _u32(a + "attention.value_length", shape.head_dim),
        _u32(a + "rope.dimension_count", shape.rotary_dim),
        _u32_array(a + "rope.dimension_sections", list(shape.rope_sections)),
        _u32(a + "ssm.conv_kernel", shape.ssm_conv_kernel),
        _u32(a + "ssm.state_size", shape.ssm_state_size),
        _u32(a + "ssm.group_count", shape.ssm_group_count),
        _u32(a + "ssm.time_step_rank", shape.ssm_time_step_rank),
        _u32(a + "ssm.inner_size", shape.ssm_inner_size),
        _u32(a + "full_attention_interval", shape.full_attention_interval),
        _f32(a + "attention.layer_norm_rms_epsilon", shape.rms_epsilon),
        _f32(a + "rope.freq_base", shape.rope_theta),
        _str("tokenizer.ggml.model", "gpt2"),
        _str("tokenizer.ggml.pre", "qwen35"),
        _str_array("tokenizer.ggml.tokens", vocab),
        _i32_array("tokenizer.ggml.token_type", [1] * len(vocab)),
        _str_array("tokenizer.ggml.merges", []),
        _u32("tokenizer.ggml.bos_token_id", shape.eos),
        _u32("tokenizer.ggml.eos_token_id", shape.eos),
    ]


def write_qwen35moe(path: str | Path, shape: Qwen35MoeShape, chunk_bytes: int = 64 << 20) -> Path:
    """Writes the synthetic Qwen3.5-MoE hybrid to `path`, streaming tensors in chunks."""
    return _write(path, qwen35_tensors(shape), qwen35_metadata(shape), chunk_bytes)


def _write(path: str | Path, tensors: list[_Tensor], meta: list[bytes], chunk_bytes: int) -> Path:
    path = Path(path)
    offsets, off = [], 0
    for t in tensors:
        off = (off + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
        offsets.append(off)
        off += t.nbytes
    directory = b"".join(
        _s(t.name) + struct.pack("<I", len(t.dims)) + b"".join(struct.pack("<Q", d) for d in t.dims)
        + struct.pack("<IQ", t.ggml_type, o) for t, o in zip(tensors, offsets))
    header = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)) + b"".join(meta) + directory
    pad = (ALIGNMENT - len(header) % ALIGNMENT) % ALIGNMENT
    with open(path, "wb") as f:
        f.write(header + b"\0" * pad)
        base = f.tell()
        for t, o in zip(tensors, offsets):
            f.write(b"\0" * (base + o - f.tell()))
            if isinstance(t.fill, np.ndarray):
                f.write(t.fill.tobytes())
                continue
            bb = BLOCK[t.ggml_type][1]
            nblocks = t.nbytes // bb
            step = max(1, chunk_bytes // bb)
            for first in range(0, nblocks, step):
                f.write(t.fill(first, min(step, nblocks - first)).tobytes())
    return path
