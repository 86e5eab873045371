"""CPU tests of the synthetic K-quant GGUF writer (pokitlms_b200.gguf): the
file parses back to the tensor directory and payloads the writer intended
(the GGUF v3 layout of the reference's reader, src/gguf_reader.cpp:173-255),
and -- where the reference's runner is built (oracle/_ref/ref_runner, from a
PokitLMs checkout) -- the reference's own Qwen3MoeRunner loads it and decodes."""
import json
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

from pokitlms_b200 import gguf, synth
from pokitlms_b200._lib import BLOCK

ROOT = Path(__file__).resolve().parents[1]
TINY = gguf.Qwen3MoeShape(layers=2, hidden=256, q_heads=2, kv_heads=1, head_dim=128, experts=4, top_k=2,
                          expert_inter=256, vocab=1024, context=256)


def _read(path):
    b = path.read_bytes()
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from(fmt, b, off)
        off += struct.calcsize(fmt)
        return v if len(v) > 1 else v[0]

    def string():
        n = take("<Q")
        nonlocal off
        s = b[off:off + n].decode()
        off += n
        return s

    def value(t):
        if t == 8:
            return string()
        if t == 9:
            et, n = take("<IQ")
            return [value(et) for _ in range(n)]
        return take({0: "<B", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q"}[t])

    assert b[:4] == b"GGUF"
    off = 4
    version, nt, nm = take("<IQQ")
    meta = {}
    for _ in range(nm):
        k = string()
        meta[k] = value(take("<I"))
    tensors = []
    for _ in range(nt):
        name = string()
        rank = take("<I")
        dims = [take("<Q") for _ in range(rank)]
        t, o = take("<IQ")
        tensors.append((name, dims, t, o))
    data = (off + gguf.ALIGNMENT - 1) // gguf.ALIGNMENT * gguf.ALIGNMENT
    return version, meta, tensors, data, b


def test_writer_layout_round_trips(tmp_path):
    path = gguf.write_qwen3moe(tmp_path / "m.gguf", TINY)
    version, meta, tensors, data, raw = _read(path)
    assert version == 3 and meta["general.architecture"] == "qwen3moe"
    assert meta["qwen3moe.expert_weights_norm"] == 1 and meta["qwen3moe.block_count"] == 2
    assert len(meta["tokenizer.ggml.tokens"]) == TINY.vocab == len(set(meta["tokenizer.ggml.tokens"]))
    assert meta["tokenizer.ggml.tokens"][:256] == gguf.byte_level_symbols()
    names = [t[0] for t in tensors]
    assert names[0] == "token_embd.weight" and names[-1] == "output.weight"
    assert len(names) == 3 + 12 * TINY.layers
    for name, dims, t, o in tensors:
        assert o % gguf.ALIGNMENT == 0
        elems, bb = BLOCK[t]
        rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        nbytes = rows * dims[0] // elems * bb
        assert data + o + nbytes <= len(raw)
    # One quantised payload equals the generator's bytes.
    name, dims, t, o = next(x for x in tensors if x[0] == "blk.1.attn_q.weight")
    want = synth.synth_matrix(t, dims[1], dims[0], TINY.seed, synth.stream_id(1, gguf.ATTN_Q))
    assert np.array_equal(np.frombuffer(raw, np.uint8, want.size, data + o), want)


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "ref_runner").exists(),
                    reason="the reference's runner is not built on this machine")
def test_reference_runner_loads_the_model(tmp_path):
    path = gguf.write_qwen3moe(tmp_path / "m.gguf", TINY)
    (tmp_path / "p.txt").write_text("1 2 3 4 5")
    r = subprocess.run([str(ROOT / "oracle" / "_ref" / "ref_runner"), str(path), str(tmp_path / "p.txt"), "6"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert 1 <= len(out["ids"]) <= 6 and all(0 <= i < TINY.vocab for i in out["ids"])


TINY35 = gguf.Qwen35MoeShape(layers=4, hidden=256, q_heads=2, kv_heads=1, head_dim=128, rotary_dim=32,
                             rope_sections=(6, 5, 5, 0), ssm_state_size=32, ssm_group_count=2,
                             ssm_time_step_rank=4, ssm_inner_size=256, experts=8, top_k=2, expert_inter=256,
                             shared_inter=256, vocab=512, context=64)


def test_qwen35_writer_layout(tmp_path):
    path = gguf.write_qwen35moe(tmp_path / "m35.gguf", TINY35)
    version, meta, tensors, data, raw = _read(path)
    a = "qwen35moe."
    assert version == 3 and meta["general.architecture"] == "qwen35moe"
    assert meta[a + "full_attention_interval"] == 4 and list(meta[a + "rope.dimension_sections"]) == [6, 5, 5, 0]
    assert meta[a + "ssm.inner_size"] == 256 and meta[a + "expert_shared_feed_forward_length"] == 256
    names = {t[0]: t for t in tensors}
    # Layer 3 is full attention (gated query: twice the query rows), 0..2 Gated DeltaNet.
    assert tuple(names["blk.3.attn_q.weight"][1]) == (256, 2 * 2 * 128) and "blk.3.attn_qkv.weight" not in names
    assert tuple(names["blk.0.attn_qkv.weight"][1]) == (256, 2 * 2 * 32 + 256) and "blk.0.attn_q.weight" not in names
    assert tuple(names["blk.0.ssm_conv1d.weight"][1]) == (4, TINY35.conv_channels)
    assert names["blk.0.ffn_down_exps.weight"][2] == TINY35.down_type(0)
    assert names["blk.1.ffn_down_exps.weight"][2] == TINY35.down_type(1)
    for name, dims, t, o in tensors:
        elems, bb = BLOCK[t]
        rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        assert data + o + rows * dims[0] // elems * bb <= len(raw)
    name, dims, t, o = names["blk.2.ssm_out.weight"]
    want = synth.synth_matrix(t, dims[1], dims[0], TINY35.seed, synth.stream_id(2, gguf.SSM_OUT))
    assert np.array_equal(np.frombuffer(raw, np.uint8, want.size, data + o), want)
    name, dims, t, o = names["blk.1.ssm_a"]
    assert np.array_equal(np.frombuffer(raw, np.float32, dims[0], data + o), gguf.ssm_f32_tensors(TINY35, 1)["a"])


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "ref_runner").exists(),
                    reason="the reference's runner is not built on this machine")
def test_reference_qwen35_runner_loads_the_model(tmp_path):
    path = gguf.write_qwen35moe(tmp_path / "m35.gguf", TINY35)
    (tmp_path / "p.txt").write_text("1 2 3 4 5")
    r = subprocess.run([str(ROOT / "oracle" / "_ref" / "ref_runner"), "--qwen35", str(path), str(tmp_path / "p.txt"),
                        "6"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert 1 <= len(out["ids"]) <= 6 and all(0 <= i < TINY35.vocab for i in out["ids"])
