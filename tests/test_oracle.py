"""CPU tests of the oracle (pokit_oracle.c): pinned to the reference's own
known-answer blocks, to golden outputs of the reference's kernels, and
bit-for-bit to the reference build where it is present."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

import cases
from oracle import oracle as O
from pokitlms_b200 import synth

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("index", [0, 1])
def test_q5k_reference_known_answers(index):
    """regression_test.cpp:86-112: decode exactly, linear within 0.01 (bias 0.75)."""
    block, expected = cases.q5k_known_answer_blocks()[index]
    decoded = O.dequantize_row(cases.Q5_K, block, 256)
    assert np.array_equal(decoded, expected)
    x = cases.check_block_input()
    dot = np.float32(0.75) + np.dot(x.astype(np.float64), expected.astype(np.float64))
    y = O.linear(cases.Q5_K, x, block, 1)[0] + np.float32(0.75)
    assert abs(y - dot) < 0.01


@pytest.mark.parametrize("builder,t", [(cases.q4k_known_answer_block, cases.Q4_K),
                                       (cases.q6k_known_answer_block, cases.Q6_K),
                                       (cases.q8_0_known_answer_block, cases.Q8_0)])
def test_layout_known_answers(builder, t):
    block, expected = builder()
    n = expected.size
    assert np.array_equal(O.dequantize_row(t, block, n), expected)
    x = cases.check_block_input()[:n]
    y = O.linear(t, x, block, 1)[0]
    assert abs(y - float(np.dot(x.astype(np.float64), expected))) < 1e-3


def test_half_to_float_exhaustive():
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.port().po_half_to_float(int(b)) for b in bits[::97]], dtype=np.float32)
    want = ref[::97]
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(want))


def test_vulkan_parity_cases_match_golden():
    """The CPU outputs of the reference's parity cases (vulkan_linear_cases.hpp),
    computed by the reference's tensor_linear, reproduced bit-for-bit."""
    g = np.load(GOLDEN / "vulkan_cases.npz")
    seen = 0
    for t, rows, cols, payload, inp in cases.vulkan_parity_cases():
        if f"t{t}_expected" not in g:
            continue
        assert sha(payload) == str(g[f"t{t}_payload_sha"]), f"generator drifted for type {t}"
        assert sha(inp) == str(g[f"t{t}_input_sha"])
        x = inp
        for rep in range(3):
            y = O.linear(t, x, payload, rows)
            assert np.array_equal(y.view(np.uint32), g[f"t{t}_expected"][rep].view(np.uint32)), (t, rep)
            x = (x * np.float32(-0.75)).astype(np.float32)
        seen += 1
    assert seen == 5


def test_moe_config1_matches_golden():
    L = cases.moe_layer()
    x = synth.activation(2048, 0)
    g = np.load(GOLDEN / "moe_config1.npz")
    assert sha(L.gate) == str(g["gate_sha"]) and sha(L.down) == str(g["down_sha"])
    assert sha(L.router) == str(g["router_sha"]) and sha(x) == str(g["x_sha"])
    out, ids, probs, logits = O.moe_forward(L, x)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(probs, g["probs"])
    assert np.array_equal(out, g["out"])


def test_moe_qwen35_shared_expert_matches_golden():
    L = cases.moe_layer(hidden=2048, inter=512, experts=64, top_k=10, seed=1, flavour=1,
                        down_type=cases.Q6_K, shared_inter=512, expert_weights_scale=2.5)
    x = synth.activation(2048, 1)
    g = np.load(GOLDEN / "moe_qwen35.npz")
    out, ids, probs, _ = O.moe_forward(L, x)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(out, g["out"])


def test_decode_chain_matches_golden():
    layers = [cases.moe_layer(hidden=2048, inter=768, experts=32, top_k=8, seed=3, layer=l,
                              with_norm=True) for l in range(4)]
    h = O.decode_layers(layers, synth.activation(2048, 3, 0), 1e-6)
    g = np.load(GOLDEN / "decode4.npz")
    assert np.array_equal(h, g["hidden"])


def test_routing_ties_go_to_lower_id():
    logits = np.array([0.5, 2.0, 2.0, -1.0, 2.0, 1.0], dtype=np.float32)
    for flavour in (0, 1):
        ids, probs = O.route(flavour, logits, 3)
        assert list(ids) == [1, 2, 4]
        assert abs(float(probs.sum()) - 1.0) < 1e-6


def test_routing_unnormalised_and_full_k():
    rng = np.random.default_rng(5)
    logits = rng.standard_normal(16).astype(np.float32)
    ids, probs = O.route(0, logits, 16, normalize=False)
    assert sorted(ids.tolist()) == list(range(16))
    p = np.exp(logits.astype(np.float64) - logits.max())
    p /= p.sum()
    assert np.allclose(probs, p[ids], rtol=1e-6)


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_routing_rejects_non_finite(bad):
    logits = np.zeros(8, dtype=np.float32)
    logits[3] = bad
    for flavour in (0, 1):
        with pytest.raises(RuntimeError):
            O.route(flavour, logits, 2)


def test_routing_rejects_bad_k():
    with pytest.raises(ValueError):
        O.route(0, np.zeros(4, dtype=np.float32), 5)
    with pytest.raises(ValueError):
        O.route(0, np.zeros(4, dtype=np.float32), 0)


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("t,cols", [(cases.Q4_K, 2048), (cases.Q4_K, 768), (cases.Q5_K, 512),
                                    (cases.Q6_K, 512), (cases.Q6_K, 768), (cases.Q8_0, 2048),
                                    (cases.F32, 2048), (cases.F32, 257)])
def test_port_is_bit_exact_with_reference_build(t, cols):
    rows = 300  # >= 256 exercises the reference's threaded row executor
    if t == cases.F32:
        w = np.random.default_rng(1).standard_normal(rows * cols).astype(np.float32)
    else:
        w = synth.synth_matrix(t, rows, cols, 9, 4)
    x = synth.activation(cols, 9)
    a = O.linear(t, x, w, rows)
    b = O.ref_linear(t, x, w, rows, threaded=True)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    if t != cases.F32:
        rb = O.row_bytes(t, cols)
        assert np.array_equal(O.dequantize_row(t, w[:rb], cols).view(np.uint32),
                              O.ref_dequantize_row(t, w[:rb], cols).view(np.uint32))


@needs_ref
def test_port_moe_bit_exact_with_reference_build():
    L = cases.moe_layer(hidden=1024, inter=512, experts=16, top_k=4, seed=11, flavour=1,
                        down_type=cases.Q5_K, shared_inter=256, expert_weights_scale=1.25)
    x = synth.activation(1024, 11)
    out, ids, probs, _ = O.moe_forward(L, x)
    r = O.RefMoe(L)
    out2, ids2, probs2 = r.forward(x)
    assert np.array_equal(ids, ids2) and np.array_equal(probs, probs2)
    assert np.array_equal(out, out2)
