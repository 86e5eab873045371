"""GPU parity tests of the MoE block through the C ABI (pokit_cuda_moe_*).

Bar (north star): routed expert ids identical to the reference except where
the top-k logit margin is below 1e-5; MoE-layer outputs within
max-abs error <= 1e-3 x the output L2-RMS.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from pokitlms_b200 import backend as B
from pokitlms_b200 import synth
from pokitlms_b200._lib import (DOWN, FFN_NORM, GATE, ROUTER, SHARED_DOWN, SHARED_GATE,
                                SHARED_ROUTER, SHARED_UP, UP, PokitCudaError)

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 1e-3


def rms(a):
    return float(np.sqrt(np.mean(np.asarray(a, dtype=np.float64) ** 2)))


def assert_moe_close(out, ref):
    assert np.all(np.isfinite(out))
    err = float(np.max(np.abs(out.astype(np.float64) - ref)))
    assert err <= TOL * rms(ref), (err, rms(ref))


def assert_routes(ids, ref_ids, logits, k):
    if not np.array_equal(ids, ref_ids):
        assert cases.route_margin(logits, k) < 1e-5, (ids, ref_ids)


def make_backend(L, layers=1, **extra):
    kw = dict(layers=layers, hidden=L.hidden, inter=L.inter, experts=L.experts, top_k=L.top_k,
              flavour=L.flavour, normalize_top_k=L.normalize,
              expert_weights_scale=L.expert_weights_scale, down_type=L.down_type)
    if L.shared_inter:
        kw.update(shared_inter=L.shared_inter)
    kw.update(extra)
    return B.CudaMoeBackend(**kw)


def upload(be, layer, L):
    be.upload_layer(layer, router=L.router, gate=L.gate, up=L.up, down=L.down,
                    ffn_norm=L.ffn_norm if L.ffn_norm is not None else np.ones(L.hidden, np.float32),
                    shared_router=L.shared_router, shared_gate=L.shared_gate,
                    shared_up=L.shared_up, shared_down=L.shared_down)


@pytest.fixture(scope="module")
def config1(cuda):
    L = cases.moe_layer()
    be = make_backend(L)
    upload(be, 0, L)
    return L, be


def test_config1_layer_matches_oracle_and_golden(config1):
    L, be = config1
    x = synth.activation(2048, 0)
    out, ids, w = be.forward_host(0, x)
    ref_out, ref_ids, ref_p, logits = O.moe_forward(L, x)
    assert_routes(ids, ref_ids, logits, L.top_k)
    assert np.allclose(w, ref_p, rtol=1e-5)
    assert_moe_close(out, ref_out)
    g = np.load(GOLDEN / "moe_config1.npz")
    assert np.array_equal(ids, g["ids"])
    assert_moe_close(out, g["out"])


def test_config1_many_tokens(config1):
    L, be = config1
    for i in range(1, 17):
        x = synth.activation(2048, 100, i)
        out, ids, _ = be.forward_host(0, x)
        ref_out, ref_ids, _, logits = O.moe_forward(L, x)
        assert_routes(ids, ref_ids, logits, L.top_k)
        assert_moe_close(out, ref_out)


def test_device_forward_and_determinism(config1):
    L, be = config1
    x = torch.from_numpy(synth.activation(2048, 7)).cuda()
    out1 = torch.empty(2048, device="cuda")
    out2 = torch.empty(2048, device="cuda")
    ids = torch.empty(L.top_k, dtype=torch.int32, device="cuda")
    w = torch.empty(L.top_k, device="cuda")
    be.forward(0, x, out1, ids, w)
    be.forward(0, x, out2)
    be.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)
    ref_out, ref_ids, ref_p, logits = O.moe_forward(L, x.cpu().numpy())
    assert_routes(ids.cpu().numpy().astype(np.uint32), ref_ids, logits, L.top_k)
    assert_moe_close(out1.cpu().numpy(), ref_out)


def test_expert_view_and_stats(config1):
    L, be = config1
    p0, n0 = be.expert_view(0, GATE, 0)
    p5, n5 = be.expert_view(0, GATE, 5)
    assert n0 == n5 == 768 * 8 * 144 and p5 - p0 == 5 * n0
    pd, nd = be.expert_view(0, DOWN, 127)
    assert nd == 2048 * 3 * 144
    s = be.stats()
    assert s["misses"] == 0 and s["hits"] > 0 and s["forward_calls"] >= 1
    assert s["capacity_bytes"] >= L.gate.nbytes + L.up.nbytes + L.down.nbytes + L.router.nbytes
    assert s["resident_bytes"] == s["bytes_read"]


@pytest.mark.parametrize("down_type", [cases.Q6_K, cases.Q5_K])
def test_qwen35_shared_expert(cuda, down_type):
    L = cases.moe_layer(hidden=2048, inter=512, experts=64, top_k=10, seed=1, flavour=1,
                        down_type=down_type, shared_inter=512, expert_weights_scale=2.5)
    be = make_backend(L)
    upload(be, 0, L)
    x = synth.activation(2048, 1)
    out, ids, w = be.forward_host(0, x)
    ref_out, ref_ids, ref_p, logits = O.moe_forward(L, x)
    assert_routes(ids, ref_ids, logits, L.top_k)
    assert np.allclose(w, ref_p * np.float32(2.5), rtol=1e-5)
    assert_moe_close(out, ref_out)
    if down_type == cases.Q6_K:
        g = np.load(GOLDEN / "moe_qwen35.npz")
        assert np.array_equal(ids, g["ids"])
        assert_moe_close(out, g["out"])
    be.close()


def test_config3_shape_layer(cuda):
    """512 experts top-10, inter 512, Q4_K gate/up, Q5_K down, Q8_0 shared."""
    L = cases.moe_layer(hidden=2048, inter=512, experts=512, top_k=10, seed=4, flavour=1,
                        down_type=cases.Q5_K, shared_inter=512)
    be = make_backend(L)
    upload(be, 0, L)
    for i in range(3):
        x = synth.activation(2048, 4, i)
        out, ids, _ = be.forward_host(0, x)
        ref_out, ref_ids, _, logits = O.moe_forward(L, x)
        assert_routes(ids, ref_ids, logits, L.top_k)
        assert_moe_close(out, ref_out)
    be.close()


@pytest.mark.parametrize("experts,top_k,downs", [
    (512, 10, ("Q5_K", "Q6_K", "Q5_K", "Q6_K")),      # configuration 3
    (128, 8, ("Q4_K", "Q6_K", "Q5_K", "Q4_K")),
])
def test_config3_decode_chain(cuda, experts, top_k, downs):
    """Qwen3.5-MoE blocks in their decode chain (moe_chain35_kernel): Q4_K
    gate/up, the down type per layer, the Q8_0 shared expert and its sigmoid
    gate, ffn_norm per layer (configuration 3: 512 experts top-10, inter 512,
    Q5_K / Q6_K down alternating)."""
    downs = [getattr(cases, d) for d in downs]
    layers = [cases.moe_layer(hidden=2048, inter=512, experts=experts, top_k=top_k, seed=6, layer=l, flavour=1,
                              down_type=downs[l], shared_inter=512, with_norm=True) for l in range(4)]
    be = make_backend(layers[0], layers=4, rms_epsilon=1e-6, layer_down_types=downs)
    for l, L in enumerate(layers):
        upload(be, l, L)
    h0 = synth.activation(2048, 6, 0)
    k0 = be.stats()["kernel_launches"]
    out = be.decode_layers_host(0, 4, h0)
    assert be.stats()["kernel_launches"] - k0 == 1          # one chain launch for the four blocks
    ref = O.decode_layers(layers, h0, 1e-6)
    assert_moe_close(out - h0, ref.astype(np.float64) - h0)
    again = be.decode_layers_host(0, 4, h0)
    assert np.array_equal(out, again)
    mid = be.decode_layers_host(1, 3, h0)                   # odd first layer
    assert_moe_close(mid - h0, O.decode_layers(layers[1:], h0, 1e-6).astype(np.float64) - h0)
    h = torch.from_numpy(h0).cuda()
    be.decode_layers(0, 2, h)
    be.decode_layers(2, 2, h)
    torch.cuda.synchronize()
    assert np.array_equal(h.cpu().numpy(), out)
    be.close()


def test_decode_chain_matches_golden(cuda):
    layers = [cases.moe_layer(hidden=2048, inter=768, experts=32, top_k=8, seed=3, layer=l,
                              with_norm=True) for l in range(4)]
    be = make_backend(layers[0], layers=4, rms_epsilon=1e-6)
    for l, L in enumerate(layers):
        upload(be, l, L)
    h0 = synth.activation(2048, 3, 0)
    out = be.decode_layers_host(0, 4, h0)
    ref = O.decode_layers(layers, h0, 1e-6)
    g = np.load(GOLDEN / "decode4.npz")
    assert np.array_equal(ref, g["hidden"])
    assert_moe_close(out, ref)
    # The captured graph replays with identical results.
    again = be.decode_layers_host(0, 4, h0)
    assert np.array_equal(out, again)
    # Device-pointer variant on a torch stream.
    h = torch.from_numpy(h0).cuda()
    be.decode_layers(0, 4, h)
    torch.cuda.synchronize()
    assert np.array_equal(h.cpu().numpy(), out)
    # Partial ranges compose: layers [0,2) then [2,4).
    h = torch.from_numpy(h0).cuda()
    be.decode_layers(0, 2, h)
    be.decode_layers(2, 2, h)
    torch.cuda.synchronize()
    assert np.array_equal(h.cpu().numpy(), out)
    be.close()


def test_non_finite_router_reports_runtime_error(cuda):
    L = cases.moe_layer(hidden=1024, inter=256, experts=16, top_k=4, seed=6)
    be = make_backend(L)
    upload(be, 0, L)
    x = synth.activation(1024, 6)
    good, _, _ = be.forward_host(0, x)
    bad_router = L.router.copy()
    bad_router[3, 5] = np.nan
    be.upload_tensor(0, ROUTER, bad_router)
    with pytest.raises(PokitCudaError) as e:
        be.forward_host(0, x)
    assert "non-finite" in str(e.value) and e.value.status == 2
    be.upload_tensor(0, ROUTER, L.router)
    again, _, _ = be.forward_host(0, x)       # the handle stays usable
    assert np.array_equal(good, again)
    be.close()


def test_upload_validation(cuda):
    L = cases.moe_layer(hidden=1024, inter=256, experts=16, top_k=4, seed=6)
    be = make_backend(L)
    with pytest.raises(ValueError):
        be.upload_tensor(0, GATE, L.gate[:-16])
    with pytest.raises(ValueError):
        be.upload_tensor(1, GATE, L.gate)
    with pytest.raises(ValueError):
        be.upload_tensor(0, SHARED_GATE, L.gate)     # no shared expert configured
    with pytest.raises(ValueError):
        be.decode_layers_host(0, 1, np.zeros(1024, np.float32))   # weights not uploaded
    assert be.tensor_bytes(0, SHARED_ROUTER) == 0
    be.close()


def _device_synth(ggml_type, rows, cols, seed, sid):
    """Host copy of a tensor from the on-device generator (byte-identical to
    the host generator, tests/test_synth.py), without the host generator's cost."""
    nblocks = rows * (cols // 256)
    buf = torch.empty(nblocks * 144, dtype=torch.uint8, device="cuda")
    B.synthesize_blocks(ggml_type, seed, sid, nblocks, buf)
    torch.cuda.synchronize()
    return buf.cpu().numpy()


def test_full_size_decode_chain_on_device_synthesis(cuda):
    """Config 2 MoE path: 48 layers x 128 experts synthesised in HBM (16.3 GB).
    At full size: the 48-layer chain is finite and deterministic, equals the
    same 48 layers run one call per layer, and every layer's output matches
    the oracle's block evaluated on the same input hidden state."""
    from oracle.oracle import MoeLayer
    layers, H, I, E, k = 48, 2048, 768, 128, 8
    be = B.CudaMoeBackend(layers=layers, hidden=H, inter=I, experts=E, top_k=k, rms_epsilon=1e-6)
    for l in range(layers):
        be.upload_tensor(l, ROUTER, synth.router_weights(E, H, 0, l))
        be.upload_tensor(l, FFN_NORM, np.ones(H, np.float32))
        for t in (GATE, UP, DOWN):
            be.synthesize_tensor(l, t, 0, synth.stream_id(l, t))
    h0 = synth.activation(H, 0, 0)
    out1 = be.decode_layers_host(0, layers, h0)
    out2 = be.decode_layers_host(0, layers, h0)
    assert np.all(np.isfinite(out1)) and np.array_equal(out1, out2)
    h = h0.copy()
    ones = np.ones(H, np.float32)
    for l in range(layers):
        nxt = be.decode_layers_host(l, 1, h)
        L = MoeLayer(hidden=H, inter=I, experts=E, top_k=k, router=synth.router_weights(E, H, 0, l),
                     gate=_device_synth(cases.Q4_K, E * I, H, 0, synth.stream_id(l, GATE)),
                     up=_device_synth(cases.Q4_K, E * I, H, 0, synth.stream_id(l, UP)),
                     down=_device_synth(cases.Q4_K, E * H, I, 0, synth.stream_id(l, DOWN)),
                     flavour=0, normalize=True, ffn_norm=ones)
        ref = O.decode_layers([L], h, 1e-6)
        # The layer's own contribution, against its RMS (the residual is exact).
        assert_moe_close(nxt - h, ref.astype(np.float64) - h)
        h = nxt
    assert np.array_equal(h, out1)
    s = be.stats()
    assert s["capacity_bytes"] >= layers * E * (2 * 884736 + 884736)
    be.close()


def test_decode_chain_kernel_matches_the_block_graph(cuda, monkeypatch):
    """Tensor-core layers of one shape decode in one persistent launch per
    call; the per-block kernel graph (POKIT_CUDA_DECODE=graph) gives the same
    hidden states, as do sub-ranges starting on either layer parity and
    repeated calls (the launch leaves its counters and accumulators at zero)."""
    layers = [cases.moe_layer(hidden=2048, inter=768, experts=64, top_k=8, seed=8, layer=l,
                              with_norm=True) for l in range(5)]
    chain = make_backend(layers[0], layers=5, rms_epsilon=1e-6)
    monkeypatch.setenv("POKIT_CUDA_DECODE", "graph")
    graph = make_backend(layers[0], layers=5, rms_epsilon=1e-6)
    monkeypatch.delenv("POKIT_CUDA_DECODE")
    for l, L in enumerate(layers):
        upload(chain, l, L)
        upload(graph, l, L)
    for i in range(3):
        h0 = synth.activation(2048, 8, i)
        n0 = chain.stats()["kernel_launches"]
        a = chain.decode_layers_host(0, 5, h0)
        assert chain.stats()["kernel_launches"] - n0 == 1
        b = graph.decode_layers_host(0, 5, h0)
        assert_moe_close(a - h0, b.astype(np.float64) - h0)
        ref = O.decode_layers(layers, h0, 1e-6)
        assert_moe_close(a - h0, ref.astype(np.float64) - h0)
        mid = chain.decode_layers_host(1, 3, h0)          # odd first layer
        assert_moe_close(mid - h0, O.decode_layers(layers[1:4], h0, 1e-6).astype(np.float64) - h0)
        one = chain.decode_layers_host(4, 1, h0)
        assert_moe_close(one - h0, O.decode_layers(layers[4:], h0, 1e-6).astype(np.float64) - h0)
    chain.close()
    graph.close()
