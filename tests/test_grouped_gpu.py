"""GPU parity tests of the batched MoE block (pokit_cuda_moe_forward_batch):
the grouped-expert tensor-core GEMM against the CPU oracle run token by token
(the reference's prefill runs one forward_into per token).

Bar: routes identical to the oracle's except where the top-k margin is below
1e-5; every token's output within max-abs error <= 1e-3 x that token's
output RMS.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from pokitlms_b200 import backend as B
from pokitlms_b200 import synth
from pokitlms_b200._lib import InvalidArgument

pytestmark = pytest.mark.gpu
TOL = 1e-3


def make_backend(L, **extra):
    kw = dict(layers=1, hidden=L.hidden, inter=L.inter, experts=L.experts, top_k=L.top_k,
              flavour=L.flavour, normalize_top_k=L.normalize,
              expert_weights_scale=L.expert_weights_scale, down_type=L.down_type)
    if L.shared_inter:
        kw.update(shared_inter=L.shared_inter)
    kw.update(extra)
    be = B.CudaMoeBackend(**kw)
    be.upload_layer(0, router=L.router, gate=L.gate, up=L.up, down=L.down,
                    ffn_norm=np.ones(L.hidden, np.float32), shared_router=L.shared_router,
                    shared_gate=L.shared_gate, shared_up=L.shared_up, shared_down=L.shared_down)
    return be


def check_batch(L, out, ids, w, ref_out, ref_ids, ref_p, logits):
    assert np.all(np.isfinite(out))
    for t in range(out.shape[0]):
        if not np.array_equal(ids[t], ref_ids[t]):
            assert cases.route_margin(logits[t], L.top_k) < 1e-5, (t, ids[t], ref_ids[t])
            continue
        assert np.allclose(w[t], ref_p[t], rtol=1e-5, atol=1e-7), t
        ref = ref_out[t].astype(np.float64)
        rms = float(np.sqrt(np.mean(ref ** 2)))
        err = float(np.max(np.abs(out[t] - ref)))
        assert err <= TOL * rms, (t, err, rms)


@pytest.mark.parametrize("tokens,experts,top_k,hidden,inter", [
    (64, 32, 4, 512, 256),      # small, skewed
    (200, 8, 2, 256, 256),      # hot experts spanning several 64-token tiles
    (1, 16, 4, 512, 512),       # a single token
    (37, 256, 8, 256, 256),     # most experts empty, ragged tiles
])
def test_grouped_bf16_given_logits(cuda, tokens, experts, top_k, hidden, inter):
    L = cases.moe_layer(hidden=hidden, inter=inter, experts=experts, top_k=top_k, seed=3)
    be = make_backend(L)
    bits, xf, logits = synth.grouped_inputs(tokens, experts, hidden, seed=tokens)
    out, ids, w = be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
    ref_out, ref_ids, ref_p = O.moe_forward_batch(L, xf, logits)
    check_batch(L, out, ids, w, ref_out, ref_ids, ref_p, logits)
    be.close()


def test_grouped_f32_layer_router(cuda):
    """F32 activations (hi + lo operand split) routed by the layer's F32 router."""
    L = cases.moe_layer(hidden=1024, inter=512, experts=32, top_k=4, seed=5)
    be = make_backend(L)
    rng = np.random.default_rng(11)
    x = rng.standard_normal((96, 1024), dtype=np.float32) * np.float32(3.0)
    out, ids, w = be.forward_batch_host(0, x)
    ref_out, ref_ids, ref_p = O.moe_forward_batch(L, x)
    logits = x @ L.router.T
    check_batch(L, out, ids, w, ref_out, ref_ids, ref_p, logits)
    be.close()


def test_grouped_qwen35_flavour(cuda):
    """Qwen3.5 routing (float softmax, expert_weights_scale) and sigmoid-form SiLU."""
    L = cases.moe_layer(hidden=512, inter=256, experts=64, top_k=10, seed=9, flavour=1,
                        expert_weights_scale=2.5)
    be = make_backend(L)
    bits, xf, logits = synth.grouped_inputs(80, 64, 512, seed=4)
    out, ids, w = be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
    ref_out, ref_ids, ref_p = O.moe_forward_batch(L, xf, logits)
    ref_w = ref_p * np.float32(2.5)
    check_batch(L, out, ids, w, ref_out, ref_ids, ref_w, logits)
    be.close()


def test_grouped_large_activations(cuda):
    """Activations of magnitude ~1e3 (power-of-two operand scaling; the
    intermediate silu(g) * u reaches ~1e7, beyond fp16 range unscaled)."""
    L = cases.moe_layer(hidden=512, inter=256, experts=16, top_k=4, seed=2)
    be = make_backend(L)
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((40, 512), dtype=np.float32) * np.float32(1000.0))
    logits = rng.standard_normal((40, 16), dtype=np.float32)
    out, ids, w = be.forward_batch_host(0, x, logits=logits)
    ref_out, ref_ids, ref_p = O.moe_forward_batch(L, x, logits)
    check_batch(L, out, ids, w, ref_out, ref_ids, ref_p, logits)
    be.close()


@pytest.mark.parametrize("bf16", [False, True])
def test_grouped_skinny_tile_boundary(cuda, bf16):
    """Experts of 1, 7, 8, 9, 16, 64, 72 and 73 tokens: tiles on both sides of
    the 8-token limit of the mma.sync path, and large experts whose last tile
    is skinny (72 = 64 + 8) or not (73 = 64 + 9)."""
    counts = [1, 7, 8, 9, 16, 64, 72, 73]
    L = cases.moe_layer(hidden=512, inter=256, experts=8, top_k=1, seed=6)
    be = make_backend(L)
    tokens = sum(counts)
    rng = np.random.default_rng(6)
    owner = np.repeat(np.arange(8), counts)
    rng.shuffle(owner)
    logits = rng.standard_normal((tokens, 8)).astype(np.float32) * np.float32(0.1)
    logits[np.arange(tokens), owner] += np.float32(4.0)
    x = rng.standard_normal((tokens, 512), dtype=np.float32)
    if bf16:
        bits, x = synth.bf16_round(x)
        out, ids, w = be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
    else:
        out, ids, w = be.forward_batch_host(0, x, logits=logits)
    assert np.array_equal(ids[:, 0], owner)
    ref_out, ref_ids, ref_p = O.moe_forward_batch(L, x, logits)
    check_batch(L, out, ids, w, ref_out, ref_ids, ref_p, logits)
    be.close()


@pytest.fixture(scope="module")
def config4(cuda):
    L = cases.moe_layer()   # hidden 2048, 128 experts top-8, inter 768, Q4_K
    be = make_backend(L)
    bits, xf, logits = synth.grouped_inputs(512, 128, 2048, seed=0)
    yield L, be, bits, xf, logits
    be.close()


def test_config4_sampled_tokens_match_oracle(config4):
    """The benchmark batch (512 tokens, Zipf-skewed routes) on the device;
    a spread of 24 tokens checked against the oracle."""
    L, be, bits, xf, logits = config4
    out, ids, w = be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
    pick = np.linspace(0, 511, 24).astype(int)
    ref_out, ref_ids, ref_p = O.moe_forward_batch(L, xf[pick], logits[pick])
    check_batch(L, out[pick], ids[pick], w[pick], ref_out, ref_ids, ref_p, logits[pick])
    # Every token routed as the oracle's selection rule says (full batch).
    for t in range(512):
        ref_i, _ = O.route(0, logits[t], L.top_k)
        if not np.array_equal(ids[t], ref_i):
            assert cases.route_margin(logits[t], L.top_k) < 1e-5


def test_config4_device_api_deterministic_and_matches_single_token(config4):
    L, be, bits, xf, logits = config4
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    lg = torch.from_numpy(logits).cuda()
    out1 = torch.empty(512, 2048, device="cuda")
    out2 = torch.empty(512, 2048, device="cuda")
    ids = torch.empty(512, 8, dtype=torch.int32, device="cuda")
    be.forward_batch(0, x, out1, logits=lg, route_ids=ids)
    be.forward_batch(0, x, out2, logits=lg)
    be.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)
    # Tokens whose routes the layer router would also pick: the batched path
    # agrees with the single-token path on the same token.
    xf_dev = torch.from_numpy(xf).cuda()
    single = torch.empty(2048, device="cuda")
    for t in (0, 255, 511):
        be.forward(0, xf_dev[t], single)
        be.synchronize()
        ref_out, ref_ids, _, ref_logits = O.moe_forward(L, xf[t])
        assert np.allclose(single.cpu().numpy(), ref_out, atol=TOL * np.sqrt(np.mean(ref_out ** 2)))
    stats = be.stats()
    assert stats["forward_calls"] >= 1024


def test_batch_rejects_bad_arguments(config4):
    L, be, bits, xf, logits = config4
    with pytest.raises(InvalidArgument):
        be.forward_batch_host(0, np.zeros((0, 2048), np.float32))
    x = torch.zeros(4, 2048, dtype=torch.float16, device="cuda")
    with pytest.raises(InvalidArgument):
        be.forward_batch(0, x, torch.empty(4, 2048, device="cuda"))


def test_non_grouped_layer_falls_back_per_token(cuda):
    """A Q6_K-down layer runs the single-token block per row (F32 only)."""
    L = cases.moe_layer(hidden=512, inter=256, experts=16, top_k=4, seed=8, down_type=cases.Q6_K)
    be = make_backend(L)
    rng = np.random.default_rng(8)
    x = rng.standard_normal((5, 512), dtype=np.float32)
    out, ids, w = be.forward_batch_host(0, x)
    ref_out, ref_ids, ref_p = O.moe_forward_batch(L, x)
    check_batch(L, out, ids, w, ref_out, ref_ids, ref_p, x @ L.router.T)
    with pytest.raises(InvalidArgument):
        be.forward_batch_host(0, synth.bf16_round(x)[0], bf16_bits=True)
    be.close()
