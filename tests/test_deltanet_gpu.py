"""GPU parity of the Gated DeltaNet mixer step (pokit_cuda_delta_net_step)
against the oracle's restatement (oracle/pokit_oracle.c, pinned bit for bit to
the reference's causal_depthwise_conv1d_step, gated_delta_recurrent_step_grouped
and rms_norm_gated by tests/test_deltanet.py), at configuration 3's mixer shape
over several tokens with the states carried on both sides: outputs within
1e-3 x their RMS, states within 1e-4 x theirs; an invalid decay sets the
status bit and leaves the state alone."""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from pokitlms_b200 import backend as B

pytestmark = pytest.mark.gpu


def _rms(a):
    return float(np.sqrt(np.mean(np.asarray(a, np.float64) ** 2)))


@pytest.mark.parametrize("shape", [cases.DELTA_NET_CFG3, dict(key_heads=2, value_heads=6, key_dim=64, value_dim=96,
                                                             conv_kernel=4, rms_epsilon=1e-6),
                                   dict(key_heads=1, value_heads=2, key_dim=256, value_dim=160, conv_kernel=4,
                                        rms_epsilon=1e-6)],
                         ids=["config3", "odd", "wide"])   # wide: heads beyond 128 (the streamed-row kernel)
def test_delta_net_steps_match_the_oracle(cuda, shape):
    t, steps = cases.delta_net_inputs(shape, seed=7, steps=6)
    C, K = t["conv_w"].shape
    vh, dv, dk = shape["value_heads"], shape["value_dim"], shape["key_dim"]
    cs = np.zeros((C, K - 1), np.float32)
    rs = np.zeros((vh, dv, dk), np.float32)
    dev = {k: torch.from_numpy(v).cuda() for k, v in t.items()}
    d_cs = torch.zeros(C, K - 1, device="cuda")
    d_rs = torch.zeros(vh, dv, dk, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(vh * dv, device="cuda")
    for s in steps:
        ref, ref_conv = O.delta_net_step(shape, s["projected"], s["gate"], s["alpha"], s["beta"], t["conv_w"], cs,
                                         t["a"], t["dt_bias"], t["norm"], rs)
        proj = torch.from_numpy(s["projected"]).cuda()
        B.delta_net_step(shape, proj, torch.from_numpy(s["gate"]).cuda(), torch.from_numpy(s["alpha"]).cuda(),
                         torch.from_numpy(s["beta"]).cuda(), dev["conv_w"], d_cs, dev["a"], dev["dt_bias"],
                         dev["norm"], d_rs, out, status)
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        assert np.all(np.isfinite(o))
        assert float(np.max(np.abs(o - ref))) <= 1e-3 * _rms(ref)
        assert float(np.max(np.abs(proj.cpu().numpy() - ref_conv))) <= 1e-5 * _rms(ref_conv)
        assert np.array_equal(d_cs.cpu().numpy(), cs)          # the conv state is a copy of inputs
        assert float(np.max(np.abs(d_rs.cpu().numpy() - rs))) <= 1e-4 * _rms(rs)
    assert int(status.item()) == 0


def test_invalid_decay_sets_the_status(cuda):
    shape = dict(key_heads=2, value_heads=4, key_dim=32, value_dim=64, conv_kernel=4, rms_epsilon=1e-6)
    t, steps = cases.delta_net_inputs(shape, seed=8, steps=1)
    t["a"][1] = np.float32(2.0)                               # log decay > 0 for head 1
    dev = {k: torch.from_numpy(v).cuda() for k, v in t.items()}
    C = t["conv_w"].shape[0]
    rs = torch.full((4, 64, 32), 0.5, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(4 * 64, device="cuda")
    s = steps[0]
    B.delta_net_step(shape, torch.from_numpy(s["projected"]).cuda(), torch.from_numpy(s["gate"]).cuda(),
                     torch.from_numpy(s["alpha"]).cuda(), torch.from_numpy(s["beta"]).cuda(), dev["conv_w"],
                     torch.zeros(C, 3, device="cuda"), dev["a"], dev["dt_bias"], dev["norm"], rs, out, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert torch.all(rs[1] == 0.5) and torch.all(out[64:128] == 0)
