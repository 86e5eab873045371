"""CPU tests of the Gated DeltaNet restatement (oracle/pokit_oracle.c):
bit-identical to the reference's own causal_depthwise_conv1d_step,
gated_delta_recurrent_step_grouped and rms_norm_gated (oracle/_ref, built from
the reference's sources) over several steps of configuration 3's mixer shape,
states included; an invalid decay is refused as the reference throws."""
import numpy as np
import pytest

import cases
from oracle import oracle as O

SMALL = dict(key_heads=2, value_heads=4, key_dim=32, value_dim=64, conv_kernel=4, rms_epsilon=1e-6)


@pytest.mark.skipif(not O.ref_available(), reason="the reference's kernels are not built here")
@pytest.mark.parametrize("shape", [SMALL, cases.DELTA_NET_CFG3], ids=["small", "config3"])
def test_restatement_matches_the_reference_bit_for_bit(shape):
    t, steps = cases.delta_net_inputs(shape, seed=3, steps=3)
    C = t["conv_w"].shape[0]
    vh, dv, dk = shape["value_heads"], shape["value_dim"], shape["key_dim"]
    st = {p: (np.zeros((C, shape["conv_kernel"] - 1), np.float32), np.zeros((vh, dv, dk), np.float32))
          for p in ("po", "ref")}
    for s in steps:
        outs = {}
        for p in ("po", "ref"):
            conv_state, state = st[p]
            outs[p] = O.delta_net_step(shape, s["projected"], s["gate"], s["alpha"], s["beta"], t["conv_w"],
                                       conv_state, t["a"], t["dt_bias"], t["norm"], state, fn_prefix=p)
        assert np.array_equal(outs["po"][0], outs["ref"][0])
        assert np.array_equal(outs["po"][1], outs["ref"][1])
        assert np.array_equal(st["po"][0], st["ref"][0]) and np.array_equal(st["po"][1], st["ref"][1])
        assert np.all(np.isfinite(outs["po"][0]))


def test_invalid_decay_is_refused():
    t, steps = cases.delta_net_inputs(SMALL, seed=4, steps=1)
    t["a"][0] = np.float32(1.0)                 # positive a: log decay > 0
    C = t["conv_w"].shape[0]
    with pytest.raises(ValueError):
        O.delta_net_step(SMALL, steps[0]["projected"], steps[0]["gate"], steps[0]["alpha"], steps[0]["beta"],
                         t["conv_w"], np.zeros((C, 3), np.float32), t["a"], t["dt_bias"], t["norm"],
                         np.zeros((4, 64, 32), np.float32))
