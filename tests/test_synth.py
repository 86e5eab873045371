"""CPU tests of the seeded synthetic block generator."""
import numpy as np
import pytest

from pokitlms_b200 import synth
from pokitlms_b200._lib import BLOCK, Q4_K, Q5_K, Q6_K, Q8_0


@pytest.mark.parametrize("t", [Q4_K, Q5_K, Q6_K, Q8_0])
def test_block_ranges_are_consistent(t):
    full = synth.synth_blocks(t, 40, 7, 3)
    bb = BLOCK[t][1]
    part = synth.synth_blocks(t, 9, 7, 3, first_block=13)
    assert np.array_equal(part, full[13 * bb:22 * bb])
    assert np.array_equal(full, synth.synth_blocks(t, 40, 7, 3))
    assert not np.array_equal(full, synth.synth_blocks(t, 40, 7, 4))


@pytest.mark.parametrize("t,offsets", [(Q4_K, (0, 2)), (Q5_K, (0, 2)), (Q6_K, (208,)),
                                       (Q8_0, (0,))])
def test_scale_fields_uniform_in_range(t, offsets):
    bb = BLOCK[t][1]
    blocks = synth.synth_blocks(t, 4000, 0, 1).reshape(-1, bb)
    for off in offsets:
        d = blocks[:, off:off + 2].copy().view(np.float16).astype(np.float32).ravel()
        assert d.min() >= np.float32(1e-3) * 0.999 and d.max() <= np.float32(1e-2) * 1.001
        assert 0.45 < float(np.mean((d - 1e-3) / 9e-3)) < 0.55


def test_q4k_scales_and_nibbles_cover_range():
    blocks = synth.synth_blocks(Q4_K, 2000, 0, 2).reshape(-1, 144)
    scales = blocks[:, 4:8] & 63
    assert scales.min() == 0 and scales.max() == 63
    nib = blocks[:, 16:] & 15
    assert nib.min() == 0 and nib.max() == 15


def test_router_and_activation_distributions():
    r = synth.router_weights(128, 2048, 0)
    assert r.dtype == np.float32 and r.shape == (128, 2048)
    assert abs(float(r.std()) - 0.02) < 1e-3
    x = synth.activation(2048, 0)
    assert abs(float(x.std()) - 1.0) < 0.05
    assert np.array_equal(x, synth.activation(2048, 0))
