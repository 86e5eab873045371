"""Oracle parity of the batched block at benchmark configuration 5's shape
(hidden 4096, expert intermediate 1536, 128 experts top-8, Q4_K experts, 64
F32 tokens), on one whole-pool handle and on 2, 4 and 8 expert-shard handles
whose partial outputs are summed in rank order (expert parallelism emulated
on one GPU).

Routing follows the benchmark's caller logits (N(0, 1) per token and
expert) with a +4 bias on four experts, so the batch holds both kinds of
tiles the grouped path has: the four hot experts get most of the 64 tokens
(tcgen05 tiles of more than 8 tokens) and the rest a few tokens each (the
skinny mma.sync tiles).  Every token is checked against the oracle
(O.moe_forward_batch, the reference's MoE block restated): route ids
identical except below the 1e-5 margin, outputs within 1e-3 x the token's
RMS.  Weights come from the on-device generator (byte-identical to the host
generator, tests/test_synth.py), copied back for the oracle.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from pokitlms_b200 import backend as B
from pokitlms_b200 import synth
from pokitlms_b200._lib import DOWN, GATE, ROUTER, UP
from pokitlms_b200.ep import shard_range

pytestmark = pytest.mark.gpu

H, I, E, K, T = 4096, 1536, 128, 8, 64
SEED = 5
HOT = (3, 40, 77, 111)


def _device_tensor(rows, cols, sid):
    nblocks = rows * (cols // 256)
    buf = torch.empty(nblocks * 144, dtype=torch.uint8, device="cuda")
    B.synthesize_blocks(cases.Q4_K, SEED, sid, nblocks, buf)
    torch.cuda.synchronize()
    return buf.cpu().numpy()


@pytest.fixture(scope="module")
def config5(cuda):
    from oracle.oracle import MoeLayer
    L = MoeLayer(hidden=H, inter=I, experts=E, top_k=K,
                 router=synth.router_weights(E, H, SEED, 0),
                 gate=_device_tensor(E * I, H, synth.stream_id(0, GATE)),
                 up=_device_tensor(E * I, H, synth.stream_id(0, UP)),
                 down=_device_tensor(E * H, I, synth.stream_id(0, DOWN)),
                 flavour=0, normalize=True)
    x = np.stack([synth.activation(H, SEED, i) for i in range(T)])
    rng = np.random.default_rng([SEED, 0x6c67])
    logits = rng.standard_normal((T, E), dtype=np.float32)
    logits[:, list(HOT)] += np.float32(4.0)
    ref, ref_ids, _ = O.moe_forward_batch(L, x, logits)
    return L, x, logits, ref, ref_ids


def _run(L, x, logits, first, count):
    be = B.CudaMoeBackend(layers=1, hidden=H, inter=I, experts=E, top_k=K, expert_first=first,
                          expert_count=count)
    be.upload_tensor(0, ROUTER, L.router)
    for t in (GATE, UP, DOWN):
        be.synthesize_tensor(0, t, SEED, synth.stream_id(0, t))
    out, ids, _ = be.forward_batch_host(0, x, logits=logits)
    be.close()
    return out, ids


def test_config5_batch_has_both_tile_kinds(config5):
    _, _, _, _, ref_ids = config5
    counts = np.bincount(ref_ids.ravel(), minlength=E)
    assert counts.max() > 8                      # tensor-core tiles
    assert ((counts > 0) & (counts <= 8)).sum() > 64   # skinny tiles


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config5_shards_match_the_oracle(config5, world):
    L, x, logits, ref, ref_ids = config5
    total = np.zeros((T, H), np.float64)
    for r in range(world):
        first, count = shard_range(E, r, world) if world > 1 else (0, 0)
        out, ids = _run(L, x, logits, first, count)
        total += out
        if world == 1:
            for t in range(T):
                if not np.array_equal(ids[t], ref_ids[t]):
                    assert cases.route_margin(logits[t], K) < 1e-5, t
    for t in range(T):
        rms = float(np.sqrt(np.mean(ref[t].astype(np.float64) ** 2)))
        err = float(np.max(np.abs(total[t] - ref[t])))
        assert err <= 1e-3 * rms, (world, t, err, rms)
