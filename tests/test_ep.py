"""Expert parallelism, host side (CPU): shard ranges, and the decomposition
the sharded path relies on -- each rank's partial MoE output (its experts'
w_r * y_r) summed across ranks by an all-reduce equals the block's output.
Runs as two gloo ranks on 127.0.0.1 with the CPU oracle standing in for the
device kernels."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from oracle import oracle as O
from pokitlms_b200.ep import shard_range


@pytest.mark.parametrize("experts,world", [(128, 1), (128, 2), (128, 8), (10, 4), (512, 8), (3, 3)])
def test_shard_ranges_cover_every_expert_once(experts, world):
    seen = []
    for r in range(world):
        first, count = shard_range(experts, r, world)
        assert count >= 1
        seen.extend(range(first, first + count))
    assert seen == list(range(experts))
    counts = [shard_range(experts, r, world)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_shard_range_rejects_bad_arguments():
    with pytest.raises(ValueError):
        shard_range(4, 4, 4)
    with pytest.raises(ValueError):
        shard_range(2, 0, 4)


def oracle_partial(L, x, logits, first, count):
    """sum over routes whose expert is in [first, first + count) of w_r * y_r,
    per token, with the oracle's kernels (src/qwen3_moe_runner.cpp:674-690)."""
    H, I = L.hidden, L.inter
    gs = L.gate.size // L.experts
    ds = L.down.size // L.experts
    out = np.zeros((x.shape[0], H), np.float32)
    for t in range(x.shape[0]):
        ids, probs = O.route(L.flavour, logits[t], L.top_k)
        for e, p in zip(ids, probs):
            if not first <= e < first + count:
                continue
            g = O.linear(cases.Q4_K, x[t], L.gate[e * gs:(e + 1) * gs], I)
            u = O.linear(cases.Q4_K, x[t], L.up[e * gs:(e + 1) * gs], I)
            a = (g / (np.float32(1) + np.exp(-g))) * u
            y = O.linear(L.down_type, a.astype(np.float32), L.down[e * ds:(e + 1) * ds], H)
            out[t] += np.float32(p) * y
    return out


def _rank(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch
    L = cases.moe_layer(hidden=256, inter=256, experts=8, top_k=3, seed=4)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 256), dtype=np.float32)
    logits = rng.standard_normal((5, 8), dtype=np.float32)
    first, count = shard_range(8, rank, world)
    part = torch.from_numpy(oracle_partial(L, x, logits, first, count))
    dist.all_reduce(part)
    if rank == 0:
        ref, _, _ = O.moe_forward_batch(L, x, logits)
        err = float(np.max(np.abs(part.numpy() - ref)))
        result.put((err, float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))))
    dist.destroy_process_group()


def test_partial_outputs_all_reduce_to_the_block_output():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    err, rms = q.get(timeout=10)
    assert err <= 1e-5 * rms
