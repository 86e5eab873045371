"""Expert-shard handles on the GPU (pokit_cuda_moe_config.expert_first /
expert_count): the partial outputs of the shards add up to the whole pool's
batched output, for uploaded and for synthesised weights, and two ranks on two
GPUs combine over NCCL through pokitlms_b200.ep (when two GPUs are visible)."""
import os
import socket

import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from pokitlms_b200 import backend as B
from pokitlms_b200 import synth
from pokitlms_b200._lib import DOWN, GATE, UP, InvalidArgument
from pokitlms_b200.ep import shard_range

pytestmark = pytest.mark.gpu
TOL = 1e-3


def make(L, first=0, count=0):
    return B.CudaMoeBackend(layers=1, hidden=L.hidden, inter=L.inter, experts=L.experts, top_k=L.top_k,
                            flavour=L.flavour, normalize_top_k=True, down_type=L.down_type,
                            expert_first=first, expert_count=count)


def upload_shard(be, L, first, count):
    gs, ds = L.gate.size // L.experts, L.down.size // L.experts
    be.upload_layer(0, router=L.router, gate=L.gate[first * gs:(first + count) * gs],
                    up=L.up[first * gs:(first + count) * gs], down=L.down[first * ds:(first + count) * ds],
                    ffn_norm=np.ones(L.hidden, np.float32))


def assert_close(out, ref):
    for t in range(out.shape[0]):
        rms = float(np.sqrt(np.mean(ref[t].astype(np.float64) ** 2)))
        assert float(np.max(np.abs(out[t] - ref[t]))) <= TOL * rms, t


@pytest.mark.parametrize("world", [2, 3])
def test_shard_partials_sum_to_the_block(cuda, world):
    L = cases.moe_layer(hidden=512, inter=256, experts=24, top_k=4, seed=6)
    bits, xf, logits = synth.grouped_inputs(48, 24, 512, seed=world)
    total = np.zeros((48, 512), np.float64)
    for r in range(world):
        first, count = shard_range(24, r, world)
        be = make(L, first, count)
        assert be.tensor_bytes(0, GATE) == count * (L.gate.size // 24)
        upload_shard(be, L, first, count)
        out, ids, _ = be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
        total += out
        be.close()
    ref, _, _ = O.moe_forward_batch(L, xf, logits)
    assert_close(total.astype(np.float32), ref)


def test_synthesised_shards_match_the_whole_pool(cuda):
    """On-device synthesis of a shard reproduces the whole tensor's blocks."""
    cfg = dict(hidden=512, inter=256, experts=16, top_k=4)
    L = cases.moe_layer(seed=0, **cfg)
    bits, xf, logits = synth.grouped_inputs(32, 16, 512, seed=1)

    def run(first, count):
        be = make(L, first, count)
        be.upload_tensor(0, 0, L.router)
        for t in (GATE, UP, DOWN):
            be.synthesize_tensor(0, t, 0, synth.stream_id(0, t))
        out, _, _ = be.forward_batch_host(0, bits, bf16_bits=True, logits=logits)
        be.close()
        return out

    whole = run(0, 0)
    parts = run(0, 7) + run(7, 9)
    assert_close(parts, whole)
    ref, _, _ = O.moe_forward_batch(L, xf, logits)   # the host generator's weights
    assert_close(whole, ref)


def test_shard_handle_refuses_the_single_token_paths(cuda):
    L = cases.moe_layer(hidden=256, inter=256, experts=8, top_k=2, seed=1)
    be = make(L, 4, 4)
    upload_shard(be, L, 4, 4)
    x = np.zeros(256, np.float32)
    with pytest.raises(InvalidArgument):
        be.forward_host(0, x)
    with pytest.raises(InvalidArgument):
        be.decode_layers_host(0, 1, x)
    with pytest.raises(InvalidArgument):
        be.expert_view(0, GATE, 0)
    p, n = be.expert_view(0, GATE, 5)
    assert n == L.gate.size // 8
    be.close()


def _nccl_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    from pokitlms_b200.ep import ExpertParallelMoe
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    L = cases.moe_layer(hidden=512, inter=256, experts=16, top_k=4, seed=2)
    ep = ExpertParallelMoe(rank=rank, world=world, layers=1, hidden=512, inter=256, experts=16, top_k=4,
                           device=rank)
    upload_shard(ep.backend, L, ep.expert_first, ep.expert_count)
    bits, xf, logits = synth.grouped_inputs(40, 16, 512, seed=9)
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    lg = torch.from_numpy(logits).cuda()
    out = torch.empty(40, 512, device="cuda")
    ep.forward_batch(0, x, out, logits=lg)
    ep.backend.synchronize()
    torch.cuda.synchronize()
    if rank == 0:
        ref, _, _ = O.moe_forward_batch(L, xf, logits)
        q.put(np.abs(out.cpu().numpy() - ref).max(axis=1) / np.sqrt(np.mean(ref.astype(np.float64) ** 2, axis=1)))
    ep.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_expert_parallel_over_nccl(cuda):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs)
    rel = q.get(timeout=10)
    assert float(rel.max()) <= TOL


def _exchange_rank(rank, world, port, q):
    """One rank of the peer-memory exchange: two eager batches of different
    sizes and input types (both exchange parities), then one batch captured in
    a CUDA graph and replayed twice (the call counter lives on the device)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    from pokitlms_b200.ep import ExpertParallelMoe
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    L = cases.moe_layer(hidden=512, inter=256, experts=16, top_k=4, seed=2)
    ep = ExpertParallelMoe(rank=rank, world=world, layers=1, hidden=512, inter=256, experts=16, top_k=4,
                           device=rank, exchange_tokens=64)
    assert ep.peer_exchange
    upload_shard(ep.backend, L, ep.expert_first, ep.expert_count)
    results = []
    bits, xf, logits = synth.grouped_inputs(40, 16, 512, seed=9)
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    out = torch.empty(40, 512, device="cuda")
    ep.forward_batch(0, x, out, logits=torch.from_numpy(logits).cuda())
    ep.backend.synchronize()
    results.append((out.cpu().numpy(), xf, logits))
    rng = np.random.default_rng(4)
    x2 = rng.standard_normal((8, 512), dtype=np.float32)
    lg2 = rng.standard_normal((8, 16), dtype=np.float32)
    x2d, lg2d = torch.from_numpy(x2).cuda(), torch.from_numpy(lg2).cuda()
    out2 = torch.empty(8, 512, device="cuda")
    ep.forward_batch(0, x2d, out2, logits=lg2d)
    ep.backend.synchronize()
    results.append((out2.cpu().numpy(), x2, lg2))
    side = torch.cuda.Stream()
    out3 = torch.empty(8, 512, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        ep.forward_batch(0, x2d, out3, logits=lg2d, stream=side)
    replays = []
    for _ in range(2):
        out3.zero_()
        g.replay()
        torch.cuda.synchronize()
        replays.append(out3.cpu().numpy())
    del g
    ep.backend.synchronize()
    q.put((rank, [r[0] for r in results], replays))
    if rank == 0:
        q.put(("inputs", [(r[1], r[2]) for r in results]))
    ep.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_expert_parallel_over_peer_memory(cuda):
    """The block's last kernel sums the two shards' partials over NVLink:
    every rank gets the oracle's output, both ranks the same values, and a
    captured batch replays to the eager result."""
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(3)]
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    inputs = next(g[1] for g in got if g[0] == "inputs")
    outs = {g[0]: g for g in got if g[0] != "inputs"}
    L = cases.moe_layer(hidden=512, inter=256, experts=16, top_k=4, seed=2)
    for i, (xi, li) in enumerate(inputs):
        ref, _, _ = O.moe_forward_batch(L, xi, li)
        rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2, axis=1))
        for rank in (0, 1):
            out = outs[rank][1][i]
            assert float((np.abs(out - ref).max(axis=1) / rms).max()) <= TOL
        assert np.array_equal(outs[0][1][i], outs[1][1][i])
    for rank in (0, 1):
        for rep in outs[rank][2]:
            assert np.array_equal(rep, outs[rank][1][1])



def _silent_rank(to_child, to_parent):
    """Rank 1 of a two-rank exchange on the same GPU as rank 0: it creates
    and maps its region but never runs a block, so rank 0 waits for a flag
    that nothing raises.  It launches no kernel, so no two kernels wait on one
    another."""
    from pokitlms_b200 import backend as B
    torch.cuda.set_device(0)
    be = B.CudaMoeBackend(layers=1, hidden=512, inter=256, experts=16, top_k=4, expert_first=8, expert_count=8,
                          device=0)
    mine = be.exchange_create(2, 1, 16)
    to_parent.put(mine)
    h0 = to_child.get(timeout=120)
    be.exchange_connect([h0, mine])
    to_parent.put("connected")
    assert to_child.get(timeout=300) == "disconnect"
    be.exchange_disconnect()
    be.close()
    to_parent.put("closed")


def test_peer_exchange_wait_runs_out_when_a_rank_never_arrives(cuda):
    """A bounded device-side wait: rank 0's combine waits for rank 1's flag,
    which rank 1 (another process, same GPU) never raises; after ~1-2 s the
    kernel gives up, sets the status word, and the handle reports a sticky
    runtime error instead of hanging."""
    import time
    import torch.multiprocessing as mp
    from pokitlms_b200._lib import PokitCudaError
    ctx = mp.get_context("spawn")
    to_child, to_parent = ctx.Queue(), ctx.Queue()
    child = ctx.Process(target=_silent_rank, args=(to_child, to_parent))
    child.start()
    L = cases.moe_layer(hidden=512, inter=256, experts=16, top_k=4, seed=2)
    be = B.CudaMoeBackend(layers=1, hidden=512, inter=256, experts=16, top_k=4, expert_first=0, expert_count=8,
                          device=0)
    upload_shard(be, L, 0, 8)
    try:
        mine = be.exchange_create(2, 0, 16)
        h1 = to_parent.get(timeout=120)
        to_child.put(mine)
        be.exchange_connect([mine, h1])
        assert to_parent.get(timeout=120) == "connected"
        rng = np.random.default_rng(5)
        x = torch.from_numpy(rng.standard_normal((4, 512), dtype=np.float32)).cuda()
        lg = torch.from_numpy(rng.standard_normal((4, 16), dtype=np.float32)).cuda()
        out = torch.empty(4, 512, device="cuda")
        t0 = time.perf_counter()
        be.forward_batch(0, x, out, logits=lg)
        with pytest.raises(PokitCudaError, match="timed out"):
            be.synchronize()
        assert time.perf_counter() - t0 < 60
        with pytest.raises(PokitCudaError):          # sticky
            be.forward_batch(0, x, out, logits=lg)
    finally:
        be.exchange_disconnect()                   # unmap rank 1's region before it is freed
        to_child.put("disconnect")
        assert to_parent.get(timeout=120) == "closed"
        child.join(60)
        be.close()
    assert child.exitcode == 0
