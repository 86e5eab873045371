"""Expert parallelism over ranks (one process per GPU, torch.distributed).

Experts are split into contiguous shards, one per rank; the router, the
routes and the hidden states are the same on every rank.  Each rank runs the
batched MoE block on the experts it holds (pokit_cuda_moe_forward_batch on an
expert-shard handle, which returns that shard's contribution
sum_{r : e_r held here} w_r * y_r per token) and the contributions are summed
across ranks: the combine step of the block, the one exchange the sharded
path needs.  Two forms: an NCCL all-reduce of the partial outputs, or (with
exchange_tokens) the block's own last kernel, which stores its partial into
every rank's memory over NVLink and adds all ranks' partials itself
(pokit_cuda_moe_exchange_create / _connect; CUDA IPC handles are swapped
once over the process group).

The reference runs every expert of a block on one host (src/qwen3_moe_runner.cpp
:643-692); the sum over shards equals its combine up to the order of the F32
additions.
"""
from __future__ import annotations

from . import backend as B


def shard_range(experts: int, rank: int, world: int) -> tuple[int, int]:
    """(first, count) of rank's contiguous expert shard; the first
    experts % world ranks hold one expert more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if experts < world:
        raise ValueError("need at least one expert per rank")
    base, extra = divmod(experts, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


class ExpertParallelMoe:
    """One rank's share of an expert-parallel MoE: a CudaMoeBackend holding
    this rank's expert shard plus the combine over the process group."""

    def __init__(self, *, rank: int, world: int, group=None, exchange_tokens: int | None = None, **config):
        self.rank, self.world, self.group = rank, world, group
        first, count = shard_range(config["experts"], rank, world)
        self.expert_first, self.expert_count = first, count
        if world == 1:
            count = 0                       # the whole pool, no shard
        self.backend = B.CudaMoeBackend(expert_first=first, expert_count=count, **config)
        self.peer_exchange = False
        if exchange_tokens and world > 1:
            import torch.distributed as dist
            mine = self.backend.exchange_create(world, rank, exchange_tokens)
            handles = [None] * world
            dist.all_gather_object(handles, mine, group=group)
            self.backend.exchange_connect(handles)
            dist.barrier(group=group)       # every rank mapped before any rank stores
            self.peer_exchange = True

    def forward_batch(self, layer: int, x, out, *, logits=None, route_ids=None, route_weights=None,
                      stream=None) -> None:
        """out[t] = MoE(x[t]) on every rank: this rank's experts, then the
        sum over ranks of the partial outputs (in the block's last kernel with
        the peer-memory exchange, else an all-reduce)."""
        import torch.distributed as dist
        self.backend.forward_batch(layer, x, out, logits=logits, route_ids=route_ids,
                                   route_weights=route_weights, stream=stream)
        if self.world > 1 and not self.peer_exchange:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)

    def close(self) -> None:
        if self.peer_exchange:
            import torch.distributed as dist
            self.backend.exchange_disconnect()   # waits for this rank's stores, unmaps the others
            dist.barrier(group=self.group)       # no rank frees its region while another still maps it
        self.backend.close()
