"""Multi-GPU plumbing for the batched leapfrog chains (one process per GPU).

HMC chains are independent, so a batch of chains is partitioned into
contiguous per-rank blocks with no data-path exchange; each rank integrates
its block with the fused chain kernel on its own GPU.  The only collective is
one all-gather of per-chain diagnostics (the final-step log density), the
exchange a sampler needs to compare chains.  Timing of a multi-rank step is
the maximum over ranks.

The functions take `torch.distributed` tensors and work with any backend:
NCCL over NVLink on the GPUs, gloo on CPU for the host-side tests.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    """The contiguous block of chains owned by one rank."""

    rank: int
    world: int
    start: int
    count: int

    @property
    def stop(self) -> int:
        return self.start + self.count


def chain_shard(n_chains: int, rank: int, world: int) -> Shard:
    """Split n_chains into `world` contiguous blocks whose sizes differ by at
    most one; rank r gets block r."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_chains < 0:
        raise ValueError("n_chains must be >= 0")
    base, extra = divmod(n_chains, world)
    start = rank * base + min(rank, extra)
    return Shard(rank, world, start, base + (1 if rank < extra else 0))


def final_logp(logp, chains: int, steps: int):
    """logp[chain][k] -> logp[chain][K-1] as a contiguous vector."""
    return logp.view(chains, steps)[:, -1].contiguous()


def gather_diagnostics(local, group=None):
    """All-gather one equal-length per-chain vector from every rank.

    Ranks with uneven shards pad to the longest shard; the result keeps only
    the real entries, in rank (= chain) order.  One collective per call."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    n = torch.tensor([local.numel()], dtype=torch.int64, device=local.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    width = max(sizes)
    padded = torch.zeros(width, dtype=local.dtype, device=local.device)
    padded[: local.numel()] = local
    out = torch.empty(world * width, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded, group=group)
    return torch.cat([out[r * width: r * width + sizes[r]] for r in range(world)])


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The step time of a multi-rank job: the slowest rank's."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
