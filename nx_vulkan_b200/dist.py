"""Multi-GPU plumbing (one process per GPU).

Leapfrog: HMC chains are independent, so a batch of chains is partitioned
into contiguous per-rank blocks with no data-path exchange; each rank
integrates its block with the fused chain kernel on its own GPU.  The only
collective is one all-gather of per-chain diagnostics (the final-step log
density), the exchange a sampler needs to compare chains.  Timing of a
multi-rank step is the maximum over ranks.

Large elementwise, broadcast, reduction and batched-matmul calls shard the
same way: contiguous 1/G slices of the flattened tensor (whole rows for
row-wise ops, whole batch entries for batched matmul), each rank running the
single-GPU kernel on its slice.  Elementwise and broadcast results need no
exchange.  A full reduction gathers the G per-rank partials and folds them in
rank order on every rank, so every rank gets the same value and the value
does not depend on timing; row-wise results are all-gathered in row order.

The functions take `torch.distributed` tensors and work with any backend:
NCCL over NVLink on the GPUs, gloo on CPU for the host-side tests.
"""
from __future__ import annotations

import math
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

    if not dist.is_initialized():  # a single process: nothing to exchange
        return local
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


def element_shard(n: int, rank: int, world: int, align: int = 1) -> Shard:
    """Contiguous slice of n elements for `rank`, with boundaries on
    multiples of `align` (e.g. the row length, so that no row is split)."""
    if align <= 0 or n % align:
        raise ValueError(f"{n} elements do not split into units of {align}")
    sh = chain_shard(n // align, rank, world)
    return Shard(rank, world, sh.start * align, sh.count * align)


# identities of the full reductions (nxv_reduce op codes: 0 sum, 1 min, 2 max)
REDUCE_IDENTITY = {0: 0.0, 1: float("inf"), 2: float("-inf")}


def fold_in_rank_order(partials, op: int) -> float:
    """Fold per-rank partials left to right in rank order.  Sums are
    compensated (Neumaier: the rounding error of every addition is carried
    and added once at the end), so the fold adds at most about one rounding
    of the total to the partials' own errors, also when slices cancel;
    min/max propagate NaN like the single-GPU kernels."""
    if op not in REDUCE_IDENTITY:
        raise ValueError(f"reduce op {op} outside 0..2")
    acc = REDUCE_IDENTITY[op]
    if op == 0:
        comp, plain = 0.0, 0.0
        for v in partials:
            v = float(v)
            plain += v
            t = acc + v
            if abs(acc) >= abs(v):
                comp += (acc - t) + v
            else:
                comp += (v - t) + acc
            acc = t
        # infinities and NaN: the plain sum's IEEE result
        return acc + comp if math.isfinite(plain) else plain
    for v in partials:
        v = float(v)
        if v != v or acc != acc:
            acc = float("nan")
        elif op == 1:
            acc = v if v < acc else acc
        else:
            acc = v if v > acc else acc
    return acc


def fold_partials(local: float, op: int, group=None, device=None) -> float:
    """Full reduction across ranks: one all-gather of every rank's partial
    (float64), then the same rank-order fold on every rank.  A rank whose
    slice is empty passes the op's identity."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        return fold_in_rank_order([local], op)
    world = dist.get_world_size(group)
    t = torch.tensor([float(local)], dtype=torch.float64, device=device)
    out = torch.empty(world, dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(out, t, group=group)
    return fold_in_rank_order(out.cpu().tolist(), op)


def gather_rows(local, group=None):
    """All-gather a row-sharded result: local is [rows_r, ...] on every rank
    (row counts may differ by rank); returns [sum rows_r, ...] in rank order."""
    tail = tuple(local.shape[1:])
    flat = gather_diagnostics(local.reshape(-1), group=group)
    return flat.reshape((-1,) + tail)


def _coll_device():
    """Tensors for collectives live on the GPU under NCCL, on the host else."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def reduce_full(nxv, x_slice, op: int, dtype: str = "f64", group=None) -> float:
    """Sum (0), min (1) or max (2) of a tensor stored as contiguous per-rank
    slices: the rank's slice through nxv_reduce / nxv_reduce_f64 on its GPU,
    then the rank-order fold.  `x_slice` is the rank's device buffer (None
    or empty for an empty slice).  f32 partials are folded in double and the
    result rounded to f32 once, like the single-GPU f32 reduce."""
    import numpy as np

    if op not in REDUCE_IDENTITY:
        raise ValueError(f"reduce op {op} outside 0..2")
    if x_slice is None or x_slice.n_bytes == 0:
        local = REDUCE_IDENTITY[op]
    else:
        if dtype == "f64":
            r = nxv.reduce_f64(x_slice, op)
        else:
            r = (nxv.sum, nxv.reduce_min, nxv.reduce_max)[op](x_slice)
        if r[0] != "ok":
            raise RuntimeError(f"reduce failed on this rank: {r[1]}")
        local = r[1]
    v = fold_partials(local, op, group=group, device=_coll_device())
    return float(np.float32(v)) if dtype == "f32" else v


def _rank_output(nxv, shape, np_dtype):
    """The rank's output tensor and the handle a kernel writes it through.

    With the CUDA library the tensor lives on the rank's GPU and the kernel
    fills it in place (a non-owning handle over the tensor's memory), so the
    result never leaves the device before the collective.  A host stand-in
    of the library (tests without a GPU; `nxv.on_host`) gets a host tensor."""
    import numpy as np
    import torch

    tdt = {np.dtype(np.float64): torch.float64, np.dtype(np.float32): torch.float32,
           np.dtype(np.int64): torch.int64}[np.dtype(np_dtype)]
    host = getattr(nxv, "on_host", False)
    dev = torch.device("cpu") if host else torch.device("cuda", torch.cuda.current_device())
    t = torch.empty(shape, dtype=tdt, device=dev)
    return t, (nxv.wrap_tensor(t) if t.numel() else None)


def _finish_rank(nxv, local, what):
    """Wait for the rank's kernel (the library runs on its own stream), then
    put the tensor where the backend's collectives run: NCCL takes device
    tensors as they are; gloo needs a host copy."""
    import torch.distributed as dist

    if not getattr(nxv, "on_host", False):
        ok = nxv.synchronize()
        if ok != "ok":
            raise RuntimeError(f"{what} failed on this rank: {ok}")
    if dist.is_initialized() and dist.get_backend() != "nccl" and local.is_cuda:
        return local.cpu()
    return local


def reduce_rows(nxv, x_rows, n_rows: int, row_len: int, op: int, dtype: str = "f64",
                group=None):
    """Per-row sum/max/min (nxv_reduce_axis op codes 0/1/2) of a row-sharded
    matrix: each rank reduces its n_rows rows on its GPU into a device tensor,
    and the results are all-gathered in row order (NCCL, device to device).
    Returns the full [total rows] vector as a torch tensor on the collective
    device (the rank's GPU under NCCL)."""
    import numpy as np

    local, h = _rank_output(nxv, (n_rows,), np.float64 if dtype == "f64" else np.float32)
    if n_rows:
        fn = nxv.reduce_axis_f64 if dtype == "f64" else nxv.reduce_axis
        ok, out = fn(x_rows, n_rows, row_len, 1, op, out=h)
        if ok != "ok":
            raise RuntimeError(f"reduce_axis failed on this rank: {out}")
    return gather_rows(_finish_rank(nxv, local, "reduce_axis"), group)


def argmax_rows(nxv, x_rows, n_rows: int, row_len: int, dtype: str = "f64", group=None):
    """Per-row argmax (lowest index on ties) of a row-sharded matrix; indices
    are within the row, so sharding by rows leaves them unchanged.  Returns
    int64 indices as a torch tensor on the collective device."""
    import numpy as np

    local, h = _rank_output(nxv, (n_rows,), np.int64)
    if n_rows:
        ok, out = nxv.argmax_axis(x_rows, n_rows, row_len, 1, dtype=dtype, out=h)
        if ok != "ok":
            raise RuntimeError(f"argmax failed on this rank: {out}")
    return gather_rows(_finish_rank(nxv, local, "argmax"), group)


def matmul_batched(nxv, a, b, n_batch: int, m: int, n: int, k: int, dtype: str = "f64",
                   group=None):
    """Batched matmul sharded by batch entry: each rank multiplies its
    n_batch entries on its GPU into a device tensor; the products are
    all-gathered in batch order.  Returns [total batch, m, n] as a torch
    tensor on the collective device."""
    import numpy as np

    local, h = _rank_output(nxv, (n_batch, m, n), np.float64 if dtype == "f64" else np.float32)
    if n_batch:
        ok, out = nxv.matmul_batched(a, b, n_batch, m, n, k, dtype=dtype, out=h)
        if ok != "ok":
            raise RuntimeError(f"matmul failed on this rank: {out}")
    return gather_rows(_finish_rank(nxv, local, "matmul"), group)
