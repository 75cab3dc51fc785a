"""Host-side multi-rank logic on CPU: world_size 2 over gloo.

Chains are sharded into contiguous blocks with no data exchange; the one
collective is the all-gather of per-chain diagnostics, and step time is the
max over ranks.  The per-rank integration here runs the CPU oracle on its
shard (test infrastructure), so the gathered diagnostics can be compared
with a single-process run over all chains."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from nx_vulkan_b200.dist import chain_shard


def test_chain_shard_covers_all_chains():
    for n in (0, 1, 7, 4096, 4097):
        for world in (1, 2, 3, 8):
            shards = [chain_shard(n, r, world) for r in range(world)]
            assert shards[0].start == 0 and shards[-1].stop == n
            for a, b in zip(shards, shards[1:]):
                assert a.stop == b.start
            assert max(s.count for s in shards) - min(s.count for s in shards) <= 1
    with pytest.raises(ValueError):
        chain_shard(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_chains, result_q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from nx_vulkan_b200.dist import chain_shard, final_logp, gather_diagnostics, max_over_ranks
    from oracle import binding as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        d, K, eps = 40, 6, 0.05
        r = np.random.default_rng(3)
        prec = r.uniform(0.5, 2.0, d)
        q0, p0 = r.normal(size=(n_chains, d)), r.normal(size=(n_chains, d))
        sh = chain_shard(n_chains, rank, world)
        sl = slice(sh.start, sh.stop)
        _, _, _, lp = orc.chain_gauss_f64(q0[sl], p0[sl], np.ones((sh.count, d)), prec, 0.0, d,
                                          sh.count, K, eps)
        diag = gather_diagnostics(final_logp(torch.from_numpy(lp), sh.count, K))
        t = max_over_ranks(1.0 + rank)
        result_q.put((rank, diag.numpy(), t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_chains", [8, 9])
def test_two_rank_gather_matches_single_process(n_chains):
    from oracle import binding as orc

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_chains, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    d, K, eps = 40, 6, 0.05
    r = np.random.default_rng(3)
    prec = r.uniform(0.5, 2.0, d)
    q0, p0 = r.normal(size=(n_chains, d)), r.normal(size=(n_chains, d))
    _, _, _, lp = orc.chain_gauss_f64(q0, p0, np.ones((n_chains, d)), prec, 0.0, d, n_chains, K, eps)
    want = lp.reshape(n_chains, K)[:, -1]
    for rank, diag, t in results:
        assert np.array_equal(diag, want)  # every rank sees every chain, in chain order
        assert t == 2.0  # max over ranks of 1 + rank
