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


# ---- sharded elementwise / reduction / batched matmul (host logic) ------------

class _Buf:
    def __init__(self, arr):
        self.arr = np.ascontiguousarray(arr)
        self.n_bytes = self.arr.nbytes


class _TensorBuf(_Buf):
    """A host stand-in's view of a torch CPU tensor (FakeNxv.wrap_tensor)."""

    def __init__(self, t):
        self.t = t
        self.arr = t.numpy()
        self.n_bytes = self.arr.nbytes


class FakeNxv:
    """Stands in for the Nx.Vulkan mirror on a machine without a GPU: the same
    call signatures and ("ok", value) results, computed with numpy; outputs
    given with out= are written in place."""

    on_host = True

    @staticmethod
    def wrap_tensor(t):
        return _TensorBuf(t)

    @staticmethod
    def _into(out, value):
        if out is None:
            return ("ok", _Buf(value))
        out.arr[...] = np.asarray(value).reshape(out.arr.shape)
        return ("ok", out)

    def reduce_f64(self, t, op):
        return ("ok", float((np.sum, np.min, np.max)[op](t.arr)))

    def sum(self, t):
        return ("ok", float(np.float32(np.sum(t.arr, dtype=np.float64))))

    def reduce_min(self, t):
        return ("ok", float(np.min(t.arr)))

    def reduce_max(self, t):
        return ("ok", float(np.max(t.arr)))

    def reduce_axis_f64(self, t, outer, r, inner, op, out=None):
        x = t.arr.reshape(outer, r, inner)
        return self._into(out, (np.sum, np.max, np.min)[op](x, axis=1).reshape(-1))

    def argmax_axis(self, t, outer, r, inner, dtype="f32", out=None):
        return self._into(out, np.argmax(t.arr.reshape(outer, r, inner), axis=1).astype(np.int64))

    def matmul_batched(self, a, b, batch, m, n, k, dtype="f64", out=None):
        return self._into(out, np.matmul(a.arr.reshape(batch, m, k), b.arr.reshape(batch, k, n)))

    def download_binary(self, t, n_bytes):
        assert n_bytes == t.n_bytes
        return ("ok", t.arr.tobytes())


def test_element_shard_keeps_rows_whole():
    from nx_vulkan_b200.dist import element_shard
    for rows, world in ((10, 3), (1, 4), (4096, 8)):
        shards = [element_shard(rows * 7, r, world, 7) for r in range(world)]
        assert shards[0].start == 0 and shards[-1].stop == rows * 7
        assert all(s.start % 7 == 0 and s.count % 7 == 0 for s in shards)
    with pytest.raises(ValueError):
        element_shard(10, 0, 2, 3)


def test_fold_in_rank_order():
    from nx_vulkan_b200.dist import fold_in_rank_order
    # compensated: the rounding error of 1e16 + 1.0 is carried, giving the exact sum
    assert fold_in_rank_order([1e16, 1.0, -1e16], 0) == 1.0
    assert fold_in_rank_order([1e300, 1e300, float("inf")], 0) == float("inf")
    assert np.isnan(fold_in_rank_order([float("inf"), 1.0, float("-inf")], 0))
    assert np.isnan(fold_in_rank_order([1.0, float("nan")], 0))
    # slices that cancel: [a, -a + tiny] gives the tiny remainder exactly
    assert fold_in_rank_order([0.1 + 0.2, -(0.1 + 0.2), 1e-17], 0) == 1e-17
    assert fold_in_rank_order([3.0, -1.0, 2.0], 1) == -1.0
    assert fold_in_rank_order([3.0, float("inf"), 2.0], 2) == float("inf")
    assert fold_in_rank_order([], 2) == float("-inf")
    assert np.isnan(fold_in_rank_order([1.0, float("nan"), 2.0], 2))
    with pytest.raises(ValueError):
        fold_in_rank_order([1.0], 3)


def _sharded_worker(rank, world, port, result_q, use_gpu):
    import torch.distributed as dist
    from datetime import timedelta

    from nx_vulkan_b200 import dist as nd

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        if use_gpu:
            from nx_vulkan_b200 import vulkan as nxv
            assert nxv.init() == "ok"

            def buf(a):
                if a.size == 0:
                    return None
                ok, t = nxv.upload_binary(np.ascontiguousarray(a).tobytes())
                assert ok == "ok", t
                return t
        else:
            nxv = FakeNxv()
            buf = _Buf
        rows, row_len, batch, m, n, k = 9, 37, 2, 6, 7, 8
        r = np.random.default_rng(11)
        x = r.normal(size=(rows, row_len))
        a, b = r.normal(size=(batch, m, k)), r.normal(size=(batch, k, n))
        sh = nd.element_shard(rows * row_len, rank, world, row_len)
        xs = x.reshape(-1)[sh.start:sh.stop]
        rs = nd.chain_shard(rows, rank, world)
        bs = nd.chain_shard(batch, rank, world)
        out = {
            "sum": nd.reduce_full(nxv, buf(xs), 0, "f64"),
            "min": nd.reduce_full(nxv, buf(xs), 1, "f64"),
            "max": nd.reduce_full(nxv, buf(xs), 2, "f64"),
            "sum32": nd.reduce_full(nxv, buf(xs.astype(np.float32)), 0, "f32"),
            "row_sum": nd.reduce_rows(nxv, buf(x[rs.start:rs.stop]), rs.count, row_len, 0),
            "row_max": nd.reduce_rows(nxv, buf(x[rs.start:rs.stop]), rs.count, row_len, 1),
            "argmax": nd.argmax_rows(nxv, buf(x[rs.start:rs.stop]), rs.count, row_len),
            "bmm": nd.matmul_batched(nxv, buf(a[bs.start:bs.stop]), buf(b[bs.start:bs.stop]),
                                     bs.count, m, n, k),
            "partials": [float(np.sum(x.reshape(-1)[s.start:s.stop]))
                         for s in (nd.element_shard(rows * row_len, q, world, row_len)
                                   for q in range(world))],
        }
        for key in ("row_sum", "row_max", "argmax", "bmm"):
            out[key] = out[key].cpu().numpy()
        result_q.put((rank, out))
    finally:
        dist.destroy_process_group()


def run_sharded(world, use_gpu=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, q, use_gpu))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return [o for _, o in sorted(results, key=lambda t: t[0])]


def check_sharded(results, world, exact_rows):
    """Every rank holds the same gathered results, equal to the unsharded
    computation; the full sum is the rank-order fold of the slice sums."""
    rows, row_len, batch, m, n, k = 9, 37, 2, 6, 7, 8
    r = np.random.default_rng(11)
    x = r.normal(size=(rows, row_len))
    a, b = r.normal(size=(batch, m, k)), r.normal(size=(batch, k, n))
    from nx_vulkan_b200.dist import fold_in_rank_order
    for o in results:
        assert o["min"] == x.min() and o["max"] == x.max()
        want_sum = fold_in_rank_order(o["partials"], 0)
        assert abs(o["sum"] - want_sum) <= 1e-12 * np.abs(x).sum()
        assert abs(o["sum"] - x.sum()) <= 1e-12 * np.abs(x).sum()
        assert abs(o["sum32"] - x.astype(np.float32).astype(np.float64).sum()) <= 1e-5 * np.abs(x).sum()
        assert np.array_equal(o["argmax"], np.argmax(x, axis=1))
        assert np.array_equal(o["row_max"], x.max(axis=1))
        if exact_rows:
            assert np.array_equal(o["row_sum"], x.sum(axis=1))
        assert np.allclose(o["row_sum"], x.sum(axis=1), rtol=1e-12, atol=1e-12 * row_len)
        bound = 2 * k * np.finfo(np.float64).eps * np.matmul(np.abs(a), np.abs(b))
        assert np.all(np.abs(o["bmm"] - np.matmul(a, b)) <= 1e-12 * np.abs(np.matmul(a, b)) + bound)
        for key in ("sum", "sum32", "row_sum", "argmax", "bmm"):   # identical on every rank
            assert np.array_equal(np.asarray(o[key]), np.asarray(results[0][key]))


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_ops_over_gloo(world):
    # world 3: one rank gets no batch entry (2 entries over 3 ranks)
    check_sharded(run_sharded(world), world, exact_rows=True)
