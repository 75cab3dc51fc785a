"""Sharded reductions, argmax and batched matmul over NCCL, one process per
GPU: the rows of x [4096, 4096] (f32 and f64, ~ N(0, 1), seed 1) are split
over two ranks, each rank reduces its rows on its own GPU into a device
tensor, and the results are all-gathered device to device.  Checked against
the oracle: argmax and max bit for bit, row sums within the f64 / f32 sum
bounds.  Needs two GPUs (skipped otherwise)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROWS, COLS = 4096, 4096


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(dt):
    return np.random.default_rng(1).normal(size=(ROWS, COLS)).astype(dt)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from nx_vulkan_b200 import dist as nd, vulkan as nxv
        assert nxv.init_devices([rank]) == "ok"
        sh = nd.chain_shard(ROWS, rank, world)
        out = {}
        for name, dt in (("f64", np.float64), ("f32", np.float32)):
            x = _data(dt)[sh.start:sh.stop]
            ok, t = nxv.upload_binary(np.ascontiguousarray(x))
            assert ok == "ok"
            rs = nd.reduce_rows(nxv, t, sh.count, COLS, 0, dtype=name)
            rm = nd.reduce_rows(nxv, t, sh.count, COLS, 1, dtype=name)
            am = nd.argmax_rows(nxv, t, sh.count, COLS, dtype=name)
            assert rs.is_cuda and am.is_cuda  # gathered on the device
            out[name] = (rs.cpu().numpy(), rm.cpu().numpy(), am.cpu().numpy())
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_sharded_rows_over_nccl_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import binding as orc

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for name, dt in (("f64", np.float64), ("f32", np.float32)):
        x = _data(dt)
        want_max = x.max(axis=1)
        want_arg = np.argmax(x, axis=1)
        want_sum = orc.reduce_axis(x.reshape(-1), ROWS, COLS, 1, 0)
        absum = np.abs(x.astype(np.float64)).sum(axis=1)
        for _, out in res:
            rs, rm, am = out[name]
            assert np.array_equal(am, want_arg)
            assert np.array_equal(rm, want_max)
            if dt == np.float64:
                assert np.all(np.abs(rs - want_sum) <= 1e-12 * np.abs(want_sum) + 4 * 2.2e-16 * absum)
            else:
                assert np.all(np.abs(rs - want_sum) <= 1e-5 * np.abs(want_sum) + 1e-6 + COLS * 2 ** -24 * absum)
        assert all(np.array_equal(res[0][1][name][i], res[1][1][name][i]) for i in range(3))
