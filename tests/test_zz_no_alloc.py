"""The leapfrog entry point that allocates nothing.

nxv_leapfrog_chain_gauss_f64_batched_noalloc serves callers that cannot
allocate device memory at call time: a host framework that keeps GPU memory
in its own allocator (EXLA preallocates most of HBM) and hands raw buffers
to the library, or a service that allocates everything at start-up.
It runs the batched Gaussian chain with its scratch in a static device
array.  These tests call it through the C ABI with raw device pointers and
check that it gives the allocating entry point's results on two calls in a
row, and that it neither touches the library's buffer pool nor accepts a
call whose scratch would not fit.

This file is collected last so that a run stopping at the first failure
has already run every other test."""
import ctypes as C

import numpy as np
import pytest

from gpu_util import close

pytestmark = pytest.mark.gpu


def _inputs(torch, chains, d, seed):
    r = np.random.default_rng(seed)
    prec = r.uniform(0.5, 2.0, d)
    q0, p0 = r.normal(size=(chains, d)), r.normal(size=(chains, d))
    m = r.uniform(0.5, 1.5, (chains, d))
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q0, p0, m, prec)]


def _outputs(torch, chains, d, K):
    outs = [torch.empty(chains * K * d, dtype=torch.float64, device="cuda") for _ in range(3)]
    outs.append(torch.empty(chains * K, dtype=torch.float64, device="cuda"))
    return outs


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _pool(lib):
    v = [C.c_ulong(0) for _ in range(5)]
    lib.nxv_pool_stats(*(C.byref(x) for x in v))
    return [x.value for x in v]


@pytest.mark.parametrize("chains,d,K,cfg", [(64, 1000, 32, None), (6, 5000, 7, None),
                                             # a register-store tile shape that would split
                                             # each chain into 4 tiles: the staged-store
                                             # kernel still takes it, so no partial sums
                                             (1024, 1000, 32, "256x1")])
def test_noalloc_matches_allocating_entry_point(nxv, monkeypatch, chains, d, K, cfg):
    if cfg:
        monkeypatch.setenv("NXV_LF_CFG", cfg)
    import torch
    from nx_vulkan_b200 import _native

    lib = _native.load()
    spv = nxv.shader_path("leapfrog_chain_gauss_f64_batched.spv")
    eps = 0.01
    for call, seed in enumerate((3, 4)):  # two calls in a row, different inputs
        ins = _inputs(torch, chains, d, seed)
        ref_out = _outputs(torch, chains, d, K)
        new_out = _outputs(torch, chains, d, K)
        torch.cuda.synchronize()
        # allocating entry point, through handles wrapping the same memory
        hin = [lib.nxv_buf_wrap(_ptr(t), t.numel() * 8) for t in ins]
        hout = [lib.nxv_buf_wrap(_ptr(t), t.numel() * 8) for t in ref_out]
        rc = lib.nxv_leapfrog_chain_gauss_f64_batched(*hout, *hin, d, chains, K, eps, 0.0, spv)
        assert rc == 0, _native.last_error()
        assert lib.nxv_synchronize() == 0
        pool_before = _pool(lib)
        rc = lib.nxv_leapfrog_chain_gauss_f64_batched_noalloc(
            *(_ptr(t) for t in new_out), *(_ptr(t) for t in ins), d, chains, K, eps, 0.0)
        assert rc == 0, _native.last_error()
        assert lib.nxv_synchronize() == 0
        assert _pool(lib) == pool_before  # no buffer taken from or returned to the pool
        for a, b in zip(ref_out[:3], new_out[:3]):
            assert torch.equal(a, b), f"call {call}: trajectories differ"
        close(new_out[3].cpu().numpy(), ref_out[3].cpu().numpy(), 1e-12, 1e-12)
        for h in hin + hout:
            lib.nxv_buf_free(h)


def test_noalloc_rejects_scratch_beyond_the_static_array(nxv):
    import torch
    from nx_vulkan_b200 import _native

    lib = _native.load()
    chains, d, K = 4096, 4096, 32  # 2 tiles per chain: 4096*32*2*8 B > 1 MiB
    small = torch.empty(8, dtype=torch.float64, device="cuda")
    p = _ptr(small)
    rc = lib.nxv_leapfrog_chain_gauss_f64_batched_noalloc(p, p, p, p, p, p, p, p, d, chains, K,
                                                          0.01, 0.0)
    assert rc == -3
    assert "static scratch" in _native.last_error()
