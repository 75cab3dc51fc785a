"""NUTS driven by the GPU chain against NUTS driven by the oracle chain.

The f64 Gaussian trajectories are bit-identical on both sides, so with the
same random stream both runs take the same tree decisions and return the
same draws.  The only difference is the reduction order of the per-step
logp and kinetic energy (tree vs sequential, ~1e-15 relative), which could
flip a decision only if a uniform draw fell within that distance of a
threshold."""
import numpy as np
import pytest

from nx_vulkan_b200 import nuts
from oracle.chain import OracleChain

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d,C,T", [(16, 8, 12), (1000, 4, 3)])
def test_nuts_gpu_matches_oracle(nxv, d, C, T):
    r = np.random.default_rng(5)
    prec = r.uniform(0.5, 2.0, d)
    t = nuts.GaussianTarget(prec)
    m = r.uniform(0.8, 1.2, d)
    eps = 0.1 if d <= 16 else 0.02
    q_init = r.normal(size=(C, d)) / np.sqrt(prec)
    gpu, cpu = nuts.GpuChain(t, m, eps), OracleChain(t, m, eps)
    qa, qb = q_init.copy(), q_init.copy()
    ra, rb = np.random.default_rng(9), np.random.default_rng(9)
    for _ in range(T):
        qa, sa = nuts.nuts_transition(gpu, t, qa, m, ra, max_depth=8)
        qb, sb = nuts.nuts_transition(cpu, t, qb, m, rb, max_depth=8)
        assert np.array_equal(qa, qb)
        assert np.array_equal(sa.depth, sb.depth) and np.array_equal(sa.n_leapfrog, sb.n_leapfrog)
    assert gpu.calls == cpu.calls


@pytest.mark.parametrize("d,C,T,depth", [(16, 64, 6, 8), (100, 256, 3, 8), (1000, 8, 2, 6)])
def test_nuts_device_tree_matches_host_tree(nxv, d, C, T, depth):
    """The tree walk on the device (nxv_nuts_*) against the host tree builder
    over the same GPU chain and the same random stream: the same depth and
    leaf count for every chain, and the same draw except where a U-turn or
    selection decision lies within rounding of its threshold (the two sum in
    different orders); at least 98 % of the draws are bit-identical."""
    import torch

    r = np.random.default_rng(7)
    prec = r.uniform(0.5, 2.0, d)
    t = nuts.GaussianTarget(prec)
    m = r.uniform(0.8, 1.2, d)
    eps = 0.1 if d <= 16 else (0.05 if d <= 100 else 0.02)
    q_init = r.normal(size=(C, d)) / np.sqrt(prec)
    host_src, dev = nuts.GpuChain(t, m, eps), nuts.DeviceTree(t, m, eps)
    qa = q_init.copy()
    same = total = same_depth = 0
    for k in range(T):
        # a fresh generator per transition, the same on both sides: a decision
        # that flips shifts the later draws of that transition only
        ra, rb = np.random.default_rng(100 + k), np.random.default_rng(100 + k)
        qa_new, sa = nuts.nuts_transition(host_src, t, qa, m, ra, max_depth=depth)
        qb_new, sb = dev.transition(torch.from_numpy(qa).cuda(), rb, max_depth=depth)
        eq = np.all(qb_new.cpu().numpy() == qa_new, axis=1)
        same += int(eq.sum())
        same_depth += int(np.sum((sa.depth == sb.depth) & (sa.n_leapfrog == sb.n_leapfrog)
                                 & (sa.divergent == sb.divergent)))
        total += C
        assert np.allclose(sa.energy, sb.energy, rtol=1e-12, atol=1e-12)
        qa = qa_new  # both continue from the host draws
    print(f"device tree: {same} of {total} draws and {same_depth} trees identical to the host's")
    assert same >= 0.98 * total and same_depth >= 0.98 * total
