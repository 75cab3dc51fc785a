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
@pytest.mark.parametrize("driver", ["layout", "levels", "host"])
def test_nuts_device_tree_matches_host_tree(nxv, d, C, T, depth, driver):
    """The tree walk on the device against the host tree builder over the
    same GPU chain and the same random numbers: the same depth and leaf
    count for every chain, and the same draw except where a U-turn or
    selection decision lies within rounding of its threshold (the two sum in
    different orders); at least 98 % of the draws are bit-identical.
    layout / levels: the device draws the momenta and uniforms (Philox) and
    keeps the tree state (one library call per transition / the per-level
    calls from Python); the host walk is given the same draws.  host: both
    draw from numpy generators with the same seed."""
    import torch

    r = np.random.default_rng(7)
    prec = r.uniform(0.5, 2.0, d)
    t = nuts.GaussianTarget(prec)
    m = r.uniform(0.8, 1.2, d)
    eps = 0.1 if d <= 16 else (0.05 if d <= 100 else 0.02)
    q_init = r.normal(size=(C, d)) / np.sqrt(prec)
    host_src, dev = nuts.GpuChain(t, m, eps), nuts.DeviceTree(t, m, eps, driver=driver)
    qa = q_init.copy()
    same = total = same_depth = 0
    for k in range(T):
        if driver in ("layout", "levels"):
            seed = 1000 + k
            p0, u = dev.randomness(C, seed, depth)
            qa_new, sa = nuts.nuts_transition(host_src, t, qa, m, None, max_depth=depth,
                                              p0=p0.cpu().numpy(), uniforms=u.cpu().numpy())
            qb_new, sb = dev.transition(torch.from_numpy(qa).cuda(), max_depth=depth, seed=seed)
        else:
            # a fresh generator per transition, the same on both sides: a
            # decision that flips shifts the later draws of that transition only
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
    print(f"device tree ({driver}): {same} of {total} draws and {same_depth} trees identical "
          f"to the host's")
    assert same >= 0.98 * total and same_depth >= 0.98 * total


@pytest.mark.parametrize("d,C,depth", [(16, 64, 8), (100, 256, 8), (1, 1, 1), (2000, 3, 5),
                                       (7, 300, 10), (2, 4, 12)])
def test_nuts_one_call_transition_matches_level_calls(nxv, d, C, depth):
    """nxv_nuts_transition_layout (the whole transition in one library call)
    against the same transition issued level by level from Python: the same
    kernels in the same order, so draws, energies, depths, leaf counts and
    divergence flags are bit-identical, over two transitions that continue
    from each other and a new seed each time."""
    import torch

    r = np.random.default_rng(17)
    prec = r.uniform(0.5, 2.0, d)
    t = nuts.GaussianTarget(prec, mu=0.3)
    m = r.uniform(0.8, 1.2, d)
    eps = 0.2 if d < 10 else (0.05 if d <= 100 else 0.02)
    if depth == 12:
        eps = 0.0005  # small steps: the trees run to the depth limit before a U-turn
    one, lev = nuts.DeviceTree(t, m, eps, driver="layout"), nuts.DeviceTree(t, m, eps, driver="levels")
    q = torch.from_numpy(r.normal(size=(C, d)) / np.sqrt(prec) + 0.3).cuda()
    for k in range(2):
        qa, sa = one.transition(q, max_depth=depth, seed=70 + k)
        qb, sb = lev.transition(q, max_depth=depth, seed=70 + k)
        assert torch.equal(qa, qb)
        for f in ("depth", "n_leapfrog", "divergent", "energy"):
            assert np.array_equal(getattr(sa, f), getattr(sb, f)), f
        assert sa.depth.max() <= depth and sa.depth.min() >= 1
        if depth == 12:
            assert sa.depth.max() == 12
        q = qa
    assert one.calls == lev.calls


def test_nuts_layout_randomness(nxv):
    """The layout driver's draws: momenta N(0, 1) / sqrt(inv_mass) and
    uniforms in [0, 1), the same for the same seed and different for another
    (Philox keys differ between the momenta and the uniforms)."""
    d, C, depth = 50, 300, 7
    r = np.random.default_rng(2)
    t = nuts.GaussianTarget(r.uniform(0.5, 2.0, d))
    m = r.uniform(0.5, 2.0, d)
    dev = nuts.DeviceTree(t, m, 0.05)
    p0, u = dev.randomness(C, 42, depth)
    p1, u1 = dev.randomness(C, 42, depth)
    p2, _ = dev.randomness(C, 43, depth)
    p0, u, p1, u1, p2 = (x.cpu().numpy() for x in (p0, u, p1, u1, p2))
    assert p0.shape == (C, d) and u.shape == (depth, 3, C)
    assert np.array_equal(p0, p1) and np.array_equal(u, u1) and not np.array_equal(p0, p2)
    z = p0 * np.sqrt(m)
    assert abs(z.mean()) < 0.02 and abs(z.std() - 1) < 0.02
    assert u.min() >= 0 and u.max() < 1 and abs(u.mean() - 0.5) < 0.01


def test_nuts_layout_sampler_moments(nxv):
    """The layout driver as a sampler: 256 chains from the target's
    distribution stay in it (mean and variance of every coordinate after
    20 transitions, within sampling error), and a tree's depth stays within
    max_depth."""
    import torch

    d, C = 20, 256
    r = np.random.default_rng(11)
    prec = r.uniform(0.5, 4.0, d)
    t = nuts.GaussianTarget(prec)
    dev = nuts.DeviceTree(t, np.ones(d), 0.2, seed=5)
    q = torch.from_numpy(r.normal(size=(C, d)) / np.sqrt(prec)).cuda()
    acc = []
    for _ in range(20):
        q, st = dev.transition(q, max_depth=6)
        assert st.depth.max() <= 6 and st.depth.min() >= 1
        acc.append(q.cpu().numpy())
    x = np.concatenate(acc) * np.sqrt(prec)  # standardised: N(0, 1) per coordinate
    assert np.all(np.abs(x.mean(axis=0)) < 0.12)
    assert np.all(np.abs(x.var(axis=0) - 1) < 0.2)


@pytest.mark.parametrize("d,C,depth", [(1, 1, 1), (3, 5, 2), (2000, 3, 5), (7, 300, 10)])
def test_nuts_layout_edge_shapes(nxv, d, C, depth):
    """The layout driver at the edges -- one dimension, one chain, a single
    level, deep trees, many chains -- against the host walk given the same
    draws, and twice in a row on one tree object (the buffers it keeps are
    reused, and the second transition continues from the first's draws)."""
    import torch

    r = np.random.default_rng(13)
    prec = r.uniform(0.5, 2.0, d)
    t = nuts.GaussianTarget(prec)
    m = r.uniform(0.8, 1.2, d)
    eps = 0.2 if d < 10 else 0.02
    host_src, dev = nuts.GpuChain(t, m, eps), nuts.DeviceTree(t, m, eps)
    qa = r.normal(size=(C, d)) / np.sqrt(prec)
    same = 0
    for k in range(2):
        p0, u = dev.randomness(C, 50 + k, depth)
        qa_new, sa = nuts.nuts_transition(host_src, t, qa, m, None, max_depth=depth,
                                          p0=p0.cpu().numpy(), uniforms=u.cpu().numpy())
        qb_new, sb = dev.transition(torch.from_numpy(qa).cuda(), max_depth=depth, seed=50 + k)
        assert sb.depth.max() <= depth and sb.depth.min() >= 1
        assert np.array_equal(sa.n_leapfrog >= 1, np.ones(C, bool))
        same += int(np.sum(np.all(qb_new.cpu().numpy() == qa_new, axis=1)
                           & (sa.depth == sb.depth) & (sa.n_leapfrog == sb.n_leapfrog)))
        qa = qa_new
    assert same >= 0.98 * 2 * C
