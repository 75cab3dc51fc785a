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
