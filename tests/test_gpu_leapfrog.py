"""Fused leapfrog chains on the GPU vs the CPU oracle.

f32 families: q/p/grad within 1e-5 relative + 1e-6 absolute after K steps
(the integrator's + - * / are bit-identical; transcendentals differ by ulps);
logp within 1e-5 relative.  f64 Gaussian: trajectories bit-identical (same
op order, no FMA), logp within 1e-12 relative (tree vs sequential sum).
f64 logistic regression: within 1e-10 relative (GEMM summation order)."""
import numpy as np
import pytest

from gpu_util import close, down, unwrap, up

pytestmark = pytest.mark.gpu

FAMILIES = {
    "normal": ("leapfrog_chain_normal", [0.3, 1.3]),
    "exponential": ("leapfrog_chain_exponential", [1.7]),
    "studentt": ("leapfrog_chain_studentt", [0.2, 1.5, 4.0, -1.1]),
    "cauchy": ("leapfrog_chain_cauchy", [-0.4, 2.0, -float(np.log(np.pi * 2.0))]),
    "halfnormal": ("leapfrog_chain_halfnormal", [1.2, -float(np.log(1.2) + 0.5 * np.log(np.pi))]),
    "weibull": ("leapfrog_chain_weibull", [1.8, 1.4, 0.0]),
}


@pytest.mark.parametrize("family", list(FAMILIES))
@pytest.mark.parametrize("n,K", [(1, 1), (8, 32), (256, 16), (257, 5), (1000, 40), (5000, 3)])
def test_chain_families_f32(nxv, orc, family, n, K):
    fn, prm = FAMILIES[family]
    if family == "weibull":
        prm = [prm[0], prm[1], n * (np.log(prm[0]) - prm[0] * np.log(prm[1]))]
    r = np.random.default_rng(n * 31 + K)
    q0 = (r.normal(size=n) * 0.5).astype(np.float32)
    p0 = r.normal(size=n).astype(np.float32)
    m = r.uniform(0.5, 1.5, n).astype(np.float32)
    eps = 0.05
    qc, pc, gc, lc = unwrap(getattr(nxv, fn)(up(nxv, q0), up(nxv, p0), up(nxv, m), K, eps, *prm))
    wq, wp, wg, wl = orc.chain_f32(family, prm, q0, p0, m, n, 1, K, eps)
    close(down(nxv, qc, np.float32), wq, 1e-5, 1e-6)
    close(down(nxv, pc, np.float32), wp, 1e-5, 1e-6)
    close(down(nxv, gc, np.float32), wg, 1e-5, 1e-6)
    close(down(nxv, lc, np.float32), wl, 1e-5, 1e-5)
    if family == "normal":  # no transcendental in the integrator: bit-exact
        assert np.array_equal(down(nxv, qc, np.float32), wq)
        assert np.array_equal(down(nxv, pc, np.float32), wp)


@pytest.mark.parametrize("n", [3, 256, 1000, 1500])
def test_chain_normal_lg_partials(nxv, orc, n):
    r = np.random.default_rng(n)
    q0, p0 = r.normal(size=n).astype(np.float32), r.normal(size=n).astype(np.float32)
    m = np.ones(n, np.float32)
    K, eps, mu, sigma = 12, 0.1, 0.2, 0.9
    qc, pc, gc, pl = unwrap(nxv.leapfrog_chain_normal_lg(up(nxv, q0), up(nxv, p0), up(nxv, m), K, eps, mu, sigma))
    nwg = (n + 255) // 256
    parts = down(nxv, pl, np.float32).reshape(K, nwg)
    wq, wp, wg, wl = orc.chain_f32("normal", [mu, sigma], q0, p0, m, n, 1, K, eps)
    assert np.array_equal(down(nxv, qc, np.float32), wq)
    close(parts.astype(np.float64).sum(axis=1), wl, 1e-5, 1e-5)
    # each partial covers its own 256-element group; group 0 carries the constant
    qk = wq.reshape(K, n)
    for w in range(nwg):
        z = (qk[:, 256 * w:256 * (w + 1)] - mu) / sigma
        want = -0.5 * (z.astype(np.float64) ** 2).sum(axis=1)
        if w == 0:
            want = want - n * (np.log(sigma) + 0.5 * np.log(2 * np.pi))
        close(parts[:, w], want, 1e-5, 1e-5)


def test_leapfrog_single_step(nxv, orc):
    r = np.random.default_rng(7)
    n = 1001
    q, p, m = (r.normal(size=n).astype(np.float32) for _ in range(3))
    m = np.abs(m) + 0.5
    qn, pn = unwrap(nxv.leapfrog_normal(up(nxv, q), up(nxv, p), up(nxv, m), 0.1, 0.3, 1.1))
    wq, wp = orc.leapfrog_step_f32(q, p, m, 0.1, 0.3, 1.1)
    assert np.array_equal(down(nxv, qn, np.float32), wq)
    assert np.array_equal(down(nxv, pn, np.float32), wp)


@pytest.mark.parametrize("n,K", [(1, 1), (8, 32), (100, 7), (1000, 32), (3000, 33)])
def test_chain_normal_f64(nxv, orc, n, K):
    r = np.random.default_rng(n + K)
    q0, p0, m = r.normal(size=n), r.normal(size=n), r.uniform(0.5, 2, n)
    eps, mu, sigma = 0.01, 0.4, 1.3
    qc, pc, gc, lc = unwrap(nxv.leapfrog_chain_normal_f64(up(nxv, q0), up(nxv, p0), up(nxv, m), K, eps, mu, sigma))
    wq, wp, wg, wl = orc.chain_gauss_f64(q0, p0, m, np.full(n, 1 / sigma**2), mu, n, 1, K, eps)
    assert np.array_equal(down(nxv, qc, np.float64), wq)
    assert np.array_equal(down(nxv, pc, np.float64), wp)
    assert np.array_equal(down(nxv, gc, np.float64), wg)
    close(down(nxv, lc, np.float64), wl, 1e-12, 1e-12)


def gauss_config(chains, d=1000, seed=3):
    """Anisotropic Gaussian workload: prec ~ U(0.5, 2) (seed 3), q0, p0 ~ N(0,1), m = 1."""
    r = np.random.default_rng(seed)
    prec = r.uniform(0.5, 2.0, d)
    q0 = r.normal(size=(chains, d))
    p0 = r.normal(size=(chains, d))
    return prec, q0, p0, np.ones((chains, d))


@pytest.mark.parametrize("chains,d,K", [(1, 1, 1), (3, 17, 5), (64, 1000, 32), (5, 4000, 9),
                                        (2, 70000, 3)])
def test_gauss_batched_vs_oracle(nxv, orc, chains, d, K):
    prec, q0, p0, m = gauss_config(chains, d)
    m = m * np.random.default_rng(1).uniform(0.5, 1.5, m.shape)
    eps = 0.01
    outs = unwrap(nxv.leapfrog_chain_gauss_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, m), up(nxv, prec),
                                                       chains, K, eps))
    want = orc.chain_gauss_f64(q0, p0, m, prec, 0.0, d, chains, K, eps)
    for t, w in zip(outs[:3], want[:3]):
        assert np.array_equal(down(nxv, t, np.float64), w)
    close(down(nxv, outs[3], np.float64), want[3], 1e-12, 1e-12)


@pytest.mark.parametrize("stages", ["0", "1", "2", "4"])
@pytest.mark.parametrize("chains,d,K", [(64, 1000, 32), (5, 2000, 9), (7, 17, 5), (3, 998, 33)])
def test_gauss_batched_tma_staged(nxv, orc, monkeypatch, stages, chains, d, K):
    """The staged-store (TMA bulk copy) kernel gives the same bits; odd rows
    that are not 16-byte multiples fall back to the register-store kernel."""
    monkeypatch.setenv("NXV_LF_TMA", stages)
    prec, q0, p0, m = gauss_config(chains, d)
    eps = 0.01
    outs = unwrap(nxv.leapfrog_chain_gauss_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, m), up(nxv, prec),
                                                       chains, K, eps))
    want = orc.chain_gauss_f64(q0, p0, m, prec, 0.0, d, chains, K, eps)
    for t, w in zip(outs[:3], want[:3]):
        assert np.array_equal(down(nxv, t, np.float64), w)
    close(down(nxv, outs[3], np.float64), want[3], 1e-12, 1e-12)


@pytest.mark.parametrize("stages", ["2", "0"])
@pytest.mark.parametrize("chains,d,K", [(1, 1, 1), (64, 1000, 32), (7, 17, 5), (5, 4000, 9), (3, 998, 33)])
def test_gauss_batched_kinetic_energy(nxv, orc, monkeypatch, stages, chains, d, K):
    """The chain with the fused kinetic energy: trajectories and logp as the
    plain chain; ke[chain][k] = 0.5 * sum(p^2 m) of the oracle's p within
    1e-12 relative (tree vs sequential order).  Covers the staged-store
    kernel, the register-store kernel and multi-tile chains (d = 4000)."""
    monkeypatch.setenv("NXV_LF_TMA", stages)
    prec, q0, p0, m = gauss_config(chains, d)
    m = m * np.random.default_rng(1).uniform(0.5, 1.5, m.shape)
    eps = 0.01
    outs = unwrap(nxv.leapfrog_chain_gauss_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, m), up(nxv, prec),
                                                       chains, K, eps, kinetic=True))
    assert len(outs) == 5
    want = orc.chain_gauss_f64(q0, p0, m, prec, 0.0, d, chains, K, eps)
    for t, w in zip(outs[:3], want[:3]):
        assert np.array_equal(down(nxv, t, np.float64), w)
    close(down(nxv, outs[3], np.float64), want[3], 1e-12, 1e-12)
    pc = want[1].reshape(chains, K, d)
    ke_want = np.array([[sum(((pc[c, k] * pc[c, k]) * m[c]).tolist()) * 0.5 for k in range(K)]
                        for c in range(chains)])
    close(down(nxv, outs[4], np.float64).reshape(chains, K), ke_want, 1e-12, 1e-12)


@pytest.mark.parametrize("family", ["normal", "weibull"])
def test_chain_families_tma_staged(nxv, orc, monkeypatch, family):
    monkeypatch.setenv("NXV_LF_TMA", "2")
    fn, prm = FAMILIES[family]
    n, K = 1000, 40
    if family == "weibull":
        prm = [prm[0], prm[1], n * (np.log(prm[0]) - prm[0] * np.log(prm[1]))]
    r = np.random.default_rng(5)
    q0 = (r.normal(size=n) * 0.5).astype(np.float32)
    p0 = r.normal(size=n).astype(np.float32)
    m = r.uniform(0.5, 1.5, n).astype(np.float32)
    qc, pc, gc, lc = unwrap(getattr(nxv, fn)(up(nxv, q0), up(nxv, p0), up(nxv, m), K, 0.05, *prm))
    wq, wp, wg, wl = orc.chain_f32(family, prm, q0, p0, m, n, 1, K, 0.05)
    assert np.array_equal(down(nxv, qc, np.float32), wq)
    assert np.array_equal(down(nxv, pc, np.float32), wp)
    close(down(nxv, lc, np.float32), wl, 1e-5, 1e-5)


@pytest.mark.parametrize("d,chains,K", [(1000, 64, 8), (3000, 5, 4), (7, 3, 3), (1000, 1, 2)])
@pytest.mark.parametrize("ke", [False, True])
def test_gauss_shared_inverse_mass(nxv, orc, d, chains, K, ke):
    """inv_mass given as one [d] row (broadcast over the chains) gives the
    same trajectories, bit for bit, as the same row repeated per chain, on
    the staged-store kernel (d <= 2048), the multi-tile kernel (d = 3000) and
    odd rows (d = 7, register stores)."""
    r = np.random.default_rng(12)
    prec = r.uniform(0.5, 2.0, d)
    q0, p0 = r.normal(size=(chains, d)), r.normal(size=(chains, d))
    row = r.uniform(0.5, 1.5, d)
    tiled = np.tile(row, (chains, 1))
    a = unwrap(nxv.leapfrog_chain_gauss_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, row), up(nxv, prec),
                                                    chains, K, 0.01, kinetic=ke))
    b = unwrap(nxv.leapfrog_chain_gauss_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, tiled), up(nxv, prec),
                                                    chains, K, 0.01, kinetic=ke))
    for ta, tb in zip(a, b):
        assert np.array_equal(down(nxv, ta, np.float64), down(nxv, tb, np.float64))
    wq, wp, wg, wl = orc.chain_gauss_f64(q0, p0, tiled, prec, 0.0, d, chains, K, 0.01)
    assert np.array_equal(down(nxv, a[0], np.float64), wq)
    assert np.array_equal(down(nxv, a[1], np.float64), wp)


def test_gauss_full_config(nxv, orc):
    """4096 chains x d=1000, L=32, eps=0.01 (the headline workload): 16 sampled
    chains against the oracle bit for bit; all chains: time reversibility
    (negate p, integrate L more steps, recover q0 to 1e-9) and energy drift."""
    chains, d, K, eps = 4096, 1000, 32, 0.01
    prec, q0, p0, m = gauss_config(chains, d)
    outs = unwrap(nxv.leapfrog_chain_gauss_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, m), up(nxv, prec),
                                                       chains, K, eps))
    qc = down(nxv, outs[0], np.float64).reshape(chains, K, d)
    pc = down(nxv, outs[1], np.float64).reshape(chains, K, d)
    lp = down(nxv, outs[3], np.float64).reshape(chains, K)
    pick = np.random.default_rng(0).choice(chains, 16, replace=False)
    wq, wp, wg, wl = orc.chain_gauss_f64(q0[pick], p0[pick], m[pick], prec, 0.0, d, 16, K, eps)
    assert np.array_equal(qc[pick].reshape(-1), wq)
    assert np.array_equal(pc[pick].reshape(-1), wp)
    close(lp[pick].reshape(-1), wl, 1e-12, 1e-12)
    # reversibility: start at the end with flipped momentum
    qe, pe = qc[:, -1].copy(), -pc[:, -1]
    back = unwrap(nxv.leapfrog_chain_gauss_f64_batched(up(nxv, qe), up(nxv, pe), up(nxv, m), up(nxv, prec),
                                                       chains, K, eps))
    qb = down(nxv, back[0], np.float64).reshape(chains, K, d)[:, -1]
    assert np.max(np.abs(qb - q0)) < 1e-9
    # Hamiltonian drift is O(eps^2)
    h0 = 0.5 * (prec * q0**2).sum(1) + 0.5 * (p0**2).sum(1)
    h1 = -lp[:, -1] + 0.5 * np.log(prec).sum() - d * 0.5 * np.log(2 * np.pi) + 0.5 * (pc[:, -1] ** 2).sum(1)
    assert np.max(np.abs(h1 - h0) / h0) < 1e-3


@pytest.mark.parametrize("N,D,C,K", [
    (50, 3, 2, 2), (1000, 20, 5, 4), (10000, 100, 16, 3),
    # two chain blocks with a partial one; the benchmark's X shape and chain count
    (10000, 100, 256, 2), (997, 7, 130, 3),
    # fewer observations than one tile, model dims at each tile-width boundary
    (5, 2, 1, 1), (333, 32, 3, 2), (333, 33, 3, 2), (777, 64, 9, 2), (777, 104, 9, 2),
    # partial tiles; one observation; slices of more than 64 tiles (the
    # running-product flush)
    (1001, 50, 33, 2), (1, 2, 1, 1), (160000, 4, 4, 1),
    # general (two-GEMM) path
    (300, 120, 4, 2)])
@pytest.mark.parametrize("split,persist", [("1", "0"), ("2", "0"), ("2", "1")])
def test_logreg_vs_oracle(nxv, orc, monkeypatch, N, D, C, K, split, persist):
    monkeypatch.setenv("NXV_LR_SPLIT", split)  # warps per 16-chain block in the fused kernel
    # 1: the whole chain call as one cooperative kernel with grid barriers
    # (used for even D that fits one wave; the others run the per-step launches)
    monkeypatch.setenv("NXV_LR_PERSIST", persist)
    r = np.random.default_rng(4)
    X = r.normal(size=(N, D))
    w = r.normal(size=D)
    y = (r.random(N) < 1 / (1 + np.exp(-X @ w))).astype(np.float64)
    q0 = r.normal(size=(C, D)) * 0.1
    p0 = r.normal(size=(C, D))
    eps = 0.002
    outs = unwrap(nxv.leapfrog_logreg_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, X), up(nxv, y), N, D, C, K, eps))
    want = orc.chain_logreg_f64(q0, p0, X, y, N, D, C, K, eps)
    assert nxv.synchronize() == "ok"  # no bounded pipeline wait ran out
    for t, wv in zip(outs, want):
        close(down(nxv, t, np.float64), wv, 1e-10, 1e-10)


def test_logreg_outputs_feed_the_next_kernels(nxv):
    """Kernels queued right after a logistic chain call -- an f64 map and a
    per-row reduction, both on programmatic dependent launch -- read the
    chain's finished outputs: the chain's kernels let their successor start
    before they complete, so no successor may load early.  Checked against
    the downloaded outputs, bit for bit."""
    r = np.random.default_rng(8)
    N, D, C, K = 4000, 64, 48, 6
    X = r.normal(size=(N, D))
    y = (r.random(N) < 0.5).astype(np.float64)
    q0, p0 = r.normal(size=(C, D)) * 0.1, r.normal(size=(C, D))
    qc, pc, gc, lg = unwrap(nxv.leapfrog_logreg_f64_batched(up(nxv, q0), up(nxv, p0), up(nxv, X),
                                                             up(nxv, y), N, D, C, K, 0.002))
    twice = unwrap(nxv.apply_binary_f64(qc, qc, "add"))          # queued behind the chain
    row_sums = unwrap(nxv.reduce_axis_f64(gc, C * K, D, 1, 0))   # likewise
    q_h = down(nxv, qc, np.float64)
    g_h = down(nxv, gc, np.float64)
    assert np.array_equal(down(nxv, twice, np.float64), q_h + q_h)
    want = g_h.reshape(C * K, D).sum(axis=1)
    got = down(nxv, row_sums, np.float64)
    assert np.allclose(got, want, rtol=1e-12, atol=1e-12 * np.abs(g_h).reshape(C * K, D).sum(axis=1).max())
