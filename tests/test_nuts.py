"""NUTS tree builder over the fused chain (host logic; the trajectory source is
the oracle here, the GPU chain in test_gpu_nuts.py)."""
import numpy as np

from nx_vulkan_b200 import nuts
from oracle import binding as orc
from oracle.chain import OracleChain


def circle(n, dt=0.1, w=1.0):
    """Leaves of a 2-D harmonic oscillator in time order: p rotates with
    angular speed w; inv_mass = 1 so p# = p."""
    t = np.arange(n) * dt
    P = np.stack([np.cos(w * t), np.sin(w * t)], axis=1)
    return P


def test_uturn_criterion_on_a_circle():
    # 8 leaves spanning 0.7 rad: no U-turn anywhere
    P = circle(8, dt=0.1)
    ok, rho = nuts.subtree_check(P, P)
    assert ok and np.allclose(rho, P.sum(axis=0))
    # 8 leaves spanning 3.5 rad (more than half a turn): U-turn
    P = circle(8, dt=0.5)
    ok, _ = nuts.subtree_check(P, P)
    assert not ok
    # the across-merge check alone: halves that are each straight but whose
    # boundary momenta oppose the other half's sum
    P = np.array([[1.0, 0.0], [1.0, 0.0], [-3.0, 0.1], [-3.0, 0.1]])
    assert not nuts.subtree_check(P, P)[0]


def test_backward_steps_are_negated_forward_steps():
    """Integrating from (q, -p) and negating the momenta gives, bit for bit,
    the states of integrating with -eps."""
    r = np.random.default_rng(1)
    c, d, K, eps = 3, 7, 9, 0.05
    prec = r.uniform(0.5, 2, d)
    q, p, m = r.normal(size=(c, d)), r.normal(size=(c, d)), r.uniform(0.5, 1.5, (c, d))
    fq, fp, _, fl = orc.chain_gauss_f64(q, -p, m, prec, 0.0, d, c, K, eps)
    bq, bp, _, bl = orc.chain_gauss_f64(q, p, m, prec, 0.0, d, c, K, -eps)
    assert np.array_equal(fq, bq)
    assert np.array_equal(-np.asarray(fp), np.asarray(bp))
    assert np.array_equal(fl, bl)


def test_speculative_policy():
    assert [nuts.speculative_steps(1 << k) for k in range(8)] == [32, 32, 32, 32, 32, 64, 128, 256]
    prec = np.array([1.0, 2.0])
    t = nuts.GaussianTarget(prec)
    src = OracleChain(t, np.ones(2), 0.1)
    rng = np.random.default_rng(3)
    q = rng.normal(size=(4, 2))
    q1, st = nuts.nuts_transition(src, t, q, np.ones(2), rng, max_depth=8)
    # every call serves whole tree levels: K >= 32 and the surplus is reused
    assert all(K >= 32 for _, K in src.calls)
    assert len(src.calls) <= 2 * int(st.depth.max())
    # levels 0 .. depth-1 consumed 1, 2, 4, ... leaves
    assert np.all(st.n_leapfrog == (1 << st.depth) - 1)


def test_nuts_samples_the_gaussian():
    """Oracle-driven NUTS on N(0, diag(1/prec)), d = 4: sample means within 5
    standard errors of 0, sample variances within 10 % of 1/prec."""
    prec = np.array([0.5, 1.0, 2.0, 4.0])
    t = nuts.GaussianTarget(prec)
    m = np.ones(4)
    src = OracleChain(t, m, 0.25)
    rng = np.random.default_rng(7)
    C, T = 16, 300
    q = rng.normal(size=(C, 4)) / np.sqrt(prec)
    draws = []
    for _ in range(T):
        q, st = nuts.nuts_transition(src, t, q, m, rng, max_depth=8)
        draws.append(q.copy())
        assert not st.divergent.any()
    x = np.concatenate(draws[50:])
    var = 1.0 / prec
    se = np.sqrt(var / x.shape[0])
    assert np.all(np.abs(x.mean(axis=0)) < 5 * se)
    assert np.all(np.abs(x.var(axis=0) / var - 1) < 0.10)


def test_leaf_store_takes_the_right_leaves():
    """The flat leaf store under the tree builder's extension rule (extend a
    chain by speculative_steps(n) leaves when fewer than n are left, then
    take n): over random direction sequences, every level's rows hold leaves
    used .. used + n - 1 of that chain and direction, in order -- the two
    blocks a chain keeps per direction always cover them."""
    rng = np.random.default_rng(11)
    C, d = 7, 3
    store = nuts._Store(d)
    leaves = {+1: nuts._Leaves(store, C), -1: nuts._Leaves(store, C)}
    for trial in range(20):
        store.size = 0
        for L in leaves.values():
            L.reset()
        for level in range(9):
            n = 1 << level
            dirs = np.where(rng.random(C) < 0.5, -1, 1)
            have = np.where(dirs > 0, leaves[+1].have, leaves[-1].have)
            used = np.where(dirs > 0, leaves[+1].used, leaves[-1].used)
            need = np.flatnonzero(have < used + n)
            if need.size:
                K = nuts.speculative_steps(n)
                # leaf labels: q[..., 0] = chain, q[..., 1] = direction, q[..., 2] = leaf number
                lab = np.zeros((need.size, K, d))
                lab[..., 0] = need[:, None]
                lab[..., 1] = dirs[need][:, None]
                lab[..., 2] = have[need][:, None] + np.arange(K)
                s0 = store.append(lab, lab, lab[..., 2])
                starts = s0 + np.arange(need.size) * K
                for sgn in (+1, -1):
                    sel = dirs[need] == sgn
                    if sel.any():
                        leaves[sgn].add_block(need[sel], starts[sel], K)
            for sgn in (+1, -1):
                rows_c = np.flatnonzero(dirs == sgn)
                if rows_c.size == 0:
                    continue
                u0 = leaves[sgn].used[rows_c].copy()
                rows = leaves[sgn].take(rows_c, n)
                got = store.q[rows]
                assert np.array_equal(got[..., 0], np.broadcast_to(rows_c[:, None], (rows_c.size, n)))
                assert np.all(got[..., 1] == sgn)
                assert np.array_equal(got[..., 2], u0[:, None] + np.arange(n))
