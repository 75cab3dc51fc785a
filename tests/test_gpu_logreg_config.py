"""The logistic-regression HMC workload at its stated size, against the oracle
with an error bound.

Workload: X f64[10000, 100] ~ N(0, 1), w* ~ N(0, 1), y ~ Bernoulli(sigmoid(X w*))
(seed 4); 256 chains from q = 0; eps = 0.002, L = 16 steps per trajectory;
momenta p ~ N(0, I) drawn on the device for every trajectory
(nx_vulkan_b200.hmc: Philox key seed + trajectory, counter chain * 100 + dim).

Every trajectory is recomputed by the oracle (oracle.c, sequential sums in
double) from the same start and momenta, and each element must satisfy

    |gpu - oracle| <= 1e-12 |oracle| + 2 E

where E is a first-order bound on the difference of two f64 evaluations that
sum in different orders:

  * one gradient, grad(q) = X^T (y - sigmoid(X q)) - q, differs by at most
    2 c u T_g per element, u = 2^-53, T_g = sum_i |x_ij| (|r_i| +
    sigmoid'(z_i) sum_j' |x_ij' q_j'|) + |q_j| (the sum of absolute terms,
    including the rounding of z = X q carried through the sigmoid), and
    c = 32 (the deterministic worst case of an n-term sum is c = n; the
    observed errors of blocked sums are a few units of u T_g);
  * the leapfrog steps carry the position error into later gradients
    through the Hessian, whose 2-norm is at most 0.25 |X|_2^2 + 1; the
    bound follows each chain's 2-norm errors of q, p and grad step by step
    (plus 2u of each rounded update), and logp's by c u T_l + |grad| e_q.

The largest ratio |gpu - oracle| / bound per output is printed.
"""
import numpy as np
import pytest

from gpu_util import down, unwrap, up

pytestmark = pytest.mark.gpu

U = 2.0 ** -53
C_SUM = 32.0
N_OBS, N_DIM, CHAINS, STEPS, EPS = 10000, 100, 256, 16, 0.002
TRAJECTORIES = 10
SEED = 4


def workload():
    r = np.random.default_rng(SEED)
    X = r.normal(size=(N_OBS, N_DIM))
    w = r.normal(size=N_DIM)
    y = (r.random(N_OBS) < 1 / (1 + np.exp(-X @ w))).astype(np.float64)
    return X, y


def terms(X, absX, y, q):
    """Per chain: T_g [C, D] (absolute terms of each gradient element) and
    T_l [C] (of logp), at positions q [C, D]."""
    z = q @ X.T
    s = np.abs(q) @ absX.T
    sig = 0.5 * (1.0 + np.tanh(0.5 * z))
    r = y - sig
    tg = (np.abs(r) + sig * (1.0 - sig) * s) @ absX + np.abs(q)
    tl = (np.abs(y * z) + np.logaddexp(0.0, z) + np.abs(r) * s).sum(1) + 0.5 * (q * q).sum(1)
    return tg, tl


def grad(X, y, q):
    z = q @ X.T
    return (y - 0.5 * (1.0 + np.tanh(0.5 * z))) @ X - q


def trajectory_bounds(X, absX, y, lam, q0, p0, qc, pc, gc):
    """Bounds [C, L] for q, p, grad (per chain and step, on every element) and
    logp, from the oracle's trajectory qc/pc/gc [C, L, D]."""
    C_, L, _ = qc.shape
    nrm = lambda a: np.sqrt((a * a).sum(-1))
    tg0, _ = terms(X, absX, y, q0)
    g_prev, p_prev = grad(X, y, q0), p0
    e_q = np.zeros(C_)
    e_p = np.zeros(C_)
    e_g = 2 * C_SUM * U * nrm(tg0)
    bq, bp, bg, bl = (np.zeros((C_, L)) for _ in range(4))
    for k in range(L):
        e_ph = e_p + 0.5 * EPS * e_g + 2 * U * (nrm(p_prev) + 0.5 * EPS * nrm(g_prev))
        e_q = e_q + EPS * e_ph + 2 * U * nrm(qc[:, k])
        tg, tl = terms(X, absX, y, qc[:, k])
        e_g = 2 * C_SUM * U * nrm(tg) + lam * e_q
        e_p = e_ph + 0.5 * EPS * e_g + 2 * U * nrm(pc[:, k])
        bq[:, k], bp[:, k], bg[:, k] = e_q, e_p, e_g
        bl[:, k] = 2 * C_SUM * U * tl + nrm(gc[:, k]) * e_q
        g_prev, p_prev = gc[:, k], pc[:, k]
    return bq, bp, bg, bl


def test_logreg_workload_trajectories_vs_oracle(nxv, orc):
    from nx_vulkan_b200 import hmc

    X, y = workload()
    absX = np.abs(X)
    lam = 0.25 * np.linalg.eigvalsh(X.T @ X).max() + 1.0
    nthr = orc.max_threads()
    tX, ty = up(nxv, X), up(nxv, y)
    q0 = up(nxv, np.zeros((CHAINS, N_DIM)))
    worst = {"q": 0.0, "p": 0.0, "grad": 0.0, "logp": 0.0}
    prev_last = None
    for tr in hmc.logreg_trajectories(q0, tX, ty, N_OBS, N_DIM, CHAINS, STEPS, EPS,
                                      TRAJECTORIES, SEED):
        q_start = down(nxv, tr.q_start, np.float64).reshape(CHAINS, N_DIM)
        p_start = down(nxv, tr.p_start, np.float64).reshape(CHAINS, N_DIM)
        # momenta: the device Philox draw (normals within 1e-12 of the oracle's)
        p_ref = orc.random_f64(CHAINS * N_DIM, hmc.momentum_key(SEED, tr.t), 1).reshape(CHAINS, N_DIM)
        assert np.all(np.abs(p_start - p_ref) <= 1e-12 * np.abs(p_ref) + 1e-14)
        # the previous trajectory's last step is this one's start, bit for bit
        if prev_last is not None:
            assert np.array_equal(q_start, prev_last)
        got = [down(nxv, t, np.float64) for t in (tr.q_chain, tr.p_chain, tr.grad_chain, tr.logp_chain)]
        want = orc.chain_logreg_f64(q_start, p_start, X, y, N_OBS, N_DIM, CHAINS, STEPS, EPS,
                                    nthreads=nthr)
        wq, wp, wg = (w.reshape(CHAINS, STEPS, N_DIM) for w in want[:3])
        wl = want[3].reshape(CHAINS, STEPS)
        bq, bp, bg, bl = trajectory_bounds(X, absX, y, lam, q_start, p_start, wq, wp, wg)
        for name, g, w, b in (("q", got[0], wq, bq[..., None]), ("p", got[1], wp, bp[..., None]),
                              ("grad", got[2], wg, bg[..., None]), ("logp", got[3], wl, bl)):
            g = g.reshape(w.shape)
            bound = 1e-12 * np.abs(w) + 2 * b
            ratio = float(np.max(np.abs(g - w) / bound))
            worst[name] = max(worst[name], ratio)
            assert ratio <= 1.0, f"trajectory {tr.t}: {name} off by {ratio:.3g} of its bound"
        prev_last = got[0].reshape(CHAINS, STEPS, N_DIM)[:, -1]
    print("largest |gpu - oracle| / bound over", TRAJECTORIES, "trajectories:",
          ", ".join(f"{k} {v:.3g}" for k, v in worst.items()))


@pytest.mark.parametrize("n,rows,width", [(7, 3, 5), (1000, 256, 100)])
def test_copy_2d_takes_strided_rows(nxv, n, rows, width):
    """nxv_buf_copy_2d: rows of `width` doubles at a pitch of n doubles."""
    from nx_vulkan_b200 import _native

    lib = _native.load()
    src = np.arange(rows * n, dtype=np.float64)
    ts = up(nxv, src)
    td = up(nxv, np.zeros(rows * width))
    off = n - width
    rc = lib.nxv_buf_copy_2d(td.handle, 0, width * 8, ts.handle, off * 8, n * 8, width * 8, rows)
    assert rc == 0, _native.last_error()
    assert np.array_equal(down(nxv, td, np.float64).reshape(rows, width),
                          src.reshape(rows, n)[:, off:])
    # a row that would leave the source buffer is refused before any copy
    assert lib.nxv_buf_copy_2d(td.handle, 0, width * 8, ts.handle, (off + 1) * 8, n * 8,
                               width * 8, rows) == -3
