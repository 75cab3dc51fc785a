"""Multinomial NUTS over the fused leapfrog chain: the tree-builder call site.

eXMC's NUTS tree builder (an external repository; the call site is described
in PLAN_FUSED_LEAPFROG.md:331-358: tree.ex:524 and :572 in
ensure_available/3) does not integrate step by step.  When a trajectory end
needs n more leaves it asks the backend for K = max(32, 2 n) speculative
leapfrog steps in one call and serves later doublings in the same direction
from the surplus; the backend returns {all_q, all_p, all_logp, all_grad} with
the sign convention and [k][i] layout of the fused chain.  This module is that
call site over the batched f64 Gaussian chain (nxv_leapfrog_chain_gauss_f64
_batched_ke, which also returns the kinetic energy of every step): all chains
of a batch that need steps at a tree level are extended by one batched call.

Integration backward in time is the same kernel started from the negated
momentum, with the momenta of the returned states negated back: the leapfrog
map is time-reversible and IEEE arithmetic is symmetric under negation, so
the states are bit-identical to integrating with -eps.

The transition is the multinomial NUTS of Betancourt (2017, "A Conceptual
Introduction to Hamiltonian Monte Carlo", sections A.3-A.4) as used by Stan
and eXMC:
  - momentum p ~ N(0, M) with M^-1 = inv_mass (diagonal), H = -logp + KE,
    KE = 0.5 sum p^2 inv_mass;
  - the tree doubles in a uniformly random direction up to max_depth;
  - a new subtree is rejected (and the tree stops) if any leaf diverges
    (H - H0 > 1000) or any of its balanced sub-subtrees makes a U-turn;
  - the generalized U-turn criterion on a (sub)tree with summed momentum rho
    and end momenta p-, p+ (velocities p# = inv_mass * p): no U-turn while
    p-# . rho > 0 and p+# . rho > 0; when two halves A, B merge, the same
    test is also applied to rho_A + p_B,first (ends p_A,first, p_B,first) and
    to rho_B + p_A,last (ends p_A,last, p_B,last);
  - the sample moves into a new subtree with probability
    min(1, W_subtree / W_tree) (biased progressive sampling), where W is
    the sum of exp(-H) over leaves, and within a subtree a leaf is chosen with
    probability proportional to exp(-H).

The tree logic runs on the host in numpy: it touches 2^depth leaves per
doubling, against 2^depth d-dimensional leapfrog steps per chain on the GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

LOG_SQRT_2PI = 0.91893853320467274178
MAX_DELTA_H = 1000.0


def speculative_steps(n_needed: int) -> int:
    """Steps integrated per backend call for n_needed leaves (eXMC policy)."""
    return max(32, 2 * n_needed)


class GaussianTarget:
    """N(mu, diag(1/prec)): logp(q) = -0.5 sum prec (q-mu)^2 + 0.5 sum log prec
    - d log sqrt(2 pi) -- the density of the batched Gaussian chain."""

    def __init__(self, prec, mu=0.0):
        self.prec = np.ascontiguousarray(prec, dtype=np.float64)
        self.mu = float(mu)
        self.const = 0.5 * float(np.log(self.prec).sum()) - self.prec.size * LOG_SQRT_2PI

    def logp(self, q):
        d = q - self.mu
        return -0.5 * ((self.prec * d) * d).sum(axis=-1) + self.const


class OracleChain:
    """Trajectory source on the CPU: the oracle's batched Gaussian chain
    (test infrastructure; the kinetic energy is computed from its p)."""

    def __init__(self, target: GaussianTarget, inv_mass, eps: float):
        from oracle import binding as orc
        self.orc, self.t, self.m, self.eps = orc, target, np.asarray(inv_mass, np.float64), eps
        self.calls = []

    def extend(self, q, p, K):
        c, d = q.shape
        m = np.broadcast_to(self.m, (c, d)).copy()
        qc, pc, gc, lp = self.orc.chain_gauss_f64(q, p, m, self.t.prec, self.t.mu, d, c, K, self.eps)
        pc = pc.reshape(c, K, d)
        ke = 0.5 * ((pc * pc) * m[:, None, :]).sum(axis=-1)
        self.calls.append((c, K))
        return qc.reshape(c, K, d), pc, lp.reshape(c, K), ke


class GpuChain:
    """Trajectory source on the GPU: nxv_leapfrog_chain_gauss_f64_batched_ke
    through the Nx.Vulkan mirror; q, p, logp and kinetic energy of every step
    come back to the host (the tree builder's view of the call)."""

    def __init__(self, target: GaussianTarget, inv_mass, eps: float):
        from nx_vulkan_b200 import vulkan as nxv
        self.nxv, self.t, self.m, self.eps = nxv, target, np.asarray(inv_mass, np.float64), eps
        ok, self.prec_h = nxv.upload_binary(self.t.prec.tobytes())
        if ok != "ok":
            raise RuntimeError(f"upload failed: {self.prec_h}")
        self.calls = []

    def _up(self, a):
        ok, h = self.nxv.upload_binary(np.ascontiguousarray(a, np.float64).tobytes())
        if ok != "ok":
            raise RuntimeError(f"upload failed: {h}")
        return h

    def _down(self, h, n):
        ok, b = self.nxv.download_binary(h, n * 8)
        if ok != "ok":
            raise RuntimeError(f"download failed: {b}")
        return np.frombuffer(b, dtype=np.float64).copy()

    def extend(self, q, p, K):
        c, d = q.shape
        m = np.broadcast_to(self.m, (c, d))
        ok, outs = self.nxv.leapfrog_chain_gauss_f64_batched(
            self._up(q), self._up(p), self._up(m), self.prec_h, c, K, self.eps, self.t.mu,
            kinetic=True)
        if ok != "ok":
            raise RuntimeError(f"chain call failed: {outs}")
        qh, ph, _gh, lh, kh = outs
        self.calls.append((c, K))
        return (self._down(qh, c * K * d).reshape(c, K, d), self._down(ph, c * K * d).reshape(c, K, d),
                self._down(lh, c * K).reshape(c, K), self._down(kh, c * K).reshape(c, K))


def _uturn_free(rho, ps_begin, ps_end):
    return float(ps_begin @ rho) > 0.0 and float(ps_end @ rho) > 0.0


def subtree_check(P, PS):
    """Balanced-tree U-turn check over leaves in time order (len a power of
    two).  P: momenta [n, d]; PS: velocities inv_mass * P.  Returns
    (ok, rho) with rho the summed momentum.  Evaluated level by level: at
    level j every node of 2^j leaves is the merge of two children A, B, and
    all of a level's merge tests (merge_check) run as one array operation;
    the sums pair children exactly as a recursive evaluation would."""
    n, d = P.shape
    rho = P
    size = 1
    while size < n:
        size *= 2
        h = size // 2
        pair = rho.reshape(-1, 2, d)
        ra, rb = pair[:, 0], pair[:, 1]
        first = np.arange(0, n, size)
        last, a_last, b_first = first + size - 1, first + h - 1, first + h
        r = ra + rb
        ea = ra + P[b_first]
        eb = rb + P[a_last]

        def dot(x, y):
            return np.einsum("ij,ij->i", x, y)

        ok = ((dot(PS[first], r) > 0) & (dot(PS[last], r) > 0)
              & (dot(PS[first], ea) > 0) & (dot(PS[b_first], ea) > 0)
              & (dot(PS[a_last], eb) > 0) & (dot(PS[last], eb) > 0))
        if not ok.all():
            return False, None
        rho = r
    return True, rho[0].copy()


def merge_check(rho_a, rho_b, p_a_last, ps_a_first, ps_a_last, p_b_first, ps_b_first, ps_b_last):
    """U-turn tests when subtree A (earlier in time) and B merge."""
    rho = rho_a + rho_b
    if not _uturn_free(rho, ps_a_first, ps_b_last):
        return False, None
    if not _uturn_free(rho_a + p_b_first, ps_a_first, ps_b_first):
        return False, None
    if not _uturn_free(rho_b + p_a_last, ps_a_last, ps_b_last):
        return False, None
    return True, rho


@dataclass
class Stats:
    depth: np.ndarray        # tree depth reached per chain
    n_leapfrog: np.ndarray   # leaves used per chain
    divergent: np.ndarray    # a subtree diverged
    energy: np.ndarray       # H of the initial point


def _logsumexp(v):
    m = float(np.max(v))
    return m + math.log(float(np.exp(v - m).sum()))


def nuts_transition(source, target: GaussianTarget, q0, inv_mass, rng, max_depth=10):
    """One NUTS transition for every chain of q0 [C, d]; returns (q, Stats).

    Leaves are drawn from `source` with speculative extension: all chains that
    need more steps at a tree level share one batched call of
    speculative_steps(2^depth) steps."""
    q0 = np.asarray(q0, np.float64)
    C, d = q0.shape
    m = np.asarray(inv_mass, np.float64)
    p0 = rng.standard_normal((C, d)) / np.sqrt(m)
    H0 = -target.logp(q0) + 0.5 * ((p0 * p0) * m).sum(axis=-1)
    # per chain: cached leaves beyond the initial point, index 0 = first step
    cache = {+1: [None] * C, -1: [None] * C}   # dict of arrays q, p, logp, ke
    used = {+1: np.zeros(C, np.int64), -1: np.zeros(C, np.int64)}
    # tree state
    sample = q0.copy()
    logw = -H0.copy()
    rho = p0.copy()
    ends = {+1: (p0.copy(), p0 * m), -1: (p0.copy(), p0 * m)}  # (p, p#) at each end
    active = np.ones(C, bool)
    depth = np.zeros(C, np.int64)
    divergent = np.zeros(C, bool)
    for level in range(max_depth):
        if not active.any():
            break
        n_new = 1 << level
        dirs = np.where(rng.random(C) < 0.5, -1, 1)
        # speculative extension: one batched call for every chain short of leaves
        need = [c for c in range(C) if active[c]
                and (0 if cache[dirs[c]][c] is None else cache[dirs[c]][c]["q"].shape[0])
                < used[dirs[c]][c] + n_new]
        if need:
            K = speculative_steps(n_new)
            qs, ps = np.empty((len(need), d)), np.empty((len(need), d))
            for i, c in enumerate(need):
                dd = dirs[c]
                cc = cache[dd][c]
                q_f, p_f = (q0[c], p0[c]) if cc is None else (cc["q"][-1], cc["p"][-1])
                qs[i], ps[i] = q_f, dd * p_f
            qk, pk, lk, kk = source.extend(qs, ps, K)
            for i, c in enumerate(need):
                dd = dirs[c]
                new = {"q": qk[i], "p": dd * pk[i], "logp": lk[i], "ke": kk[i]}
                cc = cache[dd][c]
                cache[dd][c] = new if cc is None else {k: np.concatenate([cc[k], new[k]]) for k in cc}
        for c in range(C):
            if not active[c]:
                continue
            dd = dirs[c]
            cc = cache[dd][c]
            a, b = used[dd][c], used[dd][c] + n_new
            Q, P = cc["q"][a:b], cc["p"][a:b]
            H = -cc["logp"][a:b] + cc["ke"][a:b]
            used[dd][c] = b
            depth[c] = level + 1
            if np.any(~(H - H0[c] <= MAX_DELTA_H)):  # also catches NaN
                divergent[c], active[c] = True, False
                continue
            # time order: backward leaves run away from the tree's left end
            if dd < 0:
                Q, P, H = Q[::-1], P[::-1], H[::-1]
            PS = P * m
            ok, rho_sub = subtree_check(P, PS)
            if not ok:
                active[c] = False
                continue
            w = -H
            logw_sub = _logsumexp(w)
            # leaf of the subtree, proportional to exp(-H); then biased move
            prob = np.exp(w - logw_sub)
            j = int(rng.choice(n_new, p=prob / prob.sum()))
            if rng.random() < min(1.0, math.exp(logw_sub - logw[c])):
                sample[c] = Q[j]
            logw[c] = float(np.logaddexp(logw[c], logw_sub))
            # merge with the old tree (A earlier in time, B later)
            old_p, old_ps = ends[-dd]  # far end of the old tree
            near_p, near_ps = ends[dd]  # end the subtree attaches to
            if dd > 0:
                ok, rho_new = merge_check(rho[c], rho_sub, near_p[c], old_ps[c], near_ps[c],
                                          P[0], PS[0], PS[-1])
            else:
                ok, rho_new = merge_check(rho_sub, rho[c], P[-1], PS[0], PS[-1],
                                          near_p[c], near_ps[c], old_ps[c])
            ends[dd][0][c], ends[dd][1][c] = (P[-1], PS[-1]) if dd > 0 else (P[0], PS[0])
            if not ok:
                active[c] = False
                continue
            rho[c] = rho_new
    n_leap = used[+1] + used[-1]
    return sample, Stats(depth=depth, n_leapfrog=n_leap, divergent=divergent, energy=H0)
