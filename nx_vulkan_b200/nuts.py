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

nuts_transition runs the tree logic on the host in numpy (it touches
2^depth leaves per doubling, against 2^depth d-dimensional leapfrog steps
per chain on the GPU); DeviceTree runs the same logic on the device over a
leaf store that the chain calls write into.
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


class GpuChain:
    """Trajectory source on the GPU: nxv_leapfrog_chain_gauss_f64_batched_ke
    through the Nx.Vulkan mirror; q, p, logp and kinetic energy of every step
    come back to the host (the tree builder's view of the call).  Transfers
    go through reused page-locked buffers (direct DMA, no staging copy); the
    arrays `extend` returns are views of those buffers, valid until the next
    call.  The per-chain inverse mass (the same row for every chain) is
    uploaded once per chain count."""

    def __init__(self, target: GaussianTarget, inv_mass, eps: float):
        from nx_vulkan_b200 import _native
        from nx_vulkan_b200 import vulkan as nxv
        self.nxv, self.lib = nxv, _native.load()
        self.t, self.m, self.eps = target, np.asarray(inv_mass, np.float64), eps
        ok, self.prec_h = nxv.upload_binary(self.t.prec.tobytes())
        if ok != "ok":
            raise RuntimeError(f"upload failed: {self.prec_h}")
        self.calls = []
        self.pinned = {}  # slot -> page-locked float64 array
        self.m_dev = {}   # chain count -> device buffer of inv_mass broadcast to [c, d]

    def _host(self, slot, n):
        a = self.pinned.get(slot)
        if a is None or a.size < n:
            import torch
            a = torch.empty(max(n, 1 << 16), dtype=torch.float64, pin_memory=True).numpy()
            self.pinned[slot] = a
        return a[:n]

    def _up(self, a, slot):
        # staged in a page-locked buffer: the upload is a direct DMA (and
        # returns once the copy is done, so the buffer can be reused)
        host = self._host(slot, a.size)
        host[:] = np.asarray(a, np.float64).reshape(-1)
        ok, h = self.nxv.upload_binary(host)
        if ok != "ok":
            raise RuntimeError(f"upload failed: {h}")
        return h

    def _down(self, h, n, slot):
        import ctypes
        a = self._host(slot, n)
        if self.lib.nxv_buf_download(h.handle, ctypes.c_void_p(a.ctypes.data), n * 8) != 0:
            raise RuntimeError("download failed")
        return a

    def extend(self, q, p, K):
        c, d = q.shape
        m = self.m_dev.get(c)
        if m is None:
            m = self.m_dev[c] = self._up(np.broadcast_to(self.m, (c, d)), 12)
        ok, outs = self.nxv.leapfrog_chain_gauss_f64_batched(
            self._up(q, 10), self._up(p, 11), m, self.prec_h, c, K, self.eps, self.t.mu,
            kinetic=True)
        if ok != "ok":
            raise RuntimeError(f"chain call failed: {outs}")
        qh, ph, _gh, lh, kh = outs
        self.calls.append((c, K))
        return (self._down(qh, c * K * d, 0).reshape(c, K, d), self._down(ph, c * K * d, 1).reshape(c, K, d),
                self._down(lh, c * K, 2).reshape(c, K), self._down(kh, c * K, 3).reshape(c, K))


def _dot(x, y):
    return np.einsum("...i,...i->...", x, y)


def _free(rho, ps_begin, ps_end):
    """No U-turn: both end velocities have a positive projection on rho."""
    return (_dot(ps_begin, rho) > 0) & (_dot(ps_end, rho) > 0)


def merge_check(rho_a, rho_b, p_a_last, ps_a_first, ps_a_last, p_b_first, ps_b_first, ps_b_last):
    """U-turn tests when subtree A (earlier in time) and B merge; every
    argument may carry leading batch axes.  Returns (ok, rho_a + rho_b)."""
    rho = rho_a + rho_b
    ok = (_free(rho, ps_a_first, ps_b_last) & _free(rho_a + p_b_first, ps_a_first, ps_b_first)
          & _free(rho_b + p_a_last, ps_a_last, ps_b_last))
    return ok, rho


def subtree_check(P, PS):
    """Balanced-tree U-turn check over leaves in time order.  P: momenta
    [..., n, d] with n a power of two; PS: velocities inv_mass * P.  Returns
    (ok [...], rho [..., d]), rho the summed momentum.

    Every node [a, b) of 2^j leaves is the merge of its halves [a, m) and
    [m, b), tested as in merge_check.  Every dot product comes from one Gram
    matrix per chain, H = PS . P^T (ps_i . p_j), and its running sums along
    j, G[i, b] = sum of H[i, :b] = ps_i . (p_0 + ... + p_(b-1)), so that
    ps_i . rho of [a, b) = G[i, b] - G[i, a]; each level's tests are then
    array lookups.  One matrix product replaces the per-level dot products
    over [..., n, d] arrays."""
    P, PS = np.asarray(P), np.asarray(PS)
    n, d = P.shape[-2:]
    lead = P.shape[:-2]
    H = PS @ np.swapaxes(P, -1, -2)   # [..., n, n]
    G = np.zeros(lead + (n, n + 1))
    np.cumsum(H, axis=-1, out=G[..., 1:])
    ok = np.ones(lead, bool)
    size = 1
    while size < n:
        size *= 2
        a = np.arange(0, n, size)
        m, b = a + size // 2, a + size
        first, last, a_last, b_first = a, b - 1, m - 1, m
        good = ((G[..., first, b] - G[..., first, a] > 0)       # whole node: ends vs rho
                & (G[..., last, b] - G[..., last, a] > 0)
                # rho_A + p_B,first against ps_A,first and ps_B,first
                & (G[..., first, m] - G[..., first, a] + H[..., first, b_first] > 0)
                & (G[..., b_first, m] - G[..., b_first, a] + H[..., b_first, b_first] > 0)
                # rho_B + p_A,last against ps_A,last and ps_B,last
                & (G[..., a_last, b] - G[..., a_last, m] + H[..., a_last, a_last] > 0)
                & (G[..., last, b] - G[..., last, m] + H[..., last, a_last] > 0))
        ok &= good.all(axis=-1)
    return ok, P.sum(axis=-2)


@dataclass
class Stats:
    depth: np.ndarray        # tree depth reached per chain
    n_leapfrog: np.ndarray   # leaves used per chain
    divergent: np.ndarray    # a subtree diverged
    energy: np.ndarray       # H of the initial point


class _Store:
    """Leaf rows (q, p in the sign it was integrated with -- negated for
    backward leaves --, H = -logp + KE) of both directions in one flat store
    that grows by doubling and is reused across transitions."""

    def __init__(self, d: int):
        self.d = d
        self.q = np.empty((0, d))
        self.p = np.empty((0, d))
        self.h = np.empty(0)
        self.size = 0

    def append(self, q, p, h) -> int:
        """Append the leaves of one chain call ([n, K, ...]); returns the
        first flat row (chain i's leaves start at row + i K)."""
        n, K = q.shape[:2]
        self.reserve(n * K)
        s0 = self.size
        self.q[s0: s0 + n * K] = q.reshape(n * K, self.d)
        self.p[s0: s0 + n * K] = p.reshape(n * K, self.d)
        self.h[s0: s0 + n * K] = h.reshape(n * K)
        self.size += n * K
        return s0

    def reserve(self, rows: int):
        need = self.size + rows
        if need <= self.h.shape[0]:
            return
        cap = max(need, 2 * self.h.shape[0])
        for name in ("q", "p", "h"):
            old = getattr(self, name)
            new = np.empty((cap,) + old.shape[1:])
            new[: self.size] = old[: self.size]
            setattr(self, name, new)


class _Leaves:
    """Leaves integrated beyond the initial point in one direction, for every
    chain, kept in a shared _Store; each extension appends one block of K
    leaves per extended chain.  Per chain: `have` leaves stored, `used`
    taken into the tree, and the flat start and leaf number of its current
    and previous blocks.

    A tree level takes leaves [used, used + n) of a chain, which always lie
    in those two blocks: a chain is extended only when fewer than n leaves
    are left, so the leftover of the previous block is used up by the level
    that follows the extension, and `used` never falls behind the previous
    block's first leaf again."""

    def __init__(self, store: _Store, C: int):
        self.store, self.C = store, C
        self.reset()

    def reset(self):
        C = self.C
        self.have = np.zeros(C, np.int64)
        self.used = np.zeros(C, np.int64)
        self.cur_start = np.zeros(C, np.int64)
        self.cur_base = np.zeros(C, np.int64)
        self.prev_start = np.zeros(C, np.int64)
        self.prev_base = np.zeros(C, np.int64)

    def add_block(self, rows, starts, K: int):
        """Chains `rows` got K new leaves at flat rows starts, starts + 1, ..."""
        self.prev_start[rows] = self.cur_start[rows]
        self.prev_base[rows] = self.cur_base[rows]
        self.cur_start[rows] = starts
        self.cur_base[rows] = self.have[rows]
        self.have[rows] += K

    def last(self, rows):
        """Flat row of the last stored leaf of chains `rows` (have > 0)."""
        return self.cur_start[rows] + (self.have[rows] - self.cur_base[rows]) - 1

    def take(self, rows, n: int):
        """Flat rows [len(rows), n] of the next n leaves of chains `rows`, marked used."""
        j = self.used[rows][:, None] + np.arange(n)
        cb = self.cur_base[rows][:, None]
        flat = np.where(j >= cb, self.cur_start[rows][:, None] + (j - cb),
                        self.prev_start[rows][:, None] + (j - self.prev_base[rows][:, None]))
        self.used[rows] += n
        return flat


def nuts_transition(source, target: GaussianTarget, q0, inv_mass, rng, max_depth=10,
                    p0=None, uniforms=None):
    """One NUTS transition for every chain of q0 [C, d]; returns (q, Stats).

    Leaves are drawn from `source` with speculative extension: all chains that
    need more steps at a tree level share one batched call of
    speculative_steps(2^depth) steps.  The tree logic is vectorized over the
    chains that are still building.  The momenta and the uniforms come from
    `rng` (momenta first, then per level the directions of every chain and
    the leaf and move uniforms of the chains still building), or are given:
    p0 [C, d] and uniforms [max_depth][3][C] (direction, leaf, move of chain
    c at each level), the draws DeviceTree makes on the device."""
    q0 = np.asarray(q0, np.float64)
    C, d = q0.shape
    m = np.asarray(inv_mass, np.float64)
    p0 = rng.standard_normal((C, d)) / np.sqrt(m) if p0 is None else np.asarray(p0, np.float64)
    H0 = -target.logp(q0) + 0.5 * ((p0 * p0) * m).sum(axis=-1)
    # per direction: the leaves beyond the initial point (kept on the source
    # between transitions, so the store's pages stay mapped)
    leaves = getattr(source, "_nuts_leaves", None)
    if leaves is None or leaves[+1].C != C or leaves[+1].store.d != d:
        store = _Store(d)
        leaves = {+1: _Leaves(store, C), -1: _Leaves(store, C)}
        try:
            source._nuts_leaves = leaves
        except AttributeError:
            pass
    store = leaves[+1].store
    store.size = 0
    for L in leaves.values():
        L.reset()
    sample = q0.copy()
    logw = -H0.copy()
    rho = p0.copy()
    # momentum and velocity at the tree's left (-1) and right (+1) ends
    end_p = {+1: p0.copy(), -1: p0.copy()}
    end_ps = {+1: p0 * m, -1: p0 * m}
    active = np.ones(C, bool)
    depth = np.zeros(C, np.int64)
    divergent = np.zeros(C, bool)
    for level in range(max_depth):
        if not active.any():
            break
        n_new = 1 << level
        dirs = np.where((rng.random(C) if uniforms is None else uniforms[level, 0]) < 0.5, -1, 1)
        fwd_all = dirs > 0
        have = np.where(fwd_all, leaves[+1].have, leaves[-1].have)
        used = np.where(fwd_all, leaves[+1].used, leaves[-1].used)
        # speculative extension: one batched call for every chain short of
        # leaves, in chain order; each starts from its last stored leaf in
        # that direction (the initial point when there is none), with the
        # momentum negated when integrating backward
        need = np.flatnonzero(active & (have < used + n_new))
        if need.size:
            K = speculative_steps(n_new)
            # initial point: p0 in forward sign, negated for backward chains;
            # stored leaves already hold p in their integration sign
            qs, ps = q0[need].copy(), p0[need] * dirs[need][:, None]
            for sgn in (+1, -1):
                L = leaves[sgn]
                sel = (dirs[need] == sgn) & (L.have[need] > 0)
                if sel.any():
                    f = L.last(need[sel])
                    qs[sel], ps[sel] = store.q[f], store.p[f]
            qk, pk, lk, kk = source.extend(qs, ps, K)
            s0 = store.append(qk, pk, -lk + kk)
            starts = s0 + np.arange(need.size) * K
            for sgn in (+1, -1):
                sel = dirs[need] == sgn
                if sel.any():
                    leaves[sgn].add_block(need[sel], starts[sel], K)
        # the level's new leaves of every active chain, in time order: their
        # flat rows, then one gather of p and H (q only for the sampled leaf)
        act = np.flatnonzero(active)
        A = act.size
        fwd = dirs[act] > 0
        rows = np.empty((A, n_new), np.int64)
        for sgn, sel in ((+1, fwd), (-1, ~fwd)):
            if sel.any():
                r_ = leaves[sgn].take(act[sel], n_new)
                rows[sel] = r_ if sgn > 0 else r_[:, ::-1]  # backward leaves run leftward
        P, H = store.p[rows], store.h[rows]
        P[~fwd] *= -1.0  # backward leaves were integrated with negated momentum
        depth[act] = level + 1
        # divergence (also NaN): the subtree is discarded and the tree stops
        div = ~np.all(H - H0[act, None] <= MAX_DELTA_H, axis=1)
        divergent[act] |= div
        PS = P * m
        ok_sub, rho_sub = subtree_check(P, PS)
        ok_sub &= ~div
        # a leaf of each subtree with probability proportional to exp(-H),
        # then the biased move into the subtree with min(1, W_sub / W_tree)
        w = -np.where(div[:, None], 0.0, H)
        wmax = w.max(axis=1)
        ew = np.exp(w - wmax[:, None])
        tot = ew.sum(axis=1)
        logw_sub = wmax + np.log(tot)
        cdf = np.cumsum(ew, axis=1)
        u = (rng.random(A) if uniforms is None else uniforms[level, 1][act]) * tot
        j = np.minimum((cdf < u[:, None]).sum(axis=1), n_new - 1)
        u_move = rng.random(A) if uniforms is None else uniforms[level, 2][act]
        move = u_move < np.exp(np.minimum(0.0, logw_sub - logw[act]))
        take = ok_sub & move
        sample[act[take]] = store.q[rows[take, j[take]]]
        logw[act] = np.where(ok_sub, np.logaddexp(logw[act], logw_sub), logw[act])
        # merge with the old tree: A is the earlier of (old tree, subtree) in time
        first_p, first_ps = P[:, 0], PS[:, 0]
        last_p, last_ps = P[:, -1], PS[:, -1]
        lp, lps = end_p[-1][act], end_ps[-1][act]   # old tree, left end
        rp, rps = end_p[+1][act], end_ps[+1][act]   # old tree, right end
        f = fwd[:, None]
        ok_m, rho_new = merge_check(
            np.where(f, rho[act], rho_sub), np.where(f, rho_sub, rho[act]),
            np.where(f, rp, last_p), np.where(f, lps, first_ps), np.where(f, rps, last_ps),
            np.where(f, first_p, lp), np.where(f, first_ps, lps), np.where(f, last_ps, rps))
        cont = ok_sub & ok_m
        rho[act] = np.where(cont[:, None], rho_new, rho[act])
        # the subtree's far end becomes the tree's end on its side
        for sgn, sel in ((+1, fwd), (-1, ~fwd)):
            idx = act[sel & ok_sub]
            src = (last_p, last_ps) if sgn > 0 else (first_p, first_ps)
            end_p[sgn][idx] = src[0][sel & ok_sub]
            end_ps[sgn][idx] = src[1][sel & ok_sub]
        active[act] = cont
    n_leap = leaves[+1].used + leaves[-1].used
    return sample, Stats(depth=depth, n_leapfrog=n_leap, divergent=divergent, energy=H0)


class DeviceTree:
    """The tree builder's walk on the device over a leaf store that the chain
    calls write into, so the trajectories never cross PCIe.  Gaussian
    targets, f64.  Three drivers:

    * "layout" (default): everything per transition is drawn and kept on the
      device -- momenta p0 = N(0, 1) / sqrt(inv_mass) and per-level uniforms
      from the Philox generator (`randomness`), the tree ends, depth and leaf
      counts -- and every chain's level-l leaves sit at fixed store rows.
      Each level is one start kernel, one batched chain call of 2^l steps for
      all chains and one level kernel; the whole transition is one library
      call (nxv_nuts_transition_layout), which reads one 4-byte flag per
      level (is any tree still growing).  With the same momenta and
      uniforms, nuts_transition takes the same decisions (the leaves are
      bit-identical: a chain restarted from a stored leaf continues exactly
      as the uninterrupted integration).
    * "levels": the same transition with this class issuing the per-level
      calls (nxv_nuts_start_layout, the batched chain call,
      nxv_nuts_level_layout) over torch tensors -- what a tree builder in
      another host language does with those entry points; its draws are
      bit-identical to "layout"'s.
    * "host": the host keeps the row bookkeeping of nuts_transition
      (speculative extension, as eXMC calls the chain) and draws from
      `rng` in its order; only the walk (nxv_nuts_start / _level) runs on
      the device."""

    MAX_DEPTH = 12  # leaves per level up to 2^11 (the level kernel's limit)

    def __init__(self, target: GaussianTarget, inv_mass, eps: float, driver: str = "layout",
                 seed: int = 0):
        import torch
        from nx_vulkan_b200 import _native
        from nx_vulkan_b200 import vulkan as nxv
        if driver not in ("layout", "levels", "host"):
            raise ValueError(f"driver must be 'layout', 'levels' or 'host', not {driver!r}")
        self.torch, self.nxv, self.lib = torch, nxv, _native.load()
        self.t, self.eps, self.driver = target, eps, driver
        self.m = np.ascontiguousarray(inv_mass, np.float64)
        self.dev = torch.device("cuda", torch.cuda.current_device())
        f64 = dict(dtype=torch.float64, device=self.dev)
        self.prec = torch.from_numpy(self.t.prec).to(self.dev)
        self.m_dev = torch.from_numpy(self.m).to(self.dev)
        self.sqrt_m = torch.sqrt(self.m_dev)
        self.f64 = f64
        self.cap = 0           # store rows
        self.node_cap = 0      # f64 scratch elements
        self.calls = []
        self.seed, self.count = seed & 0xFFFFFFFF, 0

    # -- device buffers -------------------------------------------------------------
    def _h(self, t, offset_elems=0, n_elems=None):
        """Non-owning handle over (part of) a torch tensor."""
        es = t.element_size()
        n = t.numel() - offset_elems if n_elems is None else n_elems
        h = self.lib.nxv_buf_wrap(self._ptr(t, offset_elems), n * es)
        if not h:
            raise RuntimeError("nxv_buf_wrap failed")
        return h

    @staticmethod
    def _ptr(t, offset_elems=0):
        import ctypes
        return ctypes.c_void_p(t.data_ptr() + offset_elems * t.element_size())

    def _call(self, fn, *args):
        rc = fn(*args)
        if rc != 0:
            raise RuntimeError(f"{fn.__name__} failed: {rc} {self.lib.nxv_last_error()}")

    def _reserve(self, rows: int, d: int):
        if rows <= self.cap:
            return
        torch = self.torch
        cap = max(rows, 2 * self.cap, 1 << 14)
        new = [torch.empty(cap * d, **self.f64), torch.empty(cap * d, **self.f64),
               torch.empty(cap, **self.f64), torch.empty(cap, **self.f64)]
        if self.cap:
            for a, b in zip(new, (self.st_q, self.st_p, self.st_logp, self.st_ke)):
                a[: b.numel()].copy_(b)
        self.st_q, self.st_p, self.st_logp, self.st_ke = new
        self.cap = cap

    def _free(self, *hs):
        for h in hs:
            self.lib.nxv_buf_free(h)

    @staticmethod
    def keys(seed: int):
        """Philox keys of a transition's momenta and of its uniforms."""
        return seed & 0xFFFFFFFF, (seed ^ 0x5BD1E995) & 0xFFFFFFFF

    def randomness(self, n_chains: int, seed: int, max_depth: int):
        """The layout driver's draws for one transition, on the device:
        p0 [C, d] = N(0, 1) / sqrt(inv_mass) (Philox normals, key keys(seed)[0],
        element c d + i) and uniforms [max_depth][3][C] (key keys(seed)[1]):
        per level the direction (forward when >= 0.5), the leaf and the move
        uniform of every chain."""
        torch = self.torch
        d = self.m.size
        z = torch.empty(n_chains * d, **self.f64)
        u = torch.empty(max_depth * 3 * n_chains, **self.f64)
        hz, hu = self._h(z), self._h(u)
        try:
            p0 = self._draw(n_chains, seed, max_depth, z, u, hz, hu)
        finally:
            self._free(hz, hu)
        return p0, u.view(max_depth, 3, n_chains)

    def transition(self, q0, rng=None, max_depth=10, seed=None):
        """One NUTS transition for every chain of q0 [C, d] (a torch CUDA
        tensor or an array); returns (q as a torch CUDA tensor, Stats).  The
        layout driver draws with Philox key `seed` (by default one integer
        from `rng`, or the tree's seed plus a transition count); the host
        driver draws from `rng`.  The library runs on torch's current stream
        during the call (the state tensors are torch's) and on its own stream
        again afterwards."""
        import ctypes
        if max_depth > self.MAX_DEPTH:
            raise ValueError(f"max_depth {max_depth} > {self.MAX_DEPTH}")
        s = self.torch.cuda.current_stream(self.dev).cuda_stream
        self.lib.nxv_set_stream(ctypes.c_void_p(s if s else 1))  # 1: the legacy default stream
        try:
            if self.driver == "host":
                return self._transition(q0, rng, max_depth)
            if seed is None:
                if rng is not None:
                    seed = int(rng.integers(1 << 32))
                else:
                    seed = (self.seed + self.count) & 0xFFFFFFFF
                    self.count += 1
            if self.driver == "layout":
                return self._transition_native(q0, seed, max_depth)
            return self._transition_layout(q0, seed, max_depth)
        finally:
            self.lib.nxv_set_stream(None)

    def _layout_state(self, C, d, max_depth):
        """Device buffers of the layout driver for C chains of dimension d and
        their library handles, made once and reused by every transition of
        that shape (the handles of the store's level ranges are kept until
        the store or the scratch grows)."""
        torch = self.torch
        st = getattr(self, "_state", None)
        if st is not None and st["shape"] == (C, d, max_depth):
            return st
        self._free_state()
        i32 = dict(dtype=torch.int32, device=self.dev)
        t = dict(
            q0=torch.empty(C, d, **self.f64), z=torch.empty(C * d, **self.f64),
            u=torch.empty(max_depth * 3 * C, **self.f64), H0=torch.empty(C, **self.f64),
            logw=torch.empty(C, **self.f64), sample=torch.empty(C, d, **self.f64),
            rho=torch.empty(C, d, **self.f64), ends_p=torch.empty(2, C, d, **self.f64),
            ends_ps=torch.empty(2, C, d, **self.f64), flags=torch.empty(4, C, **i32),
            end_row=torch.empty(2, C, dtype=torch.int64, device=self.dev),
            qs=torch.empty(C * d, **self.f64), ps=torch.empty(C * d, **self.f64))
        st = {"shape": (C, d, max_depth), "t": t, "levels": {}, "gen": None}
        fl = t["flags"]  # active, divergent, depth, n_leapfrog
        st["h"] = {k: self._h(v) for k, v in t.items() if k != "flags"}
        st["h"].update(active=self._h(fl[0]), div=self._h(fl[1]), depth=self._h(fl[2]),
                       leap=self._h(fl[3]), prec=self._h(self.prec), m=self._h(self.m_dev))
        self._state = st
        return st

    def _free_state(self):
        st = getattr(self, "_state", None)
        if st is not None:
            for hs in st["levels"].values():
                self._free(*hs)
            self._free(*st["h"].values())
            self._state = None
        nat = getattr(self, "_native", None)
        if nat is not None:
            self._free(*nat["h"].values())
            self._native = None

    def _native_state(self, C):
        """Output tensors of the one-call transition for C chains (flags and
        energies, with pinned host copies for one read per transition) and
        the handles of the target's rows (the library keeps the tree state
        and the leaf store in its own scratch)."""
        torch = self.torch
        nat = getattr(self, "_native", None)
        if nat is not None and nat["shape"] == C:
            return nat
        if nat is not None:
            self._free(*nat["h"].values())
        t = dict(flags=torch.empty(4, C, dtype=torch.int32, device=self.dev),
                 H0=torch.empty(C, **self.f64))
        h = {k: self._h(v) for k, v in t.items()}
        h.update(prec=self._h(self.prec), m=self._h(self.m_dev))
        host = dict(flags=torch.empty(4, C, dtype=torch.int32, pin_memory=True),
                    H0=torch.empty(C, dtype=torch.float64, pin_memory=True))
        self._native = {"shape": C, "t": t, "h": h, "host": host}
        return self._native

    def _transition_native(self, q0, seed, max_depth):
        torch, lib = self.torch, self.lib
        q0 = torch.as_tensor(q0, dtype=torch.float64, device=self.dev).contiguous()
        C, d = q0.shape
        nat = self._native_state(C)
        t, h, host = nat["t"], nat["h"], nat["host"]
        sample = torch.empty(C, d, **self.f64)
        # the caller's positions and the new draws are wrapped, not copied;
        # the library reads and writes them in this stream's order
        hq, hs = self._h(q0), self._h(sample)
        try:
            self._call(lib.nxv_nuts_transition_layout, hs, h["flags"], h["H0"], hq, h["m"],
                       h["prec"], self.t.mu, self.t.const, self.eps, C, d, max_depth,
                       seed & 0xFFFFFFFF)
        finally:
            self._free(hq, hs)
        host["flags"].copy_(t["flags"], non_blocking=True)
        host["H0"].copy_(t["H0"], non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        flags = host["flags"].numpy()  # active, divergent, depth, leaf count
        for level in range(int(flags[2].max())):
            self.calls.append((C, 1 << level))
        stats = Stats(depth=flags[2].astype(np.int64), n_leapfrog=flags[3].astype(np.int64),
                      divergent=flags[1].astype(bool), energy=host["H0"].numpy().copy())
        return sample, stats

    def __del__(self):
        try:
            self._free_state()
        except Exception:
            pass

    def _level_handles(self, st, level, C, d):
        """Handles of level `level`'s store rows and of the whole store (the
        level kernel reads the tree ends anywhere in it)."""
        n = 1 << level
        base = C * (n - 1)
        self._reserve(base + C * n, d)
        torch = self.torch
        if self.node_cap < C * n * d:
            self.node = torch.empty(C * n * d, **self.f64)
            self.grad_tmp = torch.empty(C * n * d, **self.f64)
            self.node_cap = C * n * d
        gen = (self.st_q.data_ptr(), self.node.data_ptr())
        if st["gen"] != gen:  # the store or the scratch moved: new handles
            for hs in st["levels"].values():
                self._free(*hs)
            st["levels"] = {}
            st["gen"] = gen
        hs = st["levels"].get(level)
        if hs is None:
            u = st["t"]["u"]
            hs = (self._h(u, level * 3 * C, 3 * C),
                  self._h(self.st_q), self._h(self.st_p), self._h(self.st_logp), self._h(self.st_ke),
                  self._h(self.node),
                  self._h(self.st_q, base * d, C * n * d), self._h(self.st_p, base * d, C * n * d),
                  self._h(self.grad_tmp, 0, C * n * d), self._h(self.st_logp, base, C * n),
                  self._h(self.st_ke, base, C * n))
            st["levels"][level] = hs
        return hs

    def _transition_layout(self, q0, seed, max_depth):
        torch, lib = self.torch, self.lib
        q0 = torch.as_tensor(q0, dtype=torch.float64).to(self.dev)
        C, d = q0.shape
        st = self._layout_state(C, d, max_depth)
        t, h = st["t"], st["h"]
        t["q0"].copy_(q0)
        p0 = self._draw(C, seed, max_depth, t["z"], t["u"], h["z"], h["u"])
        t["sample"].copy_(t["q0"])
        t["rho"].copy_(p0)
        t["ends_p"][0].copy_(p0)
        t["ends_p"][1].copy_(p0)
        torch.mul(t["ends_p"], self.m_dev, out=t["ends_ps"])
        fl = t["flags"]
        fl.zero_()
        fl[0].fill_(1)
        t["end_row"].fill_(-1)
        spv = self.nxv.shader_path("leapfrog_chain_gauss_f64_batched.spv")
        # p0 = z / sqrt(inv_mass) was written into z in place
        self._call(lib.nxv_nuts_energy, h["H0"], h["q0"], h["z"], h["prec"], h["m"], self.t.mu,
                   self.t.const, C, d)
        torch.neg(t["H0"], out=t["logw"])
        for level in range(max_depth):
            n = 1 << level
            base = C * (n - 1)
            hu, hsq, hsp, hsl, hsk, hnode, *outs = self._level_handles(st, level, C, d)
            self._call(lib.nxv_nuts_start_layout, h["qs"], h["ps"], h["q0"], h["z"], hsq, hsp,
                       h["end_row"], hu, C, d)
            self._call(lib.nxv_leapfrog_chain_gauss_f64_batched_ke, *outs, h["qs"], h["ps"], h["m"],
                       h["prec"], d, C, n, self.eps, self.t.mu, spv)
            self._call(lib.nxv_nuts_level_layout, base, n, d, hu, hsq, hsp, hsl, hsk, h["m"],
                       h["H0"], h["logw"], h["rho"], h["ends_p"], h["ends_ps"], h["sample"],
                       h["active"], h["div"], h["end_row"], h["depth"], h["leap"], hnode, C, level)
            self.calls.append((C, n))
            if level + 1 < max_depth and not bool(fl[0].any()):
                break
        flags = fl.cpu().numpy()  # one read: active, divergent, depth, leaf count
        stats = Stats(depth=flags[2].astype(np.int64), n_leapfrog=flags[3].astype(np.int64),
                      divergent=flags[1].astype(bool), energy=t["H0"].cpu().numpy())
        return t["sample"].clone(), stats

    def _draw(self, n_chains, seed, max_depth, z, u, hz, hu):
        """Fills z with p0 = N(0, 1) / sqrt(inv_mass) and u with the uniforms
        (the draws of `randomness`); returns z viewed as [C, d]."""
        d = self.m.size
        kp, ku = self.keys(seed)
        spv = self.nxv.shader_path("random_philox_f64.spv")
        self._call(self.lib.nxv_random_f64, hz, n_chains * d, kp, 1, spv)
        self._call(self.lib.nxv_random_f64, hu, max_depth * 3 * n_chains, ku, 0, spv)
        zv = z.view(n_chains, d)
        zv.div_(self.sqrt_m)
        return zv

    def _transition(self, q0, rng, max_depth):
        torch, lib = self.torch, self.lib
        q0 = torch.as_tensor(q0, dtype=torch.float64).to(self.dev).contiguous()
        C, d = q0.shape
        m = self.m
        p0_h = rng.standard_normal((C, d)) / np.sqrt(m)
        p0 = torch.from_numpy(p0_h).to(self.dev)
        H0 = torch.empty(C, **self.f64)
        hH0, hq0, hp0, hprec, hm = (self._h(x) for x in (H0, q0, p0, self.prec, self.m_dev))
        self._call(lib.nxv_nuts_energy, hH0, hq0, hp0, hprec, hm, self.t.mu, self.t.const, C, d)
        logw = -H0
        sample = q0.clone()
        rho = p0.clone()
        ends_p = torch.from_numpy(np.stack([p0_h, p0_h])).to(self.dev).contiguous()
        ends_ps = torch.from_numpy(np.stack([p0_h * m, p0_h * m])).to(self.dev).contiguous()
        active_d = torch.ones(C, dtype=torch.int32, device=self.dev)
        div_d = torch.zeros(C, dtype=torch.int32, device=self.dev)
        hlogw, hsample, hrho, hep, heps, hact, hdiv = (
            self._h(x) for x in (logw, sample, rho, ends_p, ends_ps, active_d, div_d))
        store = _Store(d)  # bookkeeping only: rows counted, data on the device
        leaves = {+1: _Leaves(store, C), -1: _Leaves(store, C)}
        active = np.ones(C, bool)
        depth = np.zeros(C, np.int64)
        grad_tmp = None
        for level in range(max_depth):
            if not active.any():
                break
            n_new = 1 << level
            dirs = np.where(rng.random(C) < 0.5, -1, 1)
            fwd_all = dirs > 0
            have = np.where(fwd_all, leaves[+1].have, leaves[-1].have)
            used = np.where(fwd_all, leaves[+1].used, leaves[-1].used)
            need = np.flatnonzero(active & (have < used + n_new))
            if need.size:
                K = speculative_steps(n_new)
                src = np.full(need.size, -1, np.int64)
                for sgn in (+1, -1):
                    L = leaves[sgn]
                    sel = (dirs[need] == sgn) & (L.have[need] > 0)
                    if sel.any():
                        src[sel] = L.last(need[sel])
                nn = need.size
                qs = torch.empty(nn * d, **self.f64)
                ps = torch.empty(nn * d, **self.f64)
                chain_t = torch.from_numpy(need.astype(np.int32)).to(self.dev)
                src_t = torch.from_numpy(src).to(self.dev)
                dir_t = torch.from_numpy(dirs[need].astype(np.int32)).to(self.dev)
                s0 = store.size
                self._reserve(s0 + nn * K, d)
                hs = [self._h(x) for x in (qs, ps, self.st_q, self.st_p, chain_t, src_t, dir_t)]
                self._call(lib.nxv_nuts_start, hs[0], hs[1], hq0, hp0, hs[2], hs[3], hs[4],
                           hs[5], hs[6], nn, C, d)
                if grad_tmp is None or grad_tmp.numel() < nn * K * d:
                    grad_tmp = torch.empty(nn * K * d, **self.f64)
                outs = [self._h(self.st_q, s0 * d, nn * K * d), self._h(self.st_p, s0 * d, nn * K * d),
                        self._h(grad_tmp, 0, nn * K * d), self._h(self.st_logp, s0, nn * K),
                        self._h(self.st_ke, s0, nn * K)]
                rc = lib.nxv_leapfrog_chain_gauss_f64_batched_ke(
                    *outs, hs[0], hs[1], hm, hprec, d, nn, K, self.eps, self.t.mu,
                    self.nxv.shader_path("leapfrog_chain_gauss_f64_batched.spv"))
                self._free(*hs, *outs)
                if rc != 0:
                    raise RuntimeError(f"chain call failed: {lib.nxv_last_error()}")
                store.size = s0 + nn * K
                starts = s0 + np.arange(nn) * K
                for sgn in (+1, -1):
                    sel = dirs[need] == sgn
                    if sel.any():
                        leaves[sgn].add_block(need[sel], starts[sel], K)
                self.calls.append((nn, K))
            act = np.flatnonzero(active)
            A = act.size
            fwd = dirs[act] > 0
            rows = np.empty((A, n_new), np.int64)
            for sgn, sel in ((+1, fwd), (-1, ~fwd)):
                if sel.any():
                    r_ = leaves[sgn].take(act[sel], n_new)
                    rows[sel] = r_ if sgn > 0 else r_[:, ::-1]  # backward leaves run leftward
            u_sel = rng.random(A)
            u_move = rng.random(A)
            depth[act] = level + 1
            if self.node_cap < A * n_new * d:
                self.node = torch.empty(A * n_new * d, **self.f64)
                self.node_cap = A * n_new * d
            lv = [torch.from_numpy(np.ascontiguousarray(rows)).to(self.dev),
                  torch.from_numpy(act.astype(np.int32)).to(self.dev),
                  torch.from_numpy(fwd.astype(np.int32)).to(self.dev),
                  torch.from_numpy(u_sel).to(self.dev), torch.from_numpy(u_move).to(self.dev)]
            hl = [self._h(x) for x in lv]
            hst = [self._h(x) for x in (self.st_q, self.st_p)]
            hst += [self._h(self.st_logp, 0, store.size), self._h(self.st_ke, 0, store.size)]
            hnode = self._h(self.node)
            rc = lib.nxv_nuts_level(*hl, A, n_new, d, *hst, hm, hH0, hlogw, hrho, hep, heps,
                                    hsample, hact, hdiv, hnode, C)
            self._free(*hl, *hst, hnode)
            if rc != 0:
                raise RuntimeError(f"nuts_level failed: {lib.nxv_last_error()}")
            # the only per-level transfer to the host: which trees keep growing
            active = active_d.cpu().numpy().astype(bool)
        stats = Stats(depth=depth, n_leapfrog=leaves[+1].used + leaves[-1].used,
                      divergent=div_d.cpu().numpy().astype(bool), energy=H0.cpu().numpy())
        self._free(hH0, hq0, hp0, hprec, hm, hlogw, hsample, hrho, hep, heps, hact, hdiv)
        return sample.view(C, d), stats
