"""The oracle's batched Gaussian chain as a NUTS trajectory source (test
infrastructure: the CPU side of the GPU-vs-oracle NUTS comparison and of the
NUTS CPU timing; the product's source is nx_vulkan_b200.nuts.GpuChain).

Same interface as GpuChain: extend(q, p, K) returns the q and p trajectories
[chain][K][d], logp [chain][K] and the kinetic energy 0.5 * sum(p^2 m)
[chain][K] of K leapfrog steps from (q, p), computed by
oracle.c's restatement of the batched chain."""
from __future__ import annotations

import numpy as np

from . import binding as orc


class OracleChain:
    def __init__(self, target, inv_mass, eps: float):
        self.t, self.m, self.eps = target, np.asarray(inv_mass, np.float64), eps
        self.calls = []

    def extend(self, q, p, K):
        c, d = q.shape
        m = np.broadcast_to(self.m, (c, d)).copy()
        qc, pc, gc, lp = orc.chain_gauss_f64(q, p, m, self.t.prec, self.t.mu, d, c, K, self.eps)
        pc = pc.reshape(c, K, d)
        ke = 0.5 * ((pc * pc) * m[:, None, :]).sum(axis=-1)
        self.calls.append((c, K))
        return qc.reshape(c, K, d), pc, lp.reshape(c, K), ke
