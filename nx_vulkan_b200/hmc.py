"""Trajectory loop of an HMC sampler over the batched chain entry points.

eXMC's sampler calls the fused leapfrog chain once per trajectory, with fresh
momenta each time; the chain's output contract is the reference's
(PLAN_FUSED_LEAPFROG.md:294-322: per step q, p, grad and logp, with a
leading chain axis here).  This module restates that loop for the Bayesian
logistic-regression workload (256 chains, X[10000, 100], eps = 0.002,
L = 16 steps, 1000 trajectories) with every step on the device:

  * momenta p ~ N(0, I) from the Philox generator (`nxv_random_f64`): the
    key is seed + trajectory and the counter is the element index
    chain * n_dim + dim, so the draw for (chain, trajectory, dim) depends on
    those three numbers and the seed only;
  * the L leapfrog steps of every chain in one
    `nxv_leapfrog_logreg_f64_batched` call;
  * the last step's positions q_chain[:, L-1, :] become the next
    trajectory's start through one strided device copy (`nxv_buf_copy_2d`).

No Metropolis correction is applied (the throughput workload advances every
chain); each trajectory's per-step logp is returned, which with the returned
momenta is the energy a correction would need.
"""
from __future__ import annotations

from typing import Iterator, NamedTuple

from . import _native, vulkan as nxv


class Trajectory(NamedTuple):
    t: int                      # trajectory index
    q_start: nxv.VulkanTensor   # [chain][n_dim] positions the trajectory started from
    p_start: nxv.VulkanTensor   # [chain][n_dim] momenta drawn for it
    q_chain: nxv.VulkanTensor   # [chain][L][n_dim]
    p_chain: nxv.VulkanTensor
    grad_chain: nxv.VulkanTensor
    logp_chain: nxv.VulkanTensor  # [chain][L]


def momentum_key(seed: int, t: int) -> int:
    """Philox key of trajectory t's momenta."""
    return (seed + t) & 0xFFFFFFFF


def draw_momenta(n_chains: int, n_dim: int, seed: int, t: int):
    """p ~ N(0, I) [chain][n_dim] for trajectory t, on the device."""
    return nxv.random_f64(n_chains * n_dim, momentum_key(seed, t), 1)


def last_step(chain: nxv.VulkanTensor, n_chains: int, steps: int, n: int):
    """chain[:, steps - 1, :] of a [chain][steps][n] f64 trajectory, as a new
    [chain][n] device tensor (one strided device copy)."""
    out = nxv._alloc(n_chains * n * 8)
    if out is None:
        return (nxv.ERROR, "alloc_failed")
    row = n * 8
    rc = _native.load().nxv_buf_copy_2d(out.handle, 0, row, chain.handle, (steps - 1) * row,
                                        steps * row, row, n_chains)
    return nxv._dispatch([out], rc)


def logreg_trajectories(q0, X, y, n_obs: int, n_dim: int, n_chains: int, steps: int,
                        eps: float, trajectories: int, seed: int) -> Iterator[Trajectory]:
    """Runs `trajectories` HMC trajectories of the logistic-regression target
    from positions q0 ([chain][n_dim] device tensor), yielding each one's
    start, momenta and outputs.  Raises RuntimeError when a device call fails."""
    q = q0
    for t in range(trajectories):
        ok, p = draw_momenta(n_chains, n_dim, seed, t)
        if ok != nxv.OK:
            raise RuntimeError(f"momenta of trajectory {t}: {p} ({_native.last_error()})")
        ok, outs = nxv.leapfrog_logreg_f64_batched(q, p, X, y, n_obs, n_dim, n_chains, steps, eps)
        if ok != nxv.OK:
            raise RuntimeError(f"trajectory {t}: {outs} ({_native.last_error()})")
        yield Trajectory(t, q, p, *outs)
        ok, q_next = last_step(outs[0], n_chains, steps, n_dim)
        if ok != nxv.OK:
            raise RuntimeError(f"start of trajectory {t + 1}: {q_next} ({_native.last_error()})")
        q = q_next
