#!/usr/bin/env python
"""Benchmark of the fused f64 HMC leapfrog chain (the hot path's headline).

Workload (one "step" = one call of the fused chain over one batch):
anisotropic Gaussian target, d = 1000, diagonal precision prec_i ~ U(0.5, 2)
(seed 3), 4096 independent chains per GPU, q0, p0 ~ N(0, 1), inv_mass = 1,
eps = 0.01, L = 32 leapfrog steps per trajectory, f64.  Outputs are the
reference contract's q/p/grad trajectories [chain][k][i] and logp [chain][k].

  value  chain-steps/s over all ranks, inputs resident in HBM: one CUDA
         event pair on the launching stream around all timed steps (and the
         collectives), three rotating input sets larger than L2 together.
  e2e    the same metric through the C ABI with host buffers: every step
         uploads q0/p0 [chain][d] and the shared inv_mass/prec rows [d] from
         pinned host memory, runs the chain
         and reads the step's result -- the per-step logp of every chain --
         back into pinned host memory (nxv_buf_upload/_download); the
         trajectories stay in their device buffers, as the reference API
         returns them.  Step i+1's upload runs on a copy stream while step i
         computes (nxv_set_stream, two input sets).  `e2e_serial` is the same
         without the overlap; `e2e_full_download` also brings the q/p/grad
         trajectories (3.2 GB per step) to the host: PCIe-bound.
  roofline  algorithmic bytes of one call / its measured duration, against
         the measured HBM copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the oracle (C restatement, OpenMP over all host cores) on a
         bounded sample of the same workload.

Multi-GPU (torchrun, one process per GPU): chains are independent, so each
rank integrates its own 4096 chains (weak scaling) and one NCCL all-gather
collects the per-chain diagnostics (final logp) each step.
`--impl reference` times the CPU restatement of the reference path instead.
`--workload logreg` runs the logistic-regression HMC workload (256 chains
split over the ranks, one trajectory with device-drawn momenta per step).
`--suite` times every other hot-path workload on one GPU.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

D, CHAINS, L, EPS = 1000, 4096, 32, 0.01
METRIC = "f64 leapfrog steps/s (chains×L)"
UNIT = "chain-steps/s"
# algorithmic bytes of one call: read q0, p0 (2*d*8 per chain), write the
# q/p/grad trajectories (3*L*d*8 per chain) and logp (L*8 per chain); the
# inverse mass (one [d] row shared by the chains) and prec are read once.
def algo_bytes(chains, d=D, steps=L):
    return chains * (2 * d * 8 + 3 * steps * d * 8 + steps * 8) + 2 * d * 8


def gauss_inputs(chains, d=D, seed=3):
    """prec [d], q0 and p0 [chains][d], inverse mass: one [d] row of ones
    shared by every chain (the workload's m = 1)."""
    r = np.random.default_rng(seed)
    prec = r.uniform(0.5, 2.0, d)
    q0 = r.normal(size=(chains, d))
    p0 = r.normal(size=(chains, d))
    return prec, q0, p0, np.ones(d)


def per_chain(m, chains):
    """The shared [d] inverse-mass row as the oracle's [chain][d] array."""
    return np.ascontiguousarray(np.broadcast_to(m, (chains, m.size)))


def max_over_ranks_ms(ms, dev, world):
    """A multi-rank step takes as long as its slowest rank."""
    if world == 1:
        return ms
    from nx_vulkan_b200.dist import max_over_ranks
    return max_over_ranks(ms, device=dev)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """SM clock and clock-event reasons sampled during the timed region.

    NVML (nvidia_ml_py) is read from a background thread every 2 ms -- the
    timed region can be a few milliseconds, shorter than nvidia-smi's
    sampling interval -- with one sample on entry and one on exit.  Without
    NVML, nvidia-smi -lms 200 is the fallback.  Read-only: no setting of the
    GPU is changed."""

    # NVML clocks-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.nvml = None
        self.samples = []  # (sm_mhz, reason bits)
        self.smax = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"nxv_clocks_{os.getpid()}.csv"

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:  # the CUDA device's own GPU, whatever CUDA_VISIBLE_DEVICES maps
            import torch
            u = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + u).encode())
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _sample(self):
        nv, h = self.nvml
        clk = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        try:
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        except AttributeError:
            rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
        self.samples.append((float(clk), int(rs)))

    def __enter__(self):
        import threading
        try:
            self.nvml = self._nvml_handle()
            nv, h = self.nvml
            self.smax = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._sample()
            self.stop = threading.Event()

            def run():
                while not self.stop.wait(0.002):
                    self._sample()

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.nvml:
            self.stop.set()
            self.thread.join()
            self._sample()
            return
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def mark(self):
        """Index of the next sample: summary(mark) covers what follows it."""
        return len(self.samples)

    def summary(self, start=0):
        if self.nvml:
            smp = self.samples[start:]
            sm = [c for c, _ in smp]
            reasons = sorted({nm for _, r in smp for nm, bit in self.REASONS.items() if r & bit})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.smax,
                    "reasons": reasons, "samples": len(sm), "source": "NVML every 2 ms"}
        if not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi -lms 200"}


def host_threads():
    """Every core this process may run on (torchrun sets OMP_NUM_THREADS=1
    for its workers, so the OpenMP default would be a single thread)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(seconds_min=10.0, seconds_max=30.0, chains=256):
    """Oracle (C restatement, all host threads) on a bounded sample."""
    from oracle import binding as orc
    nthreads = host_threads()
    prec, q0, p0, m = gauss_inputs(chains)
    m = per_chain(m, chains)
    done, t0 = 0, time.perf_counter()
    while True:
        orc.chain_gauss_f64(q0, p0, m, prec, 0.0, D, chains, L, EPS, nthreads=nthreads)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds_min or (el * (done + 1) / done) > seconds_max:
            break
    rate = done * chains * L / el
    return {"value": rate, "unit": UNIT, "cores": nthreads, "kind": "port",
            "sample": f"{done} x {chains} chains x L={L} x d={D} (f64), {el:.1f} s, "
                      f"oracle C restatement with OpenMP; nproc={os.cpu_count()}"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    per_step = []
    from oracle import binding as orc
    nthreads = host_threads()
    chains = args.chains  # the GPU arm's per-GPU batch: the same workload per step
    prec, q0, p0, m = gauss_inputs(chains)
    m = per_chain(m, chains)
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        orc.chain_gauss_f64(q0, p0, m, prec, 0.0, D, chains, L, EPS, nthreads=nthreads)
        if i >= args.warmup:
            per_step.append(time.perf_counter() - t0)
    t = sum(per_step)
    value = args.steps * chains * L / t
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded numpy: prec~U(0.5,2) seed 3, q0,p0~N(0,1))",
        "config": {"workload": "anisotropic Gaussian HMC leapfrog (reference path restated on CPU)",
                   "chains": chains, "d": D, "L": L, "eps": EPS},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": f"{chains} chains x L={L} x d={D} per step (the GPU arm's "
                                   f"per-GPU batch); the reference's "
                                   "Vulkan/Elixir stack cannot run here, so its CPU path is the "
                                   "oracle's C restatement of Nx.BinaryBackend semantics"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--chains", type=int, default=CHAINS)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--diag-every", type=int, default=1,
                    help="N > 1: steps whose final logps go out in one all-gather (default: every step)")
    ap.add_argument("--diag-depth", type=int, default=4,
                    help="N > 1: diagnostics buffers in flight (collective of step i waited for at step i + depth)")
    ap.add_argument("--workload", default="gauss", choices=["gauss", "logreg", "reduce"],
                    help="gauss: the headline anisotropic-Gaussian chain; logreg: the "
                         "logistic-regression HMC workload (256 chains over all ranks, "
                         "X[10000,100], L=16, eps=0.002, momenta drawn on the device); "
                         "reduce: the [4096,4096] row reductions, argmax and full sum "
                         "sharded by rows over the ranks, results all-gathered on the device")
    ap.add_argument("--lr-chains", type=int, default=256,
                    help="logistic workload: chains over all ranks (the workload's 256 by default)")
    ap.add_argument("--repeats", type=int, default=5,
                    help="timed regions of --steps steps each; value is their median")
    ap.add_argument("--suite", action="store_true",
                    help="measure every hot-path workload (one JSON line each) instead of the headline")
    ap.add_argument("--only", default="fused,reduce,random,misc,matmul,logreg,nuts",
                    help="suite sections to run, comma separated: fused, reduce, random, misc "
                         "(transpose, cast, logsumexp, HMC primitives, host transfers), matmul, "
                         "logreg, nuts")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.suite:
        return suite(args)
    if args.workload == "logreg":
        return logreg_main(args, rank, world, local)
    if args.workload == "reduce":
        return reduce_main(args, rank, world, local)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # The only collective is a 32 KB-per-rank diagnostics all-gather per
        # step: latency-bound, so the low-latency protocol on two channels
        # (measured on 2 B200s: 0.532 ms/step with NCCL defaults, 0.512 with
        # these, 0.506 without any collective).  User settings win.
        os.environ.setdefault("NCCL_PROTO", "LL")
        os.environ.setdefault("NCCL_MAX_NCHANNELS", "2")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from nx_vulkan_b200 import _native, vulkan as nxv
    lib = _native.load()
    assert nxv.init_devices([local]) == "ok", _native.last_error()
    # A dedicated stream: the library and the CUDA events must share it
    # (torch's default stream has handle 0, which the ABI reads as "library
    # stream").
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    lib.nxv_set_stream(C.c_void_p(stream.cuda_stream))

    chains = args.chains
    prec, q0, p0, m = gauss_inputs(chains, seed=3 + 1000 * rank)
    # Three copies of the inputs (3 x 98 MB > 2x L2) rotate between steps, so
    # no step finds its inputs in L2; the 3.2 GB of trajectory writes per step
    # never fit either.
    n_sets = 3
    in_sets = []
    for s in range(n_sets):
        ts = [torch.from_numpy(a).to(dev) for a in (q0, p0, m)] + [torch.from_numpy(prec).to(dev)]
        in_sets.append(ts)
    outs = [torch.empty(chains * L * D, dtype=torch.float64, device=dev) for _ in range(3)]
    outs.append(torch.empty(chains * L, dtype=torch.float64, device=dev))
    wrap = lambda t: lib.nxv_buf_wrap(C.c_void_p(t.data_ptr()), t.numel() * t.element_size())
    h_sets = [[wrap(t) for t in ts] for ts in in_sets]
    h_in = h_sets[0]
    h_out = [wrap(t) for t in outs]
    spv = nxv.shader_path("leapfrog_chain_gauss_f64_batched.spv")

    def step(i=0):
        rc = lib.nxv_leapfrog_chain_gauss_f64_batched(*h_out, *h_sets[i % n_sets], D, chains, L,
                                                      EPS, 0.0, spv)
        if rc != 0:
            raise RuntimeError(f"leapfrog failed: {rc} {_native.last_error()}")

    # Diagnostics exchange: the final-step logp of every chain, all-gathered
    # on a side stream so that the collective overlaps the next steps.  The
    # logps of `every` consecutive steps go out in one collective (every x
    # chains values per rank; the last group of a run is flushed even when
    # short).  `depth` buffers rotate; before buffer b is refilled the main
    # stream waits for the collective that read it `depth` groups earlier.
    depth = max(2, args.diag_depth)
    every = max(1, args.diag_every)
    diags = [torch.empty(world * every * chains, dtype=torch.float64, device=dev) for _ in range(depth)]
    lasts = [torch.empty(every * chains, dtype=torch.float64, device=dev) for _ in range(depth)]
    side_done = [None] * depth
    # High priority: the collective's CTAs are dispatched ahead of the chain
    # kernel's pending CTAs (a 4096-CTA grid), so it runs during the next
    # step instead of after that step's last wave.
    side = torch.cuda.Stream(device=dev, priority=-1)

    def diagnostics(i, final=False):
        if world == 1:
            return
        b, j = (i // every) % depth, i % every
        if j == 0 and side_done[b] is not None:
            stream.wait_event(side_done[b])
        lasts[b][j * chains:(j + 1) * chains].copy_(outs[3].view(chains, L)[:, -1])
        if j == every - 1 or final:
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                dist.all_gather_into_tensor(diags[b], lasts[b])
            side_done[b] = side.record_event()

    for i in range(args.warmup):
        step(i)
        diagnostics(i, final=i == args.warmup - 1)
    stream.wait_stream(side)
    torch.cuda.synchronize()
    repeats = max(1, args.repeats)
    groups = (args.steps + every - 1) // every
    n_launch0 = lib.nxv_launch_count()
    t0_ev, t1_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # per-step events around the chain call alone (no collective), in the
    # same timed loop: the roofline's launch time
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    rep_ms, rep_clocks, k_all = [], [], []
    # The clock sampler starts (NVML initialisation takes milliseconds, and
    # differently on every rank) before the barrier, so that the ranks leave
    # the barrier together and start their timed steps at the same moment.
    with Clocks(local) as clk:
        for rep in range(repeats):
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            mark = clk.mark()
            t0_ev.record(stream)
            for i in range(args.steps):
                kev[i][0].record(stream)
                step(rep * args.steps + i)
                kev[i][1].record(stream)
                # groups of `every` steps restart with each repeat
                diagnostics(rep * groups * every + i, final=i == args.steps - 1)
            stream.wait_stream(side)  # the final collective is inside the timed region
            t1_ev.record(stream)
            torch.cuda.synchronize()
            rep_clocks.append(clk.summary(mark))
            rep_ms.append(max_over_ranks_ms(t0_ev.elapsed_time(t1_ev), dev, world))
            k_all += [a.elapsed_time(b) for a, b in kev]
    if world > 1:
        dist.barrier()
    launches = (lib.nxv_launch_count() - n_launch0) // (args.steps * repeats) * args.steps
    t_ms = statistics.median(rep_ms)
    value = world * chains * L * args.steps / (t_ms / 1e3)
    rep_values = [world * chains * L * args.steps / (ms / 1e3) for ms in rep_ms]
    clocks = clk.summary()
    clocks["per_repeat"] = [{"sm_mhz": c.get("sm_mhz"), "reasons": c.get("reasons"),
                             "samples": c.get("samples")} for c in rep_clocks]
    # Roofline of the dominant kernel: the chain call (chain kernel + the
    # tiny constant kernel), median over every timed step of every repeat.
    k_ms = statistics.median(k_all)
    # per-rank view of a multi-GPU run: step time, the kernel alone, SM clock
    ranks_info = None
    if world > 1:
        loc = torch.tensor([t0_ev.elapsed_time(t1_ev) / args.steps, k_ms,
                            float(clocks.get("sm_mhz") or 0.0), float(len(clocks.get("reasons") or []))],
                           dtype=torch.float64, device=dev)
        allr = torch.empty(world * 4, dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(allr, loc)
        rows = allr.view(world, 4).cpu().tolist()
        ranks_info = {"step_ms": [r[0] for r in rows], "kernel_alone_ms": [r[1] for r in rows],
                      "sm_mhz": [r[2] for r in rows], "clock_event_reasons": [int(r[3]) for r in rows]}
    peak, peak_kind = peaks()
    abytes = algo_bytes(chains)
    achieved = abytes / (k_ms / 1e3) / 1e9
    # dram__bytes_read.sum + dram__bytes_write.sum of one k_chain_tma launch
    # over 1024 chains (24,633,856 + 729,063,680 B), scaled by chains; the
    # writes of that capture miss the dirty lines still in L2 at kernel end,
    # so this is a lower bound of the full launch's traffic.
    traffic = (24633856 + 729063680) / 1024 * chains if (D, L) == (1000, 32) else None

    # e2e through the C ABI with host buffers (library-owned device buffers).
    e2e = e2e_full = e2e_serial = None
    if not args.no_e2e:
        lib.nxv_set_stream(None)
        hb_in = [torch.from_numpy(a.reshape(-1)).pin_memory() for a in (q0, p0, m, prec)]
        hb_out = [torch.empty(o.numel(), dtype=torch.float64).pin_memory() for o in outs]
        d_in = [lib.nxv_buf_alloc(t.numel() * 8) for t in hb_in]
        d_out = [lib.nxv_buf_alloc(t.numel() * 8) for t in hb_out]

        def e2e_step(full):
            for h, t in zip(d_in, hb_in):
                assert lib.nxv_buf_upload(h, C.c_void_p(t.data_ptr()), t.numel() * 8) == 0
            rc = lib.nxv_leapfrog_chain_gauss_f64_batched(*d_out, *d_in, D, chains, L, EPS, 0.0, spv)
            assert rc == 0, _native.last_error()
            pairs = list(zip(d_out, hb_out)) if full else [(d_out[3], hb_out[3])]  # [3] = logp
            for h, t in pairs:
                assert lib.nxv_buf_download(h, C.c_void_p(t.data_ptr()), t.numel() * 8) == 0

        def e2e_run(full):
            for _ in range(2):
                e2e_step(full)
            n_e2e = max(3, min(args.steps, 5)) if full else max(5, args.steps)
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            for _ in range(n_e2e):
                e2e_step(full)
            el = time.perf_counter() - t0
            el_t = torch.tensor([el], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(el_t, op=dist.ReduceOp.MAX)
            el = float(el_t.item())
            down = hb_out if full else [hb_out[3]]
            return {"value": world * chains * L * n_e2e / el, "unit": UNIT,
                    "h2d_bytes_per_step": sum(t.numel() * 8 for t in hb_in),
                    "d2h_bytes_per_step": sum(t.numel() * 8 for t in down),
                    "steps": n_e2e,
                    "timing": "host wall clock around synchronous C-ABI calls, max over ranks"}

        # Pipelined through the same public calls: step i+1's inputs upload on a
        # copy stream (nxv_set_stream) while step i runs on a compute stream,
        # two device input sets alternating, events ordering the two streams.
        s_copy, s_comp = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        d_sets = [d_in, [lib.nxv_buf_alloc(t.numel() * 8) for t in hb_in]]
        up_ev = [torch.cuda.Event(), torch.cuda.Event()]
        used_ev = [torch.cuda.Event(), torch.cuda.Event()]

        def p_upload(i):
            b = i % 2
            s_copy.wait_event(used_ev[b])  # the chain of step i-2 read this set
            lib.nxv_set_stream(C.c_void_p(s_copy.cuda_stream))
            for h, t in zip(d_sets[b], hb_in):
                assert lib.nxv_buf_upload(h, C.c_void_p(t.data_ptr()), t.numel() * 8) == 0
            up_ev[b].record(s_copy)

        def p_launch(i):
            b = i % 2
            s_comp.wait_event(up_ev[b])
            lib.nxv_set_stream(C.c_void_p(s_comp.cuda_stream))
            rc = lib.nxv_leapfrog_chain_gauss_f64_batched(*d_out, *d_sets[b], D, chains, L, EPS, 0.0, spv)
            assert rc == 0, _native.last_error()
            used_ev[b].record(s_comp)

        def p_result(i):
            # the step's result to the host (waits for the chain)
            lib.nxv_set_stream(C.c_void_p(s_comp.cuda_stream))
            assert lib.nxv_buf_download(d_out[3], C.c_void_p(hb_out[3].data_ptr()), hb_out[3].numel() * 8) == 0

        def e2e_pipelined():
            n_e2e = max(5, args.steps)

            def run(n):
                # nxv_buf_upload returns once the copy is done (the caller may
                # reuse its buffer), so step i is launched first and step
                # i+1's upload runs while it computes
                p_upload(0)
                for i in range(n):
                    p_launch(i)
                    if i + 1 < n:
                        p_upload(i + 1)
                    p_result(i)

            run(3)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            run(n_e2e)
            el = time.perf_counter() - t0
            el_t = torch.tensor([el], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(el_t, op=dist.ReduceOp.MAX)
            el = float(el_t.item())
            h2d = sum(t.numel() * 8 for t in hb_in)
            return {"value": world * chains * L * n_e2e / el, "unit": UNIT,
                    "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": hb_out[3].numel() * 8, "steps": n_e2e,
                    "h2d_gbs_per_rank": h2d * n_e2e / el / 1e9,
                    "timing": "host wall clock from the first upload to the last result, max over ranks",
                    "result_read": "per-step logp [chain][k] (the metric); trajectories stay on the device",
                    "pipelined": "inputs of step i+1 upload on a copy stream while step i computes"}

        e2e_serial = e2e_run(False)
        e2e_serial["result_read"] = "per-step logp [chain][k] (the metric); trajectories stay on the device"
        e2e = e2e_pipelined()
        e2e_full = e2e_run(True)
        e2e_full["result_read"] = "all four outputs: q/p/grad trajectories and logp"
        torch.cuda.synchronize()
        for h in d_sets[0] + d_sets[1] + d_out:
            lib.nxv_buf_free(h)
        lib.nxv_set_stream(C.c_void_p(stream.cuda_stream))

    secondary = None
    if not args.no_secondary and rank == 0:
        secondary = fused_elementwise_gbs(lib, nxv, torch, dev, stream, peak)

    cpu = None
    if rank == 0 and not args.no_cpu:
        cpu = cpu_sample()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded numpy: prec~U(0.5,2) seed 3, q0,p0~N(0,1); rank r uses seed 3+1000r)",
            "config": {"workload": "anisotropic Gaussian HMC leapfrog, fused K-step chain",
                       "chains_per_gpu": chains, "d": D, "L": L, "eps": EPS,
                       "inv_mass": "1.0, one [d] row shared by the chains",
                       "parallelism": f"chains sharded, {world} rank(s), NCCL all-gather of every chain's "
                                      f"final-step logp, {every} step(s) per collective, on a high-priority "
                                      f"side stream, waited for {depth} collectives later "
                                      f"(NCCL_PROTO={os.environ.get('NCCL_PROTO')})"
                       if world > 1 else "1 GPU",
                       "l2": "inputs larger than L2: 3 rotating input sets of 66 MB (197 MB > 126 MB); "
                             "3.15 GB of trajectory writes per step",
                       "timing": f"{repeats} timed regions of {args.steps} steps, each one CUDA event "
                                 "pair on the launching stream around its steps, collectives included, "
                                 "max over ranks; value is the median region"},
            "repeats": {"n": repeats, "values": rep_values, "ms_per_step": [ms / args.steps for ms in rep_ms],
                        "spread": (max(rep_values) - min(rep_values)) / statistics.median(rep_values)},
            "gpu_launches": int(launches),
            **({"ranks": ranks_info} if ranks_info else {}),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "traffic_source": "a constant, not measured in this run: ncu "
                                           "dram__bytes_read.sum + dram__bytes_write.sum of one "
                                           "1024-chain launch, scaled by chains (lower bound: "
                                           "writes still dirty in L2 at kernel end are uncounted)",
                         "algorithmic_bytes_per_launch": abytes, "launch_ms": k_ms,
                         "launch_timing": "median of per-call CUDA events inside the timed loop",
                         "kernel": "k_chain_tma (TMA bulk stores, 2 steps per copy) + k_gauss_const",
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json), copy, of measured"},
            "clocks": clocks,
            "e2e": e2e,
            "e2e_serial": e2e_serial,
            "e2e_full_download": e2e_full,
            "cpu_baseline": cpu,
        }
        if secondary:
            line["secondary"] = secondary
        print(json.dumps(line), flush=True)
    for h in [h for hs in h_sets for h in hs] + h_out:
        lib.nxv_buf_free(h)
    lib.nxv_set_stream(None)
    if world > 1:
        dist.destroy_process_group()


LR_OBS, LR_DIM, LR_CHAINS, LR_STEPS, LR_EPS = 10000, 100, 256, 16, 0.002


def logreg_data():
    """X [10000, 100] ~ N(0, 1), w* ~ N(0, 1), y ~ Bernoulli(sigmoid(X w*)), seed 4."""
    r = np.random.default_rng(4)
    X = r.normal(size=(LR_OBS, LR_DIM))
    w = r.normal(size=LR_DIM)
    y = (r.random(LR_OBS) < 1 / (1 + np.exp(-X @ w))).astype(np.float64)
    return X, y


def dgemm_peak_tflops(torch, dev, n=4096, reps=10):
    """cuBLAS DGEMM (torch.matmul f64, n^3) in this process: the FP64 tensor
    peak the logistic gradient is held against (no FP64 figure is in the
    measured-peaks file)."""
    a = torch.randn(n, n, dtype=torch.float64, device=dev)
    b = torch.randn(n, n, dtype=torch.float64, device=dev)
    torch.matmul(a, b)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = None
    for _ in range(reps):
        e0.record()
        torch.matmul(a, b)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


def logreg_main(args, rank, world, local):
    """The logistic-regression HMC workload: 256 chains split over the ranks
    (contiguous blocks), X and y replicated, one step = one trajectory of
    L = 16 leapfrog steps with fresh momenta drawn on the device (Philox key
    seed + trajectory, counter chain * 100 + dim over the global chain
    index), the last positions carried to the next trajectory on the device,
    and an all-gather of every chain's final logp per trajectory (N > 1)."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_PROTO", "LL")
        os.environ.setdefault("NCCL_MAX_NCHANNELS", "2")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from nx_vulkan_b200 import _native, hmc, vulkan as nxv
    lib = _native.load()
    assert nxv.init_devices([local]) == "ok", _native.last_error()
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    lib.nxv_set_stream(C.c_void_p(stream.cuda_stream))
    total = args.lr_chains
    assert total % world == 0, "the chains split evenly over the ranks"
    lo, hi = rank * total // world, (rank + 1) * total // world
    cr = hi - lo
    X, y = logreg_data()
    ok, tX = nxv.upload_binary(X)
    ok2, ty = nxv.upload_binary(y)
    ok3, q0 = nxv.upload_binary(np.zeros((cr, LR_DIM)))
    assert ok == ok2 == ok3 == "ok"
    seed = 7
    lps = torch.empty(cr, dtype=torch.float64, device=dev)
    gathered = torch.empty(total, dtype=torch.float64, device=dev) if world > 1 else None
    h_lps = lib.nxv_buf_wrap(C.c_void_p(lps.data_ptr()), cr * 8)
    spv = nxv.shader_path("leapfrog_logreg_f64_batched.spv")
    # this rank's momenta: the rows [lo, hi) of the global [256][100] draw
    def momenta(t):
        ok, p = nxv.random_f64(total * LR_DIM, hmc.momentum_key(seed, t), 1)
        assert ok == "ok", _native.last_error()
        if world == 1:
            return p
        mine = nxv._alloc(cr * LR_DIM * 8)
        assert lib.nxv_buf_copy_2d(mine.handle, 0, cr * LR_DIM * 8, p.handle, lo * LR_DIM * 8,
                                   cr * LR_DIM * 8, cr * LR_DIM * 8, 1) == 0
        return mine

    state = {"q": q0, "t": 0}

    def trajectory():
        t = state["t"]
        p = momenta(t)
        ok, outs = nxv.leapfrog_logreg_f64_batched(state["q"], p, tX, ty, LR_OBS, LR_DIM, cr,
                                                   LR_STEPS, LR_EPS)
        assert ok == "ok", _native.last_error()
        ok, qn = hmc.last_step(outs[0], cr, LR_STEPS, LR_DIM)
        assert ok == "ok", _native.last_error()
        state["q"], state["t"] = qn, t + 1
        if world > 1:  # every chain's final logp: logp[:, L-1] to lps, then all-gathered
            assert lib.nxv_buf_copy_2d(h_lps, 0, 8, outs[3].handle, 8 * (LR_STEPS - 1),
                                       8 * LR_STEPS, 8, cr) == 0
            dist.all_gather_into_tensor(gathered, lps)

    for _ in range(args.warmup):
        trajectory()
    torch.cuda.synchronize()
    repeats = max(1, args.repeats)
    rep_ms = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_launch0 = lib.nxv_launch_count()
    with Clocks(local) as clk:
        for _ in range(repeats):
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(args.steps):
                trajectory()
            e1.record(stream)
            torch.cuda.synchronize()
            rep_ms.append(max_over_ranks_ms(e0.elapsed_time(e1), dev, world))
    launches = (lib.nxv_launch_count() - n_launch0) // repeats
    t_ms = statistics.median(rep_ms)
    value = total * LR_STEPS * args.steps / (t_ms / 1e3)
    peak = dgemm_peak_tflops(torch, dev) if rank == 0 else None
    flops = (LR_STEPS + 1) * 2 * 2 * cr * LR_DIM * LR_OBS  # per trajectory, this rank
    achieved = flops / (t_ms / args.steps / 1e3) / 1e12
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "f64 logistic-regression leapfrog steps/s (chains×L)", "value": value,
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_ms / args.steps, "higher_is_better": True,
            "scaling": f"strong ({total} chains in total)", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded numpy: X~N(0,1) [10000,100], w*~N(0,1), y~Bernoulli, seed 4; "
                    "q0=0; momenta from the device Philox generator)",
            "config": {"workload": "Bayesian logistic-regression HMC, one trajectory per step",
                       "chains_total": total, "chains_per_gpu": cr, "n_obs": LR_OBS,
                       "d": LR_DIM, "L": LR_STEPS, "eps": LR_EPS,
                       "timing": f"{repeats} timed regions of {args.steps} trajectories (CUDA events "
                                 "on the launching stream, max over ranks); value is the median"},
            "repeats": {"n": repeats, "ms_per_step": [ms / args.steps for ms in rep_ms]},
            "gpu_launches_per_region": int(launches),
            "roofline": {"bound": "fp64 tensor (DMMA)", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak if peak else None,
                         "flops_per_step_per_gpu": flops,
                         "peak_source": "cuBLAS DGEMM 4096^3 measured in this run (rank 0)",
                         "note": "the step's whole time, momenta draws and carries included"},
            "clocks": clk.summary(),
        }), flush=True)


def reduce_main(args, rank, world, local):
    """The reductions workload sharded by rows: x f32 and f64 [4096, 4096]
    ~ N(0, 1) (seed 1), rank r holding rows chain_shard(4096, r, N) on its
    GPU.  One step = sum over axis 1, max over axis 1, argmax over axis 1
    (each rank's rows into device tensors, all-gathered device to device in
    row order) and the full sum (rank partials all-gathered and folded in
    rank order), for f32 and f64.  Strong scaling: the matrix is fixed."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from nx_vulkan_b200 import _native, dist as nd, vulkan as nxv
    lib = _native.load()
    assert nxv.init_devices([local]) == "ok", _native.last_error()
    rows = cols = 4096
    sh = nd.chain_shard(rows, rank, world)
    x64 = np.random.default_rng(1).normal(size=(rows, cols))
    bufs = {}
    for name, dt in (("f64", np.float64), ("f32", np.float32)):
        ok, t = nxv.upload_binary(np.ascontiguousarray(x64[sh.start:sh.stop].astype(dt)))
        assert ok == "ok"
        bufs[name] = t

    def step():
        res = []
        for name, t in bufs.items():
            res.append(nd.reduce_rows(nxv, t, sh.count, cols, 0, dtype=name))
            res.append(nd.reduce_rows(nxv, t, sh.count, cols, 1, dtype=name))
            res.append(nd.argmax_rows(nxv, t, sh.count, cols, dtype=name))
            res.append(nd.reduce_full(nxv, t, 0, name))
        return res

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    rep_ms = []
    for _ in range(max(1, args.repeats)):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        rep_ms.append(max_over_ranks_ms((time.perf_counter() - t0) * 1e3, dev, world))
    t_ms = statistics.median(rep_ms) / args.steps
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        nbytes = 3 * rows * cols * (4 + 8) + rows * cols * (4 + 8)  # each op reads the matrix
        print(json.dumps({
            "metric": "sharded [4096,4096] reductions: ms per step (sum/max/argmax over axis 1 + "
                      "full sum, f32 and f64)", "value": t_ms, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "scaling": "strong", "dtype": "f32+f64", "data": "synthetic N(0,1) seed 1",
            "algorithmic_gbs": nbytes / (t_ms / 1e3) / 1e9,
            "config": {"workload": "row-sharded reductions with device all-gathers",
                       "rows_per_gpu": sh.count,
                       "timing": "host wall clock around the steps (each op waits for its kernel "
                                 "before its collective), median of repeats, max over ranks"},
            "repeats_ms_per_step": [ms / args.steps for ms in rep_ms],
        }), flush=True)


def fused_elementwise_gbs(lib, nxv, torch, dev, stream, peak):
    """tanh(exp(x*y + z) - 1.0) on f32/f64[1,048,576] (x,y,z ~ U(-1,1), seed 0), one
    fused kernel per call, rotating over buffer sets totalling > 2x L2."""
    res = {}
    n = 1 << 20
    for dt, name, code in ((torch.float32, "f32", 0), (torch.float64, "f64", 1)):
        es = 4 if code == 0 else 8
        sets = max(4, (512 << 20) // (4 * n * es))
        g = torch.Generator(device="cpu").manual_seed(0)
        bufs = []
        for s in range(sets):
            xs = [(torch.rand(n, generator=g, dtype=torch.float64) * 2 - 1).to(dt).to(dev) for _ in range(3)]
            out = torch.empty(n, dtype=dt, device=dev)
            hs = [lib.nxv_buf_wrap(C.c_void_p(t.data_ptr()), n * es) for t in xs + [out]]
            bufs.append((xs, out, hs))
        ops = (C.c_uint * 8)(1, 0, 100, 2, 106, 255, 255, 255)
        src = (C.c_uint * 8)(1, 2, 1, 0, 1, 1, 1, 1)
        imm = (C.c_double * 8)(0, 0, 0, 1.0, 0, 0, 0, 0)
        spv = nxv.shader_path("fused_elementwise_imm.spv")

        def call(s):
            _, _, hs = bufs[s % sets]
            rc = lib.nxv_fused_chain_imm(hs[3], hs[0], hs[1], hs[2], None, n, 5, ops, src, imm, code, spv)
            assert rc == 0

        # The C-ABI call costs a few microseconds of host time, more than the
        # 16 MB kernel itself, so the launch sequence is captured once in a
        # CUDA graph and replayed: the events then time the GPU only.
        modes = [("fast", "0")] + ([("exact", "1")] if code == 0 else [])
        for mode, env in modes:
            os.environ["NXV_EXACT_F32"] = env
            for s in range(sets):
                call(s)
            reps = 8 * sets
            graph = torch.cuda.CUDAGraph()
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=stream):
                for s in range(reps):
                    call(s)
            graph.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record(stream)
            for _ in range(3):
                graph.replay()
            b.record(stream)
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / (3 * reps)
            del graph
            gbs = 4 * n * es / (ms / 1e3) / 1e9
            key = f"fused_elementwise_{name}" + ("" if mode == "fast" else "_exact_math")
            res[key] = {
                "metric": "fused-elementwise HBM GB/s", "value": gbs, "unit": "GB/s",
                "frac_of_hbm": gbs / peak, "us_per_call": ms * 1e3,
                "bytes_per_call": 4 * n * es,
                "f32_math": mode if code == 0 else "f64",
                "config": f"tanh(exp(x*y+z)-1.0), {name}[1048576], {sets} rotating buffer sets "
                          f"({sets * 4 * n * es >> 20} MiB > 2x L2), {reps} launches in one CUDA graph"}
        os.environ.pop("NXV_EXACT_F32", None)
        for _, _, hs in bufs:
            for h in hs:
                lib.nxv_buf_free(h)
    return res


def suite(args):
    """Every hot-path workload on GPU 0, one JSON line each.  Launch
    sequences are captured in a CUDA graph (after a warm-up that sizes the
    library's scratch) so the events time the GPU, not the host."""
    import torch
    from nx_vulkan_b200 import _native, vulkan as nxv

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    lib = _native.load()
    assert nxv.init_devices([0]) == "ok", _native.last_error()
    lib.nxv_set_stream(C.c_void_p(stream.cuda_stream))
    peak, peak_kind = peaks()
    handles = []

    def wrap(t):
        h = lib.nxv_buf_wrap(C.c_void_p(t.data_ptr()), t.numel() * t.element_size())
        handles.append(h)
        return h

    def timed(fn, reps=20):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(reps):
                fn()
        g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(3):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / (3 * reps)

    def emit(**kw):
        print(json.dumps(kw), flush=True)

    def ck(rc):
        if rc != 0:
            raise RuntimeError(_native.last_error())

    gen = torch.Generator(device="cpu").manual_seed(0)

    want = set(args.only.split(","))

    # CPU path beside each GPU line: the oracle (the C restatement of the
    # reference's semantics) timed on a bounded sample of the same workload on
    # this host, scaled to the full workload by its size.
    from oracle import binding as orc
    nthr = host_threads()
    crng = np.random.default_rng(11)

    def cpu_est(fn, scale, cores, sample, min_s=0.2):
        if args.no_cpu:
            return None
        fn()
        reps, t0 = 0, time.perf_counter()
        while True:
            fn()
            reps += 1
            el = time.perf_counter() - t0
            if el >= min_s or reps >= 20:
                break
        return {"us_per_call": el / reps * scale * 1e6, "kind": "port", "cores": cores,
                "sample": sample}

    # -- fused elementwise chain tanh(exp(x*y+z)-1.0), size sweep ---------------
    ops = (C.c_uint * 8)(1, 0, 100, 2, 106, 255, 255, 255)
    src = (C.c_uint * 8)(1, 2, 1, 0, 1, 1, 1, 1)
    imm = (C.c_double * 8)(0, 0, 0, 1.0, 0, 0, 0, 0)
    spv = nxv.shader_path("fused_elementwise_imm.spv")
    for dt, code, sizes in ((torch.float32, 0, (1 << 20, 1 << 24, 1 << 28)),
                            (torch.float64, 1, (1 << 20, 1 << 24, 1 << 27))) if "fused" in want else ():
        es = 4 if code == 0 else 8
        for n in sizes:
            sets = max(1, min(16, (512 << 20) // (4 * n * es)))
            bufs = []
            for _ in range(sets):
                xs = [(torch.rand(n, dtype=torch.float32, device=dev) * 2 - 1).to(dt) for _ in range(3)]
                out = torch.empty(n, dtype=dt, device=dev)
                bufs.append([wrap(t) for t in xs + [out]] + [xs, out])
            it = [0]

            def call():
                hs = bufs[it[0] % sets]
                it[0] += 1
                ck(lib.nxv_fused_chain_imm(hs[3], hs[0], hs[1], hs[2], None, n, 5, ops, src, imm, code, spv))

            reps = 4 * sets if n <= (1 << 24) else 4
            ms = timed(call, reps)
            gbs = 4 * n * es / (ms / 1e3) / 1e9
            ns = min(n, 1 << 22)
            npdt = np.float32 if code == 0 else np.float64
            cx = [crng.uniform(-1, 1, ns).astype(npdt) for _ in range(3)]
            cpu = cpu_est(lambda: orc.fused(cx[0], [cx[1], cx[2]], [1, 0, 100, 2, 106], [1, 2, 1, 0, 1],
                                            [0, 0, 0, 1.0, 0], nthreads=nthr),
                          n / ns, nthr, f"{ns} elements, scaled x{n // ns}")
            emit(workload="fused chain tanh(exp(x*y+z)-1.0)", dtype=str(dt).split(".")[-1], n=n,
                 us_per_call=ms * 1e3, gbs=gbs, frac_of_hbm=gbs / peak, bytes_per_call=4 * n * es,
                 rotating_sets=sets, cpu_baseline=cpu)
            del bufs
            torch.cuda.empty_cache()

    # -- reductions + broadcast on [4096, 4096] ---------------------------------------
    R = 4096
    for dt, code in ((torch.float32, 0), (torch.float64, 1)) if "reduce" in want else ():
        es = 4 if code == 0 else 8
        # Rotating copies of x (and of the broadcast output) so that one call's
        # input is not still in the 126 MB L2 from the previous call.
        nset = 3 if code == 0 else 2
        x = torch.randn(R * R, generator=gen, dtype=torch.float64).to(dt).to(dev)
        xs = [x] + [x.clone() for _ in range(nset - 1)]
        bvec = torch.randn(R, generator=gen, dtype=torch.float64).to(dt).to(dev)
        hxs, hb = [wrap(t) for t in xs], wrap(bvec)
        o_row = torch.empty(R, dtype=dt, device=dev)
        o_idx = torch.empty(R, dtype=torch.int64, device=dev)
        o_one = torch.empty(1, dtype=dt, device=dev)
        o_fulls = [torch.empty(R * R, dtype=dt, device=dev) for _ in range(nset)]
        ho_row, ho_idx, ho_one = wrap(o_row), wrap(o_idx), wrap(o_one)
        ho_fulls = [wrap(t) for t in o_fulls]
        rspv = nxv.shader_path("reduce_axis.spv" if code == 0 else "reduce_axis_f64.spv")
        fspv = nxv.shader_path("reduce.spv" if code == 0 else "reduce_full_f64.spv")
        aspv = nxv.shader_path("argmax_axis.spv")
        bspv = nxv.shader_path("elementwise_binary_broadcast.spv" if code == 0
                               else "elementwise_binary_broadcast_f64.spv")
        shape = (C.c_uint * 4)(R, R, 0, 0)
        as_ = (C.c_uint * 4)(R, 1, 0, 0)
        bs_ = (C.c_uint * 4)(0, 1, 0, 0)
        k = [0]

        def rot(f):
            def call():
                i = k[0] % nset
                k[0] += 1
                f(i)
            return call

        cases = [
            ("sum axis 1", rot(lambda i: ck(lib.nxv_reduce_axis(ho_row, hxs[i], R, R, 1, 0, rspv))),
             R * R * es + R * es),
            ("reduce_max axis 1", rot(lambda i: ck(lib.nxv_reduce_axis(ho_row, hxs[i], R, R, 1, 1, rspv))),
             R * R * es + R * es),
            ("sum all axes", rot(lambda i: ck(lib.nxv_reduce_to_buf(ho_one, hxs[i], R * R, 0, code, fspv))),
             R * R * es),
            ("reduce_max all axes", rot(lambda i: ck(lib.nxv_reduce_to_buf(ho_one, hxs[i], R * R, 2, code, fspv))),
             R * R * es),
            ("argmax axis 1", rot(lambda i: ck(lib.nxv_argmax_axis(ho_idx, hxs[i], R, R, 1, 0, code, 8, aspv))),
             R * R * es + R * 8),
            ("x + b (rows)", rot(lambda i: ck(lib.nxv_apply_binary_broadcast(ho_fulls[i], hxs[i], hb, 0, 2, shape,
                                                                              as_, bs_, bspv))),
             2 * R * R * es + R * es),
        ]
        rs = 256  # CPU sample: 256 of the 4096 rows, scaled x16
        xc = x[: rs * R].cpu().numpy()
        bc = bvec.cpu().numpy()
        cpu_fns = {
            "sum axis 1": lambda: orc.reduce_axis(xc, rs, R, 1, 0),
            "reduce_max axis 1": lambda: orc.reduce_axis(xc, rs, R, 1, 1),
            "sum all axes": lambda: orc.reduce_full(xc, 0),
            "reduce_max all axes": lambda: orc.reduce_full(xc, 2),
            "argmax axis 1": lambda: orc.argmax_axis(xc, rs, R, 1),
            "x + b (rows)": lambda: orc.broadcast(xc, bc, 0, 2, [rs, R], [R, 1], [0, 1]),
        }
        for name, fn, nbytes in cases:
            ms = timed(fn, 10 * nset)
            gbs = nbytes / (ms / 1e3) / 1e9
            cpu = cpu_est(cpu_fns[name], R / rs, 1, f"{rs} of {R} rows, scaled x{R // rs}")
            emit(workload=f"{name} [4096,4096]", dtype=str(dt).split(".")[-1], us_per_call=ms * 1e3,
                 gbs=gbs, frac_of_hbm=gbs / peak, bytes_per_call=nbytes,
                 l2=f"{nset} rotating copies of the {R * R * es >> 20} MiB input (and output): "
                    "each call's data is out of L2", cpu_baseline=cpu)
        del x, xs, o_fulls
        torch.cuda.empty_cache()

    # -- Philox random streams (write-bound) -------------------------------------------------
    if "random" in want:
        n = 1 << 26
        for code, name in ((0, "f32"), (1, "f64")):
            es = 4 if code == 0 else 8
            outs = [torch.empty(n * es // 4, dtype=torch.float32, device=dev) for _ in range(2)]
            hs = [wrap(t) for t in outs]
            spv_r = nxv.shader_path("random_philox.spv" if code == 0 else "random_philox_f64.spv")
            for dist, dname in ((0, "uniform"), (1, "normal")):
                it = [0]

                def call():
                    h = hs[it[0] % 2]
                    it[0] += 1
                    if code == 0:
                        ck(lib.nxv_random(h, n, 7, dist, spv_r))
                    else:
                        ck(lib.nxv_random_f64(h, n, 7, dist, spv_r))

                ms = timed(call, 8)
                gbs = n * es / (ms / 1e3) / 1e9
                ns = 1 << 22
                cfn = orc.random_f32 if code == 0 else orc.random_f64
                cpu = cpu_est(lambda: cfn(ns, 7, dist), n / ns, 1, f"{ns} elements, scaled x{n // ns}")
                emit(workload=f"philox random {dname}", dtype=name, n=n, us_per_call=ms * 1e3,
                     gbs=gbs, frac_of_hbm=gbs / peak, bytes_per_call=n * es,
                     l2="two alternating outputs of 256/512 MB (larger than L2)", cpu_baseline=cpu)
            del outs
            torch.cuda.empty_cache()

    # -- transpose, cast, logsumexp, HMC primitives, host transfers ---------------------------
    if "misc" in want:
        def hbm_line(name, dtype, fn, nbytes, cpu, reps=10, **extra):
            ms = timed(fn, reps)
            gbs = nbytes / (ms / 1e3) / 1e9
            emit(workload=name, dtype=dtype, us_per_call=ms * 1e3, gbs=gbs, frac_of_hbm=gbs / peak,
                 bytes_per_call=nbytes, cpu_baseline=cpu, **extra)

        # 2-D transpose, 256 MiB in and out
        for dt, name, spv_t, (m, n) in ((torch.float32, "float32", "transpose.spv", (8192, 8192)),
                                        (torch.float64, "float64", "transpose_f64.spv", (4096, 8192))):
            es = 4 if dt == torch.float32 else 8
            a = torch.randn(m * n, dtype=dt, device=dev)
            o = torch.empty(m * n, dtype=dt, device=dev)
            ha, ho = wrap(a), wrap(o)
            sp = nxv.shader_path(spv_t)
            tc = crng.normal(size=(m // 4) * n).astype(np.float32 if es == 4 else np.float64)
            cpu = cpu_est(lambda: orc.transpose(tc, m // 4, n), 4, 1, f"{m // 4} x {n}, scaled x4")
            hbm_line(f"transpose [{m},{n}]", name,
                     lambda: ck(lib.nxv_transpose(ho, ha, m, n, sp)), 2 * m * n * es, cpu)
            del a, o
        # casts, 2^26 elements
        n = 1 << 26
        a32 = torch.randn(n, dtype=torch.float32, device=dev)
        a64 = torch.empty(n, dtype=torch.float64, device=dev)
        h32, h64 = wrap(a32), wrap(a64)
        up_spv, down_spv = nxv.shader_path("cast_f32_to_f64.spv"), nxv.shader_path("cast_f64_to_f32.spv")
        c32 = crng.normal(size=1 << 22).astype(np.float32)
        c64 = c32.astype(np.float64)
        hbm_line("cast f32 -> f64 [2^26]", "float32", lambda: ck(lib.nxv_cast(h64, h32, n, up_spv)), n * 12,
                 cpu_est(lambda: c32.astype(np.float64), 16, 1, "numpy astype of 2^22 elements, scaled x16"))
        hbm_line("cast f64 -> f32 [2^26]", "float64", lambda: ck(lib.nxv_cast(h32, h64, n, down_spv)), n * 12,
                 cpu_est(lambda: c64.astype(np.float32), 16, 1, "numpy astype of 2^22 elements, scaled x16"))
        del a32, a64
        # logsumexp over axis 1 of [4096, 4096] f32, 3 rotating copies (out of L2)
        R = 4096
        xs = [torch.randn(R * R, dtype=torch.float32, device=dev) for _ in range(3)]
        hxs = [wrap(t) for t in xs]
        o = torch.empty(R, dtype=torch.float32, device=dev)
        ho = wrap(o)
        lse_spv = nxv.shader_path("logsumexp.spv")
        k = [0]

        def lse():
            i = k[0] % 3
            k[0] += 1
            ck(lib.nxv_reduce_axis(ho, hxs[i], R, R, 1, 0, lse_spv))

        lc = xs[0][: 256 * R].cpu().numpy()
        hbm_line("logsumexp axis 1 [4096,4096]", "float32", lse, R * R * 4 + R * 4,
                 cpu_est(lambda: orc.logsumexp(lc, 256, R, 1), 16, 1, "256 of 4096 rows, scaled x16"),
                 reps=30, math="f32 exp, double sums (NXV_EXACT_F32=1: f64 exp)")
        del xs
        # HMC primitives (f32, the reference's kinetic_energy.spv / normal_logpdf.spv)
        n = 1 << 26
        pv = torch.randn(n, dtype=torch.float32, device=dev)
        mv = torch.rand(n, dtype=torch.float32, device=dev) + 0.5
        part = torch.empty((n + 255) // 256, dtype=torch.float32, device=dev)
        hp, hm, hpart = wrap(pv), wrap(mv), wrap(part)
        ke_spv = nxv.shader_path("kinetic_energy.spv")
        kp = crng.normal(size=1 << 22).astype(np.float32)
        km = (crng.random(1 << 22) + 0.5).astype(np.float32)
        hbm_line("kinetic_energy [2^26] (per-256 partials)", "float32",
                 lambda: ck(lib.nxv_kinetic_energy(hpart, hp, hm, n, ke_spv)), 2 * n * 4 + (n // 256) * 4,
                 cpu_est(lambda: orc.kinetic_energy(kp, km), 16, 1, "2^22 elements, scaled x16"))
        n2 = 1 << 24
        xv, muv, sv, ov = (torch.rand(n2, dtype=torch.float32, device=dev) + 0.5 for _ in range(4))
        hx2, hmu, hs2, ho2 = wrap(xv), wrap(muv), wrap(sv), wrap(ov)
        lp_spv = nxv.shader_path("normal_logpdf.spv")
        lx, lmu, ls = ((crng.random(1 << 22) + 0.5).astype(np.float32) for _ in range(3))
        hbm_line("normal_logpdf [2^24]", "float32",
                 lambda: ck(lib.nxv_normal_logpdf(ho2, hx2, hmu, hs2, n2, lp_spv)), 4 * n2 * 4,
                 cpu_est(lambda: orc.normal_logpdf(lx, lmu, ls), 4, 1, "2^22 elements, scaled x4"))
        del pv, mv, part, xv, muv, sv, ov
        torch.cuda.empty_cache()
        # host <-> device through the C ABI (256 MiB): pinned copies directly,
        # pageable through the library's pinned staging ring
        nb = 256 << 20
        buf = lib.nxv_buf_alloc(nb)
        pinned = torch.empty(nb, dtype=torch.uint8, pin_memory=True)
        pageable = np.ones(nb, dtype=np.uint8)
        for kind, host in (("pinned", pinned.data_ptr()), ("pageable", pageable.ctypes.data)):
            for direction in ("upload", "download"):
                f = lib.nxv_buf_upload if direction == "upload" else lib.nxv_buf_download
                ck(f(buf, C.c_void_p(host), nb))
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                reps = 5
                for _ in range(reps):
                    ck(f(buf, C.c_void_p(host), nb))
                lib.nxv_synchronize()
                torch.cuda.synchronize()
                sec = (time.perf_counter() - t0) / reps
                emit(workload=f"host {direction} 256 MiB ({kind})", us_per_call=sec * 1e6,
                     gbs=nb / sec / 1e9, timing="host wall clock around synchronous calls")
        lib.nxv_buf_free(buf)

    # -- dense matmul ---------------------------------------------------------------------
    N = 2048
    cub = {}
    for dt, code in ((torch.float64, 1), (torch.float32, 0)) if "matmul" in want else ():
        a = (torch.randn(N, N, generator=gen, dtype=torch.float64) / N ** 0.5).to(dt).to(dev)
        b = (torch.randn(N, N, generator=gen, dtype=torch.float64) / N ** 0.5).to(dt).to(dev)
        c = torch.empty(N, N, dtype=dt, device=dev)
        ha, hb2, hc = wrap(a), wrap(b), wrap(c)
        if code == 1:
            fn = lambda: ck(lib.nxv_matmul_batched(hc, ha, hb2, 1, N, N, N, 1, nxv.shader_path("matmul_batched.spv")))
        else:
            fn = lambda: ck(lib.nxv_matmul(hc, ha, hb2, N, N, N, nxv.shader_path("matmul.spv")))
        ms = timed(fn, 10)
        torch.backends.cuda.matmul.allow_tf32 = False
        ms_cublas = timed(lambda: torch.matmul(a, b, out=c), 10)
        flops = 2 * N ** 3
        cub[code] = flops / (ms_cublas / 1e3) / 1e12
        ms_ = 512
        ca = crng.normal(size=ms_ * ms_).astype(np.float32 if code == 0 else np.float64)
        cpu = cpu_est(lambda: orc.matmul(ca, ca, ms_, ms_, ms_), (N / ms_) ** 3, nthr,
                      f"{ms_}^3 (OpenMP), scaled by flops x{(N // ms_) ** 3}")
        emit(cpu_baseline=cpu, workload=f"matmul {N}x{N}x{N}", dtype=str(dt).split(".")[-1],
             kernel="DMMA mma.sync f64, 64 x 64 tiles" if code == 1 else "3xTF32 tcgen05 (TMEM accumulator, TMA 128B-swizzled tiles)",
             ms=ms, tflops=flops / (ms / 1e3) / 1e12, cublas_ms=ms_cublas, cublas_tflops=cub[code],
             frac_of_cublas=ms_cublas / ms)
    if "matmul" in want:
        a = (torch.randn(64, 256, 256, generator=gen, dtype=torch.float64) / 16).to(dev)
        b = (torch.randn(64, 256, 256, generator=gen, dtype=torch.float64) / 16).to(dev)
        c = torch.empty(64, 256, 256, dtype=torch.float64, device=dev)
        ha, hb2, hc = wrap(a), wrap(b), wrap(c)
        ms = timed(lambda: ck(lib.nxv_matmul_batched(hc, ha, hb2, 64, 256, 256, 256, 1,
                                                     nxv.shader_path("matmul_batched.spv"))), 10)
        ms_cublas = timed(lambda: torch.bmm(a, b, out=c), 10)
        flops = 64 * 2 * 256 ** 3
        cb = crng.normal(size=4 * 256 * 256)
        cpu = cpu_est(lambda: orc.matmul(cb, cb, 256, 256, 256, batch=4), 16, nthr,
                      "4 of 64 batches (OpenMP), scaled x16")
        emit(cpu_baseline=cpu, workload="batched matmul 64 x 256^3", dtype="float64", ms=ms, tflops=flops / (ms / 1e3) / 1e12,
             cublas_ms=ms_cublas, cublas_tflops=flops / (ms_cublas / 1e3) / 1e12, frac_of_cublas=ms_cublas / ms)

        # stream-K vs data-parallel schedule on shapes whose tile count leaves SMs idle
        bspv = nxv.shader_path("matmul_batched.spv")
        for code, shapes in ((1, [(1, 1024, 1024, 1024), (1, 4096, 4096, 4096), (1, 3000, 3000, 512)]),
                             (0, [(1, 128, 128, 4096), (1, 500, 400, 4000), (2, 256, 256, 2048),
                                  (1, 2560, 1024, 2048)])):
            tdt = torch.float64 if code == 1 else torch.float32
            for bt, m_, n_, k_ in shapes:
                a = torch.randn(bt, m_, k_, dtype=tdt, device=dev)
                b = torch.randn(bt, k_, n_, dtype=tdt, device=dev)
                c = torch.empty(bt, m_, n_, dtype=tdt, device=dev)
                ha, hb2, hc = wrap(a), wrap(b), wrap(c)
                # f64: the default 64 x 64 tiles against the 128 x 128 schedule
                # (stream-K tail where it pays); f32: stream-K against data-parallel
                var, alt = ("NXV_GEMM_TILE", "128") if code == 1 else ("NXV_GEMM_SK", "0")
                res = {}
                for v in (None, alt):
                    if v:
                        os.environ[var] = v
                    res[v] = timed(lambda: ck(lib.nxv_matmul_batched(hc, ha, hb2, bt, m_, n_, k_, code, bspv)), 10)
                    os.environ.pop(var, None)
                fl = 2.0 * bt * m_ * n_ * k_
                emit(workload=f"matmul {bt}x{m_}x{n_}x{k_} schedules", dtype="float64" if code else "float32",
                     ms=res[None], tflops=fl / (res[None] / 1e3) / 1e12, ms_alternative=res[alt],
                     tflops_alternative=fl / (res[alt] / 1e3) / 1e12,
                     note=("default 64 x 64 tiles vs NXV_GEMM_TILE=128 (128 x 128 tiles, stream-K tail)"
                           if code == 1 else "default schedule (stream-K tail where it pays) vs NXV_GEMM_SK=0"))
                del a, b, c

    # -- logistic-regression leapfrog -----------------------------------------------------------
    if "logreg" in want:
        Nobs, Dm, Cc, Lr = 10000, 100, 256, 16
        r = np.random.default_rng(4)
        X = r.normal(size=(Nobs, Dm))
        w = r.normal(size=Dm)
        y = (r.random(Nobs) < 1 / (1 + np.exp(-X @ w))).astype(np.float64)
        tX, ty = torch.from_numpy(X).to(dev), torch.from_numpy(y).to(dev)
        tq = torch.zeros(Cc, Dm, dtype=torch.float64, device=dev)
        tp = torch.from_numpy(r.normal(size=(Cc, Dm))).to(dev)
        outs = [torch.empty(Cc * Lr * Dm, dtype=torch.float64, device=dev) for _ in range(3)]
        outs.append(torch.empty(Cc * Lr, dtype=torch.float64, device=dev))
        hs = [wrap(t) for t in outs] + [wrap(tq), wrap(tp), wrap(tX), wrap(ty)]
        lspv = nxv.shader_path("leapfrog_logreg_f64_batched.spv")
        ms = timed(lambda: ck(lib.nxv_leapfrog_logreg_f64_batched(*hs, Nobs, Dm, Cc, Lr, 0.002, lspv)), 3)
        flops = (Lr + 1) * 2 * 2 * Cc * Dm * Nobs
        qs, ps = np.zeros((16, Dm)), r.normal(size=(16, Dm))
        cpu = cpu_est(lambda: orc.chain_logreg_f64(qs, ps, X, y, Nobs, Dm, 16, 1, 0.002, nthreads=nthr),
                      (Cc / 16) * (Lr + 1) / 2, nthr,
                      "16 chains x 1 step (2 gradients, OpenMP over chains), scaled to 256 chains x 17 gradients")
        emit(cpu_baseline=cpu, workload="logistic-regression leapfrog, 256 chains, X[10000,100], L=16 (one trajectory)",
             dtype="float64", ms_per_trajectory=ms, chain_steps_per_s=Cc * Lr / (ms / 1e3),
             gemm_tflops=flops / (ms / 1e3) / 1e12, dgemm_cublas_tflops=cub.get(1),
             seconds_for_1000_trajectories=ms)
    # -- NUTS over the speculative chain (the tree builder's call site) --------------------
    if "nuts" in want:
        from nx_vulkan_b200 import nuts
        from oracle.chain import OracleChain
        lib.nxv_set_stream(None)

        class Timed:
            """Wraps a trajectory source and accumulates the wall time of its calls."""

            def __init__(self, src):
                self.src, self.sec, self.steps = src, 0.0, 0
                self.calls = src.calls

            def extend(self, q, p, K):
                t0 = time.perf_counter()
                out = self.src.extend(q, p, K)
                self.sec += time.perf_counter() - t0
                self.steps += q.shape[0] * K
                return out

        def run_nuts(src_cls, chains, transitions, d=100, eps=0.05):
            r = np.random.default_rng(3)
            prec = r.uniform(0.5, 2.0, d)
            tg = nuts.GaussianTarget(prec)
            m = np.ones(d)
            src = Timed(src_cls(tg, m, eps))
            q = r.normal(size=(chains, d)) / np.sqrt(prec)
            rng = np.random.default_rng(4)
            q, _ = nuts.nuts_transition(src, tg, q, m, rng, max_depth=8)  # warm-up
            src.sec, src.steps = 0.0, 0
            depths, t0 = [], time.perf_counter()
            for _ in range(transitions):
                q, st = nuts.nuts_transition(src, tg, q, m, rng, max_depth=8)
                depths.append(float(st.depth.mean()))
            el = time.perf_counter() - t0
            return el, src, statistics.mean(depths)

        Cn, Tn = 256, 5
        el, src, dep = run_nuts(nuts.GpuChain, Cn, Tn)
        cel, csrc, _ = run_nuts(OracleChain, Cn, 2)
        cpu_us = cel / 2 * 1e6
        emit(workload="NUTS transitions, 256 chains, Gaussian d=100, eps=0.05, max depth 8",
             dtype="float64", us_per_call=el / Tn * 1e6, transitions_per_s=Cn * Tn / el,
             mean_tree_depth=dep, chain_call_share=src.sec / el,
             speculative_steps_per_s=src.steps / src.sec if src.sec else None,
             note="tree logic on the host (numpy), trajectories from the GPU chain with fused KE; "
                  "call share = fraction of wall time in the chain calls (kernel + transfers)",
             cpu_baseline={"us_per_call": cpu_us, "kind": "port", "cores": 1,
                           "sample": "same NUTS (same host tree logic) driven by the oracle chain, "
                                     "256 chains x 2 transitions"})
        # the tree walk on the device: leaves stay in the device store
        r = np.random.default_rng(3)
        prec = r.uniform(0.5, 2.0, 100)
        tg = nuts.GaussianTarget(prec)
        q_start = r.normal(size=(Cn, 100)) / np.sqrt(prec)
        for driver in ("layout", "levels", "host"):
            dt = nuts.DeviceTree(tg, np.ones(100), 0.05, driver=driver)
            qd = torch.from_numpy(q_start).to(dev)
            rng = np.random.default_rng(4)
            qd, _ = dt.transition(qd, rng, max_depth=8)  # warm-up
            torch.cuda.synchronize()
            depths, t0 = [], time.perf_counter()
            for _ in range(Tn):
                qd, st = dt.transition(qd, rng, max_depth=8)
                depths.append(float(st.depth.mean()))
            torch.cuda.synchronize()
            el_d = time.perf_counter() - t0
            note = ("momenta and uniforms drawn by Philox on the device, tree state on the device, "
                    "every chain's leaves at fixed store rows: per level one start kernel, one "
                    "chain call of 2^l steps for all chains and one level kernel, the whole "
                    "transition one library call (nxv_nuts_transition_layout) reading one "
                    "4-byte flag per level"
                    if driver == "layout" else
                    "the same kernels issued level by level from Python "
                    "(nxv_nuts_start_layout, the batched chain call, nxv_nuts_level_layout); "
                    "the host reads one flag per level"
                    if driver == "levels" else
                    "leaves written by the chain calls into a device store and walked there "
                    "(nxv_nuts_energy/_start/_level); the host keeps the row bookkeeping "
                    "(speculative extension), draws the random numbers and reads one active "
                    "flag per chain and level")
            emit(workload="NUTS transitions, 256 chains, Gaussian d=100, eps=0.05, max depth 8, "
                          f"tree walk on the device ({driver} driver)",
                 dtype="float64", us_per_call=el_d / Tn * 1e6, transitions_per_s=Cn * Tn / el_d,
                 mean_tree_depth=statistics.mean(depths),
                 speedup_over_host_tree=el / Tn / (el_d / Tn), note=note)
        lib.nxv_set_stream(C.c_void_p(stream.cuda_stream))

    for h in handles:
        lib.nxv_buf_free(h)
    lib.nxv_set_stream(None)


if __name__ == "__main__":
    main()
