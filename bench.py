"""Benchmark: Sinkhorn fwd+bwd throughput (cost-element-iterations per second).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg1|cfg2|cfg3|cfg4|cfg5]

One step = one pass of the hot path over one batch of synthetic input of the
chosen BASELINE configuration: for Sinkhorn, ``dot.sinkhorn(C, reg, n_iters,
tol=0)`` followed by ``result.cost.sum().backward()``; for bidirectional
softmax, forward + backward with an N(0,1) upstream gradient.  The default
workload is configs[1] (cfg2: B=256, 512x512, reg 0.05, 200 iterations), the
configuration the headline metric is quoted on.

Units: one cost-element-iteration = one element of the B x n x m cost for one
Sinkhorn iteration (fwd+bwd counted once, backward_iters = n_iters); for
bidirectional softmax one element fwd+bwd.

Timing: W untimed warm-up steps, then K steps between a barrier +
torch.cuda.synchronize() on both sides, timed with CUDA events on the
launching stream; the job time is the max over ranks.  Under torchrun each rank
runs its own batch of the workload (independent problems, no collective on the
data path): weak scaling.  ``value`` is the whole-job throughput with inputs
resident in HBM; ``e2e`` re-times the same step from pinned host memory
(host->device copy of every step's inputs and device->host read of every
step's loss inside the timed region; the next step's inputs are copied on a
second stream while the current step computes).

``--impl reference`` times the reference's own CPU implementation of the path
(its kernels_cpu.cpp compiled from source into oracle/_ref by oracle/Makefile;
the C restatement in oracle/ if that library is absent) on all host threads,
one bounded sample of the workload per step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "Sinkhorn fwd+bwd cost-elem-iters/s per GPU; achieved HBM GB/s vs peak"

CONFIGS = {
    "cfg1": dict(kind="sinkhorn", B=8, n=64, m=64, reg=1.0, iters=100, cost="uniform", marg="uniform",
                 desc="configs[0]: Sinkhorn fwd+bwd B=8 64x64 U[0,1) cost, reg 1.0, 100 it, uniform marginals"),
    "cfg2": dict(kind="sinkhorn", B=256, n=512, m=512, reg=0.05, iters=200, cost="sqdist64", marg="uniform",
                 desc="configs[1]: Sinkhorn fwd+bwd B=256 512x512 normalised sq-dist of N(0,1) 64-D clouds, "
                      "reg 0.05, 200 it, uniform marginals"),
    "cfg3": dict(kind="bidir", B=64, n=1024, m=1024, tau=0.1, dtype="f32",
                 desc="configs[2]: bidirectional softmax fwd+bwd B=64 1024x1024 N(0,1) scores, tau 0.1, fp32"),
    "cfg3bf16": dict(kind="bidir", B=64, n=1024, m=1024, tau=0.1, dtype="bf16",
                     desc="configs[2]: bidirectional softmax fwd+bwd B=64 1024x1024 N(0,1) scores, tau 0.1, bf16 "
                          "input (fp32 output and upstream gradient, bf16 input gradient)"),
    "cfg4": dict(kind="sinkhorn", B=4096, n=128, m=128, reg=0.1, iters=100, cost="uniform", marg="dirichlet",
                 desc="configs[3]: Sinkhorn fwd+bwd B=4096 128x128 U[0,1) cost, Dirichlet(1) marginals, "
                      "reg 0.1, 100 it"),
    "cfg5": dict(kind="sinkhorn_fwd", B=1, n=32768, m=32768, reg=0.01, iters=500, cost="sqdist3u",
                 marg="uniform", desc="configs[4]: Sinkhorn fwd B=1 32768x32768 sq-dist of U[0,1)^3 clouds, "
                                      "reg 0.01, 500 it"),
}


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------

def make_inputs(cfg: dict, seed: int):
    import torch

    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    B, n, m = cfg["B"], cfg["n"], cfg["m"]
    if cfg["kind"] == "bidir":
        S = torch.randn(B, n, m, generator=g)
        if cfg.get("dtype") == "bf16":
            S = S.bfloat16()
        return {"S": S, "G": torch.randn(B, n, m, generator=g)}
    if cfg["cost"] == "uniform":
        C = torch.rand(B, n, m, generator=g)
    elif cfg["cost"] == "sqdist64":
        x = torch.randn(B, n, 64, generator=g)
        y = torch.randn(B, m, 64, generator=g)
        C = torch.cdist(x, y).square()
        C = C / C.amax(dim=(1, 2), keepdim=True)
    elif cfg["cost"] == "sqdist3u":
        x = torch.rand(B, n, 3, generator=g)
        y = torch.rand(B, m, 3, generator=g)
        C = torch.cdist(x, y).square()
    else:
        raise ValueError(cfg["cost"])
    out = {"C": C.float().contiguous()}
    if cfg["marg"] == "dirichlet":
        torch.manual_seed(seed)
        d = torch.distributions.Dirichlet(torch.ones(n))
        out["a"] = d.sample((B,)).float()
        out["b"] = torch.distributions.Dirichlet(torch.ones(m)).sample((B,)).float()
    return out


def units_per_step(cfg: dict) -> int:
    if cfg["kind"] == "bidir":
        return cfg["B"] * cfg["n"] * cfg["m"]
    return cfg["B"] * cfg["n"] * cfg["m"] * cfg["iters"]


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi sampling every 100 ms, started before the warm-up (the tool
    takes a moment to print its first sample) and stopped after the timed
    region; only samples whose timestamp falls inside the marked region count.
    A region shorter than the sampling period falls back to the samples within
    0.5 s of it, and says so."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark_begin(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is not None:
            time.sleep(0.25)   # let the sample covering the region's end land
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    @staticmethod
    def _stamp(s: str):
        import datetime

        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.datetime.strptime(s.strip(), fmt).timestamp()
            except ValueError:
                pass
        return None

    def summary(self) -> dict:
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 10:
                    rows.append((self._stamp(p[0]), p[1:]))
        os.unlink(self.path)
        inside = [r for t, r in rows if t is not None and self.t0 is not None and self.t0 <= t <= self.t1]
        window = "timed region"
        if not inside:
            inside = [r for t, r in rows if t is not None and self.t0 is not None
                      and self.t0 - 0.5 <= t <= self.t1 + 0.5]
            window = "within 0.5 s of the timed region (region shorter than the 100 ms sampling period)"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [v for v in (num(r[1]) for r in inside) if v is not None]
        mx = [v for v in (num(r[2]) for r in inside) if v is not None]
        pw = [v for v in (num(r[3]) for r in inside) if v is not None]
        reasons = sorted({self.REASONS[k] for r in inside for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside), "window": window,
                "power_w_max": max(pw) if pw else None}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, cfg: dict) -> None:
    import torch
    import torch.distributed as dist

    import dot
    from dot_b200 import _lib

    rank, local_rank, world = env_rank()
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    rowshard = cfg["kind"] == "sinkhorn_fwd" and world > 1
    if cfg.get("cost") == "sqdist3u":
        # one problem (cfg5): the same seeded points on every rank; each rank
        # builds the cost rows it owns on its GPU (row sharding for world > 1)
        from dot_b200.distributed import shard_range

        g = torch.Generator(device="cpu")
        g.manual_seed(1234)
        x = torch.rand(cfg["B"], cfg["n"], 3, generator=g)
        y = torch.rand(cfg["B"], cfg["m"], 3, generator=g)
        lo, hi = shard_range(cfg["n"], rank, world) if rowshard else (0, cfg["n"])
        C_gpu = torch.cdist(x[:, lo:hi].to(dev), y.to(dev)).square().contiguous()
        inputs = {"C": C_gpu.cpu()}
        del C_gpu
    else:
        inputs = make_inputs(cfg, seed=1234 + rank)

    def barrier():
        if world > 1:
            dist.barrier()

    if cfg["kind"] == "bidir":
        S_host = inputs["S"].pin_memory()
        G_host = inputs["G"].pin_memory()
        S_dev = S_host.to(dev)
        G_dev = G_host.to(dev)

        def step(S, G):
            s = S.detach().requires_grad_(True)
            out = dot.bidirectional_softmax(s, tau=cfg["tau"])
            out.backward(G)
            return out

        host_in = (S_host, G_host)

        def step_on(bufs):
            return step(*bufs).sum()

        step_dev = lambda: step(S_dev, G_dev)  # noqa: E731
        h2d = S_host.numel() * S_host.element_size() + G_host.numel() * 4
    else:
        C_host = inputs["C"].pin_memory()
        C_dev = C_host.to(dev)
        a = inputs.get("a")
        b = inputs.get("b")
        a_dev = None if a is None else a.to(dev)
        b_dev = None if b is None else b.to(dev)
        fwd_only = cfg["kind"] == "sinkhorn_fwd"

        def step(C):
            if rowshard:
                from dot_b200.distributed import sinkhorn_rowshard

                res = sinkhorn_rowshard(C, cfg["reg"], cfg["iters"], n_total=cfg["n"])
                return res["cost"].sum()
            Cg = C if fwd_only else C.detach().requires_grad_(True)
            res = dot.sinkhorn(Cg, reg=cfg["reg"], n_iters=cfg["iters"], a=a_dev, b=b_dev, tol=0)
            loss = res.cost.sum()
            if not fwd_only:
                loss.backward()
            return loss

        host_in = (C_host,)

        def step_on(bufs):
            return step(*bufs)

        step_dev = lambda: step(C_dev)  # noqa: E731
        h2d = C_host.numel() * 4

    clocks = ClockSampler(local_rank).start()
    for _ in range(args.warmup):
        step_dev()
    torch.cuda.synchronize()

    # ---- timed region (device-resident inputs) ----
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    _lib.prof_begin(time_events=True)
    clocks.mark_begin()
    ev0.record(stream)
    for _ in range(args.steps):
        step_dev()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.mark_end()
    clocks.stop()
    prof = _lib.prof_end()
    barrier()
    ms = ev0.elapsed_time(ev1)
    t_local = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_local, op=dist.ReduceOp.MAX)
    ms_max = float(t_local.item())

    # ---- timed region (end to end from pinned host memory) ----
    # Every step's inputs are copied host -> device inside the timed region and
    # its loss is read back to the host; the copy of step k+1's inputs runs on a
    # second stream into a second set of device buffers while step k computes
    # (double buffering, as an input pipeline would).
    copy_stream = torch.cuda.Stream(dev)
    dbufs = [tuple(torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_in) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def upload(k):
        j = k % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[j])   # step k-2 is done with these buffers
            for d, h in zip(dbufs[j], host_in):
                d.copy_(h, non_blocking=True)
            ready[j].record(copy_stream)

    def run_e2e(nsteps):
        upload(0)
        for k in range(nsteps):
            if k + 1 < nsteps:
                upload(k + 1)
            stream.wait_event(ready[k % 2])
            loss = step_on(dbufs[k % 2])
            free[k % 2].record(stream)
            loss.item()  # device -> host read of the step's result

    for j in range(2):
        free[j].record(stream)
    run_e2e(1)   # untimed: first use of the e2e path's allocations
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run_e2e(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    t_e2e = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    ms_e2e = float(t_e2e.item())

    units = units_per_step(cfg)
    jobs = 1 if rowshard else world   # row sharding splits one problem; otherwise each rank runs its own batch
    value = units * jobs * args.steps / (ms_max / 1e3)
    e2e_value = units * jobs * args.steps / (ms_e2e / 1e3)
    launches = sum(v["launches"] for v in prof.values())

    if rank == 0:
        peaks = measured_peaks()
        roof = roofline(cfg, prof, peaks, args.steps,
                        elems_local=(C_dev.numel() if cfg["kind"] != "bidir" else None))
        line = {
            "metric": METRIC if cfg["kind"] != "bidir" else "bidirectional softmax fwd+bwd elements/s",
            "value": value,
            "unit": "cost-elem-iters/s" if cfg["kind"] != "bidir" else "elements/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if rowshard else "weak",
            "vs_baseline": None,
            "dtype": "f32" if cfg.get("dtype", "f32") == "f32" else "bf16-in/f32",
            "data": "synthetic (seeded; shapes and distributions of the BASELINE config)",
            "config": {"workload": cfg["desc"], **{k: cfg[k] for k in ("B", "n", "m") if k in cfg},
                       **({"reg": cfg["reg"], "n_iters": cfg["iters"], "backward_iters": cfg["iters"],
                           "tol": 0} if cfg["kind"] != "bidir" else {"tau": cfg["tau"]}),
                       "per_rank_batch": cfg["B"],
                       "l2": "inputs larger than L2 (126 MB)" if units_per_step(cfg) // max(cfg.get("iters", 1), 1) * 4
                       > 126e6 else "small working set: L2-resident by design (on-chip solver)",
                       "parallelism": (f"rows sharded x{world}, NCCL all-gather of column (max, sum) pairs "
                                       "per iteration" if rowshard else
                                       f"batch-independent x{world} (no collective)")},
            "e2e": {"value": e2e_value, "unit": "cost-elem-iters/s" if cfg["kind"] != "bidir" else "elements/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4,
                    "ms_per_step": ms_e2e / args.steps,
                    "pipeline": "each step's inputs copied from pinned host memory inside the timed region, "
                                "step k+1's on a second stream while step k computes; loss read back every step"},
            "gpu_launches": int(launches),
            "roofline": roof,
            "kernels": {k: v for k, v in prof.items() if v["launches"]},
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, sample_seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def roofline(cfg: dict, prof: dict, peaks: dict, steps: int, elems_local: int | None = None) -> dict:
    """Dominant kernel class: algorithmic bytes / measured kernel time.

    Sinkhorn: every sweep kernel (fused forward iteration, fused adjoint
    iteration, or one pass of the two-pass path) streams the B x n x m fp32
    matrix once: 4 B per element per launch.  The resident solver reads the
    cost once and writes the plan once per call (8 B per element), all
    iterations on chip; its bound is the SFU, so its roofline is reported
    against HBM only for completeness.  Bidirectional softmax: compulsory
    bytes per step, fwd = read sim + write out, bwd = read sim + read grad_out
    + write grad_sim.
    """
    B, n, m = cfg["B"], cfg["n"], cfg["m"]
    elems = B * n * m
    if elems_local is None:
        elems_local = elems
    cands = [(v["ms"], k, v) for k, v in prof.items() if v["launches"] and v["ms"] > 0]
    if not cands:
        return {"bound": "hbm", "achieved": None, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": None,
                "traffic": None}
    cands.sort(reverse=True)
    ms, k, v = cands[0]
    avg_ms = v["ms"] / v["launches"]
    if k in ("sk_fwd_iter", "sk_bwd_iter"):
        # matrix sweeps per iteration: one for the fused (m <= 1024) and the
        # wide-row cluster (8192 <= m <= 65536) kernels, two (row, then
        # column) for the general two-pass path; the merge launches of the
        # two-pass and row-shard paths move no matrix bytes
        single = (m <= 1024 and m % 4 == 0) or (8192 <= m <= 65536 and m % 32 == 0)
        sweeps = cfg["iters"] * steps * (1 if single else 2)
        total_bytes = 4 * elems_local * sweeps
        bytes_per_launch = total_bytes / v["launches"]
    elif k == "sk_resident":
        total_bytes = 20 * elems * steps   # fwd: read C, write P; bwd: read P, read C, write grad
        bytes_per_launch = total_bytes / v["launches"]
    elif k in ("bs_fwd", "bs_bwd"):
        per = 4 if cfg.get("dtype", "f32") == "f32" else 2
        per_step = (per + 4) if k == "bs_fwd" else (per + 4 + per)
        total_bytes = per_step * elems * steps
        bytes_per_launch = total_bytes / v["launches"]
    else:
        total_bytes = 8 * elems * v["launches"]
        bytes_per_launch = 8 * elems
    achieved = total_bytes / (v["ms"] / 1e3) / 1e9
    peak = peaks["hbm_gbs"]
    traffic = traffic_from_profiles(k, cfg.get("name", ""))
    if traffic is not None and k in ("sk_fwd_iter", "sk_bwd_iter"):
        # the captured figure is one full single-GPU sweep launch; average it
        # over this run's launches (row-shard merge launches move no matrix
        # bytes) and scale it to this rank's rows
        traffic *= (elems_local / elems) * (sweeps / v["launches"])
    out = {"bound": "hbm", "kernel_class": k, "achieved": achieved, "peak": peak, "unit": "GB/s",
           "frac": achieved / peak, "peak_source": peaks["source"], "avg_launch_ms": avg_ms,
           "launches": v["launches"], "algorithmic_bytes_per_launch": bytes_per_launch,
           "traffic": traffic}
    fw, bw = prof.get("sk_fwd_iter"), prof.get("sk_bwd_iter")
    if k in ("sk_fwd_iter", "sk_bwd_iter") and fw and bw and fw["ms"] > 0 and bw["ms"] > 0:
        # forward and adjoint iteration sweeps together (each streams the
        # matrix once per iteration on the single-pass paths)
        single = (m <= 1024 and m % 4 == 0) or (8192 <= m <= 65536 and m % 32 == 0)
        nsweep = (cfg["iters"] + cfg.get("bwd_iters", cfg["iters"])) * steps * (1 if single else 2)
        fb = 4 * elems_local * nsweep / ((fw["ms"] + bw["ms"]) / 1e3) / 1e9
        out["fwd_bwd"] = {"achieved": fb, "frac": fb / peak, "unit": "GB/s",
                          "ms": fw["ms"] + bw["ms"], "sweeps": nsweep}
    return out


def traffic_from_profiles(kclass: str, workload: str):
    """DRAM bytes (read + write) per launch of the dominant kernel, from the
    committed ncu summary profiles/traffic_per_launch.txt (lines:
    `<workload> <kernel class> <bytes>`), or None when not captured."""
    path = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            p = line.split()
            if len(p) >= 3 and p[0] == workload and p[1] == kclass:
                return float(p[2])
    return None


# ---------------------------------------------------------------------------
# CPU baseline / reference arm
# ---------------------------------------------------------------------------

def cpu_sample(cfg: dict, problems: int, threads: int, kind: str, seed: int = 99):
    """Time the reference CPU implementation on ``problems`` problems of the
    workload, ``threads`` at a time.  Returns (units/s, seconds, units)."""
    import numpy as np

    from oracle import oracle as O

    sub = dict(cfg)
    sub["B"] = problems
    inp = make_inputs(sub, seed)
    if cfg["kind"] == "bidir":
        S = inp["S"].float().numpy()
        G = inp["G"].numpy()
        lengths = np.tile(np.array([[cfg["n"], cfg["m"]]], np.int32), (problems, 1))
        from concurrent.futures import ThreadPoolExecutor

        def work(i):
            out, rs, cs = O.bidir_forward(S[i:i + 1], cfg["tau"], lengths[i:i + 1], kind=kind)
            O.bidir_backward(S[i:i + 1], out, G[i:i + 1], rs, cs, cfg["tau"], lengths[i:i + 1], kind=kind)

        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(work, range(problems)))
        dt = time.perf_counter() - t0
        units = problems * cfg["n"] * cfg["m"]
        return units / dt, dt, units
    C = inp["C"].numpy()
    a = None if "a" not in inp else inp["a"].numpy()
    b = None if "b" not in inp else inp["b"].numpy()
    t0 = time.perf_counter()
    O.sinkhorn_fwd_bwd_threaded(C, cfg["reg"], cfg["iters"], a, b, threads=threads, kind=kind)
    dt = time.perf_counter() - t0
    units = problems * cfg["n"] * cfg["m"] * cfg["iters"]
    return units / dt, dt, units


def cpu_kind() -> str:
    from oracle import oracle as O

    return "reference" if O.available("reference") else "restated"


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def sample_problems(cfg: dict, threads: int, seconds: float) -> int:
    """Problems per CPU sample: about `seconds` of CPU work, at least one per thread."""
    per_problem = {"cfg1": 0.011, "cfg2": 1.7, "cfg3": 0.12, "cfg3bf16": 0.12, "cfg4": 0.046, "cfg5": 1e9}
    est = per_problem.get(cfg.get("name", ""), 1.0)
    p = max(threads, int(seconds / est))
    p = (p // threads) * threads if p >= threads else threads
    return max(1, min(p, cfg["B"]))


def cpu_baseline(cfg: dict, sample_seconds: float = 15.0) -> dict:
    if cfg["kind"] == "sinkhorn_fwd":
        return {"value": None, "unit": "cost-elem-iters/s", "cores": 1, "kind": "reference",
                "sample": "not run: one iteration of the 32768^2 problem takes minutes on one core"}
    kind = cpu_kind()
    threads = cpu_threads()
    problems = sample_problems(cfg, threads, sample_seconds)
    v, dt, units = cpu_sample(cfg, problems, threads, kind)
    return {"value": v, "unit": "cost-elem-iters/s" if cfg["kind"] != "bidir" else "elements/s",
            "cores": threads, "kind": "reference" if kind == "reference" else "port",
            "sample": f"{problems} of {cfg['B']} problems of the workload, full size and iterations, "
                      f"{threads} threads (one problem per thread at a time), {dt:.1f} s wall; the reference's "
                      "CPU fwd op, then its backward op (which re-runs the forward)"}


def run_reference(args, cfg: dict) -> None:
    rank, _, world = env_rank()
    if rank != 0:
        return
    kind = cpu_kind()
    threads = cpu_threads()
    if cfg["kind"] == "sinkhorn_fwd":
        print(json.dumps({"impl": "reference", "unavailable": "cfg5 on the host CPU takes ~16 h per step"}))
        return
    problems = sample_problems(cfg, threads, args.cpu_seconds)
    for _ in range(args.warmup):
        cpu_sample(cfg, threads, threads, kind)
    vals, secs = [], []
    for _ in range(args.steps):
        v, dt, _ = cpu_sample(cfg, problems, threads, kind)
        vals.append(v)
        secs.append(dt)
    value = statistics.median(vals)
    unit = "cost-elem-iters/s" if cfg["kind"] != "bidir" else "elements/s"
    sample = (f"{problems} of {cfg['B']} problems per step at full size and iterations, {threads} host threads, "
              f"reference CPU kernels ({'oracle/_ref, compiled from the reference sources' if kind == 'reference' else 'oracle restatement'})")
    line = {
        "impl": "reference",
        "metric": METRIC if cfg["kind"] != "bidir" else "bidirectional softmax fwd+bwd elements/s",
        "value": value, "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * statistics.median(secs), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; shapes of the BASELINE config)",
        "config": {"workload": cfg["desc"], "B": cfg["B"], "n": cfg["n"], "m": cfg["m"]},
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads,
                         "kind": "reference" if kind == "reference" else "port", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU work per baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--iters", type=int, default=None, help="override the config's iteration count (profiling)")
    ap.add_argument("--rows", type=int, default=None, help="override the config's row count n (profiling)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    cfg["name"] = args.config
    if args.iters is not None and "iters" in cfg:
        cfg["iters"] = args.iters
        cfg["desc"] += f" (run with {args.iters} iterations)"
    if args.rows is not None:
        cfg["n"] = args.rows
        cfg["desc"] += f" (run with {args.rows} rows)"
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
