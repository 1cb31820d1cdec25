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

Extra keys of the default (cfg2) line: ``configs`` (N=1) -- every other
BASELINE configuration with its time per step, throughput, dominant-kernel
roofline and CPU baseline; ``rowshard_cfg5`` -- configs[4] (32768 x 32768,
reg 0.01) forward at 100 iterations, on one GPU at N=1 and rows sharded over
the N GPUs (library-owned NCCL all-gather per iteration) at N>1;
``rowshard_points_cfg5`` -- the same problem from its two point clouds
(``sinkhorn_points_rowshard``: the cost built in the half-steps); and
``batchshard_cfg4`` -- configs[3] with its 4096 problems split over the N
GPUs.  The last two are strong scaling and give the 1/2/4/8-GPU curve of the
sharded configurations when the driver runs the bench at several N.

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
METRIC_FWD = "Sinkhorn fwd cost-elem-iters/s (forward only); achieved HBM GB/s vs peak"
METRIC_BS = "bidirectional softmax fwd+bwd elements/s; achieved HBM GB/s vs peak"

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

def metric_of(cfg: dict) -> str:
    if cfg["kind"] == "bidir":
        return METRIC_BS
    return METRIC_FWD if cfg["kind"] == "sinkhorn_fwd" else METRIC


def unit_of(cfg: dict) -> str:
    return "elements/s" if cfg["kind"] == "bidir" else "cost-elem-iters/s"


def config_dict(cfg: dict, world: int) -> dict:
    """The ``config`` object of a bench line; both arms print the same one."""
    rowshard = cfg["kind"] == "sinkhorn_fwd" and world > 1
    d = {"workload": cfg["desc"], **{k: cfg[k] for k in ("B", "n", "m") if k in cfg}}
    if cfg["kind"] == "bidir":
        d.update({"tau": cfg["tau"], "dtype": cfg.get("dtype", "f32")})
    else:
        d.update({"reg": cfg["reg"], "n_iters": cfg["iters"], "tol": 0})
        if cfg["kind"] == "sinkhorn":
            d["backward_iters"] = cfg["iters"]
    d["per_rank_batch"] = cfg["B"]
    big = cfg["B"] * cfg["n"] * cfg["m"] * 4 > 126e6
    d["l2"] = ("inputs larger than L2 (126 MB)" if big else
               "small working set: L2-resident by design (on-chip solver)")
    d["parallelism"] = (f"rows sharded x{world}, NCCL all-gather of column (max, sum) pairs per iteration"
                        if rowshard else f"batch-independent x{world} (no collective)")
    return d


class Workload:
    """Device-resident inputs and the step function of one configuration on
    this rank.  ``rowshard``: configs[4] (one problem) with its rows split
    over the ranks; ``batch_split``: the batch split over the ranks (strong
    scaling through ``sinkhorn_batchshard``); otherwise every rank runs the
    whole workload on its own inputs (weak scaling)."""

    def __init__(self, cfg: dict, rank: int, world: int, dev, batch_split: bool = False):
        import torch

        import dot
        from dot_b200.distributed import shard_range, sinkhorn_batchshard, sinkhorn_rowshard

        self.cfg = cfg
        self.rowshard = cfg["kind"] == "sinkhorn_fwd" and world > 1
        if cfg.get("cost") == "sqdist3u":
            # one problem: the same seeded points on every rank; each
            # rank builds the cost rows it owns on its GPU
            g = torch.Generator(device="cpu")
            g.manual_seed(1234)
            x = torch.rand(cfg["B"], cfg["n"], 3, generator=g)
            y = torch.rand(cfg["B"], cfg["m"], 3, generator=g)
            lo, hi = shard_range(cfg["n"], rank, world) if self.rowshard else (0, cfg["n"])
            C_gpu = torch.cdist(x[:, lo:hi].to(dev), y.to(dev)).square().contiguous()
            inputs = {"C": C_gpu.cpu()}
            del C_gpu
        else:
            inputs = make_inputs(cfg, seed=1234 if batch_split else 1234 + rank)
        if cfg["kind"] == "bidir":
            S_host = inputs["S"].pin_memory()
            G_host = inputs["G"].pin_memory()
            self.S_dev, self.G_dev = S_host.to(dev), G_host.to(dev)

            def step(S, G):
                s = S.detach().requires_grad_(True)
                out = dot.bidirectional_softmax(s, tau=cfg["tau"])
                out.backward(G)
                return out

            self.host_in = (S_host, G_host)
            self.step_on = lambda bufs: step(*bufs).sum()
            self.step_dev = lambda: step(self.S_dev, self.G_dev)
            self.h2d = S_host.numel() * S_host.element_size() + G_host.numel() * 4
            self.elems_local = None
            return
        C_host = inputs["C"].pin_memory()
        self.C_dev = C_host.to(dev)
        a, b = inputs.get("a"), inputs.get("b")
        a_dev = None if a is None else a.to(dev)
        b_dev = None if b is None else b.to(dev)
        fwd_only = cfg["kind"] == "sinkhorn_fwd"
        rowshard = self.rowshard

        def step(C):
            if rowshard:
                res = sinkhorn_rowshard(C, cfg["reg"], cfg["iters"], n_total=cfg["n"])
                return res["cost"].sum()
            if batch_split:
                Cg = C.detach().requires_grad_(True)
                res = sinkhorn_batchshard(Cg, reg=cfg["reg"], n_iters=cfg["iters"], a=a_dev, b=b_dev, tol=0,
                                          device=dev)
                loss = res["cost"].sum()
                loss.backward()
                return loss
            Cg = C if fwd_only else C.detach().requires_grad_(True)
            res = dot.sinkhorn(Cg, reg=cfg["reg"], n_iters=cfg["iters"], a=a_dev, b=b_dev, tol=0)
            loss = res.cost.sum()
            if not fwd_only:
                loss.backward()
            return loss

        self.host_in = (C_host,)
        self.step_on = lambda bufs: step(*bufs)
        self.step_dev = lambda: step(self.C_dev)
        self.h2d = C_host.numel() * 4
        self.elems_local = self.C_dev.numel()
        if batch_split:
            lo, hi = shard_range(cfg["B"], rank, world)
            self.elems_local = (hi - lo) * cfg["n"] * cfg["m"]


def _barrier(world):
    import torch.distributed as dist

    if world > 1:
        dist.barrier()


def _max_over_ranks(ms: float, world: int, dev) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_device(step, steps: int, warmup: int, world: int, dev, profile: bool, clocks=None):
    """W untimed steps, then K steps between a barrier + synchronize on both
    sides, timed with CUDA events on the launching stream; returns (max-over-
    ranks ms for the K steps, per-class launch counts / kernel ms)."""
    import torch

    from dot_b200 import _lib

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize()
    _lib.prof_begin(time_events=profile)
    if clocks is not None:
        clocks.mark_begin()
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.mark_end()
    prof = _lib.prof_end()
    _barrier(world)
    return _max_over_ranks(ev0.elapsed_time(ev1), world, dev), prof


def time_e2e(wl: Workload, steps: int, world: int, dev) -> float:
    """End to end from pinned host memory: every step's inputs are copied host
    -> device inside the timed region and its loss is read back to the host;
    the copy of step k+1's inputs runs on a second stream into a second set of
    device buffers while step k computes (double buffering, as an input
    pipeline would)."""
    import torch

    stream = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    dbufs = [tuple(torch.empty(t.shape, dtype=t.dtype, device=dev) for t in wl.host_in) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def upload(k):
        j = k % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[j])   # step k-2 is done with these buffers
            for d, h in zip(dbufs[j], wl.host_in):
                d.copy_(h, non_blocking=True)
            ready[j].record(copy_stream)

    def run(nsteps):
        upload(0)
        for k in range(nsteps):
            if k + 1 < nsteps:
                upload(k + 1)
            stream.wait_event(ready[k % 2])
            loss = wl.step_on(dbufs[k % 2])
            free[k % 2].record(stream)
            loss.item()  # device -> host read of the step's result

    for j in range(2):
        free[j].record(stream)
    run(1)   # untimed: first use of the e2e path's allocations
    _barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    return _max_over_ranks(e0.elapsed_time(e1), world, dev)


def measure_config(name: str, steps: int, warmup: int, rank: int, world: int, dev, cpu_seconds: float,
                   with_cpu: bool) -> dict:
    """One secondary configuration at N=1: device-resident timing, the
    dominant kernel's roofline and the CPU baseline."""
    cfg = dict(CONFIGS[name])
    cfg["name"] = name
    wl = Workload(cfg, rank, world, dev)
    ms, prof = time_device(wl.step_dev, steps, warmup, world, dev, profile=True)
    units = units_per_step(cfg)
    value = units * world * steps / (ms / 1e3)
    out = {"workload": cfg["desc"], "metric": metric_of(cfg), "unit": unit_of(cfg), "ms_per_step": ms / steps,
           "value": value, "value_per_gpu": value / world, "steps": steps, "warmup": warmup,
           "roofline": roofline(cfg, prof, measured_peaks(), steps, elems_local=wl.elems_local),
           "kernels": {k: v for k, v in prof.items() if v["launches"]}}
    if with_cpu:
        out["cpu_baseline"] = cpu_baseline(cfg, sample_seconds=cpu_seconds)
    del wl
    import torch

    torch.cuda.empty_cache()
    return out


def measure_rowshard_cfg5(iters: int, rank: int, world: int, dev) -> dict:
    """configs[4] (32768 x 32768, reg 0.01) forward at ``iters`` iterations:
    at N=1 the single-GPU forward, at N>1 rows sharded over the ranks with the
    library's per-iteration all-gather.  A separate profiled step gives the
    per-iteration split between the sweep kernel and the exchange."""
    import torch

    cfg = dict(CONFIGS["cfg5"])
    cfg["name"] = "cfg5"
    cfg["iters"] = iters
    wl = Workload(cfg, rank, world, dev)
    steps = 3
    ms, _ = time_device(wl.step_dev, steps, 3, world, dev, profile=False)
    _, prof = time_device(wl.step_dev, 1, 0, world, dev, profile=True)
    units = cfg["B"] * cfg["n"] * cfg["m"] * iters
    peaks = measured_peaks()
    fw, ex = prof["sk_fwd_iter"], prof["sk_exchange"]
    sweep_bytes = 4 * wl.elems_local * iters
    out = {"n_gpus": world, "n_iters": iters, "ms_per_step": ms / steps, "ms_per_iter": ms / steps / iters,
           "value": units * steps / (ms / 1e3), "unit": "cost-elem-iters/s", "scaling": "strong",
           "rows_per_gpu": wl.elems_local // cfg["m"],
           "profiled_step": {"sweep_ms_per_iter": fw["ms"] / iters, "exchange_ms_per_iter": ex["ms"] / iters,
                             "note": "one step with events around every launch (breaks the launch overlap "
                                     "of the unprofiled steps)"},
           "roofline": {"bound": "hbm", "kernel_class": "sk_fwd_iter",
                        "achieved": sweep_bytes / (fw["ms"] / 1e3) / 1e9 if fw["ms"] > 0 else None,
                        "peak": peaks["hbm_gbs"], "unit": "GB/s", "peak_source": peaks["source"]}}
    r = out["roofline"]
    r["frac"] = r["achieved"] / r["peak"] if r["achieved"] else None
    del wl
    torch.cuda.empty_cache()
    return out


def measure_rowshard_points_cfg5(iters: int, rank: int, world: int, dev) -> dict:
    """configs[4] (32768 x 32768 U[0,1)^3 clouds, reg 0.01) forward at
    ``iters`` iterations from the two clouds, rows of x split over the ranks
    (``sinkhorn_points_rowshard``: the half-steps on each rank's rows, one
    NCCL all-gather of the column (max, sum) pairs per iteration); the cost
    only (no plan)."""
    import torch

    from dot_b200.distributed import shard_range, sinkhorn_points_rowshard

    cfg = CONFIGS["cfg5"]
    g = torch.Generator(device="cpu")
    g.manual_seed(1234)
    x = torch.rand(1, cfg["n"], 3, generator=g)
    y = torch.rand(1, cfg["m"], 3, generator=g).to(dev)
    lo, hi = shard_range(cfg["n"], rank, world)
    xl = x[:, lo:hi].contiguous().to(dev)

    def step():
        return sinkhorn_points_rowshard(xl, y, cfg["reg"], iters, n_total=cfg["n"], want_plan=False)["cost"]

    steps = 3
    ms, _ = time_device(step, steps, 2, world, dev, profile=False)
    units = cfg["n"] * cfg["m"] * iters
    it_s = ms / steps / 1e3
    fp32_peak = 148 * 128 * 1965e6 * world
    torch.cuda.empty_cache()
    return {"n_gpus": world, "n_iters": iters, "ms_per_step": ms / steps, "ms_per_iter": ms / steps / iters,
            "value": units / it_s, "unit": "cost-elem-iters/s", "scaling": "strong", "rows_per_gpu": hi - lo,
            "roofline": {"bound": "fp32", "achieved": 18 * units / it_s / 1e12, "unit": "T FP32 lane-ops/s",
                         "peak": fp32_peak / 1e12, "frac": 18 * units / it_s / fp32_peak,
                         "peak_source": "nominal: 128 FP32 lanes per SM per clock x 148 SMs x 1965 MHz x n_gpus"}}


def measure_batchshard_cfg4(rank: int, world: int, dev) -> dict:
    """configs[3] (B=4096, 128x128, 100 iterations, fwd+bwd) with the batch
    split over the ranks by ``sinkhorn_batchshard`` (strong scaling; the
    per-step cost gather is the only collective)."""
    import torch

    cfg = dict(CONFIGS["cfg4"])
    cfg["name"] = "cfg4"
    wl = Workload(cfg, rank, world, dev, batch_split=True)
    steps = 5
    ms, _ = time_device(wl.step_dev, steps, 3, world, dev, profile=False)
    units = units_per_step(cfg)
    del wl
    torch.cuda.empty_cache()
    return {"n_gpus": world, "ms_per_step": ms / steps, "value": units * steps / (ms / 1e3),
            "unit": "cost-elem-iters/s", "scaling": "strong", "problems_per_gpu": -(-cfg["B"] // world)}


def measure_points_cfg5(dev, n=None, iters=None, steps: int = 3, warmup: int = 3) -> dict:
    """configs[4] (32768 x 32768 U[0,1)^3 clouds, reg 0.01, 500 iterations)
    through ``dot_b200.sinkhorn_points``: the squared distances built inside
    the half-steps from the two clouds (no 4 GiB cost matrix), with and
    without writing the plan.  The iterations read no matrix from HBM; per
    element-iteration the two half-steps execute 2 ex2 and 2 x (2 d + 3) FP32
    lane operations (d = 3: 18), so the roofline is the FP32 pipe (128 lane
    operations per SM per clock) with the exponential unit (16 per SM per
    clock) beside it."""
    import torch

    import dot_b200

    cfg = CONFIGS["cfg5"]
    n = cfg["n"] if n is None else n
    iters = cfg["iters"] if iters is None else iters
    g = torch.Generator(device="cpu")
    g.manual_seed(1234)
    x = torch.rand(n, 3, generator=g).to(dev)
    y = torch.rand(cfg["m"], 3, generator=g).to(dev)
    units = n * cfg["m"] * iters
    out = {"workload": cfg["desc"] + "; cost built in the half-steps from the two clouds"
                       + (f" (run with {n} rows, {iters} iterations)" if (n, iters) != (cfg["n"], cfg["iters"]) else ""),
           "metric": METRIC_FWD, "n_gpus": 1, "unit": "cost-elem-iters/s", "steps": steps, "warmup": warmup}
    for key, plan in (("with_plan", True), ("cost_only", False)):
        def step(plan=plan):
            return dot_b200.sinkhorn_points(x, y, cfg["reg"], iters, return_plan=plan).cost
        ms, prof = time_device(step, steps, warmup, 1, dev, profile=True)
        it = prof["sk_fwd_iter"]
        out[key] = {"ms_per_step": ms / steps, "value": units * steps / (ms / 1e3),
                    "iterations_ms": it["ms"] / steps, "launches_per_step": it["launches"] // steps}
    it_s = out["cost_only"]["iterations_ms"] / 1e3
    clock = 1965e6
    fp32_peak, xu_peak = 148 * 128 * clock, 148 * 16 * clock
    fp32 = 18 * units / it_s if it_s > 0 else None
    xu = 2 * units / it_s if it_s > 0 else None
    out["roofline"] = {"bound": "fp32", "kernel_class": "sk_fwd_iter",
                       "achieved": fp32 / 1e12 if fp32 else None, "unit": "T FP32 lane-ops/s",
                       "peak": fp32_peak / 1e12, "frac": fp32 / fp32_peak if fp32 else None,
                       "peak_source": "nominal: 128 FP32 lanes per SM per clock x 148 SMs x 1965 MHz "
                                      "(packed f32x2 measured at the same lane rate)",
                       "sfu": {"achieved": xu / 1e12 if xu else None, "unit": "T ex2/s", "peak": xu_peak / 1e12,
                               "frac": xu / xu_peak if xu else None}}
    out["value"] = out["with_plan"]["value"]
    out["ms_per_step"] = out["with_plan"]["ms_per_step"]
    torch.cuda.empty_cache()
    return out


SECONDARY = ("cfg1", "cfg3", "cfg3bf16", "cfg4", "cfg5")


def run_ours(args, cfg: dict) -> None:
    import torch
    import torch.distributed as dist

    rank, local_rank, world = env_rank()
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    wl = Workload(cfg, rank, world, dev)
    rowshard = wl.rowshard

    clocks = ClockSampler(local_rank).start()
    ms_max, prof = time_device(wl.step_dev, args.steps, args.warmup, world, dev, profile=True, clocks=clocks)
    clocks.stop()
    ms_e2e = time_e2e(wl, args.steps, world, dev)

    units = units_per_step(cfg)
    jobs = 1 if rowshard else world   # row sharding splits one problem; otherwise each rank runs its own batch
    value = units * jobs * args.steps / (ms_max / 1e3)
    e2e_value = units * jobs * args.steps / (ms_e2e / 1e3)
    launches = sum(v["launches"] for v in prof.values())
    elems_local = wl.elems_local
    del wl
    torch.cuda.empty_cache()

    line = None
    if rank == 0:
        peaks = measured_peaks()
        line = {
            "metric": metric_of(cfg),
            "value": value,
            "unit": unit_of(cfg),
            "value_per_gpu": value / world,
            "value_is": "whole-job total over n_gpus (value_per_gpu = value / n_gpus)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if rowshard else "weak",
            "vs_baseline": None,
            "dtype": "f32" if cfg.get("dtype", "f32") == "f32" else "bf16-in/f32",
            "data": "synthetic (seeded; shapes and distributions of the BASELINE config)",
            "config": config_dict(cfg, world),
            "e2e": {"value": e2e_value, "unit": unit_of(cfg),
                    "h2d_bytes_per_step": h2d_bytes(cfg, elems_local),
                    "d2h_bytes_per_step": 4, "ms_per_step": ms_e2e / args.steps,
                    "pipeline": "each step's inputs copied from pinned host memory inside the timed region, "
                                "step k+1's on a second stream while step k computes; loss read back every step"},
            "gpu_launches": int(launches),
            "roofline": roofline(cfg, prof, peaks, args.steps, elems_local=elems_local),
            "kernels": {k: v for k, v in prof.items() if v["launches"]},
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, sample_seconds=args.cpu_seconds)
    if world == 1 and not args.no_configs and cfg["name"] == "cfg2":
        confs = {}
        for name in SECONDARY:
            # configs[0] is a ~0.3 ms step dominated by launch overhead: more steps steady it
            steps_c = 20 if name == "cfg1" else 3
            confs[name] = measure_config(name, steps_c, 3, rank, world, dev, args.cpu_seconds / 2,
                                         with_cpu=not args.no_cpu_baseline)
        pts = measure_points_cfg5(dev)
        if line is not None:
            line["configs"] = confs
            line["points_cfg5"] = pts
    if not args.no_scaling and cfg["name"] != "cfg5":
        rs = measure_rowshard_cfg5(100, rank, world, dev)
        rsp = measure_rowshard_points_cfg5(100, rank, world, dev)
        bsd = measure_batchshard_cfg4(rank, world, dev)
        if line is not None:
            line["rowshard_cfg5"] = rs
            line["rowshard_points_cfg5"] = rsp
            line["batchshard_cfg4"] = bsd
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        from dot_b200.distributed import release_communicators

        dist.barrier()
        release_communicators()
        dist.destroy_process_group()


def h2d_bytes(cfg: dict, elems_local) -> int:
    """Bytes copied host -> device per end-to-end step."""
    if cfg["kind"] == "bidir":
        per = 4 if cfg.get("dtype", "f32") == "f32" else 2
        return cfg["B"] * cfg["n"] * cfg["m"] * (per + 4)
    return 4 * int(elems_local)


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


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def sample_problems(cfg: dict, threads: int, seconds: float) -> int:
    """Problems per CPU sample: about `seconds` of CPU work, at least one per thread."""
    per_problem = {"cfg1": 0.011, "cfg2": 1.7, "cfg3": 0.12, "cfg3bf16": 0.12, "cfg4": 0.046}
    est = per_problem.get(cfg.get("name", ""), 1.0)
    p = max(threads, int(seconds / est))
    p = (p // threads) * threads if p >= threads else threads
    return max(1, min(p, cfg["B"]))


def cpu_cfg5_extrapolated(cfg: dict, kind: str, cols: int = 2048) -> tuple[float, str]:
    """configs[4] on the host: the reference's CPU forward op (single-threaded
    by construction) on all rows and a slice of ``cols`` columns, run for 0, 1
    and 2 iterations; the per-iteration time and the fixed part (scaling and
    plan) are scaled by m / cols and extrapolated to the configuration's
    iteration count.  Returns (units/s, description)."""
    import numpy as np
    import torch

    from oracle import oracle as O

    n, m, T = cfg["n"], cfg["m"], cfg["iters"]
    g = torch.Generator().manual_seed(99)
    x = torch.rand(1, n, 3, generator=g)
    y = torch.rand(1, cols, 3, generator=g)
    log_alpha = np.ascontiguousarray(-torch.cdist(x, y).square().float().numpy())
    t = []
    for it in (0, 1, 2):
        t0 = time.perf_counter()
        O.sinkhorn_forward(log_alpha, cfg["reg"], it, kind=kind)
        t.append(time.perf_counter() - t0)
    per_iter = max((t[2] - t[0]) / 2, 1e-9)
    full = (m / cols) * (t[0] + T * per_iter)
    desc = (f"extrapolated: the reference CPU forward op on all {n} rows x {cols} of {m} columns, timed at 0/1/2 "
            f"iterations ({t[0]:.2f}/{t[1]:.2f}/{t[2]:.2f} s), per-iteration time x {T} plus the fixed part, "
            f"scaled by {m // cols}: {full / 3600:.2f} h per step on 1 core")
    return n * m * T / full, desc


def cpu_baseline(cfg: dict, sample_seconds: float = 15.0) -> dict:
    """The reference's CPU implementation timed on this host: all host threads
    (one problem per thread at a time) and one thread (the op as-is)."""
    kind = cpu_kind()
    ckind = "reference" if kind == "reference" else "port"
    unit = unit_of(cfg)
    if cfg["kind"] == "sinkhorn_fwd":
        v, desc = cpu_cfg5_extrapolated(cfg, kind)
        return {"value": v, "value_1thread": v, "unit": unit, "cores": 1, "kind": ckind, "cpu_model": cpu_model(),
                "sample": desc + " (one problem: the single-threaded op cannot use more cores)"}
    threads = cpu_threads()
    problems = sample_problems(cfg, threads, sample_seconds)
    v, dt, _ = cpu_sample(cfg, problems, threads, kind)
    p1 = sample_problems(cfg, 1, sample_seconds / 4)
    v1, dt1, _ = cpu_sample(cfg, p1, 1, kind)
    what = ("the reference's CPU fwd op, then its backward op (which re-runs the forward)"
            if cfg["kind"] == "sinkhorn" else "the reference's CPU forward op, then its backward op")
    return {"value": v, "value_1thread": v1, "unit": unit, "cores": threads, "kind": ckind,
            "cpu_model": cpu_model(),
            "sample": f"{problems} of {cfg['B']} problems of the workload, full size and iterations, {threads} threads "
                      f"(one problem per thread at a time), {dt:.1f} s wall; 1 thread: {p1} problem(s), "
                      f"{dt1:.1f} s; {what}"}


def run_reference(args, cfg: dict) -> None:
    rank, _, world = env_rank()
    if rank != 0:
        return
    kind = cpu_kind()
    threads = cpu_threads()
    unit = unit_of(cfg)
    vals, secs = [], []
    if cfg["kind"] == "sinkhorn_fwd":
        for _ in range(args.warmup):
            cpu_cfg5_extrapolated(cfg, kind, cols=256)
        for _ in range(args.steps):
            v, desc = cpu_cfg5_extrapolated(cfg, kind)
            vals.append(v)
            secs.append(cfg["B"] * cfg["n"] * cfg["m"] * cfg["iters"] / v)
        cores = 1
        sample = desc
    else:
        problems = sample_problems(cfg, threads, args.cpu_seconds)
        for _ in range(args.warmup):
            cpu_sample(cfg, threads, threads, kind)
        for _ in range(args.steps):
            v, dt, _ = cpu_sample(cfg, problems, threads, kind)
            vals.append(v)
            secs.append(dt * cfg["B"] / problems)
        cores = threads
        sample = (f"{problems} of {cfg['B']} problems per step at full size and iterations, {threads} host threads, "
                  f"reference CPU kernels ({'oracle/_ref, compiled from the reference sources' if kind == 'reference' else 'oracle restatement'}); "
                  "ms_per_step scaled to the whole batch")
    value = statistics.median(vals)
    line = {
        "impl": "reference",
        "metric": metric_of(cfg), "value": value, "unit": unit, "value_per_gpu": value / world, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(secs),
        "higher_is_better": True, "scaling": "strong" if cfg["kind"] == "sinkhorn_fwd" and world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; shapes and distributions of the BASELINE config)",
        "config": config_dict(cfg, world),
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores,
                         "kind": "reference" if kind == "reference" else "port", "cpu_model": cpu_model(),
                         "sample": sample},
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
    ap.add_argument("--no-configs", action="store_true", help="skip the other BASELINE configs (N=1 default run)")
    ap.add_argument("--no-scaling", action="store_true",
                    help="skip the row-sharded configs[4] and batch-sharded configs[3] measurements")
    ap.add_argument("--iters", type=int, default=None, help="override the config's iteration count (profiling)")
    ap.add_argument("--rows", type=int, default=None, help="override the config's row count n (profiling)")
    ap.add_argument("--batch", type=int, default=None, help="override the config's batch size B (profiling)")
    ap.add_argument("--cols", type=int, default=None, help="override the config's row length m (profiling)")
    ap.add_argument("--points", action="store_true",
                    help="configs[4] from its two point clouds through dot_b200.sinkhorn_points (1 GPU)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    cfg["name"] = args.config
    if args.iters is not None and "iters" in cfg:
        cfg["iters"] = args.iters
        cfg["desc"] += f" (run with {args.iters} iterations)"
    if args.rows is not None:
        cfg["n"] = args.rows
        cfg["desc"] += f" (run with {args.rows} rows)"
    if args.batch is not None:
        cfg["B"] = args.batch
        cfg["desc"] += f" (run with batch {args.batch})"
    if args.cols is not None:
        cfg["m"] = args.cols
        cfg["desc"] += f" (run with {args.cols} columns)"
    if args.impl == "reference":
        run_reference(args, cfg)
    elif args.points:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps(measure_points_cfg5(torch.device("cuda", 0), n=args.rows, iters=args.iters,
                                             steps=args.steps, warmup=args.warmup)), flush=True)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
