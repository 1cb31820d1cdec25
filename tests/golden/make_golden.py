"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in the build container, where the reference sources are mounted
(default ``/root/reference``, override with ``DOT_REF``)::

    python tests/golden/make_golden.py

What it does:

1. builds the reference's CPU operator library (``src/*/registry.cpp``,
   ``torch_cpu.cpp``, ``kernels_cpu.cpp``) with ``torch.utils.cpp_extension``
   into a scratch directory under /tmp (nothing is copied into this repo);
2. imports the reference's own Python package ``dot`` against that library;
3. runs the public API -- ``dot.sinkhorn(...)`` + ``backward()``,
   ``dot.sinkhorn_from_scores(...)``, ``dot.bidirectional_softmax(...)`` +
   ``backward()`` -- on small seeded inputs and writes inputs and outputs to
   ``tests/golden/*.npz``.

The fixtures pin the oracle (tests/test_oracle_golden.py) and the CUDA path
(tests/test_sinkhorn_gpu.py, tests/test_bidir_gpu.py).  The GPU box never runs
this script; it only reads the committed .npz files.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import textwrap

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("DOT_REF", "/root/reference")
SCRATCH = os.environ.get("DOT_REF_SCRATCH", "/tmp/dot_ref_golden")


def build_reference() -> str:
    """Build the reference CPU ops; return the package dir to put on sys.path."""
    from torch.utils.cpp_extension import load

    src = os.path.join(REF, "src")
    links = os.path.join(SCRATCH, "srcs")
    os.makedirs(links, exist_ok=True)
    sources = []
    for op in ("sinkhorn", "bidirectional_softmax"):
        for f in ("registry", "torch_cpu", "kernels_cpu"):
            dst = os.path.join(links, f"{op}_{f}.cpp")
            if not os.path.exists(dst):
                os.symlink(os.path.join(src, op, f + ".cpp"), dst)
            sources.append(dst)
    bdir = os.path.join(SCRATCH, "build")
    os.makedirs(bdir, exist_ok=True)
    load(name="_C", sources=sources, extra_include_paths=[src, os.path.join(src, "sinkhorn")],
         extra_cflags=["-O3", "-DUSE_TORCH_LIBRARY"], build_directory=bdir,
         is_python_module=False, verbose=False)
    pkg = os.path.join(SCRATCH, "pkg")
    if os.path.exists(pkg):
        shutil.rmtree(pkg)
    shutil.copytree(os.path.join(REF, "dot"), os.path.join(pkg, "dot"))
    shutil.copy(os.path.join(bdir, "_C.so"), os.path.join(pkg, "dot", "_C.so"))
    return pkg


CASES = textwrap.dedent(r'''
import numpy as np, torch, dot

def gen(seed):
    g = torch.Generator(device="cpu"); g.manual_seed(seed); return g

def sqdist_cost(B, n, m, d, seed):
    g = gen(seed)
    x = torch.randn(B, n, d, generator=g); y = torch.randn(B, m, d, generator=g)
    C = torch.cdist(x, y).square()
    return (C / C.amax(dim=(1, 2), keepdim=True)).float()

def dirichlet(B, n, seed):
    torch.manual_seed(seed)
    return torch.distributions.Dirichlet(torch.ones(n)).sample((B,)).float()

def run_sinkhorn(name, C, reg, n_iters, a=None, b=None, reg_tensor=False, plan_weight=None,
                 cost_weight=None, backward_iters=None, backward_mode=None):
    Cg = C.clone().requires_grad_(True)
    r = torch.tensor(float(reg), requires_grad=True) if reg_tensor else float(reg)
    kw = {}
    if backward_iters is not None:
        kw["backward_iters"] = backward_iters
    if backward_mode is not None:
        kw["backward_mode"] = backward_mode
    res = dot.sinkhorn(Cg, reg=r, n_iters=n_iters, a=a, b=b, **kw)
    cw = torch.ones_like(res.cost) if cost_weight is None else cost_weight
    loss = (res.cost * cw).sum()
    if plan_weight is not None:
        loss = loss + (res.transport_plan * plan_weight).sum()
    loss.backward()
    out = dict(C=C.numpy(), reg=np.float32(reg), n_iters=np.int64(n_iters),
               P=res.transport_plan.detach().numpy(), cost=res.cost.detach().numpy(),
               dC=Cg.grad.numpy(), cost_weight=cw.numpy(),
               n_iters_used=np.int64(res.n_iters_used), converged=np.bool_(res.converged))
    if backward_iters is not None:
        out["backward_iters"] = np.int64(backward_iters)
    if backward_mode is not None:
        out["backward_mode"] = np.array(backward_mode)
    if a is not None: out["a"] = a.numpy()
    if b is not None: out["b"] = b.numpy()
    if plan_weight is not None: out["plan_weight"] = plan_weight.numpy()
    if reg_tensor: out["dreg"] = np.float32(r.grad.item())
    np.savez_compressed(f"{OUT}/sinkhorn_{name}.npz", **out)

# BASELINE configs[0] (cfg1), exact
g = gen(0)
run_sinkhorn("cfg1", torch.rand(8, 64, 64, generator=g), 1.0, 100)
# reference test shapes (tests/test_sinkhorn.py:226-237), softmax marginals
g = gen(1)
C = torch.rand(2, 6, 9, generator=g)
a = torch.softmax(torch.randn(2, 6, generator=g), -1); b = torch.softmax(torch.randn(2, 9, generator=g), -1)
run_sinkhorn("refmatch", C, 0.7, 75, a, b)
# differentiable reg with Dirichlet marginals (cfg4 distribution, small)
g = gen(2)
run_sinkhorn("cfg4small", torch.rand(4, 128, 128, generator=g), 0.1, 100,
             dirichlet(4, 128, 3), dirichlet(4, 128, 4), reg_tensor=True)
# finite-difference known-answer case (tests/test_sinkhorn.py:400-416)
run_sinkhorn("eye5", torch.eye(5).unsqueeze(0), 0.2, 80, reg_tensor=True)
# ragged, odd sizes, rectangular both ways
g = gen(5)
run_sinkhorn("ragged", torch.rand(3, 33, 47, generator=g), 0.1, 60)
g = gen(6)
run_sinkhorn("tall", torch.rand(2, 70, 5, generator=g), 0.5, 40)
# plan used directly in the loss (grad_P path) plus a weighted cost
g = gen(7)
run_sinkhorn("planloss", torch.rand(2, 12, 20, generator=g), 0.3, 50,
             plan_weight=torch.randn(2, 12, 20, generator=g), cost_weight=torch.tensor([0.5, -1.5]))
# cfg2 distribution (normalised squared distances), small
run_sinkhorn("cfg2small", sqdist_cost(1, 128, 128, 64, 8), 0.05, 200)
# separate backward_iters
g = gen(9)
run_sinkhorn("bwditers", torch.rand(2, 24, 24, generator=g), 0.2, 30, backward_iters=7)
# 1-D marginals broadcast over the batch
g = gen(10)
run_sinkhorn("marg1d", torch.rand(3, 16, 8, generator=g), 0.4, 25,
             torch.softmax(torch.randn(16, generator=g), -1), torch.softmax(torch.randn(8, generator=g), -1))

# unrolled backward (backward_mode='unrolled'): plan and cost in the loss,
# differentiable reg; and non-uniform marginals
g = gen(12)
run_sinkhorn("unrolled", torch.rand(2, 20, 24, generator=g), 0.2, 30, reg_tensor=True,
             plan_weight=torch.randn(2, 20, 24, generator=g), cost_weight=torch.tensor([1.0, -0.5]),
             backward_mode="unrolled")
g = gen(13)
run_sinkhorn("unrolled_marg", torch.rand(2, 16, 12, generator=g), 0.3, 25,
             torch.softmax(torch.randn(2, 16, generator=g), -1), torch.softmax(torch.randn(2, 12, generator=g), -1),
             backward_mode="unrolled")

# sinkhorn_from_scores (plan and log-plan)
g = gen(11)
la = torch.randn(2, 10, 14, generator=g)
w = torch.randn(2, 10, 14, generator=g)
lag = la.clone().requires_grad_(True)
P = dot.sinkhorn_from_scores(lag, tau=0.5, n_iters=30)
(P * w).sum().backward()
logP = dot.sinkhorn_from_scores(la, tau=0.5, n_iters=30, return_log=True)
np.savez_compressed(f"{OUT}/scores_basic.npz", log_alpha=la.numpy(), tau=np.float32(0.5),
                    n_iters=np.int64(30), plan_weight=w.numpy(), P=P.detach().numpy(),
                    logP=logP.numpy(), dlog_alpha=lag.grad.numpy())

# bidirectional softmax
def run_bs(name, sim, tau, lengths=None, seed=0):
    g = gen(seed)
    grad_out = torch.randn(sim.shape, generator=g)
    s = sim.clone().requires_grad_(True)
    if lengths is None:
        out = dot.bidirectional_softmax(s, tau=tau)
    else:
        out = dot.bidirectional_softmax_with_lengths(s, lengths, tau=tau)
    (out * grad_out).sum().backward()
    d = dict(sim=sim.float().numpy() if sim.dtype != torch.bfloat16 else sim.view(torch.int16).numpy(),
             sim_dtype=np.array(str(sim.dtype)), tau=np.float32(tau), grad_out=grad_out.numpy(),
             out=out.detach().numpy(),
             grad=(s.grad.float().numpy() if s.grad.dtype != torch.bfloat16 else s.grad.view(torch.int16).numpy()),
             grad_dtype=np.array(str(s.grad.dtype)))
    if lengths is not None: d["lengths"] = lengths.numpy()
    np.savez_compressed(f"{OUT}/bidir_{name}.npz", **d)

g = gen(20)
run_bs("basic", torch.randn(2, 10, 15, generator=g), 1.0, seed=21)
g = gen(22)
run_bs("lengths", torch.randn(2, 10, 15, generator=g), 0.5,
       torch.tensor([[8, 12], [6, 10]], dtype=torch.int32), seed=23)
g = gen(24)
run_bs("cfg3small", torch.randn(2, 64, 96, generator=g), 0.1, seed=25)
g = gen(26)
run_bs("bf16", torch.randn(2, 32, 48, generator=g).bfloat16(), 0.1, seed=27)
sim = torch.zeros(1, 5, 5)
for i in range(5): sim[0, i, i] = 10.0
run_bs("diag", sim, 0.1, seed=28)
g = gen(29)
run_bs("lengths_edge", torch.randn(3, 7, 9, generator=g), 0.3,
       torch.tensor([[7, 9], [1, 1], [3, 9]], dtype=torch.int32), seed=30)
print("ok")
''')


def main() -> None:
    pkg = build_reference()
    env = dict(os.environ)
    env["PYTHONPATH"] = pkg
    code = f"OUT = {HERE!r}\n" + CASES
    subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=SCRATCH)


if __name__ == "__main__":
    main()
