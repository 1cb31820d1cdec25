"""Build the dot_b200 C-ABI library for sm_100a with nvcc (in-tree).

``python dot_b200/build.py`` compiles every ``csrc/*.cu`` (in parallel, one
object per source under ``dot_b200/_lib/obj``) and links them into
``dot_b200/_lib/libdot_b200.so``, with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``.  The CUDA runtime is
linked statically so the library carries no dependency beyond the driver
(NCCL, used only by the row-sharded solver, is loaded at run time).
The build is skipped when the library is newer than every source.
"""

from __future__ import annotations

import glob
import os
from concurrent.futures import ThreadPoolExecutor
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIB_DIR, "libdot_b200.so")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(HERE, "csrc", "*.h")) + glob.glob(
        os.path.join(HERE, "csrc", "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    obj_dir = os.path.join(LIB_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    flags = [ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
             "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]
    nvcc = _nvcc()

    def compile_one(src: str) -> str:
        obj = os.path.join(obj_dir, os.path.splitext(os.path.basename(src))[0] + ".o")
        cmd = [nvcc] + flags + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [nvcc, ARCH, "-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
