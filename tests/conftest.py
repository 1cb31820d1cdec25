"""Shared pytest setup.

Markers: ``gpu`` -- needs a CUDA device (run on the B200 box with ``-m gpu``);
everything else runs on CPU.  The native library and the CPU oracle are built
once per session if they are missing or stale (nvcc / gcc are in the image).
"""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200)")
    import importlib.util

    # load dot_b200/build.py by path: importing the package loads the library
    spec = importlib.util.spec_from_file_location("_dot_b200_build", os.path.join(ROOT, "dot_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    if not os.path.exists(os.path.join(ROOT, "oracle", "_build", "liboracle.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
