"""The C-ABI library loads and exports every symbol include/dot_b200.h declares;
argument validation and workspace queries work without a GPU."""

import ctypes
import os
import re
import subprocess

import pytest

import dot_b200
from dot_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dot_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^DOT_API\s+[\w\s\*]+?\b(dot_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ["dot_sinkhorn_fwd", "dot_sinkhorn_bwd", "dot_bidir_fwd", "dot_bidir_bwd", "dot_last_error"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (dot_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"not exported: {missing}"
    lib = _lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s)
    assert set(_lib.exported_symbols()) == set(declared_symbols())


def test_abi_version():
    assert _lib.load().dot_abi_version() == 1


def test_workspace_queries():
    lib = _lib.load()
    assert lib.dot_sinkhorn_fwd_workspace_bytes(0, 4, 4, 10, 0.0, 1) == 0
    ws = lib.dot_sinkhorn_fwd_workspace_bytes(2, 2048, 64, 10, 1e-6, 1)
    assert ws >= 2 * 4 * 64 * 8  # column partials for 4 row chunks
    assert lib.dot_sinkhorn_bwd_workspace_bytes(2, 8, 8, 5) > 0
    assert lib.dot_bidir_bwd_workspace_bytes(2, 8, 8) > 0


@pytest.mark.parametrize("tau,iters,sign,mode,code", [
    (0.0, 10, -1.0, 0, -1), (-1.0, 10, -1.0, 0, -1), (float("nan"), 10, -1.0, 0, -1),
    (1.0, -1, -1.0, 0, -1), (1.0, 10, 0.5, 0, -1), (1.0, 10, -1.0, 3, -1)])
def test_sinkhorn_fwd_rejects_bad_arguments(tau, iters, sign, mode, code):
    lib = _lib.load()
    rc = lib.dot_sinkhorn_fwd(None, sign, None, None, 1, 4, 4, tau, iters, 0.0, mode, None, None, None, None,
                              None, None, 0, None)
    assert rc == code
    assert lib.dot_last_error().decode()


def test_null_pointers_and_workspace_are_rejected():
    lib = _lib.load()
    rc = lib.dot_sinkhorn_fwd(None, -1.0, None, None, 1, 4, 4, 1.0, 10, 0.0, 0, None, None, None, None, None,
                              None, 0, None)
    assert rc == -1 and "null" in lib.dot_last_error().decode()
    dummy = ctypes.c_void_p(16)
    rc = lib.dot_sinkhorn_fwd(dummy, -1.0, None, None, 1, 4, 4, 1.0, 10, 0.0, 0, dummy, dummy, dummy, dummy, dummy,
                              None, 0, None)
    assert rc == -3 and "workspace" in lib.dot_last_error().decode()


def test_empty_problems_are_noops():
    lib = _lib.load()
    assert lib.dot_sinkhorn_fwd(None, -1.0, None, None, 0, 4, 4, 1.0, 10, 0.0, 0, None, None, None, None, None,
                                None, 0, None) == 0
    assert lib.dot_bidir_fwd(None, 0, None, 3, 0, 5, 1.0, None, None, None, None, 0, None) == 0


def test_bidir_rejects_bad_dtype_and_tau():
    lib = _lib.load()
    assert lib.dot_bidir_fwd(None, 7, None, 1, 4, 4, 1.0, None, None, None, None, 0, None) == -4
    assert lib.dot_bidir_fwd(None, 0, None, 1, 4, 4, 0.0, None, None, None, None, 0, None) == -1


def test_error_text_is_per_call():
    lib = _lib.load()
    lib.dot_bidir_fwd(None, 0, None, 1, 4, 4, 0.0, None, None, None, None, 0, None)
    assert lib.dot_last_error().decode()
    assert lib.dot_bidir_fwd(None, 0, None, 0, 4, 4, 1.0, None, None, None, None, 0, None) == 0
    assert lib.dot_last_error().decode() == ""


def test_prof_counters_start_at_zero():
    _lib.prof_begin(False)
    res = _lib.prof_end()
    assert set(res) == set(_lib.KCLASSES)
    assert all(v["launches"] == 0 for v in res.values())


def test_package_surface_matches_reference():
    import dot

    for name in ["sinkhorn", "sinkhorn_from_scores", "spectral_preflight", "SinkhornResult", "Sinkhorn",
                 "SinkhornFromScores", "bidirectional_softmax", "bidirectional_softmax_with_lengths",
                 "BidirectionalSoftmax"]:
        assert hasattr(dot, name) and hasattr(dot_b200, name)
    for name in ["sinkhorn", "sinkhorn_log", "sinkhorn_dual_forward", "sinkhorn_spectral_preflight",
                 "sinkhorn_with_grads_unrolled", "sinkhorn_with_grads_implicit", "bidirectional_softmax",
                 "bidirectional_softmax_backward"]:
        assert hasattr(dot._ops, name)
