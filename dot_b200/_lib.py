"""Loader for the dot_b200 C-ABI library (``_lib/libdot_b200.so``).

The library is built in-tree by :mod:`dot_b200.build`.  Importing the package
loads it; if it is missing or was built for another ABI version the import
fails loudly -- there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libdot_b200.so")
ABI_VERSION = 1

DOT_F32, DOT_BF16, DOT_F16 = 0, 1, 2
KCLASSES = ("sk_fwd_iter", "sk_fwd_epi", "sk_bwd_iter", "sk_bwd_epi", "sk_resident", "bs_fwd", "bs_bwd",
            "sk_exchange")

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_f = ctypes.c_float
_i = ctypes.c_int
_sz = ctypes.c_size_t

_SIGS = {
    "dot_last_error": (ctypes.c_char_p, []),
    "dot_abi_version": (_i, []),
    "dot_sinkhorn_fwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _i, _f, _i]),
    "dot_sinkhorn_fwd": (_i, [_vp, _f, _vp, _vp, _i64, _i64, _i64, _f, _i, _f, _i, _vp, _vp, _vp, _vp, _vp,
                              _vp, _sz, _vp]),
    "dot_sinkhorn_fwd_noalloc": (_i, [_vp, _f, _vp, _vp, _i64, _i64, _i64, _f, _i, _f, _i, _vp, _vp, _vp, _vp,
                                      _vp, _vp]),
    "dot_sinkhorn_bwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _i]),
    "dot_sinkhorn_bwd": (_i, [_vp, _f, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f, _i, _vp, _vp, _vp, _sz,
                              _vp]),
    "dot_sinkhorn_fwd_hist": (_i, [_vp, _f, _vp, _vp, _i64, _i64, _i64, _f, _i, _f, _vp, _vp, _vp, _vp, _vp, _vp,
                                   _vp, _vp, _sz, _vp]),
    "dot_sinkhorn_bwd_unrolled_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "dot_sinkhorn_bwd_unrolled": (_i, [_vp, _f, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f, _i, _vp, _vp, _vp,
                                       _sz, _vp]),
    "dot_sinkhorn_rows_colpairs_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "dot_sinkhorn_rows_colpairs": (_i, [_vp, _f, _vp, _i64, _i64, _i64, _i64, _f, _vp, _vp, _vp, _vp, _vp, _sz,
                                        _vp]),
    "dot_sinkhorn_col_merge": (_i, [_vp, _i, _vp, _i64, _i64, _vp, _vp]),
    "dot_sinkhorn_plan_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "dot_sinkhorn_plan": (_i, [_vp, _f, _vp, _vp, _i64, _i64, _i64, _f, _i, _vp, _vp, _vp, _sz, _vp]),
    "dot_sinkhorn_fwd_rowshard_workspace_bytes": (_sz, [_i64, _i64, _i64, _i]),
    "dot_sinkhorn_fwd_rowshard": (_i, [_vp, _f, _vp, _vp, _i64, _i64, _i64, _i64, _f, _i, _vp, _vp, _vp, _vp, _vp,
                                       _vp, _vp, _sz, _vp]),
    "dot_sq_dist": (_i, [_vp, _vp, _i64, _i64, _i64, _i, _f, _vp, _vp]),
    "dot_sinkhorn_points_fwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _i, _i, _f, _i, _i]),
    "dot_sinkhorn_points_fwd": (_i, [_vp, _vp, _i64, _i64, _i64, _i, _f, _vp, _vp, _f, _i, _f, _vp, _vp, _vp, _vp,
                                     _vp, _vp, _sz, _vp]),
    "dot_sinkhorn_points_fwd_rowshard_workspace_bytes": (_sz, [_i64, _i64, _i64, _i, _i]),
    "dot_sinkhorn_points_fwd_rowshard": (_i, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i, _i64, _f, _f, _i, _vp, _vp,
                                              _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "dot_nccl_unique_id": (_i, [_vp]),
    "dot_nccl_comm_init": (_i, [ctypes.POINTER(_vp), _i, _vp, _i]),
    "dot_nccl_comm_destroy": (_i, [_vp]),
    "dot_bidir_fwd_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "dot_bidir_fwd": (_i, [_vp, _i, _vp, _i64, _i64, _i64, _f, _vp, _vp, _vp, _vp, _sz, _vp]),
    "dot_bidir_bwd_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "dot_bidir_bwd": (_i, [_vp, _i, _vp, _i64, _i64, _i64, _f, _vp, _vp, _vp, _vp, _i, _vp, _vp, _sz, _vp]),
    "dot_prof_begin": (_i, [_i]),
    "dot_prof_end": (_i, [ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_double)]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"dot_b200: native library not found at {LIB_PATH}; build it with "
            "`python dot_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.dot_abi_version() != ABI_VERSION:
        raise ImportError(f"dot_b200: library ABI {lib.dot_abi_version()} != expected {ABI_VERSION}")
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().dot_last_error().decode(errors="replace")
        if rc == -4:
            raise NotImplementedError(f"{what}: {msg}")
        if rc == -1:
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


def ptr(t: torch.Tensor | None):
    return None if t is None else _vp(t.data_ptr())


def stream_of(t: torch.Tensor):
    return _vp(torch.cuda.current_stream(t.device).cuda_stream)


def workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def prof_begin(time_events: bool = False) -> None:
    check(load().dot_prof_begin(1 if time_events else 0), "dot_prof_begin")


def prof_end() -> dict:
    """Launch counts and (if timed) summed milliseconds per kernel class."""
    n = len(KCLASSES)
    launches = (ctypes.c_int64 * n)()
    ms = (ctypes.c_double * n)()
    check(load().dot_prof_end(launches, ms), "dot_prof_end")
    return {k: {"launches": int(launches[i]), "ms": float(ms[i])} for i, k in enumerate(KCLASSES)}
