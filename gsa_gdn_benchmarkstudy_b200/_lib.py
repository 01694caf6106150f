"""ctypes binding of ``libgsa_b200.so`` (the C ABI in ``include/gsa_b200.h``).

The library is the only compute path of this package: there is no CPU or
PyTorch fallback.  If the shared object is missing, or the current device is
not an sm_100 GPU, every call raises ``RuntimeError``.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgsa_b200.so"

GSA_OK = 0
GSA_DTYPE_BF16 = 0
GSA_DTYPE_F32 = 1
GSA_FUSED_AUTO, GSA_FUSED_ALWAYS, GSA_FUSED_NEVER = 0, 1, 2

# Every exported symbol of include/gsa_b200.h with (restype, argtypes).
_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
SIGNATURES: dict[str, tuple] = {
    "gsa_version": (_i32, []),
    "gsa_set_fused_selection": (_i32, [_i32]),
    "gsa_status_string": (ctypes.c_char_p, [_i32]),
    "gsa_last_error_string": (ctypes.c_char_p, []),
    "gsa_device_error": (_i32, [ctypes.POINTER(_i32), _i32]),
    "gsa_bitmask_words": (_i64, [_i32]),
    "gsa_rope_gates": (
        _i32,
        [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "gsa_indexer_scores": (
        _i32,
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _f32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _vp, _i64, _i32, _vp],
    ),
    "gsa_indexer_topk_workspace_size": (_i64, [_i32, _i32, _i32]),
    "gsa_indexer_topk": (
        _i32,
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _f32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i32, _vp, _i64, _vp, _vp, _vp, _i64, _vp],
    ),
    "gsa_indexer_topk_noalloc": (
        _i32,
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _f32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i32, _vp, _vp, _vp, _i64, _vp],
    ),
    "gsa_topk_select": (
        _i32,
        [_vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _i64, _vp],
    ),
    "gsa_row_variance": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp]),
    "gsa_adaptive_k_width": (_i32, [_i32, _i32]),
    "gsa_topk_select_adaptive": (
        _i32,
        [_vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _vp,
         _vp, _i64, _vp],
    ),
    "gsa_indexer_topk_adaptive_workspace_size": (_i64, [_i32, _i32, _i32]),
    "gsa_indexer_topk_adaptive": (
        _i32,
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _f32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i32, _i32, _i32, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp],
    ),
    "gsa_masked_attention": (
        _i32,
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _f32, _i32, _i32,
         _i32, _i32, _i32, _i32, _vp],
    ),
    "gsa_gather_attention": (
        _i32,
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _vp, _i64, _f32, _i32, _i32, _i32,
         _i32, _i32, _i32, _vp],
    ),
    "gsa_output_gate": (
        _i32,
        [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp],
    ),
    "gsa_fused_projection": (
        _i32,
        [_vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _i64,
         _vp, _vp, _vp, _vp, _i64, _vp],
    ),
    "gsa_fused_projection_rows": (_i64, [_i32, _i32, _i32]),
    "gsa_fused_projection_rest_width": (_i64, [_i32, _i32, _i32]),
    "gsa_fused_projection_pack": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load the shared library (once) and attach the C signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p.name} is not built: run `python -m gsa_gdn_benchmarkstudy_b200.build` "
                "(there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def status_string(rc: int) -> str:
    return load().gsa_status_string(rc).decode()


def last_error() -> str:
    return load().gsa_last_error_string().decode()


def check(rc: int, what: str) -> None:
    """Raise RuntimeError for a non-zero gsa_status_t."""
    if rc != GSA_OK:
        raise RuntimeError(f"{what} failed: {status_string(rc)} ({last_error()})")


def device_error(reset: bool = True) -> int:
    """Synchronise and return the device-side error word (0 = none)."""
    out = ctypes.c_int(0)
    check(load().gsa_device_error(ctypes.byref(out), 1 if reset else 0), "gsa_device_error")
    return out.value


@contextlib.contextmanager
def fused_selection(mode: int):
    """Inside the block, gsa_indexer_topk uses the given selection
    (GSA_FUSED_ALWAYS / GSA_FUSED_NEVER / GSA_FUSED_AUTO) process-wide; the
    automatic choice is restored afterwards."""
    check(load().gsa_set_fused_selection(int(mode)), "gsa_set_fused_selection")
    try:
        yield
    finally:
        check(load().gsa_set_fused_selection(GSA_FUSED_AUTO), "gsa_set_fused_selection")
