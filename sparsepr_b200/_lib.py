"""ctypes binding of ``libsparsepr_b200.so`` (the C ABI in ``include/sparsepr_b200.h``).

The library is built in-tree by ``sparsepr_b200.build``.  Loading is lazy; a
missing library raises ``RuntimeError`` (there is no fallback path).
"""

from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsparsepr_b200.so")

SPR_OK = 0
STATUS_NAMES = {
    -1: "SPR_ERR_SHAPE", -2: "SPR_ERR_DTYPE", -3: "SPR_ERR_ALIGN", -4: "SPR_ERR_LAUNCH",
    -5: "SPR_ERR_TIMEOUT", -6: "SPR_ERR_UNIMPLEMENTED", -7: "SPR_ERR_WORKSPACE", -8: "SPR_ERR_ARG",
}
SPR_F32, SPR_BF16, SPR_F16 = 0, 1, 2
PRECISION = {"tf32": 0, "fp32": 1}

_P = C.c_void_p
_I = C.c_int
_I64 = C.c_int64
_F = C.c_float
_SZ = C.c_size_t

# name -> (restype, argtypes); mirrors include/sparsepr_b200.h exactly.
PROTOTYPES = {
    "spr_version": (_I, []),
    "spr_last_error": (C.c_char_p, []),
    "spr_kmeans_workspace_bytes": (_SZ, [_I64, _I64, _I, _I]),
    "spr_kmeans_lloyd": (_I, [_P, _I, _I64, _I64, _I, _I, _I, _F, _I, _I, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "spr_kmeans_assign": (_I, [_P, _I, _I64, _I64, _I, _I, _P, _I, _P, _P, _SZ, _P]),
    "spr_label_sort": (_I, [_P, _I64, _I64, _I, _P, _P, _P, _P, _SZ, _P]),
    "spr_centroid_means": (_I, [_P, _I, _P, _P, _I64, _I64, _I, _I, _P, _P, _P, _P]),
    "spr_permute_rows": (_I, [_P, _P, _P, _I64, _I64, _I, _I, _I, _P]),
    "spr_attention_mass_scores": (_I, [_P, _P, _P, _I64, _I, _I, _I64, _I, _P, _P]),
    "spr_attention_mass_scores_status": (_I, [_P]),
    "spr_attention_mass_scores_status_async": (_I, [_P, _P]),
    "spr_role_projection_workspace_bytes": (_SZ, [_I64, _I64, _I]),
    "spr_role_projection": (_I, [_P, _P, _I64, _I64, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "spr_role_projection_status": (_I, [_P]),
    "spr_role_projection_status_async": (_I, [_P, _P]),
    "spr_probe_representatives": (_I, [_P, _P, _P, _I64, _I64, _I, _I, _P, _P]),
    "spr_cholesky_qr": (_I, [_P, _I64, _I, _I, C.c_float, _P, _P, _P]),
    "spr_ridge_cholesky": (_I, [_P, _P, _I64, _I, C.c_float, C.c_float, _P, _P, _P]),
    "spr_svg_ear_value_scores_workspace_bytes": (_SZ, [_I64, _I, _I, _I64]),
    "spr_svg_ear_value_scores": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I, _I, _I64, _I, _P, _P, _SZ, _P]),
    "spr_wan_qkv_norm_rope_layout": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I, _I, C.c_float, _P, _P,
                                          _P, _P]),
    "spr_select_budget": (_I, [_P, _P, _P, _I64, _I, _I, _P, _P, _P, _P]),
    "spr_block_sparse_attn": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _P, _P, _SZ,
                                   _P]),
    "spr_probe_rows_attn_workspace_bytes": (_SZ, [_I64, _I64, _I]),
    "spr_probe_rows_attn": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "spr_block_sparse_attn_workspace_bytes": (_SZ, [_I64, _I64, _I]),
    "spr_block_sparse_attn_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _P]),
    "spr_block_sparse_attn_noalloc_status": (_I, [_P]),
    "spr_selftest_bounded_wait": (_I, [_P, _I, _I64, _P]),
    "spr_sym_eig": (_I, [_P, _I64, _I, _I, _P, _P, _P]),
    "spr_sym_eig_top": (_I, [_P, _I64, _I, _I, _I, _P, _P, _P]),
    "spr_chol_solve": (_I, [_P, _P, _I64, _I, _I, _P, _P]),
    "spr_repair_apply": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _F, _P, _P, _I, _P, _P]),
}

class SprRepairState(C.Structure):
    """``SprRepairState`` of include/sparsepr_b200.h (device pointers)."""

    _fields_ = [("x_mean", _P), ("x_scale", _P), ("y_mean", _P), ("left", _P), ("basis", _P), ("rank", _I),
                ("alpha", _F), ("probe_rows", _P), ("probe_dense", _P), ("m", _I)]


_lock = threading.Lock()
_lib = None


def load(path: str | None = None):
    """Load the shared library once and bind every prototype."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"sparsepr_b200 native library not found at {p}; build it with "
                "`python -m sparsepr_b200.build` (there is no CPU fallback)."
            )
        lib = C.CDLL(p)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def call(name: str, *args) -> int:
    """Invoke an entry point; a non-zero status raises RuntimeError with the library message."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != SPR_OK:
        msg = lib.spr_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed with {STATUS_NAMES.get(status, status)}: {msg}")
    return status


def query(name: str, *args):
    """Invoke a non-status entry point (sizes, version)."""
    return getattr(load(), name)(*args)
