"""ctypes binding of ``libeinsparse.so`` (the C ABI declared in ``include/einsparse.h``).

There is no fallback: if the shared library is missing or fails to load,
``lib()`` raises ``EinsparseUnavailable``. Device buffers come from torch's
caching allocator and are passed as raw pointers; every call runs on torch's
current CUDA stream.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("EINSPARSE_LIB", os.path.join(HERE, "libeinsparse.so"))

ES_OK, ES_ERR_INVALID, ES_ERR_INDEX, ES_ERR_WORKSPACE, ES_ERR_CUDA, ES_ERR_UNSUPPORTED, ES_ERR_TIMEOUT = range(7)
ES_F32, ES_BF16, ES_F64, ES_I32, ES_I64 = range(5)
ES_PREC_AUTO, ES_PREC_EXACT, ES_PREC_TC = range(3)
ES_DUP_LAST, ES_DUP_SUM = range(2)

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_vp = ctypes.c_void_p
c_sz = ctypes.c_size_t
c_i64p = ctypes.POINTER(ctypes.c_int64)
c_i32p = ctypes.POINTER(ctypes.c_int32)

# name -> (restype, argtypes); pointers to device memory are c_void_p,
# host arrays (shape, tile, keys) are POINTER types.
SIGNATURES = {
    "es_version": (c_int, []),
    "es_launch_count": (c_i64, []),
    "es_launch_count_reset": (None, []),
    "es_status_string": (ctypes.c_char_p, [c_int]),
    "es_tile_coo_workspace_size": (c_sz, [c_i64, c_int, c_i64p, c_i64p]),
    "es_tile_coo_plan": (c_int, [c_vp, c_vp, c_int, c_i64, c_int, c_i64p, c_i64p, c_vp, c_sz, c_vp, c_vp, c_vp]),
    "es_tile_coo_fill": (c_int, [c_vp, c_int, c_i64, c_int, c_i64p, c_i64p, c_vp, c_sz, c_i64, c_vp, c_vp, c_int,
                                 c_vp]),
    "es_coo_coalesce_workspace_size": (c_sz, [c_i64, c_int, c_i64p]),
    "es_coo_coalesce": (c_int, [c_vp, c_vp, c_int, c_i64, c_int, c_i64p, c_int, c_vp, c_sz, c_vp, c_vp, c_int, c_vp,
                                c_vp, c_vp]),
    "es_tile_dense_workspace_size": (c_sz, [c_int, c_i64p, c_i64p]),
    "es_tile_dense_plan": (c_int, [c_vp, c_int, c_int, c_i64p, c_i64p, c_vp, c_sz, c_vp, c_vp]),
    "es_tile_dense_fill": (c_int, [c_vp, c_int, c_int, c_i64p, c_i64p, c_vp, c_sz, c_i64, c_vp, c_vp, c_int, c_vp]),
    "es_join_workspace_size": (c_sz, [c_i64, c_i64]),
    "es_join_plan": (c_int, [c_vp, c_i64, c_int, c_vp, c_i64, c_int, c_i32p, c_int, c_i64p, c_vp, c_sz, c_vp, c_vp,
                             c_vp]),
    "es_join_fill": (c_int, [c_i64, c_i64, c_int, c_vp, c_sz, c_i64, c_vp, c_vp, c_int, c_vp]),
    "es_join_static": (c_int, [c_vp, c_i64, c_int, c_vp, c_i64, c_int, c_i32p, c_int, c_i64p, c_vp, c_vp, c_int, c_i64,
                               c_vp, c_vp, c_vp]),
    "es_segments_workspace_size": (c_sz, [c_i64]),
    "es_segments_plan": (c_int, [c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_i64, c_i32p, c_int, c_i64p, c_vp, c_sz,
                                 c_vp, c_vp, c_vp]),
    "es_segments_fill": (c_int, [c_vp, c_vp, c_i64, c_int, c_i64p, c_vp, c_sz, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp,
                                 c_int, c_vp, c_vp]),
    "es_output_coords": (c_int, [c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_i64, c_i32p, c_int, c_vp, c_vp]),
    "es_direct_workspace_size": (c_sz, [c_i64, c_int, c_i64, c_int, c_int, c_i64p, c_i64p]),
    "es_direct_plan": (c_int, [c_vp, c_i64, c_int, c_vp, c_i64, c_int, c_int, c_i64p, c_i64p, c_vp, c_sz, c_vp, c_vp,
                               c_vp]),
    "es_direct_fill": (c_int, [c_vp, c_i64, c_int, c_i64, c_int, c_int, c_i64p, c_i64p, c_vp, c_sz, c_i64, c_i64, c_vp,
                               c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "es_tile_einsum_workspace_size": (c_sz, [ctypes.c_char_p, c_i64p, c_int, c_i64p, c_int, c_int, c_int, c_i64,
                                              c_i64, c_i64, c_i64, c_i64, c_int]),
    "es_tile_einsum": (c_int, [ctypes.c_char_p, c_i64p, c_int, c_i64p, c_int, c_vp, c_int, c_i64, c_vp, c_int, c_i64,
                               c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_int, c_int, c_vp,
                               c_sz, c_vp, c_vp]),
    "es_tile_einsum_ev": (c_int, [ctypes.c_char_p, c_i64p, c_int, c_i64p, c_int, c_vp, c_int, c_i64, c_vp, c_int,
                                  c_i64, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_int, c_int,
                                  c_vp, c_sz, c_vp, c_vp, c_vp, c_vp]),
    "es_tile_einsum_path": (c_int, [ctypes.c_char_p, c_i64p, c_int, c_i64p, c_int, c_int, c_int, c_int]),
    "es_out_tile_shape": (c_int, [ctypes.c_char_p, c_i64p, c_int, c_i64p, c_int, c_i64p]),
    "es_segsum_workspace_size": (c_sz, [c_i64]),
    "es_sparsity_stats_workspace_size": (c_sz, [c_i64, c_int, c_i64p, c_i64p, c_int]),
    "es_sparsity_stats": (c_int, [c_vp, c_vp, c_int, c_i64, c_int, c_i64p, c_i64p, c_int, c_vp, c_sz, c_vp, c_vp, c_vp,
                                  c_vp]),
    "es_segsum_plan": (c_int, [c_vp, c_i64, c_int, c_i64p, c_vp, c_sz, c_vp, c_vp, c_vp]),
    "es_segsum_fill": (c_int, [c_vp, c_int, c_i64, c_i64, c_int, c_i64p, c_vp, c_sz, c_i64, c_vp, c_vp, c_int, c_vp]),
    "es_segsum_groups": (c_int, [c_i64, c_int, c_i64p, c_vp, c_sz, c_i64, c_vp, c_vp, c_vp]),
    "es_scatter_add_workspace_size": (c_sz, [c_i64]),
    "es_scatter_add_rows": (c_int, [c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_sz, c_vp, c_vp, c_vp]),
}


class EinsparseUnavailable(RuntimeError):
    """The native library could not be loaded; there is no CPU fallback."""


class EinsparseError(RuntimeError):
    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: {msg} (status {status})")
        self.status = status


_LIB = None
_LOCK = threading.Lock()


def load(path: str = LIB_PATH):
    """Load the library and bind every symbol of ``SIGNATURES``."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not os.path.exists(path):
            raise EinsparseUnavailable(
                f"{path} not found; build it with `python -m einjax_b200.build` (nvcc, sm_100a)")
        try:
            lib = ctypes.CDLL(path)
        except OSError as e:  # pragma: no cover
            raise EinsparseUnavailable(f"cannot load {path}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
        return lib


def lib():
    return _LIB if _LIB is not None else load()


def i64arr(vals):
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)


def i32arr(vals):
    vals = [int(v) for v in vals]
    return (ctypes.c_int32 * max(1, len(vals)))(*vals)


def device_error(fn: str, err: int, msg: str):
    """Raise for a non-zero device-side error slot (read with the counts): a
    bounded device wait that ran out (ES_ERR_TIMEOUT, outputs invalid) raises
    EinsparseError; anything else is a bad input and raises ValueError(msg)."""
    e = int(err) & 0xFFFFFFFF
    if e == ES_OK:
        return
    if e == ES_ERR_TIMEOUT:
        raise EinsparseError(fn, e, lib().es_status_string(e).decode())
    raise ValueError(msg)


def check(fn: str, status: int):
    if status != ES_OK:
        msg = lib().es_status_string(status).decode()
        if status in (ES_ERR_INVALID, ES_ERR_INDEX):
            raise ValueError(f"{fn}: {msg}")
        raise EinsparseError(fn, status, msg)


def _dtype_code(dt) -> int:
    import torch
    return {torch.float32: ES_F32, torch.bfloat16: ES_BF16, torch.float64: ES_F64}[dt]
