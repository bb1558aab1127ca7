"""ctypes binding of libxspmm_b200.so (the C ABI declared in include/xspmm_b200.h).

Loading fails loudly when the library has not been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libxspmm_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "xspmm_b200.h")

STATUS = {
    0: "OK", 1: "INVALID_ARGUMENT", 2: "UNSUPPORTED", 3: "CUDA_ERROR", 4: "OUT_OF_MEMORY",
    5: "NCCL_ERROR", 6: "TIMEOUT", 7: "INTERNAL",
}


class XSpMMError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class Timings(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in (
        "clustering_ms", "permutation_ms", "conversion_ms", "spmm_ms", "unpermutation_ms",
        "total_pipeline_ms")]


class DistPlanInfo(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("row_begin", ctypes.c_int64), ("row_end", ctypes.c_int64),
                ("block_begin", ctypes.c_int64), ("block_end", ctypes.c_int64),
                ("nnz_blocks", ctypes.c_int64), ("nnz_blocks_total", ctypes.c_int64),
                ("clustered", ctypes.c_int32), ("value_bytes", ctypes.c_int32),
                ("device_bytes", ctypes.c_int64)]


class PlanInfo(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("block_rows", ctypes.c_int64), ("block_cols", ctypes.c_int64),
                ("nnz_blocks", ctypes.c_int64), ("clustered", ctypes.c_int32),
                ("value_bytes", ctypes.c_int32), ("tcgen05_ready", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("tcgen05_tiles", ctypes.c_int64),
                ("device_bytes", ctypes.c_int64)]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float

_lib = None


def _sig(IT):
    return {
        "bcsr_spmm": [_P, IT, IT, IT, IT, IT, _P, _P, _P, _P, _P, IT, IT, IT, _P],
        "cluster": [_P, IT, IT, IT, _P, _P, _F, IT, _P],
        "permute": [_P, IT, IT, IT, _P, _P, _P, _P, _P, _P, _P],
        "count": [_P, IT, IT, IT, _P, _P, IT, IT, _P, _P],
        "fill": [_P, IT, IT, IT, _P, _P, _P, IT, IT, _P, _P, _P],
        "unpermute": [_P, _P, _P, _P, IT, IT],
        "pipeline": [_P, IT, IT, IT, _P, _P, _P, _P, _P, IT, IT, ctypes.c_int, _P],
        "plan_csr": [_P, IT, IT, IT, _P, _P, _P, IT, ctypes.c_int, ctypes.POINTER(_P), _P],
        "plan_bcsr": [_P, IT, IT, IT, IT, IT, _P, _P, _P, IT, IT, ctypes.POINTER(_P)],
    }


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build the CUDA library first (python -m xspmm_b200.build). "
            "xspmm_b200 has no CPU fallback.")
    L = ctypes.CDLL(LIB_PATH)
    L.xspmm_create.argtypes = [ctypes.c_int, _P, ctypes.POINTER(_P)]
    L.xspmm_destroy.argtypes = [_P]
    L.xspmm_set_stream.argtypes = [_P, _P]
    L.xspmm_get_device.argtypes = [_P, ctypes.POINTER(ctypes.c_int)]
    L.xspmm_get_launch_count.argtypes = [_P, ctypes.POINTER(ctypes.c_uint64)]
    L.xspmm_reset_launch_count.argtypes = [_P]
    L.xspmm_set_tier1_kernel.argtypes = [_P, ctypes.c_int]
    L.xspmm_status_string.argtypes = [ctypes.c_int]
    L.xspmm_status_string.restype = ctypes.c_char_p
    L.xspmm_last_error.argtypes = []
    L.xspmm_last_error.restype = ctypes.c_char_p
    L.xspmm_malloc.argtypes = [_P, ctypes.POINTER(_P), ctypes.c_size_t]
    L.xspmm_free.argtypes = [_P, _P]
    for k in ("h2d", "d2h", "d2d"):
        getattr(L, "xspmm_memcpy_" + k).argtypes = [_P, _P, _P, ctypes.c_size_t]
    L.xspmm_synchronize.argtypes = [_P]
    for suf, IT in (("i32", _I32), ("i64", _I64)):
        s = _sig(IT)
        for vt in ("f16f32", "bf16f32", "f32f32"):
            getattr(L, f"xspmm_bcsr_spmm_{vt}_{suf}").argtypes = s["bcsr_spmm"]
            getattr(L, f"xspmm_spmm_csr_{vt}_{suf}").argtypes = s["pipeline"]
            getattr(L, f"xspmm_plan_csr_{vt}_{suf}").argtypes = s["plan_csr"]
            getattr(L, f"xspmm_plan_bcsr_{vt}_{suf}").argtypes = s["plan_bcsr"]
        getattr(L, f"xspmm_cluster_jaccard_{suf}").argtypes = s["cluster"]
        getattr(L, f"xspmm_csr_to_bcsr_count_{suf}").argtypes = s["count"]
        for v in ("f16", "bf16", "f32"):
            getattr(L, f"xspmm_permute_rows_{v}_{suf}").argtypes = s["permute"]
            getattr(L, f"xspmm_csr_to_bcsr_fill_{v}_{suf}").argtypes = s["fill"]
            getattr(L, f"xspmm_unpermute_dense_{v}_{suf}").argtypes = s["unpermute"]
    L.xspmm_plan_execute.argtypes = [_P, _P, _P, _I64]
    L.xspmm_plan_get_info.argtypes = [_P, ctypes.POINTER(PlanInfo)]
    L.xspmm_plan_destroy.argtypes = [_P]
    L.xspmm_permute_rows_noalloc_i32.argtypes = [_P, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _P,
                                                  _P, _P]
    L.xspmm_dist_partition.argtypes = [_P, _I64, _I32, ctypes.c_double, _P]
    L.xspmm_dist_unique_id.argtypes = [_P, _I32]
    L.xspmm_dist_comm_init.argtypes = [_P, _I32, _I32, _P, _I32, _I32, ctypes.POINTER(_P)]
    L.xspmm_dist_comm_wrap.argtypes = [_P, _I32, ctypes.POINTER(_P)]
    L.xspmm_dist_comm_destroy.argtypes = [_P]
    for suf, IT in (("i32", _I32), ("i64", _I64)):
        for vt in ("f16f32", "bf16f32", "f32f32"):
            getattr(L, f"xspmm_dist_plan_csr_{vt}_{suf}").argtypes = [
                _P, _P, IT, IT, IT, _P, _P, _P, IT, ctypes.c_int, ctypes.c_double,
                ctypes.POINTER(_P)]
    L.xspmm_dist_plan_get_info.argtypes = [_P, ctypes.POINTER(DistPlanInfo)]
    L.xspmm_dist_plan_execute.argtypes = [_P, _P, _P, _I64, _I32, _I32]
    L.xspmm_dist_gather.argtypes = [_P, _P, _P, _I64, _I32, _I32]
    L.xspmm_dist_plan_destroy.argtypes = [_P]
    _lib = L
    return L


def check(status: int) -> None:
    if status != 0:
        msg = lib().xspmm_last_error().decode(errors="replace")
        raise XSpMMError(status, msg)


def declared_symbols() -> list[str]:
    """Every function the C header declares (used by the ABI export test)."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(xspmm_\w+)\s*\(", text)))
