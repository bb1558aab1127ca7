"""CPU checkers for the xSpMM hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this package, and
only to check GPU results or to time the CPU path beside the GPU. The xspmm_b200 product never
imports it; a product call that reached this code would be a CPU fallback.

Two libraries are wrapped:

* ``liboracle.so`` -- the C restatement in ``xspmm_oracle.c`` (clustering literal and fast-exact,
  row permutation, CSR->BCSR, fp64 BCSR SpMM, dense unpermute).
* ``_ref/libxspmm_ref.so`` -- the reference's own host code (compute_1d_jaccard_clustering,
  apply_permutation, csr_to_bcsr) compiled from its sources by ``oracle/Makefile``. It pins the
  restatement. It is built in the development container (where the reference tree exists) and
  travels to the GPU box prebuilt.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(HERE, "liboracle.so")
_REF = os.path.join(HERE, "_ref", "libxspmm_ref.so")

_lib = None
_ref = None

_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_I64 = ctypes.c_int64


def build() -> None:
    """Compile liboracle.so and, when the reference tree is present, _ref/libxspmm_ref.so."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build()
        L = ctypes.CDLL(_LIB)
        L.orc_cluster_literal.argtypes = [_I64, _I64, _i64p, _i64p, ctypes.c_float, _I64, _i64p]
        L.orc_cluster_fast.argtypes = [_I64, _I64, _i64p, _i64p, ctypes.c_float, _I64, _i64p]
        L.orc_permute_rows.argtypes = [_I64, _i64p, _i64p, ctypes.c_void_p, ctypes.c_int, _i64p,
                                       _i64p, _i64p, ctypes.c_void_p]
        L.orc_csr_to_bcsr_count.argtypes = [_I64, _I64, _i64p, _i64p, _I64, _I64, _i64p]
        L.orc_csr_to_bcsr_count.restype = _I64
        L.orc_csr_to_bcsr_fill.argtypes = [_I64, _I64, _i64p, _i64p, ctypes.c_void_p, ctypes.c_int,
                                           _I64, _I64, _i64p, _i64p, ctypes.c_void_p]
        L.orc_bcsr_spmm_f64.argtypes = [_I64, _I64, _I64, _I64, _I64, _i64p, _i64p, _f32p, _f32p,
                                        _f64p]
        L.orc_unpermute_dense.argtypes = [_I64, _I64, _i64p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_int]
        L.orc_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF)


def ref_lib():
    global _ref
    if _ref is None:
        if not os.path.exists(_REF):
            raise FileNotFoundError("compiled reference host code absent: " + _REF)
        L = ctypes.CDLL(_REF)
        for suf, ip, I in (("i32", _i32p, ctypes.c_int32), ("i64", _i64p, ctypes.c_int64)):
            f = getattr(L, "ref_cluster_" + suf)
            f.argtypes = [I, I, I, ip, ip, ctypes.c_float, I, ip]
            f = getattr(L, "ref_permute_" + suf)
            f.argtypes = [I, I, I, ip, ip, _f32p, ip, ip, ip, _f32p]
            f = getattr(L, "ref_csr_to_bcsr_" + suf)
            f.argtypes = [I, I, I, ip, ip, _f32p, I, I, ctypes.POINTER(ctypes.c_int64)]
            f.restype = ctypes.c_void_p
            f = getattr(L, "ref_bcsr_copy_" + suf)
            f.argtypes = [ctypes.c_void_p, ip, ip, _f32p]
            f = getattr(L, "ref_bcsr_free_" + suf)
            f.argtypes = [ctypes.c_void_p]
        L.ref_read_mtx.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32),
                                   ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64)]
        L.ref_read_mtx.restype = ctypes.c_void_p
        L.ref_mtx_copy.argtypes = [ctypes.c_void_p, _i32p, _i32p, _f32p]
        L.ref_mtx_free.argtypes = [ctypes.c_void_p]
        L.ref_gen.argtypes = [ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                              ctypes.c_float, ctypes.c_float, ctypes.c_int,
                              ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64)]
        L.ref_gen.restype = ctypes.c_void_p
        L.ref_gen_copy.argtypes = [ctypes.c_void_p, _i32p, _i32p, _f32p]
        L.ref_gen_free.argtypes = [ctypes.c_void_p]
        _ref = L
    return _ref


def _c64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _nnz(rp):
    return int(rp[-1]) if len(rp) else 0


# ------------------------------------------------------------------------------------------------
# C restatement
# ------------------------------------------------------------------------------------------------
def cluster_literal(rp, ci, M, K, tau=0.5, w=16) -> np.ndarray:
    perm = np.zeros(M, dtype=np.int64)
    rc = lib().orc_cluster_literal(M, K, _c64(rp), _c64(ci if len(ci) else [0]), tau, w, perm)
    if rc != 0:
        raise RuntimeError(f"orc_cluster_literal failed: {rc}")
    return perm


def cluster_fast(rp, ci, M, K, tau=0.5, w=16) -> np.ndarray:
    perm = np.zeros(M, dtype=np.int64)
    rc = lib().orc_cluster_fast(M, K, _c64(rp), _c64(ci if len(ci) else [0]), tau, w, perm)
    if rc != 0:
        raise RuntimeError(f"orc_cluster_fast failed: {rc}")
    return perm


def permute_rows(rp, ci, vals, perm):
    M = len(rp) - 1
    nnz = _nnz(rp)
    vals = np.ascontiguousarray(vals)
    orp = np.zeros(M + 1, dtype=np.int64)
    oci = np.zeros(max(nnz, 1), dtype=np.int64)
    ov = np.zeros(max(nnz, 1), dtype=vals.dtype)
    rc = lib().orc_permute_rows(M, _c64(rp), _c64(ci if len(ci) else [0]),
                                vals.ctypes.data if nnz else ov.ctypes.data, vals.itemsize,
                                _c64(perm), orp, oci, ov.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"orc_permute_rows failed: {rc}")
    return orp, oci[:nnz], ov[:nnz]


def csr_to_bcsr(rp, ci, vals, M, K, rb=16, cb=16):
    """Returns (bcsr_row_ptr[nbr+1], bcsr_col_ind[nnzb], bcsr_values[nnzb, rb, cb])."""
    nbr = (M + rb - 1) // rb
    rp = _c64(rp)
    ci = _c64(ci if len(ci) else [0])
    vals = np.ascontiguousarray(vals)
    brp = np.zeros(nbr + 1, dtype=np.int64)
    nnzb = lib().orc_csr_to_bcsr_count(M, K, rp, ci, rb, cb, brp)
    if nnzb < 0:
        raise RuntimeError(f"orc_csr_to_bcsr_count failed: {nnzb}")
    bci = np.zeros(max(nnzb, 1), dtype=np.int64)
    bv = np.zeros((max(nnzb, 1), rb, cb), dtype=vals.dtype)
    vptr = vals.ctypes.data if len(vals) else bv.ctypes.data
    rc = lib().orc_csr_to_bcsr_fill(M, K, rp, ci, vptr, vals.itemsize, rb, cb, brp, bci,
                                    bv.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"orc_csr_to_bcsr_fill failed: {rc}")
    return brp, bci[:nnzb], bv[:nnzb]


def bcsr_spmm_f64(M, K, N, brp, bci, bvals, B, rb=16, cb=16) -> np.ndarray:
    C = np.zeros((M, N), dtype=np.float64)
    bv = np.ascontiguousarray(np.asarray(bvals, dtype=np.float32).reshape(-1))
    if bv.size == 0:
        bv = np.zeros(1, dtype=np.float32)
    Bf = np.ascontiguousarray(np.asarray(B, dtype=np.float32).reshape(-1))
    if Bf.size == 0:
        Bf = np.zeros(1, dtype=np.float32)
    rc = lib().orc_bcsr_spmm_f64(M, K, N, rb, cb, _c64(brp), _c64(bci if len(bci) else [0]), bv,
                                 Bf, C.reshape(-1) if C.size else np.zeros(1))
    if rc != 0:
        raise RuntimeError(f"orc_bcsr_spmm_f64 failed: {rc}")
    return C


def unpermute_dense(inp: np.ndarray, perm) -> np.ndarray:
    inp = np.ascontiguousarray(inp)
    M, N = inp.shape
    out = np.zeros_like(inp)
    if M == 0:
        return out
    rc = lib().orc_unpermute_dense(M, N, _c64(perm), inp.ctypes.data, out.ctypes.data,
                                   inp.itemsize)
    if rc != 0:
        raise RuntimeError(f"orc_unpermute_dense failed: {rc}")
    return out


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ------------------------------------------------------------------------------------------------
# The reference's own host code
# ------------------------------------------------------------------------------------------------
def _idx(dtype):
    return ("i32", np.int32) if np.dtype(dtype) == np.int32 else ("i64", np.int64)


def ref_cluster(rp, ci, M, K, tau=0.5, w=16, index_dtype=np.int64) -> np.ndarray:
    suf, it = _idx(index_dtype)
    rp = np.ascontiguousarray(rp, dtype=it)
    ci = np.ascontiguousarray(ci if len(ci) else [0], dtype=it)
    perm = np.zeros(max(M, 1), dtype=it)
    rc = getattr(ref_lib(), "ref_cluster_" + suf)(M, K, _nnz(rp), rp, ci, tau, w, perm)
    if rc != 0:
        raise RuntimeError("reference clustering raised")
    return perm[:M]


def ref_permute(rp, ci, vals, perm, K, index_dtype=np.int64):
    suf, it = _idx(index_dtype)
    M = len(rp) - 1
    nnz = _nnz(rp)
    rp = np.ascontiguousarray(rp, dtype=it)
    ci = np.ascontiguousarray(ci if nnz else [0], dtype=it)
    v = np.ascontiguousarray(np.asarray(vals, dtype=np.float32) if nnz else np.zeros(1, np.float32))
    orp = np.zeros(M + 1, dtype=it)
    oci = np.zeros(max(nnz, 1), dtype=it)
    ov = np.zeros(max(nnz, 1), dtype=np.float32)
    rc = getattr(ref_lib(), "ref_permute_" + suf)(M, K, nnz, rp, ci, v,
                                                   np.ascontiguousarray(perm, dtype=it), orp, oci, ov)
    if rc != 0:
        raise RuntimeError("reference apply_permutation raised")
    return orp, oci[:nnz], ov[:nnz]


def ref_csr_to_bcsr(rp, ci, vals, M, K, rb=16, cb=16, index_dtype=np.int64):
    suf, it = _idx(index_dtype)
    L = ref_lib()
    nnz = _nnz(rp)
    rp = np.ascontiguousarray(rp, dtype=it)
    ci = np.ascontiguousarray(ci if nnz else [0], dtype=it)
    v = np.ascontiguousarray(np.asarray(vals, dtype=np.float32) if nnz else np.zeros(1, np.float32))
    nnzb = ctypes.c_int64(0)
    h = getattr(L, "ref_csr_to_bcsr_" + suf)(M, K, nnz, rp, ci, v, rb, cb, ctypes.byref(nnzb))
    if not h:
        raise RuntimeError("reference csr_to_bcsr raised")
    nb = nnzb.value
    nbr = (M + rb - 1) // rb
    brp = np.zeros(nbr + 1, dtype=it)
    bci = np.zeros(max(nb, 1), dtype=it)
    bv = np.zeros((max(nb, 1), rb, cb), dtype=np.float32)
    getattr(L, "ref_bcsr_copy_" + suf)(h, brp, bci, bv)
    getattr(L, "ref_bcsr_free_" + suf)(h)
    return brp, bci[:nb], bv[:nb]


def ref_read_mtx(path):
    """The reference's matrix_utils::io::read_mtx<float> (utils/matrix_io.hpp:27-98) on `path`:
    (rows, cols, row_ptr int32, col_ind int32, values fp32). Raises RuntimeError if it threw."""
    L = ref_lib()
    r, c, n = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_int64(0)
    h = L.ref_read_mtx(os.fsencode(path), ctypes.byref(r), ctypes.byref(c), ctypes.byref(n))
    if not h:
        raise RuntimeError("reference read_mtx raised")
    rp = np.zeros(r.value + 1, dtype=np.int32)
    ci = np.zeros(max(n.value, 1), dtype=np.int32)
    v = np.zeros(max(n.value, 1), dtype=np.float32)
    L.ref_mtx_copy(h, rp, ci, v)
    L.ref_mtx_free(h)
    return r.value, c.value, rp, ci[:n.value], v[:n.value]


REF_GEN_KINDS = {"banded": 0, "triangular": 1, "hessenberg": 2, "arrowhead": 3, "checkers": 4,
                 "block_diagonal": 5, "near_symmetric": 6, "power_law": 7}


def ref_generate(kind, a, b=0, c=0, f1=0.0, f2=0.0, seed=42):
    """The reference's own generator `kind` (utils/matrix_gen.hpp:68-323, float values, int32
    indices); parameters as in ref_gen of ref_driver.cpp. Returns (rows, row_ptr, col_ind,
    values)."""
    L = ref_lib()
    rows, n = ctypes.c_int32(0), ctypes.c_int64(0)
    h = L.ref_gen(REF_GEN_KINDS[kind], a, b, c, f1, f2, seed, ctypes.byref(rows), ctypes.byref(n))
    if not h:
        raise RuntimeError("reference generator raised")
    rp = np.zeros(rows.value + 1, dtype=np.int32)
    ci = np.zeros(max(n.value, 1), dtype=np.int32)
    v = np.zeros(max(n.value, 1), dtype=np.float32)
    L.ref_gen_copy(h, rp, ci, v)
    L.ref_gen_free(h)
    return rows.value, rp, ci[:n.value], v[:n.value]
