"""Shared helpers for the tests: golden fixtures, error metrics, CSR helpers."""
from __future__ import annotations

import glob
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_cases():
    return sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


def load_golden(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


def errors(expected: np.ndarray, actual: np.ndarray, floor_rel: float):
    """Error metrics of the reference's utils/matrix_compare.hpp:23-65 (max abs, max relative
    with abs fallback when expected == 0, relative Frobenius) plus a guarded max relative error
    |d| / max(|expected|, floor_rel * rms(expected)) that stays meaningful where sums cancel."""
    e = np.asarray(expected, dtype=np.float64)
    a = np.asarray(actual, dtype=np.float64)
    d = np.abs(a - e)
    ae = np.abs(e)
    strict = np.where(ae > 0, d / np.where(ae > 0, ae, 1), d)
    rms = float(np.sqrt(np.mean(e * e))) if e.size else 0.0
    floor = max(floor_rel * rms, np.finfo(np.float64).tiny)
    guarded = d / np.maximum(ae, floor)
    fro = float(np.sqrt((d * d).sum()))
    efro = float(np.sqrt((e * e).sum()))
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "max_rel_strict": float(strict.max()) if d.size else 0.0,
        "max_rel_guarded": float(guarded.max()) if d.size else 0.0,
        "rel_frobenius": fro / efro if efro > 0 else fro,
    }


# tolerances written in the north star: max relative error 1e-3 (fp16 in / fp32 out), 1e-5 (fp32)
TOL = {np.dtype(np.float16): 1e-3, np.dtype(np.float32): 1e-5}


def dense_from_csr(M, K, rp, ci, v):
    A = np.zeros((M, K), dtype=np.float64)
    for r in range(M):
        for j in range(rp[r], rp[r + 1]):
            A[r, ci[j]] = v[j]  # last duplicate wins, as in the conversion
    return A


def fp32_block_emulation(M, N, brp, bci, bv, B, rb=16, cb=16):
    """C computed the way the reference kernel's arithmetic runs (src/common/spmm_math.hpp:68-114):
    block by block in col_ind order, each block's 16-term products summed and added to an fp32
    running sum. Used to bound the error any fp32-accumulating implementation has on long rows."""
    nbr = len(brp) - 1
    K = B.shape[0]
    nbk = max((K + cb - 1) // cb, int(np.max(bci)) + 1 if len(bci) else 1)
    Bp = np.zeros((nbk * cb, N), dtype=np.float32)
    Bp[:K] = B.astype(np.float32)
    C = np.zeros((nbr * rb, N), dtype=np.float32)
    lens = np.diff(brp)
    vals = np.asarray(bv, dtype=np.float32).reshape(-1, rb, cb)
    for t in range(int(lens.max()) if nbr else 0):
        rows = np.nonzero(lens > t)[0]
        j = brp[rows] + t
        blk = vals[j]                                          # (R, rb, cb)
        bsl = Bp[(bci[j][:, None] * cb + np.arange(cb)[None, :])]  # (R, cb, N)
        part = np.einsum("rik,rkn->rin", blk.astype(np.float64), bsl.astype(np.float64))
        idx = (rows[:, None] * rb + np.arange(rb)[None, :]).reshape(-1)
        C[idx] = (C[idx] + part.reshape(-1, N).astype(np.float32)).astype(np.float32)
    return C[:M]
