"""Matrix Market (coordinate format) input and output, producing the host CSR that CSRMatrix
uploads.

Reading follows the acceptance rules of the reference's reader (utils/matrix_io.hpp:27-98,
`matrix_utils::io::read_mtx`) so that a file yields the same CSR under both:

* lines that are empty or start with ``%`` are skipped everywhere (the ``%%MatrixMarket`` banner
  included); the first other line holds ``rows cols nnz``;
* an entry line is ``row col [value ...]`` with 1-based indices; a line whose first two tokens
  are not integers is skipped; a missing value (pattern files) reads as 1.0; only the first value
  token is used (the real part of a complex entry); entries outside [1, rows] x [1, cols] are
  dropped;
* values are parsed as fp32 and then converted to the requested value type;
* entries are sorted by (row, col); the CSR has int32 indices, and ``nnz`` is the number of kept
  entries (the header's count is only a size hint).

Two points where the reference is unspecified or does not apply are decided here:

* duplicates of one (row, col) keep their file order (a stable sort; the reference's std::sort
  leaves their order unspecified, and CSR->BCSR keeps the last one);
* ``expand_symmetry=True`` (off by default, like the reference) mirrors the off-diagonal entries
  of ``symmetric``, ``skew-symmetric`` and ``hermitian`` files as the Matrix Market format defines.

The bulk of a file is parsed with pandas' C tokenizer when pandas is available and the file is
regular; any line the fast path cannot take sends the whole file through the line-by-line parser,
which implements the rules above directly.
"""
from __future__ import annotations

import io
import os
import re
from dataclasses import dataclass

import numpy as np


@dataclass
class HostCSRMatrix:
    """Host CSR as the reference's reader returns it (num_rows, num_cols, row_ptr, col_ind,
    values; int32 indices)."""
    num_rows: int
    num_cols: int
    row_ptr: np.ndarray
    col_ind: np.ndarray
    values: np.ndarray

    @property
    def nnz(self) -> int:
        return int(self.row_ptr[-1]) if len(self.row_ptr) else 0


def _is_skipped(line: str) -> bool:
    return len(line) == 0 or line[0] == "%"


_FLOAT_TOKEN = r"[+-]?(?:\d+\.?\d*|\.\d+)(?:[eE][+-]?\d+)?"
_INT = re.compile(r"\s*([+-]?\d+)")
_FLOAT = re.compile(r"\s*(" + _FLOAT_TOKEN + ")")


def _split_header(text: str):
    """(rows, cols, nnz_hint, banner, offset of the first entry line)."""
    pos = 0
    banner = ""
    while pos < len(text):
        end = text.find("\n", pos)
        if end < 0:
            end = len(text)
        line = text[pos:end].rstrip("\r")
        nxt = end + 1
        if line.startswith("%%MatrixMarket") and not banner:
            banner = line
        if _is_skipped(line):
            pos = nxt
            continue
        vals, p = [], 0
        for _ in range(3):  # istream >> rows >> cols >> nnz
            m = _INT.match(line, p)
            if not m:
                raise ValueError("Failed to parse MTX dimensions.")
            vals.append(int(m.group(1)))
            p = m.end()
        return vals[0], vals[1], vals[2], banner, nxt
    raise ValueError("Failed to parse MTX dimensions.")


def _entries_slow(body: str):
    """Line by line, reading each line's fields the way `istringstream >> int >> int >> float`
    does: each extraction skips whitespace and takes the longest numeric prefix from where the
    previous one stopped."""
    rows, cols, vals = [], [], []
    for raw in body.split("\n"):
        line = raw.rstrip("\r")
        if _is_skipped(line):
            continue
        m1 = _INT.match(line)
        if not m1:
            continue
        m2 = _INT.match(line, m1.end())
        if not m2:
            continue
        m3 = _FLOAT.match(line, m2.end())
        # an exponent marker without digits is taken into the number and fails the extraction
        if m3 and line[m3.end():m3.end() + 1] in ("e", "E"):
            m3 = None
        rows.append(int(m1.group(1)))
        cols.append(int(m2.group(1)))
        vals.append(m3.group(1) if m3 else "1")
    return (np.asarray(rows, dtype=np.int64), np.asarray(cols, dtype=np.int64),
            np.asarray(vals, dtype=str))


def _entries_fast(body: str):
    """pandas C tokenizer over a regular body (2 to 4 numeric columns, '%' comments); None when
    the body is not regular enough for it."""
    try:
        import pandas as pd
    except Exception:  # pragma: no cover - pandas is optional
        return None
    if not body.strip():
        return (np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros(0, dtype=str))
    try:
        df = pd.read_csv(io.StringIO(body), sep=r"\s+", header=None, comment="%",
                         engine="c", float_precision="round_trip", dtype=str,
                         names=range(4), skip_blank_lines=True)
    except Exception:
        return None
    if df.shape[1] < 2:
        return None
    rc = df.iloc[:, :2]
    if rc.isna().any().any():
        return None
    r_s, c_s = rc.iloc[:, 0].to_numpy(str), rc.iloc[:, 1].to_numpy(str)
    if not (np.char.isdigit(np.char.lstrip(r_s, "+-")).all()
            and np.char.isdigit(np.char.lstrip(c_s, "+-")).all()):
        return None
    rows = r_s.astype(np.int64)
    cols = c_s.astype(np.int64)
    if df.shape[1] >= 3:
        vs = df.iloc[:, 2]
        present = vs.dropna()
        # only plain decimal tokens here; anything else ("nan", "1.0abc", ...) is read the
        # way an istream would, by the line parser
        if len(present) and not present.str.fullmatch(_FLOAT_TOKEN).all():
            return None
        v = vs.fillna("1").to_numpy(str)
    else:
        v = np.full(len(rows), "1")
    return rows, cols, v


def _to_f32(tokens: np.ndarray) -> np.ndarray:
    """Decimal tokens to the nearest fp32 (as strtof rounds). Parsing goes through fp64; where
    that lands exactly on the midpoint of two fp32 neighbours the fp64 rounding may have
    decided the tie, so those few values are settled against the exact decimal."""
    v64 = tokens.astype(np.float64)
    f = v64.astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):  # neighbours of the largest fp32
        up = np.nextafter(f, np.float32(np.inf))
        dn = np.nextafter(f, np.float32(-np.inf))
        f64 = f.astype(np.float64)
        tie_up = v64 == (f64 + up.astype(np.float64)) / 2
        tie_dn = v64 == (f64 + dn.astype(np.float64)) / 2
    idx = np.nonzero((tie_up | tie_dn) & np.isfinite(v64))[0]
    if len(idx):
        from decimal import Decimal
        for i in idx:
            exact = Decimal(str(tokens[i]))
            mid = Decimal(float(v64[i]))
            if exact == mid:
                continue  # a true tie: round-half-even already applied
            if tie_up[i] and exact > mid:
                f[i] = up[i]
            elif tie_dn[i] and exact < mid:
                f[i] = dn[i]
    return f


def read_mtx(path: str, value_dtype=np.float32, expand_symmetry: bool = False) -> HostCSRMatrix:
    """Read a Matrix Market coordinate file into a host CSR (int32 indices, `value_dtype`
    values). Raises RuntimeError if the file cannot be opened and ValueError if it has no
    dimension line."""
    try:
        with open(path, "rb") as f:
            text = f.read().decode("utf-8", errors="replace")
    except OSError as e:
        raise RuntimeError("Could not open MTX file: " + str(path)) from e
    M, K, _nnz_hint, banner, off = _split_header(text)
    body = text[off:]
    got = _entries_fast(body)
    if got is None:
        got = _entries_slow(body)
    rows, cols, v = got
    keep = (rows >= 1) & (rows <= M) & (cols >= 1) & (cols <= K)
    rows, cols, v = rows[keep] - 1, cols[keep] - 1, v[keep]
    v32 = _to_f32(v)  # values are read as fp32, as the reference does
    if expand_symmetry:
        kind = banner.lower().split()
        sym = next((k for k in ("skew-symmetric", "symmetric", "hermitian") if k in kind), None)
        if sym is not None:
            off_diag = rows != cols
            mv = v32[off_diag]
            if sym == "skew-symmetric":
                mv = -mv
            rows, cols, v32 = (np.concatenate([rows, cols[off_diag]]),
                               np.concatenate([cols, rows[off_diag]]),
                               np.concatenate([v32, mv]))
    order = np.lexsort((cols, rows))  # stable: duplicates keep file order
    rows, cols, v32 = rows[order], cols[order], v32[order]
    row_ptr = np.zeros(M + 1, dtype=np.int32)
    if len(rows):
        np.cumsum(np.bincount(rows, minlength=M), out=row_ptr[1:])
    return HostCSRMatrix(M, K, row_ptr, cols.astype(np.int32),
                         v32.astype(value_dtype, copy=False))


def write_mtx(path: str, M: int, K: int, row_ptr, col_ind, values, comment: str = "") -> None:
    """Write a CSR as a general real coordinate Matrix Market file (1-based; values printed with
    enough digits to read back the same fp32)."""
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    col_ind = np.asarray(col_ind, dtype=np.int64)
    vals = np.asarray(values, dtype=np.float32)
    nnz = int(row_ptr[-1]) if len(row_ptr) else 0
    rows = np.repeat(np.arange(M, dtype=np.int64), np.diff(row_ptr))
    with open(path, "w") as f:
        f.write("%%MatrixMarket matrix coordinate real general\n")
        for line in comment.splitlines():
            f.write("%" + line + "\n")
        f.write(f"{M} {K} {nnz}\n")
        if nnz:
            body = np.column_stack([rows + 1, col_ind[:nnz] + 1])
            txt = [f"{r} {c} {v!r}" for (r, c), v in zip(body.tolist(),
                                                          vals[:nnz].astype(np.float64).tolist())]
            f.write("\n".join(txt) + "\n")


def block_counts(executor, A_host: HostCSRMatrix, hw: int = 16, tau: float = 0.5):
    """Nonzero 16x16 blocks before and after clustering, on the device (the report of the
    reference's examples/04_real_matrices_benchmark.cpp:132-155): returns (before, after)."""
    import torch

    from . import api
    A = api.CSRMatrix.from_host(executor, A_host.num_rows, A_host.num_cols, A_host.row_ptr,
                                A_host.col_ind, A_host.values, index_dtype=torch.int32)
    before = api.csr_to_bcsr(executor, A, hw, hw).num_blocks
    perm = torch.empty(A_host.num_rows, dtype=torch.int32, device=executor.device)
    api.compute_1d_jaccard_clustering(executor, A, tau, hw, perm)
    P = api.apply_permutation(executor, A, perm)
    after = api.csr_to_bcsr(executor, P, hw, hw).num_blocks
    return int(before), int(after)


__all__ = ["HostCSRMatrix", "read_mtx", "write_mtx", "block_counts"]

if __name__ == "__main__":  # pragma: no cover
    import sys
    m = read_mtx(sys.argv[1])
    print(os.path.basename(sys.argv[1]), m.num_rows, m.num_cols, m.nnz)
