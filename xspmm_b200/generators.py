"""Structured sparse-matrix families for regression inputs: the families and parameters of the
reference's utils/matrix_gen.hpp:68-334 (banded, triangular, Hessenberg, arrowhead, checkers,
block diagonal, near-symmetric, power-law, dense, row shuffle).

Each generator returns a host CSR ``(row_ptr, col_ind, values)`` (int64 indices, columns
ascending within a row) with values drawn from U[0.1, 1.0), the value distribution of the
reference (utils/matrix_gen.hpp:16-20). The random streams are numpy's (PCG64, default seed
42), not the reference's mt19937, so the randomly masked families give different matrices for
the same seed; the deterministic structures (banded, arrowhead, checkers) are identical to the
reference's. All of them are vectorized (the reference loops over every (i, j) of arrowhead and
checkers), so sizes in the millions of rows are fine.
"""
from __future__ import annotations

import numpy as np


def _vals(rng, n, dtype):
    return rng.uniform(0.1, 1.0, n).astype(np.float32).astype(dtype)


def _from_rows_cols(M, rows, cols, rng, dtype):
    order = np.lexsort((cols, rows))
    rows, cols = rows[order], cols[order].astype(np.int64)
    rp = np.zeros(M + 1, dtype=np.int64)
    if len(rows):
        np.cumsum(np.bincount(rows, minlength=M), out=rp[1:])
    return rp, cols, _vals(rng, len(cols), dtype)


def _range_rows(starts, ends):
    """Row ids and column ids of the contiguous column ranges [starts[i], ends[i]] (inclusive)."""
    lens = np.maximum(ends - starts + 1, 0)
    rows = np.repeat(np.arange(len(starts), dtype=np.int64), lens)
    offs = np.arange(lens.sum(), dtype=np.int64) - np.repeat(np.cumsum(lens) - lens, lens)
    return rows, np.repeat(starts, lens) + offs


def banded(size: int, bandwidth: int, seed: int = 42, dtype=np.float32):
    """Every (i, j) with |i - j| <= bandwidth (bandwidth 1: tridiagonal)
    (utils/matrix_gen.hpp:68-92)."""
    rng = np.random.default_rng(seed)
    i = np.arange(size, dtype=np.int64)
    rows, cols = _range_rows(np.maximum(0, i - bandwidth), np.minimum(size - 1, i + bandwidth))
    return _from_rows_cols(size, rows, cols, rng, dtype)


def _masked(size, rows, cols, keep_always, density, rng, dtype):
    keep = keep_always | (rng.random(len(rows)) < density)
    return _from_rows_cols(size, rows[keep], cols[keep], rng, dtype)


def triangular(size: int, upper: bool, density: float, seed: int = 42, dtype=np.float32):
    """Upper (j >= i) or lower (j <= i) triangle, each entry kept with probability `density`,
    the diagonal always (utils/matrix_gen.hpp:95-123)."""
    rng = np.random.default_rng(seed)
    i = np.arange(size, dtype=np.int64)
    s, e = (i, np.full(size, size - 1)) if upper else (np.zeros(size, np.int64), i)
    rows, cols = _range_rows(s, e)
    return _masked(size, rows, cols, rows == cols, density, rng, dtype)


def hessenberg(size: int, upper: bool, density: float, seed: int = 42, dtype=np.float32):
    """Upper Hessenberg (zeros below the first subdiagonal) or lower (above the first
    superdiagonal); entries kept with probability `density`, the three central diagonals always
    (utils/matrix_gen.hpp:126-154)."""
    rng = np.random.default_rng(seed)
    i = np.arange(size, dtype=np.int64)
    if upper:
        s, e = np.maximum(0, i - 1), np.full(size, size - 1)
    else:
        s, e = np.zeros(size, np.int64), np.minimum(size - 1, i + 1)
    rows, cols = _range_rows(s, e)
    return _masked(size, rows, cols, np.abs(rows - cols) <= 1, density, rng, dtype)


def arrowhead(size: int, width: int, seed: int = 42, dtype=np.float32):
    """Dense first `width` rows and columns plus the diagonal (utils/matrix_gen.hpp:157-181)."""
    rng = np.random.default_rng(seed)
    w = min(max(width, 0), size)
    i = np.arange(size, dtype=np.int64)
    # rows < w are full; later rows hold columns [0, w) and their diagonal
    full_r, full_c = _range_rows(np.zeros(w, np.int64), np.full(w, size - 1))
    rest = i[w:]
    head_r, head_c = _range_rows(np.zeros(len(rest), np.int64), np.full(len(rest), w - 1))
    rows = np.concatenate([full_r, head_r + w, rest])
    cols = np.concatenate([full_c, head_c, rest])
    return _from_rows_cols(size, rows, cols, rng, dtype)


def checkers(rows: int, cols: int, block_size: int, seed: int = 42, dtype=np.float32):
    """Alternating dense and empty block_size x block_size tiles: (i / bs + j / bs) odd is
    nonzero (utils/matrix_gen.hpp:184-211)."""
    rng = np.random.default_rng(seed)
    bs = max(int(block_size), 1)
    nbc = (cols + bs - 1) // bs
    r_list, c_list = [], []
    for parity in (0, 1):  # rows of even / odd block rows take the odd / even block columns
        tiles = np.arange(1 - parity, nbc, 2, dtype=np.int64)
        tcols = (tiles[:, None] * bs + np.arange(bs)[None, :]).reshape(-1)
        tcols = tcols[tcols < cols]
        rsel = np.nonzero((np.arange(rows) // bs) % 2 == parity)[0]
        r_list.append(np.repeat(rsel, len(tcols)))
        c_list.append(np.tile(tcols, len(rsel)))
    return _from_rows_cols(rows, np.concatenate(r_list), np.concatenate(c_list), rng, dtype)


def block_diagonal(size: int, block_size: int, density: float, seed: int = 42,
                   dtype=np.float32):
    """Diagonal blocks of block_size, entries kept with probability `density`, the diagonal
    always (utils/matrix_gen.hpp:214-243)."""
    rng = np.random.default_rng(seed)
    i = np.arange(size, dtype=np.int64)
    s = (i // block_size) * block_size
    rows, cols = _range_rows(s, np.minimum(size - 1, s + block_size - 1))
    return _masked(size, rows, cols, rows == cols, density, rng, dtype)


def near_symmetric(size: int, density: float, drop_rate: float, seed: int = 42,
                   dtype=np.float32):
    """A symmetric pattern (each i <= j kept with probability `density`) whose two mirrored
    entries are then each dropped with probability `drop_rate` (utils/matrix_gen.hpp:246-281).
    Sampled per upper-triangle entry, so intended for sizes up to a few thousand."""
    rng = np.random.default_rng(seed)
    iu, ju = np.triu_indices(size)
    pick = rng.random(len(iu)) < density
    iu, ju = iu[pick].astype(np.int64), ju[pick].astype(np.int64)
    keep_ij = rng.random(len(iu)) > drop_rate
    keep_ji = (iu != ju) & (rng.random(len(iu)) > drop_rate)
    rows = np.concatenate([iu[keep_ij], ju[keep_ji]])
    cols = np.concatenate([ju[keep_ij], iu[keep_ji]])
    return _from_rows_cols(size, rows, cols, rng, dtype)


def power_law(rows: int, cols: int, alpha: float, seed: int = 42, dtype=np.float32):
    """Scale-free rows: row degree floor(u^(-1/(alpha-1))) for u ~ U[0.001, 1), clamped to
    [1, cols], columns a uniform sample without replacement (utils/matrix_gen.hpp:284-323)."""
    rng = np.random.default_rng(seed)
    u = rng.uniform(0.001, 1.0, rows).astype(np.float32)
    deg = np.floor(np.power(u, np.float32(-1.0 / (alpha - 1.0)))).astype(np.int64)
    deg = np.clip(deg, 1, cols)
    r_list, c_list = [], []
    for r in range(rows):
        d = int(deg[r])
        c = rng.choice(cols, d, replace=False) if d < cols else np.arange(cols)
        r_list.append(np.full(d, r, np.int64))
        c_list.append(np.asarray(c, np.int64))
    return _from_rows_cols(rows, np.concatenate(r_list) if r_list else np.zeros(0, np.int64),
                           np.concatenate(c_list) if c_list else np.zeros(0, np.int64), rng, dtype)


def dense(rows: int, cols: int, seed: int = 42, dtype=np.float32) -> np.ndarray:
    """Row-major dense rows x cols matrix of U[0.1, 1) values (utils/matrix_gen.hpp:326-333)."""
    rng = np.random.default_rng(seed)
    return _vals(rng, rows * cols, dtype).reshape(rows, cols)


def shuffle_rows(row_ptr, col_ind, values, seed: int = 42):
    """Rows in a random order (utils/matrix_gen.hpp:25-62); returns (row_ptr, col_ind, values,
    order) with new row i = old row order[i]."""
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    M = len(row_ptr) - 1
    order = np.random.default_rng(seed).permutation(M)
    lens = np.diff(row_ptr)[order]
    rp = np.zeros(M + 1, dtype=np.int64)
    np.cumsum(lens, out=rp[1:])
    src = np.repeat(row_ptr[:-1][order], lens) + (np.arange(rp[-1]) - np.repeat(rp[:-1], lens))
    return rp, np.asarray(col_ind)[src], np.asarray(values)[src], order


FAMILIES = {
    "banded": lambda n, seed=42, dtype=np.float32: banded(n, 8, seed, dtype),
    "tridiagonal": lambda n, seed=42, dtype=np.float32: banded(n, 1, seed, dtype),
    "upper_triangular": lambda n, seed=42, dtype=np.float32: triangular(n, True, 0.02, seed, dtype),
    "lower_hessenberg": lambda n, seed=42, dtype=np.float32: hessenberg(n, False, 0.02, seed, dtype),
    "arrowhead": lambda n, seed=42, dtype=np.float32: arrowhead(n, 20, seed, dtype),
    "checkers": lambda n, seed=42, dtype=np.float32: checkers(n, n, 16, seed, dtype),
    "block_diagonal": lambda n, seed=42, dtype=np.float32: block_diagonal(n, 32, 0.3, seed, dtype),
    "near_symmetric": lambda n, seed=42, dtype=np.float32: near_symmetric(n, 0.01, 0.1, seed, dtype),
    "power_law": lambda n, seed=42, dtype=np.float32: power_law(n, n, 2.1, seed, dtype),
}
"""A default parameter set per family for square n x n regression inputs."""

__all__ = ["banded", "triangular", "hessenberg", "arrowhead", "checkers", "block_diagonal",
           "near_symmetric", "power_law", "dense", "shuffle_rows", "FAMILIES"]
