"""Seeded synthetic inputs with the shapes and value distributions of the five benchmark configs.

The reference ships generators in utils/matrix_gen.hpp (mt19937, seed 42); the benchmark configs
used here define their own distributions, so these generators are written from the config text
(numpy PCG64, default seed 42). Every generator returns a :class:`Problem` holding a CSR matrix A
(int64 indices, rows sorted by column), the dense right-hand side B (row-major K x N) and metadata.

Config summary (all synthetic, no public dataset is involved):

1. plumbing    4096 x 4096 fp32, entries kept independently with p=0.01, U[-1,1]; B 4096x128 fp32
2. hidden-block 16384^2 fp16, 1024^2 grid of 16x16 blocks kept with p=0.005, each entry of a kept
               block kept with p=0.5, N(0,1); rows randomly permuted; B 16384x256 fp16 N(0,1)
3. pruned LLM  4096 x 11008 fp16 N(0,0.02) magnitude-pruned to 10% density; B 11008 x N fp16 N(0,1)
4. banded FEM  2,000,000^2 fp16, entries with |i-j|<=32 kept with p=0.4, U[-1,1]; rows randomly
               permuted; B 2,000,000 x 64 fp16
5. GNN R-MAT   2^20 nodes, 16 * 2^20 sampled edges (a,b,c,d = .57,.19,.19,.05), duplicates merged,
               self-loops kept, values 1/deg(row) fp16; B 2^20 x 128 fp16 N(0,1)

Every generator takes size parameters so the tests can build scaled-down instances with the same
structure.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class Problem:
    name: str
    M: int
    K: int
    N: int
    row_ptr: np.ndarray  # int64 [M+1]
    col_ind: np.ndarray  # int64 [nnz]
    values: np.ndarray  # float16 or float32 [nnz]
    B: np.ndarray  # [K, N], same dtype as values
    clustering: bool = True
    meta: dict = field(default_factory=dict)

    @property
    def nnz(self) -> int:
        return int(self.row_ptr[-1])

    @property
    def value_dtype(self):
        return self.values.dtype


def csr_from_coo(M: int, rows: np.ndarray, cols: np.ndarray, vals: np.ndarray, K: int):
    """Sort COO triplets by (row, col) and return (row_ptr, col_ind, values)."""
    order = np.lexsort((cols, rows))
    rows = rows[order]
    cols = cols[order].astype(np.int64)
    vals = vals[order]
    counts = np.bincount(rows, minlength=M).astype(np.int64)
    row_ptr = np.zeros(M + 1, dtype=np.int64)
    np.cumsum(counts, out=row_ptr[1:])
    return row_ptr, cols, vals


def permute_csr_rows(row_ptr: np.ndarray, col_ind: np.ndarray, values: np.ndarray,
                     order: np.ndarray):
    """New row i = old row order[i] (entries keep their order)."""
    lens = np.diff(row_ptr)[order]
    new_rp = np.zeros(len(order) + 1, dtype=np.int64)
    np.cumsum(lens, out=new_rp[1:])
    starts = row_ptr[:-1][order]
    # index of every output entry in the input arrays
    rep_start = np.repeat(starts - new_rp[:-1], lens)
    src = np.arange(new_rp[-1], dtype=np.int64) + rep_start
    return new_rp, col_ind[src], values[src]


def cfg1_plumbing(seed: int = 42, M: int = 4096, K: int = 4096, N: int = 128,
                  density: float = 0.01) -> Problem:
    rng = np.random.default_rng(seed)
    mask = rng.random((M, K), dtype=np.float32) < density
    rows, cols = np.nonzero(mask)
    vals = rng.uniform(-1.0, 1.0, rows.size).astype(np.float32)
    row_ptr = np.zeros(M + 1, dtype=np.int64)
    np.cumsum(np.bincount(rows, minlength=M), out=row_ptr[1:])
    B = rng.uniform(-1.0, 1.0, (K, N)).astype(np.float32)
    return Problem("cfg1_plumbing", M, K, N, row_ptr, cols.astype(np.int64), vals, B,
                   clustering=False, meta={"density": density, "seed": seed})


def cfg2_hidden_block(seed: int = 42, n: int = 16384, N: int = 256, block_density: float = 0.005,
                      fill: float = 0.5, bs: int = 16) -> Problem:
    rng = np.random.default_rng(seed)
    nb = n // bs
    bmask = rng.random((nb, nb), dtype=np.float32) < block_density
    bi, bj = np.nonzero(bmask)
    emask = rng.random((bi.size, bs, bs), dtype=np.float32) < fill
    blk, ii, jj = np.nonzero(emask)
    rows = bi[blk].astype(np.int64) * bs + ii
    cols = bj[blk].astype(np.int64) * bs + jj
    vals = rng.standard_normal(rows.size, dtype=np.float32).astype(np.float16)
    shuffle = rng.permutation(n)  # new row r holds old row shuffle[r]
    inv = np.empty(n, dtype=np.int64)
    inv[shuffle] = np.arange(n)
    row_ptr, col_ind, values = csr_from_coo(n, inv[rows], cols, vals, n)
    B = rng.standard_normal((n, N), dtype=np.float32).astype(np.float16)
    return Problem("cfg2_hidden_block", n, n, N, row_ptr, col_ind, values, B, clustering=True,
                   meta={"block_density": block_density, "fill": fill, "hidden_blocks": int(bi.size),
                         "seed": seed})


def cfg3_pruned_llm(seed: int = 42, M: int = 4096, K: int = 11008, N: int = 256,
                    keep: float = 0.1) -> Problem:
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02)
    thr = np.quantile(np.abs(W), 1.0 - keep)
    mask = np.abs(W) > thr
    rows, cols = np.nonzero(mask)
    vals = W[rows, cols].astype(np.float16)
    del W
    row_ptr = np.zeros(M + 1, dtype=np.int64)
    np.cumsum(np.bincount(rows, minlength=M), out=row_ptr[1:])
    B = rng.standard_normal((K, N), dtype=np.float32).astype(np.float16)
    return Problem("cfg3_pruned_llm", M, K, N, row_ptr, cols.astype(np.int64), vals, B,
                   clustering=True, meta={"keep": keep, "seed": seed})


def cfg4_banded(seed: int = 42, n: int = 2_000_000, N: int = 64, half_bw: int = 32,
                fill: float = 0.4, chunk: int = 1 << 18) -> Problem:
    rng = np.random.default_rng(seed)
    offs = np.arange(-half_bw, half_bw + 1, dtype=np.int64)
    lens = np.zeros(n, dtype=np.int64)
    col_parts = []
    for r0 in range(0, n, chunk):
        r1 = min(n, r0 + chunk)
        cols = np.arange(r0, r1, dtype=np.int64)[:, None] + offs[None, :]
        keep = (rng.random(cols.shape, dtype=np.float32) < fill) & (cols >= 0) & (cols < n)
        lens[r0:r1] = keep.sum(axis=1)
        col_parts.append(cols[keep])
    col_ind = np.concatenate(col_parts)
    row_ptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lens, out=row_ptr[1:])
    values = rng.uniform(-1.0, 1.0, col_ind.size).astype(np.float16)
    shuffle = rng.permutation(n)
    row_ptr, col_ind, values = permute_csr_rows(row_ptr, col_ind, values, shuffle)
    B = rng.uniform(-1.0, 1.0, (n, N)).astype(np.float16)
    return Problem("cfg4_banded", n, n, N, row_ptr, col_ind, values, B, clustering=True,
                   meta={"half_bandwidth": half_bw, "fill": fill, "seed": seed})


def cfg5_rmat(seed: int = 42, scale: int = 20, edge_factor: int = 16, N: int = 128,
              a: float = 0.57, b: float = 0.19, c: float = 0.19) -> Problem:
    rng = np.random.default_rng(seed)
    n = 1 << scale
    E = edge_factor * n
    src = np.zeros(E, dtype=np.int64)
    dst = np.zeros(E, dtype=np.int64)
    for level in range(scale):
        r = rng.random(E, dtype=np.float32)
        bit = np.int64(1) << (scale - 1 - level)
        down = r >= (a + b)  # quadrants c and d
        right = ((r >= a) & (r < a + b)) | (r >= a + b + c)  # quadrants b and d
        src |= down.astype(np.int64) * bit
        dst |= right.astype(np.int64) * bit
    key = np.unique(src * n + dst)  # dedupe; self-loops kept
    rows = key // n
    cols = key % n
    deg = np.bincount(rows, minlength=n).astype(np.float64)
    vals = (1.0 / deg[rows]).astype(np.float16)
    row_ptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(deg.astype(np.int64), out=row_ptr[1:])
    B = rng.standard_normal((n, N), dtype=np.float32).astype(np.float16)
    return Problem("cfg5_rmat", n, n, N, row_ptr, cols, vals, B, clustering=True,
                   meta={"scale": scale, "edge_factor": edge_factor, "abcd": [a, b, c, 1 - a - b - c],
                         "dedupe": True, "self_loops": "kept", "seed": seed})


def random_csr(M: int, K: int, density: float, seed: int = 0, dtype=np.float32,
               empty_row_frac: float = 0.0, dup_frac: float = 0.0, shuffle_cols: bool = False):
    """Small random CSR for edge-case tests.

    empty_row_frac forces that share of rows to be empty; dup_frac appends that share of extra
    entries that repeat an existing (row, col); shuffle_cols leaves columns unsorted inside rows.
    """
    rng = np.random.default_rng(seed)
    mask = rng.random((M, K)) < density
    if empty_row_frac > 0 and M > 0:
        mask[rng.random(M) < empty_row_frac, :] = False
    rows, cols = np.nonzero(mask)
    rows = rows.astype(np.int64)
    cols = cols.astype(np.int64)
    if dup_frac > 0 and rows.size > 0:
        nd = max(1, int(rows.size * dup_frac))
        pick = rng.integers(0, rows.size, nd)
        rows = np.concatenate([rows, rows[pick]])
        cols = np.concatenate([cols, cols[pick]])
    vals = rng.uniform(-1.0, 1.0, rows.size).astype(dtype)
    order = np.argsort(rows, kind="stable")  # keep duplicates in generation order
    rows, cols, vals = rows[order], cols[order], vals[order]
    row_ptr = np.zeros(M + 1, dtype=np.int64)
    np.cumsum(np.bincount(rows, minlength=M), out=row_ptr[1:])
    if shuffle_cols:
        for r in range(M):
            s, e = row_ptr[r], row_ptr[r + 1]
            p = rng.permutation(e - s) + s
            cols[s:e] = cols[p]
            vals[s:e] = vals[p]
    return row_ptr, cols, vals


CONFIGS = {
    "cfg1": cfg1_plumbing,
    "cfg2": cfg2_hidden_block,
    "cfg3": cfg3_pruned_llm,
    "cfg4": cfg4_banded,
    "cfg5": cfg5_rmat,
}
