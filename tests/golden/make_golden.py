"""Generate the golden fixtures in tests/golden/ by running the reference's own host code.

The reference xSpMM ships no golden vectors or known-answer tests. These fixtures are produced by
its own CPU functions -- compute_1d_jaccard_clustering, apply_permutation, csr_to_bcsr -- compiled
from its unmodified sources by oracle/Makefile into oracle/_ref/libxspmm_ref.so and driven through
its CpuExecutor. Inputs are small seeded matrices with the structure of the five benchmark configs
plus the edge cases the path has (empty matrix, empty rows, row counts that are not multiples of
16, duplicate and unsorted columns, several thresholds and block widths).

Run from the repository root (needs the reference tree, so only in the development container):
    python tests/golden/make_golden.py
Each case becomes tests/golden/<name>.npz holding the input CSR (int64 indices, float32 values),
M, K, tau, w and the reference outputs:
    perm                       -- compute_1d_jaccard_clustering(A, tau, w)
    p_row_ptr/p_col_ind/p_vals -- apply_permutation(A, perm)
    b_row_ptr/b_col_ind/b_vals -- csr_to_bcsr(A, 16, 16)                (unpermuted input)
    pb_row_ptr/pb_col_ind/pb_vals -- csr_to_bcsr(apply_permutation(A, perm), 16, 16)
The clustering output of the int32 instantiation is checked equal to the int64 one here.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from xspmm_b200 import synth  # noqa: E402


def checkers(M, K, pattern, seed):
    """Alternating dense/empty pattern x pattern tiles, rows shuffled (shape of the reference's
    examples/01 checkers input)."""
    rng = np.random.default_rng(seed)
    r, c = np.meshgrid(np.arange(M), np.arange(K), indexing="ij")
    mask = ((r // pattern + c // pattern) % 2) == 1
    rows, cols = np.nonzero(mask)
    vals = rng.uniform(0.1, 1.0, rows.size).astype(np.float32)
    rp = np.zeros(M + 1, dtype=np.int64)
    np.cumsum(np.bincount(rows, minlength=M), out=rp[1:])
    order = rng.permutation(M)
    return synth.permute_csr_rows(rp, cols.astype(np.int64), vals, order)


def cases():
    out = []
    P = synth.cfg1_plumbing(seed=1, M=128, K=128, N=8, density=0.05)
    out.append(("cfg1_small", P.row_ptr, P.col_ind, P.values, P.M, P.K, 0.5, 16))
    P = synth.cfg2_hidden_block(seed=2, n=512, N=8, block_density=0.06)
    out.append(("cfg2_small", P.row_ptr, P.col_ind, P.values, P.M, P.K, 0.5, 16))
    P = synth.cfg3_pruned_llm(seed=3, M=64, K=176, N=8)
    out.append(("cfg3_small", P.row_ptr, P.col_ind, P.values, P.M, P.K, 0.5, 16))
    P = synth.cfg4_banded(seed=4, n=512, N=8)
    out.append(("cfg4_small", P.row_ptr, P.col_ind, P.values, P.M, P.K, 0.5, 16))
    P = synth.cfg5_rmat(seed=5, scale=9, N=8)
    out.append(("cfg5_small", P.row_ptr, P.col_ind, P.values, P.M, P.K, 0.5, 16))
    rp, ci, v = checkers(64, 64, 4, seed=6)
    out.append(("checkers_p4", rp, ci, v, 64, 64, 0.5, 16))
    rp, ci, v = synth.random_csr(0, 20, 0.1, seed=7)
    out.append(("empty_matrix", rp, ci, v, 0, 20, 0.5, 16))
    rp, ci, v = synth.random_csr(40, 40, 0.0, seed=8)
    out.append(("all_rows_empty", rp, ci, v, 40, 40, 0.5, 16))
    rp, ci, v = synth.random_csr(1, 50, 0.3, seed=9)
    out.append(("single_row", rp, ci, v, 1, 50, 0.5, 16))
    rp, ci, v = synth.random_csr(37, 29, 0.15, seed=10, empty_row_frac=0.3)
    out.append(("ragged_37x29_empty_rows", rp, ci, v, 37, 29, 0.5, 16))
    rp, ci, v = synth.random_csr(53, 70, 0.1, seed=11, dup_frac=0.2, shuffle_cols=True)
    out.append(("duplicates_unsorted", rp, ci, v, 53, 70, 0.5, 16))
    for tau in (0.0, 0.3, 0.8, 1.0):
        rp, ci, v = synth.random_csr(70, 90, 0.05, seed=12)
        out.append((f"tau_{tau}", rp, ci, v, 70, 90, tau, 16))
    for w in (1, 4, 7):
        rp, ci, v = synth.random_csr(60, 80, 0.05, seed=13)
        out.append((f"width_{w}", rp, ci, v, 60, 80, 0.5, w))
    return out


def main():
    if not oracle.ref_available():
        oracle.build()
    for name, rp, ci, v, M, K, tau, w in cases():
        rp = np.asarray(rp, dtype=np.int64)
        ci = np.asarray(ci, dtype=np.int64)
        v = np.asarray(v, dtype=np.float32)
        perm = oracle.ref_cluster(rp, ci, M, K, tau, w)
        perm32 = oracle.ref_cluster(rp, ci, M, K, tau, w, index_dtype=np.int32)
        assert np.array_equal(perm, perm32), name
        prp, pci, pv = oracle.ref_permute(rp, ci, v, perm, K)
        brp, bci, bv = oracle.ref_csr_to_bcsr(rp, ci, v, M, K, 16, 16)
        pbrp, pbci, pbv = oracle.ref_csr_to_bcsr(prp, pci, pv, M, K, 16, 16)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), M=M, K=K, tau=np.float32(tau), w=w,
                            row_ptr=rp, col_ind=ci, vals=v, perm=perm,
                            p_row_ptr=prp, p_col_ind=pci, p_vals=pv,
                            b_row_ptr=brp, b_col_ind=bci, b_vals=bv,
                            pb_row_ptr=pbrp, pb_col_ind=pbci, pb_vals=pbv)
        print(f"{name:28s} M={M:5d} K={K:5d} nnz={int(rp[-1]):6d} nnzb={int(brp[-1]):5d}"
              f" -> {int(pbrp[-1]):5d}")


if __name__ == "__main__":
    main()
