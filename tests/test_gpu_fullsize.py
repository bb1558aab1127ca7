"""Parity at the configs' full sizes.

* cfg1/cfg2/cfg3 (4096^2 1 %, 16384^2 hidden blocks, 4096 x 11008 pruned): the GPU's clustering
  permutation, permuted CSR and BCSR (structure and values) against the reference itself -- its
  host code compiled from its sources (oracle/_ref) -- bit for bit.
* cfg4 (2,000,000 rows) and cfg5 (R-MAT 2^20): the permutation and the permuted BCSR structure
  against SHA-256 digests of the oracle's (tests/golden/fullsize.json, made by
  tests/golden/make_fullsize.py; the oracle's fast exact clustering is pinned to the reference's
  loop at 2^13-2^15 rows in tests/test_oracle.py).
* C: the Tier-2 call on full cfg2 (N=256) against the fp64 oracle on every entry; on full cfg4
  and cfg5, 512 sampled rows against an fp64 product of the host CSR rows (C is in the caller's
  row order, so no clustering is needed on the host). Tolerance 1e-3 guarded (fp16 inputs)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import GOLDEN, errors
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu


def _digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<i4").tobytes()).hexdigest()


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3"])
def test_fullsize_structure_vs_compiled_reference(executor, name):
    if not oracle.ref_available():
        pytest.skip("compiled reference absent")
    P = {"cfg1": lambda: synth.cfg1_plumbing(), "cfg2": lambda: synth.cfg2_hidden_block(N=8),
         "cfg3": lambda: synth.cfg3_pruned_llm(N=8)}[name]()
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    perm = torch.zeros(P.M, dtype=torch.int32, device=executor.device)
    xs.compute_1d_jaccard_clustering(executor, A, 0.5, 16, perm)
    ref_perm = oracle.ref_cluster(P.row_ptr, P.col_ind, P.M, P.K, 0.5, 16)
    assert np.array_equal(_np(perm), ref_perm), "clustering permutation"
    Pm = xs.apply_permutation(executor, A, perm)
    rrp, rci, rv = oracle.ref_permute(P.row_ptr, P.col_ind, P.values, ref_perm, P.K)
    assert np.array_equal(_np(Pm.row_ptr), rrp) and np.array_equal(_np(Pm.col_ind), rci)
    assert np.array_equal(_np(Pm.values).astype(np.float32).view(np.uint32), rv.view(np.uint32))
    Bm = xs.csr_to_bcsr(executor, Pm, 16, 16)
    brp, bci, bv = oracle.ref_csr_to_bcsr(rrp, rci, rv, P.M, P.K)
    assert np.array_equal(_np(Bm.row_ptr), brp) and np.array_equal(_np(Bm.col_ind), bci)
    assert np.array_equal(_np(Bm.values).reshape(-1).astype(np.float32).view(np.uint32),
                          np.asarray(bv, np.float32).reshape(-1).view(np.uint32))


@pytest.mark.parametrize("name", ["cfg4_banded_2M", "cfg5_rmat_2^20"])
def test_fullsize_structure_vs_oracle_digests(executor, name):
    gold = json.load(open(os.path.join(GOLDEN, "fullsize.json")))[name]
    P = synth.cfg4_banded(N=8) if name.startswith("cfg4") else synth.cfg5_rmat(N=8)
    assert (P.M, P.nnz) == (gold["M"], gold["nnz"]), "generator output changed"
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    perm = torch.zeros(P.M, dtype=torch.int32, device=executor.device)
    xs.compute_1d_jaccard_clustering(executor, A, 0.5, 16, perm)
    assert _digest(_np(perm)) == gold["perm_sha256"], "clustering permutation"
    Pm = xs.apply_permutation(executor, A, perm)
    del A
    Bm = xs.csr_to_bcsr(executor, Pm, 16, 16)
    assert Bm.num_blocks == gold["nnzb"]
    assert _digest(_np(Bm.row_ptr)) == gold["bcsr_row_ptr_sha256"]
    assert _digest(_np(Bm.col_ind)) == gold["bcsr_col_ind_sha256"]


def test_fullsize_cfg2_tier2_c(executor):
    P = synth.cfg2_hidden_block(N=256)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    B = torch.as_tensor(P.B).to(executor.device)
    C = torch.full((P.M, P.N), float("nan"), device=executor.device)
    xs.spmm(executor, A, B, C, P.N, 16, True)
    perm = oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K)
    prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values, perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
    ref = oracle.unpermute_dense(oracle.bcsr_spmm_f64(P.M, P.K, P.N, brp, bci, bv, P.B), perm)
    e = errors(ref, _np(C), 1e-3)
    print("cfg2 full Tier-2:", e)
    assert e["max_rel_guarded"] <= 1e-3, e


@pytest.mark.parametrize("name", ["cfg4", "cfg5"])
def test_fullsize_tier2_c_sampled_rows(executor, name):
    P = synth.cfg4_banded(N=64) if name == "cfg4" else synth.cfg5_rmat(N=128)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    B = torch.as_tensor(P.B).to(executor.device)
    C = torch.full((P.M, P.N), float("nan"), device=executor.device)
    xs.spmm(executor, A, B, C, P.N, 16, True)
    rows = np.sort(np.random.default_rng(7).choice(P.M, 512, replace=False))
    got = _np(C[torch.as_tensor(rows, device=executor.device)]).astype(np.float64)
    Bh = P.B.astype(np.float64)
    ref = np.stack([P.values[P.row_ptr[r]:P.row_ptr[r + 1]].astype(np.float64) @
                    Bh[P.col_ind[P.row_ptr[r]:P.row_ptr[r + 1]]] for r in rows])
    assert np.isfinite(got).all()
    e = errors(ref, got, 1e-3)
    print(name, "full Tier-2, sampled rows:", e)
    assert e["max_rel_guarded"] <= 1e-3, e
