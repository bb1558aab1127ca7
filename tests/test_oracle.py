"""CPU tests of the checker itself: the C restatement (oracle/) against the golden fixtures made by
the reference's own host code, against that compiled code directly, and the SpMM restatement
against a dense fp64 product. No GPU."""
import os

import numpy as np
import pytest

import oracle
from tests.util import golden_cases, load_golden, dense_from_csr
from xspmm_b200 import synth

CASES = golden_cases()


def test_fixtures_present():
    assert len(CASES) >= 15


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(p)[:-4] for p in CASES])
def test_oracle_matches_golden(path):
    g = load_golden(path)
    M, K, tau, w = int(g["M"]), int(g["K"]), float(g["tau"]), int(g["w"])
    rp, ci, v = g["row_ptr"], g["col_ind"], g["vals"]
    assert np.array_equal(oracle.cluster_literal(rp, ci, M, K, tau, w), g["perm"])
    assert np.array_equal(oracle.cluster_fast(rp, ci, M, K, tau, w), g["perm"])
    prp, pci, pv = oracle.permute_rows(rp, ci, v, g["perm"])
    assert np.array_equal(prp, g["p_row_ptr"])
    assert np.array_equal(pci, g["p_col_ind"])
    assert np.array_equal(pv.view(np.uint32), g["p_vals"].view(np.uint32))
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, v, M, K, 16, 16)
    assert np.array_equal(brp, g["b_row_ptr"])
    assert np.array_equal(bci, g["b_col_ind"])
    assert np.array_equal(bv.view(np.uint32), g["b_vals"].view(np.uint32))
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, M, K, 16, 16)
    assert np.array_equal(brp, g["pb_row_ptr"])
    assert np.array_equal(bci, g["pb_col_ind"])
    assert np.array_equal(bv.view(np.uint32), g["pb_vals"].view(np.uint32))


def _random_case(seed):
    rng = np.random.default_rng(seed)
    M = int(rng.integers(0, 90))
    K = int(rng.integers(1, 220))
    dens = float(rng.choice([0.0, 0.01, 0.05, 0.2, 0.6]))
    rp, ci, v = synth.random_csr(M, K, dens, seed=seed,
                                 empty_row_frac=float(rng.choice([0, 0.3])),
                                 dup_frac=float(rng.choice([0, 0.1])),
                                 shuffle_cols=bool(rng.integers(0, 2)))
    tau = float(rng.choice([0.5, 0.5, 0.3, 0.8, 0.0, 1.0, 1.5, -0.1]))
    w = int(rng.choice([16, 16, 4, 7, 1]))
    return M, K, rp, ci, v, tau, w


@pytest.mark.parametrize("seed", range(40))
def test_fast_clustering_equals_literal(seed):
    M, K, rp, ci, v, tau, w = _random_case(seed)
    assert np.array_equal(oracle.cluster_fast(rp, ci, M, K, tau, w),
                          oracle.cluster_literal(rp, ci, M, K, tau, w))


@pytest.mark.skipif(not oracle.ref_available(), reason="compiled reference not built here")
@pytest.mark.parametrize("seed", range(40, 70))
def test_oracle_equals_compiled_reference(seed):
    M, K, rp, ci, v, tau, w = _random_case(seed)
    perm = oracle.ref_cluster(rp, ci, M, K, tau, w)
    assert np.array_equal(oracle.cluster_fast(rp, ci, M, K, tau, w), perm)
    assert np.array_equal(oracle.ref_cluster(rp, ci, M, K, tau, w, index_dtype=np.int32), perm)
    for a, b in zip(oracle.permute_rows(rp, ci, v, perm), oracle.ref_permute(rp, ci, v, perm, K)):
        assert np.array_equal(a, b)
    for rb, cb in ((16, 16), (4, 8), (1, w)):
        for a, b in zip(oracle.csr_to_bcsr(rp, ci, v, M, K, rb, cb),
                        oracle.ref_csr_to_bcsr(rp, ci, v, M, K, rb, cb)):
            assert np.array_equal(a, b)


@pytest.mark.skipif(not oracle.ref_available(), reason="compiled reference not built here")
@pytest.mark.parametrize("name,kw", [("cfg2", dict(n=2048)), ("cfg4", dict(n=4096)),
                                     ("cfg5", dict(scale=11)), ("cfg3", dict(M=256, K=688))])
def test_fast_clustering_on_config_structure(name, kw):
    P = synth.CONFIGS[name](**kw)
    assert np.array_equal(oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K),
                          oracle.ref_cluster(P.row_ptr, P.col_ind, P.M, P.K))


@pytest.mark.parametrize("seed", range(6))
def test_spmm_restatement_equals_dense_product(seed):
    rng = np.random.default_rng(seed)
    M, K, N = int(rng.integers(1, 70)), int(rng.integers(1, 70)), int(rng.integers(1, 20))
    rp, ci, v = synth.random_csr(M, K, 0.1, seed=seed, dup_frac=0.05)
    B = rng.standard_normal((K, N)).astype(np.float32)
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, v, M, K)
    C = oracle.bcsr_spmm_f64(M, K, N, brp, bci, bv, B)
    ref = dense_from_csr(M, K, rp, ci, v) @ B.astype(np.float64)
    assert np.allclose(C, ref, rtol=1e-12, atol=1e-12)


def test_unpermute_restatement():
    rng = np.random.default_rng(3)
    X = rng.standard_normal((9, 5)).astype(np.float32)
    perm = rng.permutation(9)
    out = oracle.unpermute_dense(X, perm)
    assert np.array_equal(out[perm], X)


@pytest.mark.skipif(not oracle.ref_available(), reason="compiled reference not built here")
@pytest.mark.parametrize("name,kw", [("cfg5", dict(scale=15)), ("cfg4", dict(n=1 << 16))])
def test_fast_clustering_pinned_at_the_largest_reference_sizes(name, kw):
    """The oracle's fast exact clustering equals the reference's own loop (compiled from its
    sources) on the R-MAT generator at 2^15 rows and the banded one at 2^16 rows -- about the
    largest the reference's dense-bitset loop finishes in seconds (10 s and 9 s here). The GPU
    tests compare full-size results with the fast clustering's digests."""
    P = synth.CONFIGS[name](**kw)
    perm = oracle.ref_cluster(P.row_ptr, P.col_ind, P.M, P.K)
    assert np.array_equal(oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K), perm)
    rp, ci, v = oracle.ref_permute(P.row_ptr, P.col_ind, P.values, perm, P.K)
    for a, b in zip(oracle.csr_to_bcsr(rp, ci, v, P.M, P.K),
                    oracle.ref_csr_to_bcsr(rp, ci, v, P.M, P.K)):
        assert np.array_equal(a, b)
