"""Generator families (xspmm_b200.generators) on the CPU: the deterministic structures equal the
reference's own generators (utils/matrix_gen.hpp, compiled into oracle/_ref); the random ones
keep the properties their definitions state; and on every family the oracle's clustering and
conversion equal the reference's host code on the reference's own generated matrices."""
import numpy as np
import pytest

import oracle
from xspmm_b200 import generators as gen

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="compiled reference absent")


def _dense_pattern(rp, ci, M, K):
    D = np.zeros((M, K), dtype=bool)
    for r in range(M):
        D[r, ci[rp[r]:rp[r + 1]]] = True
    return D


def _check_csr(rp, ci, v, M, K):
    assert rp[0] == 0 and np.all(np.diff(rp) >= 0) and rp[-1] == len(ci) == len(v)
    for r in range(M):
        row = ci[rp[r]:rp[r + 1]]
        assert np.all(np.diff(row) > 0), "columns ascending and distinct"
        assert row.size == 0 or (row[0] >= 0 and row[-1] < K)
    assert v.size == 0 or (v.min() >= 0.1 and v.max() < 1.0)


@needs_ref
@pytest.mark.parametrize("size,bw", [(1, 0), (17, 1), (100, 8), (40, 200), (64, 0)])
def test_banded_equals_reference(size, bw):
    rp, ci, v = gen.banded(size, bw)
    _, rrp, rci, _ = oracle.ref_generate("banded", size, bw)
    np.testing.assert_array_equal(rp, rrp)
    np.testing.assert_array_equal(ci, rci)
    _check_csr(rp, ci, v, size, size)


@needs_ref
@pytest.mark.parametrize("size,w", [(50, 0), (50, 3), (30, 60), (1, 1)])
def test_arrowhead_equals_reference(size, w):
    rp, ci, v = gen.arrowhead(size, w)
    _, rrp, rci, _ = oracle.ref_generate("arrowhead", size, w)
    np.testing.assert_array_equal(rp, rrp)
    np.testing.assert_array_equal(ci, rci)


@needs_ref
@pytest.mark.parametrize("rows,cols,bs", [(37, 53, 1), (37, 53, 4), (64, 64, 16), (20, 100, 7)])
def test_checkers_equals_reference(rows, cols, bs):
    rp, ci, v = gen.checkers(rows, cols, bs)
    _, rrp, rci, _ = oracle.ref_generate("checkers", rows, cols, bs)
    np.testing.assert_array_equal(rp, rrp)
    np.testing.assert_array_equal(ci, rci)


def test_random_family_properties():
    n = 300
    rp, ci, v = gen.triangular(n, True, 0.05, seed=1)
    D = _dense_pattern(rp, ci, n, n)
    assert np.all(np.diag(D)) and not np.any(np.tril(D, -1))
    rp, ci, v = gen.triangular(n, False, 0.05, seed=1)
    D = _dense_pattern(rp, ci, n, n)
    assert np.all(np.diag(D)) and not np.any(np.triu(D, 1))
    rp, ci, v = gen.hessenberg(n, True, 0.05, seed=2)
    D = _dense_pattern(rp, ci, n, n)
    assert not np.any(np.tril(D, -2)) and np.all(np.diag(D, -1)) and np.all(np.diag(D, 1))
    rp, ci, v = gen.hessenberg(n, False, 0.05, seed=2)
    D = _dense_pattern(rp, ci, n, n)
    assert not np.any(np.triu(D, 2)) and np.all(np.diag(D, -1))
    rp, ci, v = gen.block_diagonal(n, 32, 0.3, seed=3)
    D = _dense_pattern(rp, ci, n, n)
    ii, jj = np.nonzero(D)
    assert np.all(ii // 32 == jj // 32) and np.all(np.diag(D))
    rp, ci, v = gen.near_symmetric(n, 0.05, 0.0, seed=4)  # no drops: symmetric
    D = _dense_pattern(rp, ci, n, n)
    assert np.array_equal(D, D.T)
    rp, ci, v = gen.power_law(n, 200, 2.1, seed=5)
    deg = np.diff(rp)
    assert deg.min() >= 1 and deg.max() <= 200
    for f, K in ((gen.triangular(n, True, 0.05), n), (gen.hessenberg(n, True, 0.05), n),
                 (gen.block_diagonal(n, 32, 0.3), n), (gen.near_symmetric(n, 0.05, 0.2), n),
                 (gen.power_law(n, 200, 2.1), 200)):
        _check_csr(*f, n, K)


def test_shuffle_rows_is_a_row_permutation():
    rp, ci, v = gen.banded(50, 3)
    srp, sci, sv, order = gen.shuffle_rows(rp, ci, v, seed=9)
    assert sorted(order.tolist()) == list(range(50))
    for i, old in enumerate(order):
        np.testing.assert_array_equal(sci[srp[i]:srp[i + 1]], ci[rp[old]:rp[old + 1]])
        np.testing.assert_array_equal(sv[srp[i]:srp[i + 1]], v[rp[old]:rp[old + 1]])


def test_dense_values():
    d = gen.dense(7, 9, seed=1)
    assert d.shape == (7, 9) and d.min() >= 0.1 and d.max() < 1.0


REF_CASES = [
    ("banded", dict(a=300, b=5)),
    ("triangular", dict(a=200, b=1, f1=0.05)),
    ("hessenberg", dict(a=200, b=0, f1=0.05)),
    ("arrowhead", dict(a=200, b=6)),
    ("checkers", dict(a=150, b=170, c=8)),
    ("block_diagonal", dict(a=300, b=24, f1=0.4)),
    ("near_symmetric", dict(a=250, f1=0.03, f2=0.2)),
    ("power_law", dict(a=300, b=300, f1=2.1)),
]


@needs_ref
@pytest.mark.parametrize("kind,kw", REF_CASES, ids=[k for k, _ in REF_CASES])
@pytest.mark.parametrize("shuffled", [False, True], ids=["plain", "shuffled"])
def test_oracle_equals_reference_on_reference_families(kind, kw, shuffled):
    M, rp, ci, v = oracle.ref_generate(kind, **kw)
    K = kw.get("b", M) if kind in ("checkers", "power_law") else M
    if shuffled:
        rp, ci, v, _ = gen.shuffle_rows(rp, ci, v, seed=3)
    rp = np.asarray(rp, np.int64)
    ci = np.asarray(ci, np.int64)
    perm = oracle.cluster_fast(rp, ci, M, K)
    np.testing.assert_array_equal(perm, oracle.ref_cluster(rp, ci, M, K))
    prp, pci, pv = oracle.permute_rows(rp, ci, np.asarray(v, np.float32), perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, M, K)
    rbrp, rbci, rbv = oracle.ref_csr_to_bcsr(prp, pci, pv, M, K)
    np.testing.assert_array_equal(brp, rbrp)
    np.testing.assert_array_equal(bci, rbci)
    np.testing.assert_array_equal(np.asarray(bv, np.float32).reshape(-1), rbv.reshape(-1))
