"""Matrix Market input: the Python reader (xspmm_b200.mtx) and the C++ header
(include/xspmm/io/matrix_market.hpp) against the reference's own read_mtx (utils/matrix_io.hpp,
compiled into oracle/_ref) on the same files, including the malformed lines its parser tolerates.
CPU only."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from xspmm_b200 import mtx

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="compiled reference absent")

HAND_WRITTEN = {
    "basic": "%%MatrixMarket matrix coordinate real general\n% a comment\n3 4 4\n"
             "1 1 1.5\n3 4 2\n2 2 -0.25e1\n1 2 7\n",
    "pattern": "%%MatrixMarket matrix coordinate pattern general\n4 4 3\n4 1\n1 4\n2 2\n",
    "complex_real_part": "%%MatrixMarket matrix coordinate complex general\n2 2 2\n"
                         "1 1 1.25 -3\n2 1 -0.5 8\n",
    "blank_and_comment_lines": "%%MatrixMarket matrix coordinate real general\n%\n\n5 5 3\n\n"
                               "% mid comment\n5 5 1\n\n1 3 2\n3 1 3\n",
    "out_of_range_dropped": "%%MatrixMarket matrix coordinate real general\n3 3 5\n"
                            "0 1 1\n4 1 1\n1 0 1\n1 4 1\n-2 1 1\n2 2 9\n",
    "malformed_lines": "%%MatrixMarket matrix coordinate real general\n3 3 8\n"
                       "1x 2 5\n2 3x 6\n1 1 abc\n1 2 1.5xyz\n2 1 nan\n3 3 2e\n3 1 4E+\n"
                       "2 2 .5\n3 2 +7.\n  % not a comment\n1 3\t-1e-3\n",
    "unsorted": "%%MatrixMarket matrix coordinate real general\n4 4 6\n4 4 1\n1 3 2\n2 1 3\n"
                "1 1 4\n4 2 5\n3 3 6\n",
    "rounding": "%%MatrixMarket matrix coordinate real general\n2 3 5\n1 1 0.1\n1 2 1e-8\n"
                "1 3 3.4028235e38\n2 1 16777217\n2 2 1.0000000596046448\n",
    "header_extra_tokens": "%%MatrixMarket matrix coordinate real general\n2 2 1 junk\n1 1 3\n",
    "empty_matrix": "%%MatrixMarket matrix coordinate real general\n3 2 0\n",
}


def _write(tmp_path, name, text):
    p = tmp_path / (name + ".mtx")
    p.write_text(text)
    return str(p)


def _random_file(tmp_path, seed, M=300, K=200, nnz=4000, dups=False):
    rng = np.random.default_rng(seed)
    r = rng.integers(1, M + 1, nnz)
    c = rng.integers(1, K + 1, nnz)
    if not dups:
        key = np.unique(r * (K + 1) + c)
        r, c = key // (K + 1), key % (K + 1)
        order = rng.permutation(len(r))
        r, c = r[order], c[order]
    v = rng.standard_normal(len(r)) * 10.0 ** rng.integers(-6, 6, len(r))
    lines = [f"{a} {b} {x:.9g}" for a, b, x in zip(r, c, v)]
    text = f"%%MatrixMarket matrix coordinate real general\n{M} {K} {len(r)}\n" + "\n".join(lines) + "\n"
    return _write(tmp_path, f"rand{seed}", text)


def _same_as_ref(path, got):
    M, K, rp, ci, v = oracle.ref_read_mtx(path)
    assert (got.num_rows, got.num_cols) == (M, K)
    np.testing.assert_array_equal(got.row_ptr, rp)
    np.testing.assert_array_equal(got.col_ind, ci)
    np.testing.assert_array_equal(got.values.view(np.uint32), v.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("name", sorted(HAND_WRITTEN))
def test_python_reader_matches_reference(tmp_path, name):
    p = _write(tmp_path, name, HAND_WRITTEN[name])
    _same_as_ref(p, mtx.read_mtx(p))


@needs_ref
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_python_reader_matches_reference_random(tmp_path, seed):
    p = _random_file(tmp_path, seed)
    _same_as_ref(p, mtx.read_mtx(p))


@needs_ref
def test_duplicates_same_multiset_stable_order(tmp_path):
    text = ("%%MatrixMarket matrix coordinate real general\n3 3 5\n"
            "2 2 1\n1 1 5\n2 2 2\n1 1 6\n2 2 3\n")
    p = _write(tmp_path, "dups", text)
    got = mtx.read_mtx(p)
    M, K, rp, ci, v = oracle.ref_read_mtx(p)
    np.testing.assert_array_equal(got.row_ptr, rp)
    np.testing.assert_array_equal(got.col_ind, ci)
    for r in range(M):  # same values per row; the order of equal keys is ours: file order
        a, b = got.values[got.row_ptr[r]:got.row_ptr[r + 1]], v[rp[r]:rp[r + 1]]
        np.testing.assert_array_equal(np.sort(a), np.sort(b))
    np.testing.assert_array_equal(got.values, [5, 6, 1, 2, 3])


def test_missing_dimensions_raise(tmp_path):
    with pytest.raises(ValueError):
        mtx.read_mtx(_write(tmp_path, "nodims", "%%MatrixMarket matrix coordinate real general\n"))
    with pytest.raises(ValueError):
        mtx.read_mtx(_write(tmp_path, "baddims", "% c\n3 x 4\n1 1 1\n"))
    with pytest.raises(RuntimeError):
        mtx.read_mtx(str(tmp_path / "does_not_exist.mtx"))


def test_write_read_round_trip(tmp_path):
    rng = np.random.default_rng(3)
    M, K = 50, 70
    mask = rng.random((M, K)) < 0.05
    rows, cols = np.nonzero(mask)
    vals = rng.standard_normal(len(rows)).astype(np.float32)
    rp = np.zeros(M + 1, dtype=np.int64)
    np.cumsum(np.bincount(rows, minlength=M), out=rp[1:])
    p = str(tmp_path / "rt.mtx")
    mtx.write_mtx(p, M, K, rp, cols, vals, comment="round trip")
    got = mtx.read_mtx(p)
    np.testing.assert_array_equal(got.row_ptr, rp)
    np.testing.assert_array_equal(got.col_ind, cols)
    np.testing.assert_array_equal(got.values, vals)


def test_expand_symmetry(tmp_path):
    text = ("%%MatrixMarket matrix coordinate real symmetric\n3 3 3\n1 1 1\n3 1 2\n3 2 -4\n")
    p = _write(tmp_path, "sym", text)
    plain = mtx.read_mtx(p)
    assert plain.nnz == 3  # the reference reads the stored triangle only
    full = mtx.read_mtx(p, expand_symmetry=True)
    dense = np.zeros((3, 3), np.float32)
    for r in range(3):
        for j in range(full.row_ptr[r], full.row_ptr[r + 1]):
            dense[r, full.col_ind[j]] = full.values[j]
    np.testing.assert_array_equal(dense, dense.T)
    skew = _write(tmp_path, "skew", text.replace("symmetric", "skew-symmetric").replace("1 1 1\n", ""))
    s = mtx.read_mtx(skew, expand_symmetry=True)
    dense = np.zeros((3, 3), np.float32)
    for r in range(3):
        for j in range(s.row_ptr[r], s.row_ptr[r + 1]):
            dense[r, s.col_ind[j]] = s.values[j]
    np.testing.assert_array_equal(dense, -dense.T)


def test_fp16_values(tmp_path):
    p = _write(tmp_path, "h", HAND_WRITTEN["basic"])
    got = mtx.read_mtx(p, value_dtype=np.float16)
    assert got.values.dtype == np.float16
    np.testing.assert_array_equal(got.values, mtx.read_mtx(p).values.astype(np.float16))


CPP_DRIVER = r"""
#include <cstdio>
#include <cstring>
#include "xspmm/io/matrix_market.hpp"
int main(int argc, char** argv) {
    for (int i = 1; i < argc; ++i) {
        try {
            auto m = matrix_utils::io::read_mtx<float>(argv[i]);
            std::printf("%d %d %zu\n", m.num_rows, m.num_cols, m.values.size());
            for (int x : m.row_ptr) std::printf("%d ", x);
            std::printf("\n");
            for (int x : m.col_ind) std::printf("%d ", x);
            std::printf("\n");
            for (float v : m.values) { unsigned u; std::memcpy(&u, &v, 4); std::printf("%u ", u); }
            std::printf("\n");
        } catch (const std::exception& e) {
            std::printf("ERR\n\n\n\n");
        }
    }
    return 0;
}
"""


@needs_ref
@pytest.mark.skipif(shutil.which("g++") is None, reason="no g++")
def test_cpp_header_matches_reference(tmp_path):
    src = tmp_path / "drv.cpp"
    src.write_text(CPP_DRIVER)
    exe = tmp_path / "drv"
    subprocess.run(["g++", "-std=c++20", "-O2", "-I" + os.path.join(ROOT, "include"), str(src),
                    "-o", str(exe)], check=True)
    paths = [_write(tmp_path, n, t) for n, t in sorted(HAND_WRITTEN.items())]
    paths += [_random_file(tmp_path, s) for s in (4, 5)]
    out = subprocess.run([str(exe)] + paths, check=True, capture_output=True, text=True).stdout
    lines = out.split("\n")
    for i, p in enumerate(paths):
        head, rp, ci, vb = lines[4 * i:4 * i + 4]
        M, K, rrp, rci, rv = oracle.ref_read_mtx(p)
        assert head == f"{M} {K} {len(rv)}", p
        assert [int(x) for x in rp.split()] == rrp.tolist()
        assert [int(x) for x in ci.split()] == rci.tolist()
        assert [int(x) for x in vb.split()] == rv.view(np.uint32).tolist()
