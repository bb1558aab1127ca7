"""GPU test of the reference-shaped C++ API (include/xspmm/xspmm.hpp): builds
tests/cpp/pipeline_example.cpp against the headers and libxspmm_b200.so, runs it on a seeded
hidden-block matrix and checks its outputs against the CPU oracle: the clustering permutation
bit-exact, C from the Tier-2 call and from the explicit clustering -> permute -> convert -> Tier 1
-> unpermute chain within tolerance, and the two C's identical to each other."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from tests.util import errors
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_api_pipeline(tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if shutil.which("g++") is None:
        pytest.skip("no host C++ compiler")
    exe = tmp_path / "pipeline_example"
    lib_dir = os.path.join(ROOT, "xspmm_b200")
    subprocess.run(["g++", "-std=c++20", "-O2", "-I" + os.path.join(ROOT, "include"),
                    "-I/usr/local/cuda/include", os.path.join(ROOT, "tests", "cpp", "pipeline_example.cpp"),
                    "-L" + lib_dir, "-lxspmm_b200", "-Wl,-rpath," + lib_dir, "-o", str(exe)],
                   check=True)
    P = synth.cfg2_hidden_block(seed=13, n=2048, N=40, block_density=0.02)
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as f:
        np.array([P.M, P.K, P.N, P.nnz], dtype=np.int64).tofile(f)
        P.row_ptr.astype(np.int32).tofile(f)
        P.col_ind.astype(np.int32).tofile(f)
        P.values.astype(np.float16).tofile(f)
        P.B.astype(np.float16).tofile(f)
    out = tmp_path / "out.bin"
    r = subprocess.run([str(exe), str(inp), str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    raw = open(out, "rb").read()
    M, N = P.M, P.N
    perm = np.frombuffer(raw, dtype=np.int32, count=M)
    off = 4 * M
    C1 = np.frombuffer(raw, dtype=np.float32, count=M * N, offset=off).reshape(M, N)
    C2 = np.frombuffer(raw, dtype=np.float32, count=M * N, offset=off + 4 * M * N).reshape(M, N)
    tm = np.frombuffer(raw, dtype=np.float64, count=6, offset=off + 8 * M * N)
    ref_perm = oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K)
    assert np.array_equal(perm, ref_perm)
    prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values, ref_perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
    ref = oracle.unpermute_dense(oracle.bcsr_spmm_f64(M, P.K, N, brp, bci, bv, P.B), ref_perm)
    assert errors(ref, C1, 1e-3)["max_rel_guarded"] <= 1e-3
    assert np.array_equal(C1.view(np.uint32), C2.view(np.uint32))
    assert tm[5] > 0 and tm[0] > 0
    C3 = np.frombuffer(raw, dtype=np.float32, count=M * N, offset=off + 8 * M * N + 48).reshape(M, N)
    assert np.array_equal(C1.view(np.uint32), C3.view(np.uint32))  # SpMMPlan: same product


def test_cpp_dist_api(tmp_path):
    """tests/cpp/dist_example.cpp: the matrix split over the process's GPUs (one thread each; one
    GPU gives one rank), B broadcast from rank 0, C gathered there in the caller's row order and
    compared with the CPU oracle; every rank holds its share of the blocks."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if shutil.which("g++") is None:
        pytest.skip("no host C++ compiler")
    exe = tmp_path / "dist_example"
    lib_dir = os.path.join(ROOT, "xspmm_b200")
    subprocess.run(["g++", "-std=c++20", "-O2", "-pthread", "-I" + os.path.join(ROOT, "include"),
                    "-I/usr/local/cuda/include",
                    os.path.join(ROOT, "tests", "cpp", "dist_example.cpp"),
                    "-L" + lib_dir, "-lxspmm_b200", "-Wl,-rpath," + lib_dir, "-o", str(exe)],
                   check=True)
    P = synth.cfg4_banded(n=1 << 14, N=24)
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as f:
        np.array([P.M, P.K, P.N, P.nnz], dtype=np.int64).tofile(f)
        P.row_ptr.astype(np.int32).tofile(f)
        P.col_ind.astype(np.int32).tofile(f)
        P.values.astype(np.float16).tofile(f)
        P.B.astype(np.float16).tofile(f)
    nranks = min(torch.cuda.device_count(), 2)
    out = tmp_path / "out.bin"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([str(exe), str(nranks), str(inp), str(out)], capture_output=True,
                       text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    raw = open(out, "rb").read()
    M, N = P.M, P.N
    C = np.frombuffer(raw, dtype=np.float32, count=M * N).reshape(M, N)
    blocks = np.frombuffer(raw, dtype=np.int64, count=nranks, offset=4 * M * N)
    total = int(np.frombuffer(raw, dtype=np.int64, count=1, offset=4 * M * N + 8 * nranks)[0])
    assert int(blocks.sum()) == total > 0
    perm = oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K)
    prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values, perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
    ref = oracle.unpermute_dense(oracle.bcsr_spmm_f64(M, P.K, N, brp, bci, bv, P.B), perm)
    assert errors(ref, C, 1e-3)["max_rel_guarded"] <= 1e-3
