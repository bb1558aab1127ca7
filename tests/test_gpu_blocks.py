"""GPU tests of block sizes other than 16.

* Tier 2 with hw_block_size != 16: the reference clusters with column blocks of width hw and
  converts to hw x hw blocks, then runs its 16x16 kernel on them (src/cuda/unstructured_mtx_mul.cu
  :83, :102, :39), so its C is wrong for hw != 16. Here the permutation must equal the reference's
  clustering with w = hw (the oracle, and the compiled reference where present) and C must be
  A * B within the fp16 tolerance (1e-3 guarded) -- through the one-shot call, a plan and a
  one-rank distributed plan.
* Tier 1 on an r x c BCSR (csr_to_bcsr with that shape): C = A * B, accumulated in fp64 and
  rounded once, so within 1e-6 (guarded) of the fp64 oracle for fp16 and fp32 values."""
import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import errors
from xspmm_b200 import dist as xd
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu


def _ref_c(P, B, w):
    perm = oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K, 0.5, w)
    prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values, perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
    return perm, oracle.unpermute_dense(
        oracle.bcsr_spmm_f64(P.M, P.K, B.shape[1], brp, bci, bv, B), perm)


@pytest.mark.parametrize("hw,idx", [(8, torch.int32), (32, torch.int64), (5, torch.int32),
                                    (1, torch.int64)])
def test_tier2_other_block_widths(executor, hw, idx):
    P = synth.cfg2_hidden_block(seed=50 + hw, n=2048, N=40, block_density=0.03)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=idx)
    perm = torch.zeros(P.M, dtype=idx, device=executor.device)
    xs.compute_1d_jaccard_clustering(executor, A, 0.5, hw, perm)
    ref_perm, ref = _ref_c(P, P.B, hw)
    assert np.array_equal(perm.cpu().numpy(), ref_perm)
    if oracle.ref_available():
        assert np.array_equal(ref_perm, oracle.ref_cluster(P.row_ptr, P.col_ind, P.M, P.K, 0.5, hw))
    B = torch.as_tensor(P.B).to(executor.device)
    C = torch.full((P.M, P.N), float("nan"), device=executor.device)
    t = xs.SpMMTimings()
    xs.spmm(executor, A, B, C, P.N, hw, True, t)
    e = errors(ref, C.cpu().numpy(), 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e
    assert t.clustering_ms > 0
    with xs.SpMMPlan(executor, A, hw, True) as plan:
        C2 = torch.full((P.M, P.N), float("nan"), device=executor.device)
        plan.execute(B, C2, P.N)
        assert torch.equal(C, C2)
    with xd.DistComm(executor, 1, 0, xd.unique_id(), timeout_ms=30000) as comm:
        with xd.DistPlan(comm, A, hw, True) as dp:
            Cl = torch.full((dp.num_rows, P.N), float("nan"), device=executor.device)
            dp.execute(B, Cl, P.N)
            C3 = torch.full((P.M, P.N), float("nan"), device=executor.device)
            dp.gather(Cl, C3, P.N)
            assert torch.equal(C, C3)


@pytest.mark.parametrize("rb,cb", [(8, 8), (3, 5), (32, 8), (1, 16), (16, 1), (7, 33)])
@pytest.mark.parametrize("vt", [np.float16, np.float32])
def test_tier1_other_block_shapes(executor, rb, cb, vt):
    rng = np.random.default_rng(rb * 100 + cb)
    M, K, N = 301, 277, (37 if vt == np.float16 else 130)
    rp, ci, v = synth.random_csr(M, K, 0.04, seed=rb + cb, empty_row_frac=0.1)
    v = np.asarray(v, vt)
    A = xs.CSRMatrix.from_host(executor, M, K, rp, ci, v,
                               index_dtype=torch.int32 if rb % 2 else torch.int64)
    Ab = xs.csr_to_bcsr(executor, A, rb, cb)
    assert (Ab.r_block, Ab.c_block) == (rb, cb)
    B = rng.standard_normal((K, N)).astype(vt)
    C = torch.full((M, N), float("nan"), device=executor.device)
    xs.spmm(Ab, torch.as_tensor(B).to(executor.device), C, N)
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, v, M, K, rb, cb)
    ref = oracle.bcsr_spmm_f64(M, K, N, brp, bci, bv, B, rb, cb)
    got = C.cpu().numpy()
    assert np.isfinite(got).all()
    e = errors(ref, got, 1e-6)
    assert e["max_rel_guarded"] <= 1e-6, e
