"""The Tier-2 pipeline on every generator family (xspmm_b200.generators, rows shuffled as the
reference's examples do before clustering): clustering permutation and permuted BCSR bit-exact
against the oracle, C within the fp16 tolerance, through the C ABI."""
import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import errors
from xspmm_b200 import generators as gen

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("family", sorted(gen.FAMILIES))
def test_family_pipeline(executor, family):
    n, N = 1500, 64
    rp, ci, v = gen.FAMILIES[family](n, seed=11, dtype=np.float16)
    rp, ci, v, _ = gen.shuffle_rows(rp, ci, v, seed=12)
    B = np.random.default_rng(13).standard_normal((n, N)).astype(np.float16)
    A = xs.CSRMatrix.from_host(executor, n, n, rp, ci, v, index_dtype=torch.int32)
    perm = torch.zeros(n, dtype=torch.int32, device=executor.device)
    xs.compute_1d_jaccard_clustering(executor, A, 0.5, 16, perm)
    ref_perm = oracle.cluster_fast(rp, ci, n, n)
    assert np.array_equal(perm.cpu().numpy(), ref_perm)
    P = xs.apply_permutation(executor, A, perm)
    Bm = xs.csr_to_bcsr(executor, P, 16, 16)
    prp, pci, pv = oracle.permute_rows(rp, ci, v, ref_perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, n, n)
    assert np.array_equal(Bm.row_ptr.cpu().numpy(), brp)
    assert np.array_equal(Bm.col_ind.cpu().numpy(), bci)
    assert np.array_equal(Bm.values.cpu().numpy().reshape(-1).view(np.uint16),
                          bv.reshape(-1).view(np.uint16))
    C = torch.full((n, N), float("nan"), dtype=torch.float32, device=executor.device)
    t = xs.SpMMTimings()
    xs.spmm(executor, A, torch.as_tensor(B).to(executor.device), C, N, 16, True, t)
    ref = oracle.unpermute_dense(oracle.bcsr_spmm_f64(n, n, N, brp, bci, bv, B), ref_perm)
    e = errors(ref, C.cpu().numpy(), 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e  # the fixed bar, long block rows included
    assert t.total_pipeline_ms > 0
