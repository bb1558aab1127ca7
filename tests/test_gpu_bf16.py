"""GPU tests of bf16 inputs (values and B in bf16, C in fp32): every Tier-1 kernel (mma.sync and
tcgen05 with the bf16 instruction forms, the gather kernels of a plan, the block-shape kernel),
Tier 2 with clustering, and a one-rank distributed plan, against the fp64 oracle run on the same
bf16-rounded numbers. bf16 x bf16 products are exact in fp32 and every path accumulates in fp32 or
better, so the bar is the fp16 one: 1e-3, guarded. The permutation depends on the pattern only,
so it must equal the fp16 matrix's."""
import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import errors
from xspmm_b200 import dist as xd
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu


def _bf16(a):
    """bf16-rounded copy (as float32 numbers) and the bf16 tensor."""
    t = torch.as_tensor(np.asarray(a, np.float32)).to(torch.bfloat16)
    return t.float().numpy(), t


def _problem(P, seed):
    v32, v16 = _bf16(P.values.astype(np.float32))
    B32, B16 = _bf16(np.random.default_rng(seed).standard_normal((P.K, P.N)))
    return v32, v16, B32, B16


def _oracle(P, v32, B32, perm=None):
    rp, ci, v = P.row_ptr, P.col_ind, v32
    if perm is not None:
        rp, ci, v = oracle.permute_rows(rp, ci, v, perm)
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, v, P.M, P.K)
    ref = oracle.bcsr_spmm_f64(P.M, P.K, B32.shape[1], brp, bci, bv, B32)
    return oracle.unpermute_dense(ref, perm) if perm is not None else ref


@pytest.mark.parametrize("kind", ["mma", "tc"])
@pytest.mark.parametrize("idx", [torch.int32, torch.int64])
def test_bf16_tier1_tensor_core_kernels(executor, kind, idx):
    P = synth.cfg3_pruned_llm(seed=61, M=512, K=2048, N=256)
    v32, v16, B32, B16 = _problem(P, 62)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, v16,
                               value_dtype=torch.bfloat16, index_dtype=idx)
    Ab = xs.csr_to_bcsr(executor, A, 16, 16)
    assert Ab.values.dtype == torch.bfloat16
    executor.set_tier1_kernel(kind)
    try:
        C = torch.full((P.M, P.N), float("nan"), device=executor.device)
        xs.spmm(Ab, B16.to(executor.device), C, P.N)
    finally:
        executor.set_tier1_kernel("auto")
    e = errors(_oracle(P, v32, B32), C.cpu().numpy(), 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, (kind, e)


def test_bf16_plan_gather_and_block_kernels(executor):
    """R-MAT rows (gather kernels, hub rows chunked) plus dense block rows (mma.sync)."""
    P = synth.cfg5_rmat(seed=63, scale=12, N=64)
    v32, v16, B32, B16 = _problem(P, 64)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, v16,
                               value_dtype=torch.bfloat16, index_dtype=torch.int32)
    with xs.SpMMPlan(executor, A, 16, False) as plan:
        C1 = torch.full((P.M, P.N), float("nan"), device=executor.device)
        C2 = torch.full((P.M, P.N), float("nan"), device=executor.device)
        plan.execute(B16.to(executor.device), C1, P.N)
        plan.execute(B16.to(executor.device), C2, P.N)
        assert torch.equal(C1, C2)
    e = errors(_oracle(P, v32, B32), C1.cpu().numpy(), 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e


@pytest.mark.parametrize("idx", [torch.int32, torch.int64])
def test_bf16_tier2_clustering_and_dist(executor, idx):
    P = synth.cfg2_hidden_block(seed=65, n=2048, N=48, block_density=0.03)
    v32, v16, B32, B16 = _problem(P, 66)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, v16,
                               value_dtype=torch.bfloat16, index_dtype=idx)
    A16 = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                                 index_dtype=idx)
    p_bf, p_f16 = (torch.zeros(P.M, dtype=idx, device=executor.device) for _ in range(2))
    xs.compute_1d_jaccard_clustering(executor, A, 0.5, 16, p_bf)
    xs.compute_1d_jaccard_clustering(executor, A16, 0.5, 16, p_f16)
    assert torch.equal(p_bf, p_f16)
    perm = p_bf.cpu().numpy()
    Ap = xs.apply_permutation(executor, A, p_bf)
    rp, ci, v = oracle.permute_rows(P.row_ptr, P.col_ind, v32, perm)
    assert np.array_equal(Ap.values.float().cpu().numpy(), v)  # the bits moved unchanged
    B = B16.to(executor.device)
    C = torch.full((P.M, P.N), float("nan"), device=executor.device)
    xs.spmm(executor, A, B, C, P.N, 16, True)
    ref = _oracle(P, v32, B32, perm)
    e = errors(ref, C.cpu().numpy(), 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e
    with xd.DistComm(executor, 1, 0, xd.unique_id(), timeout_ms=30000) as comm:
        with xd.DistPlan(comm, A) as dp:
            Cl = torch.full((dp.num_rows, P.N), float("nan"), device=executor.device)
            dp.execute(B, Cl, P.N)
            C3 = torch.full((P.M, P.N), float("nan"), device=executor.device)
            dp.gather(Cl, C3, P.N)
            assert torch.equal(C, C3)


def test_bf16_other_block_shape(executor):
    M, K, N = 200, 150, 40
    rp, ci, v = synth.random_csr(M, K, 0.05, seed=67)
    v32, v16 = _bf16(np.asarray(v, np.float32))
    B32, B16 = _bf16(np.random.default_rng(68).standard_normal((K, N)))
    A = xs.CSRMatrix.from_host(executor, M, K, rp, ci, v16, value_dtype=torch.bfloat16,
                               index_dtype=torch.int32)
    Ab = xs.csr_to_bcsr(executor, A, 8, 4)
    C = torch.full((M, N), float("nan"), device=executor.device)
    xs.spmm(Ab, B16.to(executor.device), C, N)
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, v32, M, K, 8, 4)
    ref = oracle.bcsr_spmm_f64(M, K, N, brp, bci, bv, B32, 8, 4)
    e = errors(ref, C.cpu().numpy(), 1e-6)
    assert e["max_rel_guarded"] <= 1e-6, e
