"""GPU tests of the tcgen05/TMEM Tier-1 kernel (block rows stacked to M=128, TMA-fed), forced
through xspmm_set_tier1_kernel, against the fp64 oracle and against the mma.sync kernel."""
import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import errors, fp32_block_emulation
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu


def _run(executor, kind, M, K, N, rp, ci, v, seed=0, row_map=None):
    rng = np.random.default_rng(seed)
    B = rng.standard_normal((K, N)).astype(np.float16)
    A = xs.CSRMatrix.from_host(executor, M, K, rp, ci, np.asarray(v, np.float16),
                               index_dtype=torch.int32)
    Ab = xs.csr_to_bcsr(executor, A, 16, 16)
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=executor.device)
    executor.set_tier1_kernel(kind)
    try:
        xs.api._tier1(Ab, torch.as_tensor(B).to(executor.device), C, N,
                      out_row_map=None if row_map is None else
                      torch.as_tensor(row_map.astype(np.int32)).to(executor.device))
        executor.synchronize()
    finally:
        executor.set_tier1_kernel("auto")
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, np.asarray(v, np.float16), M, K)
    ref = oracle.bcsr_spmm_f64(M, K, N, brp, bci, bv, B)
    if row_map is not None:
        ref = oracle.unpermute_dense(ref, row_map)
    got = C.cpu().numpy()
    assert np.isfinite(got).all(), "C not fully written"
    e = errors(ref, got, 1e-3)
    bound = 1e-3
    if e["max_rel_guarded"] > bound:  # long rows: no worse than twice an fp32 emulation
        emu = fp32_block_emulation(M, N, brp, bci, bv, B)
        if row_map is not None:
            emu = oracle.unpermute_dense(emu, row_map)
        e["fp32_emulation_guarded"] = errors(ref, emu, 1e-3)["max_rel_guarded"]
        bound = 2.0 * e["fp32_emulation_guarded"]
    assert e["max_rel_guarded"] <= bound, e
    return got


@pytest.mark.parametrize("N", [256, 264, 1024])
def test_tc_dense_blocks(executor, N):
    P = synth.cfg3_pruned_llm(seed=5, M=512, K=2048, N=8)
    c_tc = _run(executor, "tc", P.M, P.K, N, P.row_ptr, P.col_ind, P.values, seed=N)
    c_mma = _run(executor, "mma", P.M, P.K, N, P.row_ptr, P.col_ind, P.values, seed=N)
    assert errors(c_mma.astype(np.float64), c_tc, 1e-3)["max_rel_guarded"] <= 2e-3


def test_tc_without_split(executor):
    # short union lists (K = 256) and 8 groups: one CTA per tile, no partial reduction
    P = synth.cfg3_pruned_llm(seed=6, M=1024, K=256, N=8)
    _run(executor, "tc", P.M, P.K, 512, P.row_ptr, P.col_ind, P.values, seed=1)


def test_tc_ragged_edges(executor):
    # M and K not multiples of 16, last group partial, N not a multiple of 256
    P = synth.cfg3_pruned_llm(seed=7, M=500, K=2040, N=8)
    _run(executor, "tc", P.M, P.K, 72, P.row_ptr, P.col_ind, P.values, seed=2)


def test_tc_scattered_blocks_zero_fill(executor):
    # most stacked blocks are missing: they must read as zeros
    rp, ci, v = synth.random_csr(300, 400, 0.01, seed=8, empty_row_frac=0.2)
    _run(executor, "tc", 300, 400, 48, rp, ci, v, seed=3)


def test_tc_row_map(executor):
    P = synth.cfg3_pruned_llm(seed=9, M=384, K=1024, N=8)
    perm = np.random.default_rng(4).permutation(P.M)
    _run(executor, "tc", P.M, P.K, 256, P.row_ptr, P.col_ind, P.values, seed=4, row_map=perm)


def test_tc_falls_back_when_n_unaligned(executor):
    P = synth.cfg3_pruned_llm(seed=10, M=256, K=512, N=8)
    _run(executor, "tc", P.M, P.K, 20, P.row_ptr, P.col_ind, P.values, seed=5)


def test_tc_pipeline_dense(executor):
    """Tier-2 on the dense-block structure takes the tcgen05 kernel automatically."""
    P = synth.cfg3_pruned_llm(seed=12, M=512, K=2048, N=256)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    B = torch.as_tensor(P.B).to(executor.device)
    C = torch.zeros((P.M, P.N), dtype=torch.float32, device=executor.device)
    xs.spmm(executor, A, B, C, P.N, 16, True)
    perm = oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K)
    prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values, perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
    ref = oracle.unpermute_dense(oracle.bcsr_spmm_f64(P.M, P.K, P.N, brp, bci, bv, P.B), perm)
    e = errors(ref, C.cpu().numpy(), 1e-3)
    emu = oracle.unpermute_dense(fp32_block_emulation(P.M, P.N, brp, bci, bv, P.B), perm)
    assert e["max_rel_guarded"] <= max(1e-3, 2.0 * errors(ref, emu, 1e-3)["max_rel_guarded"]), e
