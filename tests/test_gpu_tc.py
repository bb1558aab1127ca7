"""GPU tests of the tcgen05/TMEM Tier-1 kernel (block rows stacked to M=128, TMA-fed, partials of
16 union entries added to a running sum with round-to-nearest FADD), forced through
xspmm_set_tier1_kernel or taken automatically, against the fp64 oracle and the mma.sync kernel.

The bar is the north star's fixed max relative error 1e-3 (guarded metric of tests.util.errors)
on every case, long block rows included. The error of an IEEE fp32 emulation of the reference's
block loop is computed beside it for the record only: on the full pruned-LLM matrix that
emulation itself exceeds 1e-3 (1.4e-3 at N = 128), so it is not used as a bound."""
import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import errors, fp32_block_emulation
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _run(executor, kind, M, K, N, rp, ci, v, seed=0, row_map=None, cols=None):
    """Tier-1 on the BCSR of (rp, ci, v) with the kernel `kind`; C checked against the fp64
    oracle (on the columns `cols` only when given: every column of C depends only on the same
    column of B)."""
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
    got = C.cpu().numpy()
    assert np.isfinite(got).all(), "C not fully written"
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, np.asarray(v, np.float16), M, K)
    Bc = B if cols is None else np.ascontiguousarray(B[:, cols])
    ref = oracle.bcsr_spmm_f64(M, K, Bc.shape[1], brp, bci, bv, Bc)
    if row_map is not None:
        ref = oracle.unpermute_dense(ref, row_map)
    gc = got if cols is None else got[:, cols]
    e = errors(ref, gc, TOL)
    if cols is None and M * N <= (1 << 22):
        emu = fp32_block_emulation(M, N, brp, bci, bv, B)
        if row_map is not None:
            emu = oracle.unpermute_dense(emu, row_map)
        e["fp32_emulation_guarded"] = errors(ref, emu, TOL)["max_rel_guarded"]
    print(f"tcgen05 {kind} M={M} K={K} N={N}: {e}")
    assert e["max_rel_guarded"] <= TOL, e
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


@pytest.mark.parametrize("K", [16 * 17, 16 * 33, 16 * 48])
def test_tc_group_boundaries(executor, K):
    # union lists of 17, 33 and 48 entries: a last accumulation group of 1, 1 and 16 entries
    P = synth.cfg3_pruned_llm(seed=11, M=256, K=K, N=8)
    _run(executor, "tc", P.M, P.K, 256, P.row_ptr, P.col_ind, P.values, seed=6)


def mixed_dense_problem(seed=0, M=2048, K=4096):
    """Block rows 0..63: 200 of the 256 block columns as 16x16 blocks filled to 50 %; block rows
    64..127: rows of 2 nonzeros, and a hub row of 2000 nonzeros every 151 rows; fp16 N(0,1).
    The block grid is dense enough (50 %, 127 blocks per block row) for the automatic choice to
    take the tcgen05 kernel, with long mixed block rows: the case that drifted past 1e-3 when
    the kernel carried one TMEM accumulator over the whole union list."""
    rng = np.random.default_rng(seed)
    nbc = (K + 15) // 16
    rows, cols = [], []
    bcs = None
    for r in range(M):
        if r < M // 2:
            if r % 16 == 0:
                bcs = np.sort(rng.choice(nbc, 200, replace=False))
            c = np.concatenate([bc * 16 + np.sort(rng.choice(16, 8, replace=False)) for bc in bcs])
        elif r % 151 == 0:
            c = np.sort(rng.choice(K, 2000, replace=False))
        else:
            c = np.sort(rng.choice(K, 2, replace=False))
        rows.append(np.full(len(c), r))
        cols.append(c)
    rows, cols = np.concatenate(rows), np.concatenate(cols)
    rp = np.zeros(M + 1, np.int64)
    np.cumsum(np.bincount(rows, minlength=M), out=rp[1:])
    v = rng.standard_normal(len(cols)).astype(np.float16)
    return synth.Problem("mixed_dense", M, K, 8, rp, cols.astype(np.int64), v, None)


@pytest.mark.parametrize("N", [64, 256])
def test_tc_mixed_density_forced(executor, N):
    P = mixed_dense_problem(seed=N)
    _run(executor, "tc", P.M, P.K, N, P.row_ptr, P.col_ind, P.values, seed=N)


@pytest.mark.parametrize("N", [256, 512])
def test_tc_mixed_density_auto_plan(executor, N):
    """The automatic choice takes tcgen05 on this matrix (checked through the plan), and the
    result meets 1e-3 without any emulation-based allowance."""
    P = mixed_dense_problem(seed=100 + N)
    B = np.random.default_rng(N).standard_normal((P.K, N)).astype(np.float16)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    with xs.SpMMPlan(executor, A, 16, False) as plan:
        C = torch.full((P.M, N), float("nan"), device=executor.device)
        plan.execute(torch.as_tensor(B).to(executor.device), C, N)
        assert plan.info()["tcgen05_ready"], "the automatic choice should take tcgen05 here"
        got = C.cpu().numpy()
    brp, bci, bv = oracle.csr_to_bcsr(P.row_ptr, P.col_ind, P.values, P.M, P.K)
    ref = oracle.bcsr_spmm_f64(P.M, P.K, N, brp, bci, bv, B)
    e = errors(ref, got, TOL)
    print(f"mixed auto N={N}: {e}")
    assert e["max_rel_guarded"] <= TOL, e


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
    e = errors(ref, C.cpu().numpy(), TOL)
    assert e["max_rel_guarded"] <= TOL, e


@pytest.mark.parametrize("N,ncheck", [(256, None), (4096, 256)])
def test_tc_full_cfg3(executor, N, ncheck):
    """The full pruned-LLM matrix (4096 x 11008, every one of the 176,128 blocks present, block
    rows of 688 blocks) through the tcgen05 kernel, at N = 256 on
    every column and at N = 4096 on 256 sampled columns."""
    P = synth.cfg3_pruned_llm(N=8)
    cols = None
    if ncheck is not None:
        cols = np.sort(np.random.default_rng(N).choice(N, ncheck, replace=False))
    _run(executor, "tc", P.M, P.K, N, P.row_ptr, P.col_ind, P.values, seed=N, cols=cols)
