"""GPU tests of the plan (xspmm_plan_*): the Tier-2 stages built once and executed many times.
Products from a plan must equal the one-shot Tier-2 / Tier-1 calls bit for bit (same BCSR, same
kernel) and the fp64 oracle within the fp16-input tolerance."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import errors, fp32_block_emulation
from xspmm_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _oracle_tier2(P, B, clustering):
    rp, ci, v = P.row_ptr, P.col_ind, P.values
    perm = None
    if clustering:
        perm = oracle.cluster_fast(rp, ci, P.M, P.K)
        rp, ci, v = oracle.permute_rows(rp, ci, v, perm)
    brp, bci, bv = oracle.csr_to_bcsr(rp, ci, v, P.M, P.K)
    ref = oracle.bcsr_spmm_f64(P.M, P.K, B.shape[1], brp, bci, bv, B)
    emu = fp32_block_emulation(P.M, B.shape[1], brp, bci, bv, B)
    if perm is not None:
        ref = oracle.unpermute_dense(ref, perm)
        emu = oracle.unpermute_dense(emu, perm)
    return ref, emu


def _close(ref, emu, got):
    """Fixed bar 1e-3 (guarded); the IEEE fp32 emulation's error is reported, not a bound."""
    e = errors(ref, got, 1e-3)
    e["fp32_emulation_guarded"] = errors(ref, emu, 1e-3)["max_rel_guarded"]
    assert e["max_rel_guarded"] <= 1e-3, e


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_plan_csr_matches_tier2_and_oracle(executor, index_dtype):
    P = synth.cfg2_hidden_block(seed=21, n=1024, N=64, block_density=0.03)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=index_dtype)
    t = xs.SpMMTimings()
    plan = xs.SpMMPlan(executor, A, 16, True, t)
    info = plan.info()
    assert info["clustered"] == 1 and info["rows"] == P.M and info["value_bytes"] == 2
    assert t.clustering_ms > 0 and t.spmm_ms == 0
    rng = np.random.default_rng(3)
    for it in range(3):  # the same plan, different right-hand sides
        B = rng.standard_normal((P.K, P.N)).astype(np.float16)
        Bd = torch.as_tensor(B).to(executor.device)
        C_plan = torch.full((P.M, P.N), float("nan"), device=executor.device)
        C_once = torch.full((P.M, P.N), float("nan"), device=executor.device)
        plan.execute(Bd, C_plan, P.N)
        xs.spmm(executor, A, Bd, C_once, P.N, 16, True)
        got = C_plan.cpu().numpy()
        assert np.array_equal(got, C_once.cpu().numpy())
        ref, emu = _oracle_tier2(P, B, True)
        _close(ref, emu, got)
    plan.close()


def test_plan_csr_f32_without_clustering(executor):
    rp, ci, v = synth.random_csr(333, 270, 0.05, seed=4, empty_row_frac=0.1)
    v = np.asarray(v, np.float32)
    A = xs.CSRMatrix.from_host(executor, 333, 270, rp, ci, v, index_dtype=torch.int64)
    B = np.random.default_rng(5).standard_normal((270, 40)).astype(np.float32)
    with xs.SpMMPlan(executor, A, 16, False) as plan:
        assert plan.info()["clustered"] == 0
        C = torch.full((333, 40), float("nan"), device=executor.device)
        plan.execute(torch.as_tensor(B).to(executor.device), C, 40)
        brp, bci, bv = oracle.csr_to_bcsr(rp, ci, v, 333, 270)
        ref = oracle.bcsr_spmm_f64(333, 270, 40, brp, bci, bv, B)
        assert errors(ref, C.cpu().numpy(), 1e-5)["max_rel_guarded"] <= 1e-5


@pytest.mark.parametrize("kind", ["mma", "tc"])
def test_plan_bcsr_matches_tier1(executor, kind):
    P = synth.cfg3_pruned_llm(seed=22, M=512, K=1024, N=8)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    Ab = xs.csr_to_bcsr(executor, A, 16, 16)
    executor.set_tier1_kernel(kind)
    try:
        plan = xs.SpMMPlan.from_bcsr(Ab)
        assert plan.info()["tcgen05_ready"] == (1 if kind == "tc" else 0)
        rng = np.random.default_rng(6)
        for N in (256, 72, 20):  # 20: not a multiple of 8, the tcgen05 plan falls back to mma
            B = torch.as_tensor(rng.standard_normal((P.K, N)).astype(np.float16)).to(
                executor.device)
            C_plan = torch.full((P.M, N), float("nan"), device=executor.device)
            C_once = torch.full((P.M, N), float("nan"), device=executor.device)
            plan.execute(B, C_plan, N)
            xs.spmm(Ab, B, C_once, N)
            assert np.array_equal(C_plan.cpu().numpy(), C_once.cpu().numpy()), N
        plan.close()
    finally:
        executor.set_tier1_kernel("auto")


def test_plan_dense_structure_prepares_tcgen05_tiles(executor):
    P = synth.cfg3_pruned_llm(seed=23, M=512, K=2048, N=256)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    with xs.SpMMPlan(executor, A, 16, True) as plan:
        info = plan.info()
        assert info["tcgen05_ready"] == 1
        assert 0 < info["tcgen05_tiles"] <= info["nnz_blocks"]
        assert info["device_bytes"] >= info["tcgen05_tiles"] * 128 * 16 * 2
        C = torch.full((P.M, P.N), float("nan"), device=executor.device)
        plan.execute(torch.as_tensor(P.B).to(executor.device), C, P.N)
        ref, emu = _oracle_tier2(P, P.B, True)
        _close(ref, emu, C.cpu().numpy())


def test_plan_empty_and_all_zero_matrices(executor):
    # no rows: nothing to do
    A0 = xs.CSRMatrix.from_host(executor, 0, 10, np.zeros(1, np.int32), np.zeros(0, np.int32),
                                np.zeros(0, np.float16), index_dtype=torch.int32)
    with xs.SpMMPlan(executor, A0, 16, True) as p0:
        assert p0.info()["nnz_blocks"] == 0
        p0.execute(torch.zeros((10, 8), dtype=torch.float16, device=executor.device),
                   torch.zeros((0, 8), device=executor.device), 8)
    # rows but no entries: C is all zeros
    A1 = xs.CSRMatrix.from_host(executor, 37, 29, np.zeros(38, np.int32), np.zeros(0, np.int32),
                                np.zeros(0, np.float16), index_dtype=torch.int32)
    with xs.SpMMPlan(executor, A1, 16, True) as p1:
        C = torch.full((37, 16), float("nan"), device=executor.device)
        p1.execute(torch.ones((29, 16), dtype=torch.float16, device=executor.device), C, 16)
        assert (C.cpu().numpy() == 0).all()


def test_handle_with_live_plan_cannot_be_destroyed(executor):
    ex = xs.CudaExecutor(executor.device_id)
    rp, ci, v = synth.random_csr(64, 64, 0.1, seed=9)
    A = xs.CSRMatrix.from_host(ex, 64, 64, rp, ci, np.asarray(v, np.float16),
                               index_dtype=torch.int32)
    plan = xs.SpMMPlan(ex, A, 16, True)
    L = _lib.lib()
    assert L.xspmm_destroy(ex._h) == 1
    assert b"plans" in L.xspmm_last_error()
    plan.close()
    assert L.xspmm_destroy(ex._h) == 0
    ex._h = None


def test_plan_rejects_bad_arguments(executor):
    rp, ci, v = synth.random_csr(64, 64, 0.1, seed=10)
    A = xs.CSRMatrix.from_host(executor, 64, 64, rp, ci, np.asarray(v, np.float16),
                               index_dtype=torch.int32)
    with pytest.raises(xs.XSpMMError, match="INVALID_ARGUMENT"):
        xs.SpMMPlan(executor, A, 0, True)  # hw_block_size 0
    L = _lib.lib()
    h = ctypes.c_void_p()
    assert L.xspmm_plan_bcsr_f16f32_i32(executor.handle, 4, 4, 0, 8, 8, None, None, None, 64, 64,
                                        ctypes.byref(h)) == 2
    with xs.SpMMPlan(executor, A, 16, True) as plan:
        assert L.xspmm_plan_execute(plan._h, None, None, 8) == 1
        with pytest.raises(ValueError):
            plan.execute(torch.zeros((64, 8), device=executor.device),
                         torch.zeros((64, 8), device=executor.device), 8)


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_plan_splits_long_block_rows(executor, index_dtype):
    """Block rows longer than a work slice (here 512 blocks) are cut into slices whose partial
    sums are added in a fixed order; C must match the oracle and be the same on every run."""
    P = synth.cfg3_pruned_llm(seed=24, M=96, K=8192, N=8)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=index_dtype)
    executor.set_tier1_kernel("mma")
    try:
        with xs.SpMMPlan(executor, A, 16, False) as plan:
            N = 72
            B = np.random.default_rng(7).standard_normal((P.K, N)).astype(np.float16)
            Bd = torch.as_tensor(B).to(executor.device)
            C1 = torch.full((P.M, N), float("nan"), device=executor.device)
            C2 = torch.full((P.M, N), float("nan"), device=executor.device)
            plan.execute(Bd, C1, N)
            plan.execute(Bd, C2, N)
            assert torch.equal(C1, C2)
            P.B = B
            P.N = N
            ref, emu = _oracle_tier2(P, B, False)
            _close(ref, emu, C1.cpu().numpy())
    finally:
        executor.set_tier1_kernel("auto")


def test_plan_power_law_rows(executor):
    """R-MAT graph with hub rows through a plan (the work list orders rows and splits hubs)."""
    P = synth.cfg5_rmat(seed=3, scale=13, N=64)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    with xs.SpMMPlan(executor, A, 16, False) as plan:
        C = torch.full((P.M, P.N), float("nan"), device=executor.device)
        plan.execute(torch.as_tensor(P.B).to(executor.device), C, P.N)
        ref, emu = _oracle_tier2(P, P.B, False)
        _close(ref, emu, C.cpu().numpy())


def _mixed_problem(seed, M=4000, K=6000):
    """Rows 0..399 in 16x16 blocks filled to 50 % (20 block columns per block row), rows 400..
    ultra-sparse (2 nonzeros), with a hub row of 2000 nonzeros every 151 rows; fp16 values. The
    block grid stays below the density at which a plan takes the tcgen05 kernel, so the mma.sync
    and gather kernels share it."""
    rng = np.random.default_rng(seed)
    nbc = (K + 15) // 16
    rows, cols = [], []
    bcs = None
    for r in range(M):
        if r < 400:
            if r % 16 == 0:
                bcs = rng.choice(nbc - 1, 20, replace=False)
            c = np.sort(np.concatenate([bc * 16 + rng.choice(16, 8, replace=False) for bc in bcs]))
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
    return synth.Problem("mixed", M, K, 8, rp, cols.astype(np.int64), v, None)


@pytest.mark.parametrize("N,clustering", [(64, False), (130, True), (256, False), (37, True)])
def test_plan_sparse_block_rows(executor, N, clustering):
    """Block rows of nearly empty blocks run on the gather kernels (spmm_sparse.cu), the rest on
    the mma.sync block kernel; C must match the oracle and be the same bits on every run."""
    P = _mixed_problem(40 + N)
    B = np.random.default_rng(N).standard_normal((P.K, N)).astype(np.float16)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32 if N % 2 else torch.int64)
    with xs.SpMMPlan(executor, A, 16, clustering) as plan:
        Bd = torch.as_tensor(B).to(executor.device)
        C1 = torch.full((P.M, N), float("nan"), device=executor.device)
        C2 = torch.full((P.M, N), float("nan"), device=executor.device)
        plan.execute(Bd, C1, N)
        plan.execute(Bd, C2, N)
        assert torch.equal(C1, C2)
        ref, emu = _oracle_tier2(P, B, clustering)
        got = C1.cpu().numpy()
        _close(ref[:400], emu[:400], got[:400])  # dense rows: the block kernel
        _close(ref[400:], emu[400:], got[400:])  # 2-nonzero and hub rows: the gather kernels
        assert plan.info()["device_bytes"] > 0


def _ragged_rows_problem(seed, M=3000, K=60000):
    """Rows of every length the gather kernels' warp tasks split on: runs of empty and
    one-nonzero rows longer than a task's 32 rows, rows of 2-5, of exactly 127/128/129 (a task's
    nonzero budget) and 200/256 (a task of their own), 257 and 3000 (cut into chunks), all in
    nearly empty 16x16 blocks (columns spread over K); fp16 values."""
    rng = np.random.default_rng(seed)
    lens = np.zeros(M, np.int64)
    pattern = [0] * 40 + [1] * 70 + [2, 3, 4, 5] * 10 + [127, 128, 129, 1, 0, 200, 256, 257] + [3000]
    for i in range(M):
        lens[i] = pattern[(i * 7 + seed) % len(pattern)] if i >= 200 else (i % 3)
    lens[-1] = 1
    rp = np.zeros(M + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    cols = np.concatenate([np.sort(rng.choice(K, n, replace=False)) for n in lens if n > 0])
    v = rng.standard_normal(len(cols)).astype(np.float16)
    return synth.Problem("ragged", M, K, 8, rp, cols.astype(np.int64), v, None)


@pytest.mark.parametrize("N,clustering", [(128, False), (256, True), (36, False), (7, True),
                                          (24, True), (200, False)])
def test_plan_gather_row_tasks(executor, N, clustering):
    """Every row of a ragged, nearly empty matrix goes through the gather kernels (the
    tensor-core gather when N is a multiple of 8 -- 24 and 200 end in a partial 64-column tile --
    the SIMT one otherwise): C is within the fp16 bar (1e-3 guarded) of the fp64 oracle, empty
    rows are exact zeros, and repeated products are the same bits."""
    P = _ragged_rows_problem(N)
    B = np.random.default_rng(N + 1).standard_normal((P.K, N)).astype(np.float16)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32 if N % 2 == 0 else torch.int64)
    with xs.SpMMPlan(executor, A, 16, clustering) as plan:
        Bd = torch.as_tensor(B).to(executor.device)
        C1 = torch.full((P.M, N), float("nan"), device=executor.device)
        C2 = torch.full((P.M, N), float("nan"), device=executor.device)
        plan.execute(Bd, C1, N)
        plan.execute(Bd, C2, N)
        assert torch.equal(C1, C2)
        ref, _ = _oracle_tier2(P, B, clustering)
        got = C1.cpu().numpy()
        assert np.isfinite(got).all()
        e = errors(ref, got, 1e-3)
        assert e["max_rel_guarded"] <= 1e-3, e
        empty = np.diff(P.row_ptr) == 0
        assert np.all(got[empty] == 0.0)


def test_plan_all_sparse_and_forced_block_kernel_agree(executor):
    """An R-MAT matrix whose block rows all take the gather path, against the same plan forced
    onto the block kernel: both within the tolerance of the oracle, and within it of each other."""
    P = synth.cfg5_rmat(seed=5, scale=12, N=128)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    ref, emu = _oracle_tier2(P, P.B, False)
    Bd = torch.as_tensor(P.B).to(executor.device)
    outs = []
    for kind in ("auto", "mma"):
        executor.set_tier1_kernel(kind)
        try:
            with xs.SpMMPlan(executor, A, 16, False) as plan:
                C = torch.full((P.M, P.N), float("nan"), device=executor.device)
                plan.execute(Bd, C, P.N)
                outs.append(C.cpu().numpy())
        finally:
            executor.set_tier1_kernel("auto")
        _close(ref, emu, outs[-1])
    assert errors(outs[1], outs[0], 1e-3)["max_rel_guarded"] <= 1e-3


def _as_f32(P, seed):
    v = np.random.default_rng(seed).uniform(-1.0, 1.0, len(P.values)).astype(np.float32)
    return synth.Problem(P.name, P.M, P.K, P.N, P.row_ptr, P.col_ind, v, None)


@pytest.mark.parametrize("N,clustering", [(64, False), (130, True), (33, False)])
def test_plan_sparse_block_rows_fp32(executor, N, clustering):
    """fp32 plans split the same way at a higher fill: the 50 %-filled block rows (128 nonzeros
    per block) stay on the SIMT block kernel, the rest go to the gather kernels. Both accumulate
    in fp64, so every row meets the fp32 tolerance (1e-5, guarded) against the fp64 oracle, and
    repeated products are the same bits."""
    P = _as_f32(_mixed_problem(60 + N), N)
    B = np.random.default_rng(N).uniform(-1.0, 1.0, (P.K, N)).astype(np.float32)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int64 if N % 2 else torch.int32)
    with xs.SpMMPlan(executor, A, 16, clustering) as plan:
        Bd = torch.as_tensor(B).to(executor.device)
        C1 = torch.full((P.M, N), float("nan"), device=executor.device)
        C2 = torch.full((P.M, N), float("nan"), device=executor.device)
        plan.execute(Bd, C1, N)
        plan.execute(Bd, C2, N)
        assert torch.equal(C1, C2)
        ref, _ = _oracle_tier2(P, B, clustering)
        e = errors(ref, C1.cpu().numpy(), 1e-5)
        assert e["max_rel_guarded"] <= 1e-5, e


def test_plan_fp32_split_matches_block_kernel(executor):
    """cfg1-shaped fp32 matrix (4096^2, 1 % uniform: ~2.6 nonzeros per block, every block row
    takes the gather path) through a plan and through the one-shot pipeline, against the plan
    forced onto the block kernel: all within 1e-5 (guarded) of the fp64 oracle."""
    P = synth.cfg1_plumbing(seed=3)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    ref, _ = _oracle_tier2(P, P.B, False)
    Bd = torch.as_tensor(P.B).to(executor.device)
    for kind in ("auto", "mma"):
        executor.set_tier1_kernel(kind)
        try:
            with xs.SpMMPlan(executor, A, 16, False) as plan:
                C = torch.full((P.M, P.N), float("nan"), device=executor.device)
                plan.execute(Bd, C, P.N)
            e = errors(ref, C.cpu().numpy(), 1e-5)
            assert e["max_rel_guarded"] <= 1e-5, (kind, e)
        finally:
            executor.set_tier1_kernel("auto")
    C = torch.full((P.M, P.N), float("nan"), device=executor.device)
    xs.spmm(executor, A, Bd, C, P.N, 16, False)
    e = errors(ref, C.cpu().numpy(), 1e-5)
    assert e["max_rel_guarded"] <= 1e-5, e


@pytest.mark.parametrize("N,index_dtype", [(96, torch.int32), (33, torch.int64)])
def test_plan_fp32_cut_long_block_rows(executor, N, index_dtype):
    """fp32 arrowhead (dense first 16 rows and columns): block row 0 holds every block column
    while the others hold two, so a plan cuts it into pieces whose fp64 partials are added in a
    fixed order. C within 1e-5 (guarded) of the fp64 oracle, the same bits on every product, and
    within 1e-5 of the uncut block kernel."""
    from xspmm_b200 import generators as gen
    n = 1500
    rp, ci, v = gen.arrowhead(n, 16, seed=N)
    P = synth.Problem("arrowhead", n, n, N, rp, ci, v.astype(np.float32), None)
    B = np.random.default_rng(N).uniform(-1.0, 1.0, (n, N)).astype(np.float32)
    A = xs.CSRMatrix.from_host(executor, n, n, rp, ci, P.values, index_dtype=index_dtype)
    ref, _ = _oracle_tier2(P, B, False)
    Bd = torch.as_tensor(B).to(executor.device)
    with xs.SpMMPlan(executor, A, 16, False) as plan:
        C1 = torch.full((n, N), float("nan"), device=executor.device)
        C2 = torch.full((n, N), float("nan"), device=executor.device)
        plan.execute(Bd, C1, N)
        plan.execute(Bd, C2, N)
    assert torch.equal(C1, C2)
    e = errors(ref, C1.cpu().numpy(), 1e-5)
    assert e["max_rel_guarded"] <= 1e-5, e
    executor.set_tier1_kernel("mma")
    try:
        with xs.SpMMPlan(executor, A, 16, False) as plan:
            C3 = torch.full((n, N), float("nan"), device=executor.device)
            plan.execute(Bd, C3, N)
    finally:
        executor.set_tier1_kernel("auto")
    e = errors(ref, C3.cpu().numpy(), 1e-5)
    assert e["max_rel_guarded"] <= 1e-5, e
