"""C against an independent implementation: cuSPARSE SpMM (through torch.sparse, fp32, inputs
widened exactly from fp16) on the original CSR, as the reference's examples cross-check against
the vendor library (examples/01_uspmm_checkers.cpp:168-183, examples/05_core_spmm_benchmark.cpp:205-218).
Tier-2 with clustering on and off, both Tier-1 kernels; the guarded tolerance of tests.util."""
import numpy as np
import pytest
import torch

import xspmm_b200 as xs
from tests.util import errors
from xspmm_b200 import generators as gen
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu


def _vendor(P, dev):
    A = torch.sparse_csr_tensor(torch.as_tensor(P.row_ptr.astype(np.int64)),
                                torch.as_tensor(P.col_ind.astype(np.int64)),
                                torch.as_tensor(P.values.astype(np.float32)),
                                size=(P.M, P.K)).to(dev)
    B = torch.as_tensor(P.B.astype(np.float32)).to(dev)
    return torch.sparse.mm(A, B).cpu().numpy().astype(np.float64)


def _ours(ex, P, clustering, idx=torch.int32):
    A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values, index_dtype=idx)
    C = torch.full((P.M, P.N), float("nan"), dtype=torch.float32, device=ex.device)
    xs.spmm(ex, A, torch.as_tensor(P.B).to(ex.device), C, P.N, 16, clustering)
    return C.cpu().numpy()


@pytest.mark.parametrize("clustering", [False, True])
def test_fp32_plumbing_config_vs_cusparse(executor, clustering):
    # cuSPARSE accumulates in fp32, so near-zero outputs carry its rounding (~1e-7 of the row
    # scale): the bound is relative to max(|C|, rms(C)) here, the fp64 oracle tests the rest
    P = synth.cfg1_plumbing(seed=3)  # full size: 4096^2 fp32, 1 %, N = 128
    e = errors(_vendor(P, executor.device), _ours(executor, P, clustering), 1.0)
    assert e["max_rel_guarded"] <= 1e-5 and e["rel_frobenius"] <= 1e-6, e


@pytest.mark.parametrize("clustering", [False, True])
def test_fp16_hidden_block_vs_cusparse(executor, clustering):
    P = synth.cfg2_hidden_block(seed=4, n=4096, N=128, block_density=0.01)
    e = errors(_vendor(P, executor.device), _ours(executor, P, clustering, torch.int64), 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e


@pytest.mark.parametrize("kernel", ["mma", "tc"])
def test_fp16_pruned_llm_vs_cusparse(executor, kernel):
    P = synth.cfg3_pruned_llm(seed=5, M=1024, K=2048, N=256)
    executor.set_tier1_kernel(kernel)
    try:
        got = _ours(executor, P, True)
    finally:
        executor.set_tier1_kernel("auto")
    e = errors(_vendor(P, executor.device), got, 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e


def test_power_law_vs_cusparse(executor):
    rp, ci, v = gen.power_law(3000, 3000, 2.1, seed=6, dtype=np.float16)
    rng = np.random.default_rng(7)
    P = synth.Problem("power_law", 3000, 3000, 64, rp, ci, v,
                      rng.standard_normal((3000, 64)).astype(np.float16))
    e = errors(_vendor(P, executor.device), _ours(executor, P, True), 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e
