"""GPU test of xspmm_permute_rows_noalloc_i32, the row permutation for callers that cannot
allocate device memory while they run (a process whose device memory is reserved by its own pool,
or code that must avoid the synchronization cudaMalloc/cudaFree can cause). Its scratch is a fixed
array inside the library, shared by all calls on a device.

The test calls it through the C ABI twice in a row, on different inputs, and checks each result
bit for bit against the allocating entry point (xspmm_permute_rows_*_i32) -- the second call also
shows that what the first call left in the shared scratch does not leak into the next result. The
file is named so pytest collects it last; it also runs alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from xspmm_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t.numel() else ctypes.c_void_p(0)


def _permute_both(executor, M, K, rp, ci, v, perm):
    L = _lib.lib()
    dev = executor.device
    t = lambda a, dt: torch.as_tensor(np.ascontiguousarray(a, dtype=dt)).to(dev)  # noqa: E731
    vt = torch.float16 if v.dtype == np.float16 else torch.float32
    vb = 2 if vt == torch.float16 else 4
    rp_t, ci_t, perm_t = t(rp, np.int32), t(ci, np.int32), t(perm, np.int32)
    v_t = torch.as_tensor(v).to(dev)
    nnz = int(rp[-1])
    outs = []
    for noalloc in (True, False):
        orp = torch.full((M + 1,), -7, dtype=torch.int32, device=dev)
        oci = torch.full((max(nnz, 1),), -7, dtype=torch.int32, device=dev)
        ov = torch.full((max(nnz, 1),), -7, dtype=vt, device=dev)
        if noalloc:
            rc = L.xspmm_permute_rows_noalloc_i32(executor.handle, M, K, nnz, _p(rp_t), _p(ci_t),
                                                  _p(v_t), vb, _p(perm_t), _p(orp), _p(oci), _p(ov))
        else:
            fn = getattr(L, "xspmm_permute_rows_%s_i32" % ("f16" if vb == 2 else "f32"))
            rc = fn(executor.handle, M, K, nnz, _p(rp_t), _p(ci_t), _p(v_t), _p(perm_t), _p(orp),
                    _p(oci), _p(ov))
        _lib.check(rc)
        torch.cuda.synchronize()
        outs.append((orp.cpu().numpy(), oci.cpu().numpy()[:nnz], ov.cpu().numpy()[:nnz]))
    return outs


def test_noalloc_permutation_matches_allocating_entry_point_twice(executor):
    # first call: a large hidden-block matrix (multi-tile scan), fp16
    P = synth.cfg2_hidden_block(seed=21, n=8192, N=8)
    perm = np.random.default_rng(1).permutation(P.M)
    (a_rp, a_ci, a_v), (b_rp, b_ci, b_v) = _permute_both(executor, P.M, P.K, P.row_ptr,
                                                         P.col_ind, P.values, perm)
    assert np.array_equal(a_rp, b_rp) and np.array_equal(a_ci, b_ci)
    assert np.array_equal(a_v.view(np.uint16), b_v.view(np.uint16))
    # second call right after: a different, smaller fp32 matrix with empty rows
    rp, ci, v = synth.random_csr(777, 300, 0.03, seed=22, empty_row_frac=0.3)
    perm = np.random.default_rng(2).permutation(777)
    (a_rp, a_ci, a_v), (b_rp, b_ci, b_v) = _permute_both(executor, 777, 300, rp, ci,
                                                         v.astype(np.float32), perm)
    assert np.array_equal(a_rp, b_rp) and np.array_equal(a_ci, b_ci)
    assert np.array_equal(a_v.view(np.uint32), b_v.view(np.uint32))


def test_noalloc_rejects_rows_beyond_its_limit(executor):
    L = _lib.lib()
    dummy = torch.zeros(4, dtype=torch.int32, device=executor.device)
    rc = L.xspmm_permute_rows_noalloc_i32(executor.handle, (1 << 21) + 1, 10, 0, _p(dummy),
                                          _p(dummy), _p(dummy), 4, _p(dummy), _p(dummy),
                                          _p(dummy), _p(dummy))
    assert rc == 1  # INVALID_ARGUMENT, nothing launched
    assert b"no-allocation limit" in L.xspmm_last_error()
