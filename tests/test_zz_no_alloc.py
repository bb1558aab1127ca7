"""GPU test of xspmm_permute_rows_noalloc_i32, the row permutation for callers that cannot
allocate device memory while they run (a process whose device memory is reserved by its own pool,
or code that must avoid the synchronization cudaMalloc/cudaFree can cause). Its scratch is a fixed
array inside the library, shared by all calls on a device.

The test calls it through the C ABI twice in a row, on different inputs, and checks each result
bit for bit against the allocating entry point (xspmm_permute_rows_*_i32) and against the CPU
oracle's row permutation (oracle.permute_rows, itself pinned to the reference's
apply_permutation) -- the second call also shows that what the first call left in the shared
scratch does not leak into the next result. A third case of more than a million rows runs the
scan of row lengths over hundreds of scratch tiles. Around every no-allocation call the high-water
mark of the device's default memory pool (where the library's own scratch would come from) is
reset and read back: it must not rise. The file is named so pytest collects it last; it also runs
alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from xspmm_b200 import _lib, synth

pytestmark = pytest.mark.gpu

_CU_MEMPOOL_ATTR_USED_MEM_CURRENT = 7
_CU_MEMPOOL_ATTR_USED_MEM_HIGH = 8


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t.numel() else ctypes.c_void_p(0)


class _PoolWatch:
    """Used-memory high-water mark of a device's default memory pool (CUDA driver API)."""

    def __init__(self, ordinal):
        self.cu = ctypes.CDLL("libcuda.so.1")
        dev = ctypes.c_int()
        assert self.cu.cuDeviceGet(ctypes.byref(dev), ctypes.c_int(ordinal)) == 0
        self.pool = ctypes.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), dev) == 0

    def _get(self, attr):
        v = ctypes.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, ctypes.c_int(attr), ctypes.byref(v)) == 0
        return v.value

    def reset(self):
        """High-water mark := current use; returns the current use."""
        zero = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolSetAttribute(self.pool, ctypes.c_int(_CU_MEMPOOL_ATTR_USED_MEM_HIGH),
                                             ctypes.byref(zero)) == 0
        return self._get(_CU_MEMPOOL_ATTR_USED_MEM_CURRENT)

    def high(self):
        return self._get(_CU_MEMPOOL_ATTR_USED_MEM_HIGH)


def _permute_both(executor, M, K, rp, ci, v, perm):
    L = _lib.lib()
    dev = executor.device
    t = lambda a, dt: torch.as_tensor(np.ascontiguousarray(a, dtype=dt)).to(dev)  # noqa: E731
    vt = torch.float16 if v.dtype == np.float16 else torch.float32
    vb = 2 if vt == torch.float16 else 4
    rp_t, ci_t, perm_t = t(rp, np.int32), t(ci, np.int32), t(perm, np.int32)
    v_t = torch.as_tensor(v).to(dev)
    nnz = int(rp[-1])
    watch = _PoolWatch(dev.index if dev.index is not None else 0)
    outs = []
    for noalloc in (True, False):
        orp = torch.full((M + 1,), -7, dtype=torch.int32, device=dev)
        oci = torch.full((max(nnz, 1),), -7, dtype=torch.int32, device=dev)
        ov = torch.full((max(nnz, 1),), -7, dtype=vt, device=dev)
        torch.cuda.synchronize()
        if noalloc:
            used = watch.reset()
            rc = L.xspmm_permute_rows_noalloc_i32(executor.handle, M, K, nnz, _p(rp_t), _p(ci_t),
                                                  _p(v_t), vb, _p(perm_t), _p(orp), _p(oci), _p(ov))
            torch.cuda.synchronize()
            assert watch.high() <= used, "the no-allocation entry point took pool memory"
        else:
            fn = getattr(L, "xspmm_permute_rows_%s_i32" % ("f16" if vb == 2 else "f32"))
            rc = fn(executor.handle, M, K, nnz, _p(rp_t), _p(ci_t), _p(v_t), _p(perm_t), _p(orp),
                    _p(oci), _p(ov))
        _lib.check(rc)
        torch.cuda.synchronize()
        outs.append((orp.cpu().numpy(), oci.cpu().numpy()[:nnz], ov.cpu().numpy()[:nnz]))
    return outs


def _check(outs, rp, ci, v, perm, view):
    (a_rp, a_ci, a_v), (b_rp, b_ci, b_v) = outs
    o_rp, o_ci, o_v = oracle.permute_rows(rp, ci, v, perm)
    for got_rp, got_ci, got_v in ((a_rp, a_ci, a_v), (b_rp, b_ci, b_v)):
        assert np.array_equal(got_rp, o_rp) and np.array_equal(got_ci, o_ci)
        assert np.array_equal(got_v.view(view), np.asarray(o_v).view(view))


def test_noalloc_permutation_matches_allocating_entry_point_and_oracle_twice(executor):
    # first call: a large hidden-block matrix (a scan over several tiles), fp16
    P = synth.cfg2_hidden_block(seed=21, n=8192, N=8)
    perm = np.random.default_rng(1).permutation(P.M)
    outs = _permute_both(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values, perm)
    _check(outs, P.row_ptr, P.col_ind, P.values, perm, np.uint16)
    # second call right after: a different, smaller fp32 matrix with empty rows
    rp, ci, v = synth.random_csr(777, 300, 0.03, seed=22, empty_row_frac=0.3)
    v = v.astype(np.float32)
    perm = np.random.default_rng(2).permutation(777)
    outs = _permute_both(executor, 777, 300, rp, ci, v, perm)
    _check(outs, rp, ci, v, perm, np.uint32)


def test_noalloc_permutation_over_a_million_rows(executor):
    # 2^20 + 3 rows of 0..3 entries: the row-length scan spans hundreds of scratch tiles
    rng = np.random.default_rng(23)
    M, K = (1 << 20) + 3, 5000
    lens = rng.integers(0, 4, M)
    rp = np.zeros(M + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    ci = rng.integers(0, K, int(rp[-1])).astype(np.int64)
    v = rng.standard_normal(int(rp[-1])).astype(np.float16)
    perm = rng.permutation(M)
    outs = _permute_both(executor, M, K, rp, ci, v, perm)
    _check(outs, rp, ci, v, perm, np.uint16)


def test_noalloc_rejects_rows_beyond_its_limit(executor):
    L = _lib.lib()
    dummy = torch.zeros(4, dtype=torch.int32, device=executor.device)
    rc = L.xspmm_permute_rows_noalloc_i32(executor.handle, (1 << 21) + 1, 10, 0, _p(dummy),
                                          _p(dummy), _p(dummy), 4, _p(dummy), _p(dummy),
                                          _p(dummy), _p(dummy))
    assert rc == 1  # INVALID_ARGUMENT, nothing launched
    assert b"no-allocation limit" in L.xspmm_last_error()
