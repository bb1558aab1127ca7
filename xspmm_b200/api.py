"""Python mirror of the reference xSpMM API for the hot path, over the C ABI.

Names, argument order and meaning follow the reference's C++ API (include/xspmm/xspmm.hpp,
include/xspmm/clustering.hpp, include/xspmm/matrix/{csr,bcsr,conversion}.hpp,
include/xspmm/core/{executor,timings}.hpp) so tests and benchmarks read like the reference's own
examples. Device buffers are torch tensors (torch is used for memory and streams only); every
computation is a call into libxspmm_b200.so. Errors map like the reference's: bad dimensions raise
ValueError (std::invalid_argument), everything else XSpMMError (std::runtime_error).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import XSpMMError, check, lib

_VAL = {torch.float16: "f16", torch.float32: "f32", torch.bfloat16: "bf16"}
_IDX = {torch.int32: "i32", torch.int64: "i64"}
_IT_C = {torch.int32: ctypes.c_int32, torch.int64: ctypes.c_int64}


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() > 0 else ctypes.c_void_p(0)


def _torch_dtype(x, default):
    if x is None:
        return default
    if isinstance(x, torch.dtype):
        return x
    return {np.dtype(np.float16): torch.float16, np.dtype(np.float32): torch.float32,
            np.dtype(np.int32): torch.int32, np.dtype(np.int64): torch.int64}[np.dtype(x)]


def _host_values(values, value_dtype, n):
    """The first n values as a CPU tensor of value_dtype. numpy has no bf16: bf16 values come as
    a torch tensor, or as float32/float16 numbers rounded to bf16 (round to nearest even)."""
    if isinstance(values, torch.Tensor):
        return values[:n].detach().to("cpu", value_dtype).contiguous()
    if value_dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(values[:n], dtype=np.float32)).to(torch.bfloat16)
    vt = {torch.float16: np.float16, torch.float32: np.float32}[value_dtype]
    return torch.from_numpy(np.ascontiguousarray(values[:n], dtype=vt))


@dataclass
class SpMMTimings:
    """Mirrors xspmm::SpMMTimings (include/xspmm/core/timings.hpp:7-14)."""
    clustering_ms: float = 0.0
    permutation_ms: float = 0.0
    conversion_ms: float = 0.0
    spmm_ms: float = 0.0
    unpermutation_ms: float = 0.0
    total_pipeline_ms: float = 0.0


class CudaExecutor:
    """Mirrors xspmm::CudaExecutor (include/xspmm/core/executor.hpp:37-51): a device plus the
    library handle. Work is enqueued on torch's current stream of that device at call time."""

    def __init__(self, device_id: int = 0):
        self.device_id = int(device_id)
        self.device = torch.device("cuda", self.device_id)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            check(lib().xspmm_create(self.device_id, ctypes.c_void_p(stream), ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        lib().xspmm_set_stream(self._h, ctypes.c_void_p(
            torch.cuda.current_stream(self.device).cuda_stream))
        return self._h

    def allocate(self, nbytes: int) -> torch.Tensor:
        return torch.empty(int(nbytes), dtype=torch.uint8, device=self.device)

    def copy_from_host(self, dst: torch.Tensor, src) -> None:
        dst.copy_(torch.as_tensor(np.ascontiguousarray(src)).view(dst.dtype).reshape(dst.shape))

    def copy_to_host(self, src: torch.Tensor) -> np.ndarray:
        return src.cpu().numpy()

    def synchronize(self) -> None:
        check(lib().xspmm_synchronize(self.handle))

    def launch_count(self) -> int:
        c = ctypes.c_uint64()
        check(lib().xspmm_get_launch_count(self._h, ctypes.byref(c)))
        return int(c.value)

    def reset_launch_count(self) -> None:
        check(lib().xspmm_reset_launch_count(self._h))

    def set_tier1_kernel(self, kind: str) -> None:
        """'auto', 'mma' (mma.sync m16n8k16) or 'tc' (tcgen05/TMEM) for the fp16 Tier-1 SpMM."""
        check(lib().xspmm_set_tier1_kernel(self._h, {"auto": 0, "mma": 1, "tc": 2}[kind]))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib._lib is not None:
            try:
                _lib._lib.xspmm_destroy(h)
            except Exception:
                pass
            self._h = None


class CSRMatrix:
    """Mirrors xspmm::CSRMatrix<ValueType, IndexType> (include/xspmm/matrix/csr.hpp:15-60)."""

    def __init__(self, exec: CudaExecutor, num_rows: int, num_cols: int, nnz: int,
                 value_dtype=torch.float16, index_dtype=torch.int64):
        if num_rows < 0 or num_cols < 0 or nnz < 0:
            raise ValueError("CSR dimensions must be non-negative.")
        self.exec = exec
        self.num_rows, self.num_cols, self.nnz = int(num_rows), int(num_cols), int(nnz)
        self.value_dtype = _torch_dtype(value_dtype, torch.float16)
        self.index_dtype = _torch_dtype(index_dtype, torch.int64)
        d = exec.device
        self.row_ptr = torch.zeros(self.num_rows + 1, dtype=self.index_dtype, device=d)
        self.col_ind = torch.empty(self.nnz, dtype=self.index_dtype, device=d)
        self.values = torch.empty(self.nnz, dtype=self.value_dtype, device=d)

    @classmethod
    def from_host(cls, exec, num_rows, num_cols, row_ptr, col_ind, values,
                  index_dtype=torch.int64, value_dtype=None):
        """values: numpy (fp16/fp32) or a torch tensor (also bf16); value_dtype overrides the
        values' own type (float numbers are rounded to it)."""
        if value_dtype is None:
            value_dtype = (values.dtype if isinstance(values, torch.Tensor)
                           else _torch_dtype(np.asarray(values).dtype, torch.float16))
        m = cls(exec, num_rows, num_cols, int(row_ptr[-1]) if len(row_ptr) else 0,
                value_dtype=value_dtype, index_dtype=index_dtype)
        m.copy_from_host(row_ptr, col_ind, values)
        return m

    def copy_from_host(self, row_ptr, col_ind, values) -> None:
        it = {torch.int32: np.int32, torch.int64: np.int64}[self.index_dtype]
        self.row_ptr.copy_(torch.from_numpy(np.ascontiguousarray(row_ptr, dtype=it)))
        if self.nnz > 0:
            self.col_ind.copy_(torch.from_numpy(np.ascontiguousarray(col_ind[: self.nnz], dtype=it)))
            self.values.copy_(_host_values(values, self.value_dtype, self.nnz))

    def get_num_rows(self): return self.num_rows
    def get_num_cols(self): return self.num_cols
    def get_nnz(self): return self.nnz
    def get_row_ptr(self): return self.row_ptr
    def get_col_ind(self): return self.col_ind
    def get_values(self): return self.values
    def get_executor(self): return self.exec


class BCSRMatrix:
    """Mirrors xspmm::BCSRMatrix<ValueType, IndexType> (include/xspmm/matrix/bcsr.hpp:15-103).
    Also records the true row/column counts of the matrix it was converted from (num_rows,
    num_cols), which the reference's BCSR does not carry; they default to the block grid extent."""

    def __init__(self, exec: CudaExecutor, num_block_rows: int, num_block_cols: int,
                 num_blocks: int, r_block: int, c_block: int, value_dtype=torch.float16,
                 index_dtype=torch.int64, num_rows: int | None = None,
                 num_cols: int | None = None):
        if num_block_rows < 0 or num_block_cols < 0 or num_blocks < 0:
            raise ValueError("BCSR dimensions must be non-negative.")
        self.exec = exec
        self.num_block_rows, self.num_block_cols = int(num_block_rows), int(num_block_cols)
        self.num_blocks, self.r_block, self.c_block = int(num_blocks), int(r_block), int(c_block)
        self.value_dtype = _torch_dtype(value_dtype, torch.float16)
        self.index_dtype = _torch_dtype(index_dtype, torch.int64)
        self.num_rows = self.num_block_rows * self.r_block if num_rows is None else int(num_rows)
        self.num_cols = self.num_block_cols * self.c_block if num_cols is None else int(num_cols)
        d = exec.device
        self.row_ptr = torch.zeros(self.num_block_rows + 1, dtype=self.index_dtype, device=d)
        self.col_ind = torch.empty(self.num_blocks, dtype=self.index_dtype, device=d)
        self.values = torch.empty(self.num_blocks * self.r_block * self.c_block,
                                  dtype=self.value_dtype, device=d)

    def copy_from_host(self, row_ptr, col_ind, values) -> None:
        it = {torch.int32: np.int32, torch.int64: np.int64}[self.index_dtype]
        self.row_ptr.copy_(torch.from_numpy(np.ascontiguousarray(row_ptr, dtype=it)))
        if self.num_blocks > 0:
            self.col_ind.copy_(torch.from_numpy(np.ascontiguousarray(col_ind, dtype=it)))
            flat = values.reshape(-1) if isinstance(values, torch.Tensor) else np.asarray(values).reshape(-1)
            self.values.copy_(_host_values(flat, self.value_dtype, self.values.numel()))

    def get_num_block_rows(self): return self.num_block_rows
    def get_num_block_cols(self): return self.num_block_cols
    def get_num_blocks(self): return self.num_blocks
    def get_r_block(self): return self.r_block
    def get_c_block(self): return self.c_block
    def get_bcsr_row_ptr(self): return self.row_ptr
    def get_bcsr_col_ind(self): return self.col_ind
    def get_bcsr_values(self): return self.values
    def get_executor(self): return self.exec


def _it(t: torch.dtype):
    return _IT_C[t]


def _check_dev(exec: CudaExecutor, *ts):
    for t in ts:
        if t is not None and t.numel() > 0 and t.device != exec.device:
            raise ValueError(f"tensor on {t.device}, executor on {exec.device}")


def _tier1(A: BCSRMatrix, B: torch.Tensor, C: torch.Tensor, N: int, out_row_map=None):
    exec = A.exec
    if B.dtype != A.value_dtype:
        raise ValueError("B must have the value type of A")
    if C.dtype != torch.float32:
        raise ValueError("C must be float32")
    _check_dev(exec, A.row_ptr, B, C, out_row_map)
    IT = _it(A.index_dtype)
    fn = getattr(lib(), f"xspmm_bcsr_spmm_{_VAL[A.value_dtype]}f32_{_IDX[A.index_dtype]}")
    check(fn(exec.handle, IT(A.num_block_rows), IT(A.num_block_cols), IT(A.num_blocks),
             IT(A.r_block), IT(A.c_block), _p(A.row_ptr), _p(A.col_ind), _p(A.values), _p(B),
             _p(C), IT(A.num_rows), IT(A.num_cols), IT(N), _p(out_row_map)))


def _tier2(exec: CudaExecutor, A: CSRMatrix, B, C, N, hw_block_size=16, optimize_pattern=True,
           timings: SpMMTimings | None = None):
    if B.dtype != A.value_dtype:
        raise ValueError("B must have the value type of A")
    if C.dtype != torch.float32:
        raise ValueError("C must be float32")
    _check_dev(exec, A.row_ptr, B, C)
    IT = _it(A.index_dtype)
    t = _lib.Timings()
    fn = getattr(lib(), f"xspmm_spmm_csr_{_VAL[A.value_dtype]}f32_{_IDX[A.index_dtype]}")
    check(fn(exec.handle, IT(A.num_rows), IT(A.num_cols), IT(A.nnz), _p(A.row_ptr),
             _p(A.col_ind), _p(A.values), _p(B), _p(C), IT(N), IT(hw_block_size),
             1 if optimize_pattern else 0, ctypes.byref(t) if timings is not None else None))
    if timings is not None:
        for f in ("clustering_ms", "permutation_ms", "conversion_ms", "spmm_ms",
                  "unpermutation_ms", "total_pipeline_ms"):
            setattr(timings, f, getattr(t, f))


def spmm(*args, **kwargs):
    """Tier 1: spmm(A_bcsr, B, C, N)   (include/xspmm/xspmm.hpp:14-18)
    Tier 2: spmm(exec, A_csr, B, C, N, hw_block_size=16, optimize_pattern=True, timings=None)
            (include/xspmm/xspmm.hpp:24-32). B and C are device tensors (row-major K x N, M x N)."""
    if args and isinstance(args[0], BCSRMatrix):
        return _tier1(*args, **kwargs)
    return _tier2(*args, **kwargs)


class SpMMPlan:
    """The Tier-2 stages done once for repeated products with the same A (xspmm_plan_* in
    include/xspmm_b200.h). The reference recomputes them in every Tier-2 call
    (src/cuda/unstructured_mtx_mul.cu:56-130) and leaves reuse to Tier-1 callers (README.md:127).

    SpMMPlan(exec, A_csr, hw_block_size=16, optimize_pattern=True, timings=None) runs clustering,
    permutation and CSR->BCSR (timings, if given, receives their times); SpMMPlan.from_bcsr(A)
    adopts a BCSR matrix, whose arrays it keeps referenced. plan.execute(B, C, N) then computes
    C = A * B with C's rows in A's original order."""

    def __init__(self, exec: CudaExecutor | None = None, A: CSRMatrix | None = None,
                 hw_block_size: int = 16, optimize_pattern: bool = True,
                 timings: SpMMTimings | None = None, *, _handle=None, _keep=None,
                 _value_dtype=None):
        self._h = None
        if _handle is not None:
            self.exec, self._h, self._keep, self.value_dtype = exec, _handle, _keep, _value_dtype
            return
        _check_dev(exec, A.row_ptr)
        IT = _it(A.index_dtype)
        t = _lib.Timings()
        h = ctypes.c_void_p()
        fn = getattr(lib(), f"xspmm_plan_csr_{_VAL[A.value_dtype]}f32_{_IDX[A.index_dtype]}")
        check(fn(exec.handle, IT(A.num_rows), IT(A.num_cols), IT(A.nnz), _p(A.row_ptr),
                 _p(A.col_ind), _p(A.values), IT(hw_block_size), 1 if optimize_pattern else 0,
                 ctypes.byref(h), ctypes.byref(t) if timings is not None else None))
        self.exec, self._h, self._keep, self.value_dtype = exec, h, None, A.value_dtype
        if timings is not None:
            for f in ("clustering_ms", "permutation_ms", "conversion_ms", "spmm_ms",
                      "unpermutation_ms", "total_pipeline_ms"):
                setattr(timings, f, getattr(t, f))

    @classmethod
    def from_bcsr(cls, A: BCSRMatrix) -> "SpMMPlan":
        exec = A.exec
        IT = _it(A.index_dtype)
        h = ctypes.c_void_p()
        fn = getattr(lib(), f"xspmm_plan_bcsr_{_VAL[A.value_dtype]}f32_{_IDX[A.index_dtype]}")
        check(fn(exec.handle, IT(A.num_block_rows), IT(A.num_block_cols), IT(A.num_blocks),
                 IT(A.r_block), IT(A.c_block), _p(A.row_ptr), _p(A.col_ind), _p(A.values),
                 IT(A.num_rows), IT(A.num_cols), ctypes.byref(h)))
        return cls(exec, _handle=h, _keep=A, _value_dtype=A.value_dtype)

    def execute(self, B: torch.Tensor, C: torch.Tensor, N: int) -> None:
        if self._h is None:
            raise ValueError("plan is closed")
        if B.dtype != self.value_dtype:
            raise ValueError("B must have the value type of A")
        if C.dtype != torch.float32:
            raise ValueError("C must be float32")
        _check_dev(self.exec, B, C)
        self.exec.handle  # binds torch's current stream to the handle
        check(lib().xspmm_plan_execute(self._h, _p(B), _p(C), ctypes.c_int64(N)))

    def info(self) -> dict:
        inf = _lib.PlanInfo()
        check(lib().xspmm_plan_get_info(self._h, ctypes.byref(inf)))
        return {f: getattr(inf, f) for f, _ in _lib.PlanInfo._fields_ if f != "reserved"}

    def close(self) -> None:
        if self._h is not None:
            self.exec.handle
            check(lib().xspmm_plan_destroy(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def compute_1d_jaccard_clustering(exec: CudaExecutor, A: CSRMatrix, dist_thresh: float,
                                  block_width: int, perm_out: torch.Tensor) -> None:
    """include/xspmm/clustering.hpp:19-25. perm_out: device tensor of A's index type, M entries."""
    _check_dev(exec, A.row_ptr, perm_out)
    if perm_out.dtype != A.index_dtype or perm_out.numel() < A.num_rows:
        raise ValueError("perm_out must hold num_rows entries of the index type")
    IT = _it(A.index_dtype)
    check(getattr(lib(), f"xspmm_cluster_jaccard_{_IDX[A.index_dtype]}")(
        exec.handle, IT(A.num_rows), IT(A.num_cols), IT(A.nnz), _p(A.row_ptr), _p(A.col_ind),
        ctypes.c_float(dist_thresh), IT(block_width), _p(perm_out)))


def apply_permutation(target_exec: CudaExecutor, A: CSRMatrix, perm: torch.Tensor) -> CSRMatrix:
    """include/xspmm/clustering.hpp:34-38."""
    _check_dev(target_exec, A.row_ptr, perm)
    out = CSRMatrix(target_exec, A.num_rows, A.num_cols, A.nnz, A.value_dtype, A.index_dtype)
    IT = _it(A.index_dtype)
    check(getattr(lib(), f"xspmm_permute_rows_{_VAL[A.value_dtype]}_{_IDX[A.index_dtype]}")(
        target_exec.handle, IT(A.num_rows), IT(A.num_cols), IT(A.nnz), _p(A.row_ptr),
        _p(A.col_ind), _p(A.values), _p(perm), _p(out.row_ptr), _p(out.col_ind), _p(out.values)))
    return out


def csr_to_bcsr(target_exec: CudaExecutor, csr: CSRMatrix, r_block: int, c_block: int) -> BCSRMatrix:
    """include/xspmm/matrix/conversion.hpp:19-22 (here on the device)."""
    _check_dev(target_exec, csr.row_ptr)
    if r_block < 1 or c_block < 1:
        raise ValueError("block sizes must be positive")
    IT = _it(csr.index_dtype)
    nbr = -(-csr.num_rows // r_block)
    nbc = -(-csr.num_cols // c_block)
    brp = torch.zeros(nbr + 1, dtype=csr.index_dtype, device=target_exec.device)
    nnzb = ctypes.c_int64()
    check(getattr(lib(), f"xspmm_csr_to_bcsr_count_{_IDX[csr.index_dtype]}")(
        target_exec.handle, IT(csr.num_rows), IT(csr.num_cols), IT(csr.nnz), _p(csr.row_ptr),
        _p(csr.col_ind), IT(r_block), IT(c_block), _p(brp), ctypes.byref(nnzb)))
    out = BCSRMatrix(target_exec, nbr, nbc, nnzb.value, r_block, c_block, csr.value_dtype,
                     csr.index_dtype, num_rows=csr.num_rows, num_cols=csr.num_cols)
    out.row_ptr = brp
    check(getattr(lib(), f"xspmm_csr_to_bcsr_fill_{_VAL[csr.value_dtype]}_{_IDX[csr.index_dtype]}")(
        target_exec.handle, IT(csr.num_rows), IT(csr.num_cols), IT(csr.nnz), _p(csr.row_ptr),
        _p(csr.col_ind), _p(csr.values), IT(r_block), IT(c_block), _p(brp), _p(out.col_ind),
        _p(out.values)))
    return out


def unpermute_dense_matrix(exec: CudaExecutor, in_matrix: torch.Tensor, out_matrix: torch.Tensor,
                           perm: torch.Tensor, M: int, N: int) -> None:
    """include/xspmm/xspmm.hpp:35-40."""
    _check_dev(exec, in_matrix, out_matrix, perm)
    v = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[in_matrix.dtype]
    IT = _it(perm.dtype)
    check(getattr(lib(), f"xspmm_unpermute_dense_{v}_{_IDX[perm.dtype]}")(
        exec.handle, _p(in_matrix), _p(out_matrix), _p(perm), IT(M), IT(N)))
