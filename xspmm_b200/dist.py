"""One matrix split by block rows over GPUs, through the C ABI's xspmm_dist_* entries.

The reference runs on one device; its Tier-1 product is independent per block row given B
(src/common/spmm_math.hpp:68-114). The library's distributed plan (xspmm_b200/csrc/dist.cu) keeps
one NCCL communicator per rank (one process or thread per GPU), clusters on every rank (the
permutation is deterministic), counts the permuted matrix's blocks, splits the block rows into
ranges balanced by nonzero blocks, and builds only this rank's BCSR. A product broadcasts B
(optionally) and writes this rank's rows of C; a gather collects C on a root in the caller's row
order (the reference's unpermute, src/cuda/mtx_permutation.cu:71-85).

Communicator set-up needs a unique id made on one rank and handed to the others; the caller moves
it (here: any torch.distributed group, or a file). Every wait on NCCL work is bounded: a rank that
never joins or stops makes the others' calls fail with TIMEOUT (status 6) instead of hanging.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib
from .api import CSRMatrix, CudaExecutor, _IDX, _VAL, _it, _p

ID_BYTES = 128


def partition(row_ptr, parts: int, row_weight: float = 0.0):
    """The library's block-row split (xspmm_dist_partition): boundaries of `parts` ranges."""
    import numpy as np
    rp = np.ascontiguousarray(row_ptr, dtype=np.int64)
    out = np.zeros(parts + 1, dtype=np.int64)
    check(lib().xspmm_dist_partition(rp.ctypes.data_as(ctypes.c_void_p), len(rp) - 1, int(parts),
                                     float(row_weight), out.ctypes.data_as(ctypes.c_void_p)))
    return out


def unique_id() -> bytes:
    """A new communicator's id (made on one rank)."""
    buf = (ctypes.c_ubyte * ID_BYTES)()
    check(lib().xspmm_dist_unique_id(buf, ID_BYTES))
    return bytes(buf)


def share_unique_id(group=None) -> bytes:
    """Rank 0 makes the id and every rank of a torch.distributed group (gloo or NCCL) gets it."""
    import torch.distributed as dist
    t = torch.zeros(ID_BYTES, dtype=torch.uint8)
    if dist.get_rank(group) == 0:
        t.copy_(torch.frombuffer(bytearray(unique_id()), dtype=torch.uint8))
    if dist.get_backend(group) == "nccl":
        tc = t.cuda()
        dist.broadcast(tc, src=0, group=group)
        t = tc.cpu()
    else:
        dist.broadcast(t, src=0, group=group)
    return bytes(t.numpy().tobytes())


class DistComm:
    """An NCCL communicator of the library (xspmm_dist_comm_init): joins within timeout_ms."""

    def __init__(self, exec: CudaExecutor, nranks: int, rank: int, uid: bytes,
                 timeout_ms: int = 60000):
        self.exec, self.nranks, self.rank = exec, int(nranks), int(rank)
        buf = (ctypes.c_ubyte * ID_BYTES).from_buffer_copy(uid[:ID_BYTES])
        h = ctypes.c_void_p()
        check(lib().xspmm_dist_comm_init(exec.handle, self.nranks, self.rank, buf, ID_BYTES,
                                         int(timeout_ms), ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if getattr(self, "_h", None) is not None:
            check(lib().xspmm_dist_comm_destroy(self._h))
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


class DistPlan:
    """This rank's share of A (xspmm_dist_plan_csr_*): every rank passes the whole CSR."""

    def __init__(self, comm: DistComm, A: CSRMatrix, hw_block_size: int = 16,
                 optimize_pattern: bool = True, row_weight: float = 0.0):
        self.comm, self.exec, self.value_dtype = comm, comm.exec, A.value_dtype
        IT = _it(A.index_dtype)
        h = ctypes.c_void_p()
        fn = getattr(lib(), f"xspmm_dist_plan_csr_{_VAL[A.value_dtype]}f32_{_IDX[A.index_dtype]}")
        check(fn(self.exec.handle, comm.handle, IT(A.num_rows), IT(A.num_cols), IT(A.nnz),
                 _p(A.row_ptr), _p(A.col_ind), _p(A.values), IT(hw_block_size),
                 1 if optimize_pattern else 0, ctypes.c_double(row_weight), ctypes.byref(h)))
        self._h = h
        self.K = A.num_cols
        inf = self.info()
        self.row_begin, self.row_end = inf["row_begin"], inf["row_end"]
        self.num_rows = self.row_end - self.row_begin

    def info(self) -> dict:
        inf = _lib.DistPlanInfo()
        check(lib().xspmm_dist_plan_get_info(self._h, ctypes.byref(inf)))
        return {f: getattr(inf, f) for f, _ in _lib.DistPlanInfo._fields_}

    def execute(self, B: torch.Tensor, C_local: torch.Tensor, N: int, bcast_root: int = -1,
                timeout_ms: int = 60000) -> None:
        """C_local (num_rows x N) = this rank's rows of A * B; bcast_root >= 0 broadcasts B
        from that rank first (in place)."""
        if B.dtype != self.value_dtype or C_local.dtype != torch.float32:
            raise ValueError("B must have A's value type and C_local must be float32")
        self.exec.handle  # binds torch's current stream
        check(lib().xspmm_dist_plan_execute(self._h, _p(B), _p(C_local), ctypes.c_int64(N),
                                            int(bcast_root), int(timeout_ms)))

    def gather(self, C_local: torch.Tensor, C: torch.Tensor | None, N: int, root: int = 0,
               timeout_ms: int = 60000) -> None:
        """C (M x N, the caller's row order) on `root` from every rank's C_local."""
        self.exec.handle
        check(lib().xspmm_dist_gather(self._h, _p(C_local), _p(C), ctypes.c_int64(N), int(root),
                                      int(timeout_ms)))

    def close(self) -> None:
        if getattr(self, "_h", None) is not None:
            self.exec.handle
            check(lib().xspmm_dist_plan_destroy(self._h))
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
