"""Block-row sharding of one BCSR matrix over ranks (one process per GPU).

The reference runs on one device only; its Tier-1 product C = A * B
(include/xspmm/xspmm.hpp:14-18) is independent per block row given B, so a matrix splits into
contiguous block-row ranges with no exchange inside the product:

* partition: rank p owns block rows [r_p, r_{p+1}), chosen on the BCSR row pointer (the prefix
  sum of nonzero blocks) so that every rank gets about the same number of blocks, optionally plus
  a per-block-row weight where empty rows dominate;
* B: one broadcast per distinct B (torch.distributed over NCCL);
* C: each rank writes rows [16 r_p, 16 r_{p+1}) of C in the matrix's own row order (the clustered
  order for a Tier-2 matrix) into local memory. Gathering or unpermuting C is left to the caller.

Host logic only; every product runs in libxspmm_b200.so through an SpMMPlan.
"""
from __future__ import annotations

import numpy as np
import torch

from .api import BCSRMatrix, SpMMPlan


def partition_block_rows(row_ptr, parts: int, row_weight: float = 0.0) -> np.ndarray:
    """Boundaries r_0 = 0 <= r_1 <= ... <= r_parts = nbr of `parts` contiguous block-row ranges
    balancing  blocks + row_weight * block_rows  per range. r_p is the first block row whose
    weighted prefix reaches p * total / parts (a lower bound on the prefix), so a range is empty
    only when a single block row outweighs a whole share."""
    rp = np.asarray(row_ptr, dtype=np.float64)
    if parts < 1:
        raise ValueError("parts must be >= 1")
    nbr = len(rp) - 1
    if nbr < 0:
        raise ValueError("row_ptr must hold at least one entry")
    w = (rp - rp[0]) + row_weight * np.arange(nbr + 1, dtype=np.float64)
    total = w[-1]
    targets = total * np.arange(parts + 1, dtype=np.float64) / parts
    b = np.searchsorted(w, targets, side="left").astype(np.int64)
    b[0], b[-1] = 0, nbr
    return np.maximum.accumulate(np.minimum(b, nbr))


def shard_slice(row_ptr, r0: int, r1: int):
    """(b0, b1, rebased row pointer) of block rows [r0, r1): the shard's blocks are the
    contiguous range [b0, b1) of the matrix's col_ind / values (256 values per block)."""
    rp = np.asarray(row_ptr)
    if not (0 <= r0 <= r1 <= len(rp) - 1):
        raise ValueError("block-row range outside the matrix")
    b0, b1 = int(rp[r0]), int(rp[r1])
    return b0, b1, rp[r0:r1 + 1] - rp[r0]


class BlockRowShard:
    """Block rows [r0, r1) of a BCSR matrix as a product plan of their own: views of the
    matrix's col_ind/values, a rebased row pointer, and C rows [16 r0, min(16 r1, M))."""

    def __init__(self, A: BCSRMatrix, r0: int, r1: int):
        if not (0 <= r0 <= r1 <= A.num_block_rows):
            raise ValueError("block-row range outside the matrix")
        if A.r_block != 16 or A.c_block != 16:
            raise ValueError("Tier-1 SpMM supports 16x16 blocks only")
        self.r0, self.r1 = int(r0), int(r1)
        self.row_begin = 16 * self.r0
        self.row_end = min(16 * self.r1, A.num_rows)
        self.num_rows = max(0, self.row_end - self.row_begin)
        rp = A.row_ptr[self.r0:self.r1 + 1]
        b0, b1 = int(rp[0].item()), int(rp[-1].item())
        sub = BCSRMatrix.__new__(BCSRMatrix)
        sub.exec = A.exec
        sub.num_block_rows, sub.num_block_cols = self.r1 - self.r0, A.num_block_cols
        sub.num_blocks, sub.r_block, sub.c_block = b1 - b0, 16, 16
        sub.value_dtype, sub.index_dtype = A.value_dtype, A.index_dtype
        sub.num_rows, sub.num_cols = self.num_rows, A.num_cols
        sub.row_ptr = (rp - b0).contiguous()
        sub.col_ind = A.col_ind[b0:b1]
        sub.values = A.values[b0 * 256:b1 * 256]
        self.A = sub
        self.nnz_blocks = b1 - b0
        self.plan = SpMMPlan.from_bcsr(sub) if sub.num_block_rows > 0 else None

    def execute(self, B: torch.Tensor, C_local: torch.Tensor, N: int) -> None:
        """C_local (num_rows x N, fp32) = rows [row_begin, row_end) of A * B."""
        if self.plan is not None:
            self.plan.execute(B, C_local, N)

    def close(self) -> None:
        if self.plan is not None:
            self.plan.close()
            self.plan = None


def broadcast_b(B: torch.Tensor, src: int = 0, group=None) -> None:
    """B in place on every rank from `src` (the one exchange step of the sharded product)."""
    import torch.distributed as dist
    dist.broadcast(B, src=src, group=group)
