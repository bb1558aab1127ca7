"""GPU tests of the block-row sharded product (xspmm_b200/shard.py): every shard on one GPU
against the unsharded product and the oracle, and (when the box has two GPUs) two NCCL ranks,
one per GPU, with B broadcast from rank 0."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import xspmm_b200 as xs
from tests.util import errors
from xspmm_b200 import synth
from xspmm_b200.shard import BlockRowShard, broadcast_b, partition_block_rows

pytestmark = pytest.mark.gpu


def _problem():
    return synth.cfg2_hidden_block(seed=31, n=2048, N=64, block_density=0.03)


def _check(P, brp, bci, bv, got, perm=None):
    ref = oracle.bcsr_spmm_f64(P.M, P.K, P.N, brp, bci, bv, P.B)
    e = errors(ref, got, 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e


@pytest.mark.parametrize("parts", [1, 3, 8])
@pytest.mark.parametrize("kind", ["mma", "tc"])
def test_shards_on_one_gpu_equal_the_whole(executor, parts, kind):
    P = _problem()
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    Ab = xs.csr_to_bcsr(executor, A, 16, 16)
    B = torch.as_tensor(P.B).to(executor.device)
    executor.set_tier1_kernel(kind)
    try:
        whole = torch.full((P.M, P.N), float("nan"), device=executor.device)
        xs.spmm(Ab, B, whole, P.N)
        bounds = partition_block_rows(Ab.row_ptr.cpu().numpy(), parts)
        pieces = []
        for p in range(parts):
            sh = BlockRowShard(Ab, int(bounds[p]), int(bounds[p + 1]))
            C = torch.full((sh.num_rows, P.N), float("nan"), device=executor.device)
            sh.execute(B, C, P.N)
            pieces.append(C)
            sh.close()
        got = torch.cat(pieces).cpu().numpy()
    finally:
        executor.set_tier1_kernel("auto")
    assert got.shape == (P.M, P.N) and np.isfinite(got).all()
    if kind == "mma":  # a block row's sum does not depend on the other block rows
        assert np.array_equal(got, whole.cpu().numpy())
    brp, bci, bv = oracle.csr_to_bcsr(P.row_ptr, P.col_ind, P.values, P.M, P.K)
    _check(P, brp, bci, bv, got)


def _nccl_rank(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ex = xs.CudaExecutor(rank)
        P = _problem()
        A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                                   index_dtype=torch.int32)
        Ab = xs.csr_to_bcsr(ex, A, 16, 16)
        bounds = partition_block_rows(Ab.row_ptr.cpu().numpy(), world)
        B = (torch.as_tensor(P.B).to(ex.device) if rank == 0
             else torch.zeros(P.B.shape, dtype=torch.float16, device=ex.device))
        broadcast_b(B, src=0)
        sh = BlockRowShard(Ab, int(bounds[rank]), int(bounds[rank + 1]))
        C = torch.full((sh.num_rows, P.N), float("nan"), device=ex.device)
        sh.execute(B, C, P.N)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"c{rank}.npy"), C.cpu().numpy())
        sh.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_ranks_nccl(tmp_path):
    world, port = 2, 29611 + os.getpid() % 1000
    mp.start_processes(_nccl_rank, args=(world, port, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    got = np.concatenate([np.load(tmp_path / f"c{r}.npy") for r in range(world)])
    P = _problem()
    brp, bci, bv = oracle.csr_to_bcsr(P.row_ptr, P.col_ind, P.values, P.M, P.K)
    assert got.shape == (P.M, P.N) and np.isfinite(got).all()
    _check(P, brp, bci, bv, got)
