"""CPU tests of the block-row sharding host logic (xspmm_b200/shard.py): the partition, the
shard slices, and a two-rank gloo run of the sharded product computed with the oracle."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from xspmm_b200 import synth
from xspmm_b200.shard import partition_block_rows, shard_slice


def _random_row_ptr(rng, nbr, max_blocks):
    return np.concatenate([[0], np.cumsum(rng.integers(0, max_blocks + 1, nbr))]).astype(np.int64)


@pytest.mark.parametrize("parts", [1, 2, 3, 7, 8])
def test_partition_is_contiguous_and_balanced(parts):
    rng = np.random.default_rng(parts)
    for trial in range(20):
        nbr = int(rng.integers(0, 300))
        rp = _random_row_ptr(rng, nbr, int(rng.integers(1, 50)))
        b = partition_block_rows(rp, parts)
        assert len(b) == parts + 1 and b[0] == 0 and b[-1] == nbr
        assert np.all(np.diff(b) >= 0)
        blocks = np.diff(rp[b])
        assert blocks.sum() == rp[-1]
        biggest_row = int(np.diff(rp).max()) if nbr else 0
        # each share is within one block row of the even split
        assert np.all(blocks <= rp[-1] / parts + biggest_row + 1e-9)


def test_partition_with_empty_rows_weight():
    rp = np.array([0] + [0] * 90 + list(range(1, 11)), dtype=np.int64)  # 90 empty then 10 rows
    b0 = partition_block_rows(rp, 2)
    b1 = partition_block_rows(rp, 2, row_weight=1.0)
    assert b0[1] > 90  # blocks only: the empty rows all land on rank 0
    assert b1[1] < b0[1]  # a per-row weight moves empty rows to the other rank


def test_partition_more_parts_than_rows():
    rp = np.array([0, 5, 6], dtype=np.int64)
    b = partition_block_rows(rp, 8)
    assert b[0] == 0 and b[-1] == 2 and np.all(np.diff(b) >= 0)


def test_shard_slices_cover_the_matrix():
    rng = np.random.default_rng(3)
    rp = _random_row_ptr(rng, 57, 9)
    b = partition_block_rows(rp, 4)
    seen = 0
    for p in range(4):
        b0, b1, sub = shard_slice(rp, b[p], b[p + 1])
        assert b0 == seen and sub[0] == 0 and sub[-1] == b1 - b0
        assert np.array_equal(sub, rp[b[p]:b[p + 1] + 1] - rp[b[p]])
        seen = b1
    assert seen == rp[-1]
    with pytest.raises(ValueError):
        shard_slice(rp, 3, 2)


def _rank_main(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P = synth.cfg1_plumbing(seed=11, M=300, K=200, N=12, density=0.05)
        brp, bci, bv = oracle.csr_to_bcsr(P.row_ptr, P.col_ind, P.values, P.M, P.K)
        bounds = partition_block_rows(brp, world)
        # the partition is computed independently on every rank: it must agree
        allb = [torch.zeros(world + 1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allb, torch.as_tensor(bounds))
        assert all(torch.equal(x, allb[0]) for x in allb)
        B = torch.as_tensor(P.B) if rank == 0 else torch.zeros(P.B.shape, dtype=torch.float32)
        dist.broadcast(B, src=0)
        r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
        b0, b1, sub = shard_slice(brp, r0, r1)
        m_local = max(0, min(16 * r1, P.M) - 16 * r0)
        C_local = np.zeros((m_local, P.N))
        if r1 > r0:
            C_local = oracle.bcsr_spmm_f64(m_local, P.K, P.N, sub, bci[b0:b1], bv[b0:b1],
                                           B.numpy())
        np.save(os.path.join(result_dir, f"c{rank}.npy"), C_local)
    finally:
        dist.destroy_process_group()


def test_two_ranks_gloo_sharded_product(tmp_path):
    world, port = 2, 29511 + os.getpid() % 1000
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    P = synth.cfg1_plumbing(seed=11, M=300, K=200, N=12, density=0.05)
    brp, bci, bv = oracle.csr_to_bcsr(P.row_ptr, P.col_ind, P.values, P.M, P.K)
    full = oracle.bcsr_spmm_f64(P.M, P.K, P.N, brp, bci, bv, P.B)
    got = np.concatenate([np.load(tmp_path / f"c{r}.npy") for r in range(world)])
    assert np.array_equal(got, full)
