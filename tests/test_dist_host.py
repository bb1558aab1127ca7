"""Host-side logic of the multi-GPU path, on CPU: the library's block-row split
(xspmm_dist_partition, the rule xspmm_dist_plan_csr_* uses) equals xspmm_b200.shard's, every rank
of a gloo group computes the same split with no message, the communicator id reaches every rank,
and a rank that never joins makes the others fail after the group's time limit instead of
hanging. No GPU work: the failures are made on the host."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from xspmm_b200 import dist as xd
from xspmm_b200 import shard


def _row_ptr(seed, nbr, empty_frac=0.0):
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, 40, nbr)
    lens[rng.random(nbr) < empty_frac] = 0
    if nbr > 3:
        lens[rng.integers(0, nbr)] += 5000  # a hub block row
    rp = np.zeros(nbr + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    return rp


@pytest.mark.parametrize("seed", range(8))
def test_library_partition_equals_python_rule(seed):
    rng = np.random.default_rng(seed)
    rp = _row_ptr(seed, int(rng.integers(1, 3000)), empty_frac=float(rng.choice([0, 0.5])))
    for parts in (1, 2, 3, 4, 8, 16):
        for w in (0.0, 1.0, 37.5):
            got = xd.partition(rp, parts, w)
            exp = shard.partition_block_rows(rp, parts, w)
            assert np.array_equal(got, exp), (parts, w)
            assert got[0] == 0 and got[-1] == len(rp) - 1 and np.all(np.diff(got) >= 0)


def test_partition_edge_cases():
    assert np.array_equal(xd.partition(np.array([0]), 4), [0, 0, 0, 0, 0])  # no block rows
    assert np.array_equal(xd.partition(np.array([0, 0, 0]), 2), shard.partition_block_rows([0, 0, 0], 2))
    with pytest.raises(Exception):
        xd.partition(np.array([0, 5, 3]), 2)  # not monotone


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        if mode == "partition":
            rp = _row_ptr(77, 5000, empty_frac=0.3)  # every rank builds the same matrix
            b = np.asarray(xd.partition(rp, world, 1.0), np.int64)
            import torch
            t = torch.as_tensor(b)
            outs = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(outs, t)
            q.put((rank, all(np.array_equal(o.numpy(), b) for o in outs)))
        elif mode == "id":
            xd.unique_id = lambda: bytes(range(128))  # no NCCL on a CPU box: a fixed id
            q.put((rank, xd.share_unique_id() == bytes(range(128))))
        elif mode == "never_joins":
            if rank == 1:
                q.put((rank, "left"))
                q.close()
                q.join_thread()  # the message is out before the process ends
                os._exit(0)  # leaves without taking part in the collective
            xd.unique_id = lambda: bytes(range(128))
            try:
                xd.share_unique_id()
                q.put((rank, "no error"))
            except Exception as e:  # the group's time limit ends the wait
                q.put((rank, "error: " + type(e).__name__))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "exception: " + repr(e)))


def _run(world, mode, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        res[r] = v
    for p in ps:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return res


def test_gloo_ranks_compute_the_same_partition():
    assert _run(2, "partition") == {0: True, 1: True}


def test_gloo_unique_id_reaches_every_rank():
    assert _run(2, "id") == {0: True, 1: True}


def test_gloo_rank_that_never_joins_ends_the_wait():
    res = _run(2, "never_joins")
    assert res[1] == "left"
    assert res[0].startswith("error") or res[0].startswith("exception"), res[0]
