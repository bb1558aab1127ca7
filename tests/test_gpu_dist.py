"""GPU tests of the multi-GPU C-ABI entries (xspmm_dist_*): a matrix split by block rows over an
NCCL communicator, B broadcast, C gathered and unpermuted on a root.

* one rank: the distributed plan's product, gathered, is the same bits as the ordinary plan's
  (SpMMPlan) and within 1e-3 of the fp64 oracle;
* a communicator whose second rank never joins: the init returns TIMEOUT after its time limit
  (the communicator is aborted) and the device stays usable for a new one;
* two ranks on two GPUs (skipped with fewer): each holds about half of the blocks, C gathered on
  rank 0 matches the oracle. Child processes, NVLS off (a rank that leaves must not be bound to an
  NVLink multicast object)."""
import os
import tempfile
import time

import numpy as np
import pytest
import torch

import oracle
import xspmm_b200 as xs
from tests.util import errors
from xspmm_b200 import dist as xd
from xspmm_b200 import synth

pytestmark = pytest.mark.gpu


def _oracle_c(P, B, clustering=True):
    perm = oracle.cluster_fast(P.row_ptr, P.col_ind, P.M, P.K) if clustering else np.arange(P.M)
    prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values, perm)
    brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
    return oracle.unpermute_dense(oracle.bcsr_spmm_f64(P.M, P.K, B.shape[1], brp, bci, bv, B),
                                  perm)


@pytest.mark.parametrize("clustering,idx", [(True, torch.int32), (False, torch.int64)])
def test_dist_single_rank_matches_plan_and_oracle(executor, clustering, idx):
    P = synth.cfg2_hidden_block(seed=41, n=4096, N=96, block_density=0.02)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=idx)
    N = P.N
    with xd.DistComm(executor, 1, 0, xd.unique_id(), timeout_ms=30000) as comm:
        with xd.DistPlan(comm, A, 16, clustering) as dp:
            inf = dp.info()
            assert inf["row_begin"] == 0 and inf["row_end"] == P.M
            assert inf["nnz_blocks"] == inf["nnz_blocks_total"] > 0
            B = torch.as_tensor(P.B).to(executor.device)
            Cl = torch.full((dp.num_rows, N), float("nan"), device=executor.device)
            dp.execute(B, Cl, N, bcast_root=0)
            C = torch.full((P.M, N), float("nan"), device=executor.device)
            dp.gather(Cl, C, N, root=0)
            got = C.cpu().numpy()
    with xs.SpMMPlan(executor, A, 16, clustering) as plan:
        C2 = torch.full((P.M, N), float("nan"), device=executor.device)
        plan.execute(B, C2, N)
        assert np.array_equal(got.view(np.uint32), C2.cpu().numpy().view(np.uint32))
    e = errors(_oracle_c(P, P.B, clustering), got, 1e-3)
    assert e["max_rel_guarded"] <= 1e-3, e


def test_dist_rank_that_never_joins_times_out(executor):
    t0 = time.time()
    with pytest.raises(xs.XSpMMError) as ei:
        xd.DistComm(executor, 2, 0, xd.unique_id(), timeout_ms=3000)  # rank 1 never comes
    assert ei.value.status == 6, ei.value  # TIMEOUT
    assert time.time() - t0 < 60
    # the device is still usable: a new one-rank communicator and a product work
    P = synth.cfg2_hidden_block(seed=42, n=1024, N=16, block_density=0.03)
    A = xs.CSRMatrix.from_host(executor, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    with xd.DistComm(executor, 1, 0, xd.unique_id(), timeout_ms=30000) as comm:
        with xd.DistPlan(comm, A) as dp:
            B = torch.as_tensor(P.B).to(executor.device)
            Cl = torch.empty((dp.num_rows, P.N), device=executor.device)
            dp.execute(B, Cl, P.N)
            C = torch.empty((P.M, P.N), device=executor.device)
            dp.gather(Cl, C, P.N)
            e = errors(_oracle_c(P, P.B), C.cpu().numpy(), 1e-3)
            assert e["max_rel_guarded"] <= 1e-3, e


def _two_rank_worker(rank, world, idfile, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    ex = xs.CudaExecutor(rank)
    try:
        if rank == 0:
            uid = xd.unique_id()
            with open(idfile + ".tmp", "wb") as f:
                f.write(uid)
            os.replace(idfile + ".tmp", idfile)
        else:
            for _ in range(600):  # bounded wait for rank 0's id
                if os.path.exists(idfile):
                    break
                time.sleep(0.05)
            uid = open(idfile, "rb").read()
        P = synth.cfg4_banded(n=1 << 15, N=32)
        A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                                   index_dtype=torch.int32)
        with xd.DistComm(ex, world, rank, uid, timeout_ms=60000) as comm:
            with xd.DistPlan(comm, A) as dp:
                inf = dp.info()
                B = (torch.as_tensor(P.B).to(ex.device) if rank == 0 else
                     torch.zeros(P.B.shape, dtype=torch.float16, device=ex.device))
                Cl = torch.empty((max(dp.num_rows, 1), P.N), device=ex.device)
                dp.execute(B, Cl, P.N, bcast_root=0, timeout_ms=60000)
                C = torch.empty((P.M, P.N), device=ex.device) if rank == 0 else None
                dp.gather(Cl, C, P.N, root=0, timeout_ms=60000)
                res = {"blocks": inf["nnz_blocks"], "total": inf["nnz_blocks_total"]}
                if rank == 0:
                    e = errors(_oracle_c(P, P.B), C.cpu().numpy(), 1e-3)
                    res["err"] = e["max_rel_guarded"]
        q.put((rank, res))
    except Exception as e:
        q.put((rank, {"exception": repr(e)}))


def test_dist_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    idfile = os.path.join(tempfile.mkdtemp(), "nccl_id")
    ps = [ctx.Process(target=_two_rank_worker, args=(r, 2, idfile, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=120)
    assert "exception" not in res[0] and "exception" not in res[1], res
    tot = res[0]["total"]
    assert res[0]["blocks"] + res[1]["blocks"] == tot
    assert abs(res[0]["blocks"] - res[1]["blocks"]) <= 0.1 * tot  # about half each
    assert res[0]["err"] <= 1e-3, res
