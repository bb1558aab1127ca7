"""Benchmark of the xSpMM hot path on B200 (one JSON line on rank 0).

Workload (default, BASELINE.json configs[4], "GNN aggregation" -- the largest config that fits one
GPU): A is an R-MAT adjacency of 2^20 nodes (a,b,c,d = .57,.19,.19,.05, 16 sampled edges per
node, duplicates merged, self-loops kept), fp16 values 1/deg(row); B is 2^20 x 128 fp16 N(0,1);
C fp32; clustering on; the config repeats the Tier-1 product 1000 times. Synthetic, seeded (42).
--workload cfg4 runs the banded 2,000,000-row config instead.

Metric: SpMM effective TFLOPS (2*nnz*N/s) at 1/2/4/8 B200; clustering+convert ms.
  value : one step = one product C = A*B on the clustered matrix (the config's repeated unit),
          block rows split over the ranks by nonzero blocks (one plan per rank, B broadcast once
          with NCCL, each rank writes its own rows of C), inputs resident in HBM, device time
          (CUDA events on the launching stream) max over ranks, L2 flushed (256 MiB write) before
          every step outside the timed interval. Strong scaling: one matrix whatever N.
  clustering_plus_conversion_ms / plan_ms : the plan's stages (clustering, row permutation,
          CSR->BCSR), timed once.
  tier2 : one whole xspmm::spmm(exec, A_csr, B, C, N, 16, true, &timings) call on rank 0 through
          the C ABI -- device-resident (with the stage times of SpMMTimings) and end to end (CSR
          and B up from pinned host memory, C down, inside the interval).
  e2e   : the product through the public API with B uploaded from pinned host memory (rank 0)
          and broadcast, and each rank's rows of C copied back, every step.
  cpu_baseline / --impl reference : the reference's CPU path on a bounded sample of the same
          generator (2^15 rows): its host code (compiled from its sources, oracle/_ref) clusters,
          permutes and converts once (single thread, as written); the product is the oracle's
          fp64 BCSR SpMM on all host cores (the reference has no CPU SpMM).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SpMM effective TFLOPS (2*nnz*N/s) at 1/2/4/8 B200; clustering+convert ms"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) of one Tier-1 product, summed over its launches, from a one-pass ncu
# capture of this bench at full size on one B200 (profiles/tier1_gather_cfg5.md, which gives the
# command); keyed by (workload, N, ranks). Other workloads report null.
TRAFFIC = {("cfg5_gnn_rmat_2^20", 128, 1): 1175840384}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        d["source"] = "measured"
        return d
    d = dict(PEAKS_FALLBACK)
    d["source"] = "fallback"
    return d


# ------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, device_index: int):
        self.dev = device_index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), "--query-gpu=" + ",".join(self.FIELDS),
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(self.FIELDS):
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        for r in self.rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                "sw_power_cap"), r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


# ------------------------------------------------------------------------------------------------
# workloads (synthetic, seeded)
# ------------------------------------------------------------------------------------------------
def _workload(name, rows_log2=0):
    """(label, N, problem factory, CPU-sample factory, sample description). rows_log2 > 0 builds
    the banded / R-MAT generator at 2^rows_log2 rows instead of full size (profiling cases)."""
    from xspmm_b200 import synth
    if name == "cfg5" and rows_log2:
        return (f"cfg5_gnn_rmat_2^{rows_log2}", 128,
                lambda N: synth.cfg5_rmat(scale=rows_log2, N=N),
                lambda N: synth.cfg5_rmat(scale=15, N=N), "R-MAT 2^15 rows, seed 42")
    if name == "cfg4" and rows_log2:
        return (f"cfg4_banded_2^{rows_log2}", 64, lambda N: synth.cfg4_banded(n=1 << rows_log2, N=N),
                lambda N: synth.cfg4_banded(n=1 << 15, N=N), "banded 2^15 rows, seed 42")
    if name == "cfg5":
        return ("cfg5_gnn_rmat_2^20", 128, lambda N: synth.cfg5_rmat(N=N),
                lambda N: synth.cfg5_rmat(scale=15, N=N),
                "R-MAT 2^15 rows, same generator (a,b,c,d = .57,.19,.19,.05, 16 edges per row, "
                "dedupe, values 1/deg), seed 42")
    if name == "cfg4":
        return ("cfg4_banded_2M", 64, lambda N: synth.cfg4_banded(N=N),
                lambda N: synth.cfg4_banded(n=1 << 15, N=N),
                "banded 2^15 rows, same generator (half-bandwidth 32, 40 % fill, rows shuffled), "
                "seed 42")
    if name == "cfg2":
        return ("cfg2_hidden_block", 256, lambda N: synth.cfg2_hidden_block(N=N),
                lambda N: synth.cfg2_hidden_block(N=N), "the full hidden-block matrix")
    raise ValueError(name)


def _config(args, P, label, N, world):
    """The workload description both arms print (identical keys and values)."""
    return {"workload": label, "M": P.M, "K": P.K, "N": N, "nnz": P.nnz, "seed": 42,
            "value_dtype": "fp16", "accumulate": "fp32", "index": "int32", "hw_block": 16,
            "clustering": True,
            "step": "one SpMM product C = A*B on the clustered matrix (the repeated unit of the "
                    "config's repeated products); clustering + permutation + conversion reported "
                    "separately and in the tier2 object",
            "parallelism": (f"block rows of the clustered matrix split over {world} rank(s), "
                            "balanced by nonzero blocks; B broadcast once (NCCL); C rows local"),
            "l2": "flushed before every timed step (256 MiB write, outside the timed interval)"}


def _ref_stage_times(S):
    """The reference's host code (compiled from its sources) on problem S: clustering,
    permutation and conversion, single-threaded as written; returns (kind, stage seconds, BCSR,
    perm). Falls back to the oracle restatement when the compiled reference is absent."""
    import oracle
    t0 = time.perf_counter()
    if oracle.ref_available():
        perm = oracle.ref_cluster(S.row_ptr, S.col_ind, S.M, S.K, 0.5, 16)
        t1 = time.perf_counter()
        prp, pci, pv = oracle.ref_permute(S.row_ptr, S.col_ind, S.values, perm, S.K)
        t2 = time.perf_counter()
        brp, bci, bv = oracle.ref_csr_to_bcsr(prp, pci, pv, S.M, S.K)
        kind = "reference"
    else:
        perm = oracle.cluster_literal(S.row_ptr, S.col_ind, S.M, S.K, 0.5, 16)
        t1 = time.perf_counter()
        prp, pci, pv = oracle.permute_rows(S.row_ptr, S.col_ind, S.values.astype(np.float32), perm)
        t2 = time.perf_counter()
        brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, S.M, S.K)
        kind = "port"
    t3 = time.perf_counter()
    return kind, {"clustering_ms": (t1 - t0) * 1e3, "permutation_ms": (t2 - t1) * 1e3,
                  "conversion_ms": (t3 - t2) * 1e3}, (brp, bci, bv), perm


def cpu_baseline(args, name, N, budget_s):
    """CPU baseline on a bounded sample of the workload: the reference's host code for
    clustering/permutation/conversion (single thread; the reference has no threading) and, for the
    product, the oracle's fp64 BCSR SpMM on all host cores (the reference has no CPU SpMM). The
    value is the product's effective TFLOPS on the sample -- the same metric as the GPU arm."""
    import oracle
    label, _, _, make_sample, desc = _workload(name)
    S = make_sample(N)
    kind, stages, (brp, bci, bv), perm = _ref_stage_times(S)
    Bf = S.B.astype(np.float32)
    runs = []
    t_start = time.perf_counter()
    while not runs or (time.perf_counter() - t_start < budget_s and len(runs) < 20):
        t0 = time.perf_counter()
        oracle.bcsr_spmm_f64(S.M, S.K, N, brp, bci, bv, Bf)
        runs.append(time.perf_counter() - t0)
    t = sum(runs) / len(runs)
    return {
        "value": round(2.0 * S.nnz * N / t / 1e12, 6), "unit": "TFLOPS",
        "cores": oracle.num_threads(), "kind": kind,
        "sample": (f"{desc} (M={S.M}, nnz={S.nnz}); product = oracle fp64 BCSR SpMM "
                   f"({oracle.num_threads()} OpenMP threads) x{len(runs)}; clustering/permutation/"
                   f"conversion = the reference's host code, 1 thread, once"),
        "spmm_ms": round(t * 1e3, 3),
        "stage_ms": {k: round(v, 3) for k, v in stages.items()},
        "clustering_plus_conversion_ms": round(stages["clustering_ms"] + stages["conversion_ms"], 3),
        "cpu_model": _cpu_model(), "nproc": os.cpu_count(),
    }


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


# ------------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------------
def run_gpu(args):
    import datetime

    import torch
    import torch.distributed as dist

    import xspmm_b200 as xs
    from xspmm_b200 import dist as xd
    from xspmm_b200.shard import broadcast_b

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def rmax(x):
        if world == 1:
            return x
        t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def rsum(x):
        if world == 1:
            return x
        t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    label, N0, make, _, _ = _workload(args.workload, args.rows_log2)
    N = args.n_cols or N0
    P = make(N)  # every rank builds the same seeded matrix on its host
    ex = xs.CudaExecutor(local)
    stream = torch.cuda.current_stream(dev)
    A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flops = 2.0 * P.nnz * N

    # ---- Tier-2: the whole pipeline in one call (rank 0), device-resident and end to end ------
    tier2 = None
    if rank == 0 and args.tier2_steps > 0:
        B0 = torch.as_tensor(P.B).to(dev)
        C0 = torch.empty((P.M, N), dtype=torch.float32, device=dev)
        xs.spmm(ex, A, B0, C0, N, 16, True)
        torch.cuda.synchronize()
        st = {k: 0.0 for k in ("clustering_ms", "permutation_ms", "conversion_ms", "spmm_ms",
                               "total_pipeline_ms")}
        ms2 = []
        for i in range(args.tier2_steps):
            flush.fill_(float(i))
            e0, e1 = ev(), ev()
            t = xs.SpMMTimings()
            e0.record(stream)
            xs.spmm(ex, A, B0, C0, N, 16, True, t)
            e1.record(stream)
            torch.cuda.synchronize()
            ms2.append(e0.elapsed_time(e1))
            for k in st:
                st[k] += getattr(t, k) / args.tier2_steps
        # end to end: CSR and B up from pinned host memory, C down, inside the interval
        h_rp = torch.from_numpy(P.row_ptr.astype(np.int32)).pin_memory()
        h_ci = torch.from_numpy(P.col_ind.astype(np.int32)).pin_memory()
        h_v = torch.from_numpy(P.values).pin_memory()
        h_B = torch.from_numpy(P.B).pin_memory()
        h_C = torch.empty((P.M, N), dtype=torch.float32).pin_memory()
        Ae = xs.CSRMatrix(ex, P.M, P.K, P.nnz, torch.float16, torch.int32)
        Be = torch.empty_like(B0)
        e2e2 = []
        for i in range(args.tier2_steps):
            flush.fill_(float(i))
            e0, e1 = ev(), ev()
            e0.record(stream)
            Ae.row_ptr.copy_(h_rp, non_blocking=True)
            Ae.col_ind.copy_(h_ci, non_blocking=True)
            Ae.values.copy_(h_v, non_blocking=True)
            Be.copy_(h_B, non_blocking=True)
            xs.spmm(ex, Ae, Be, C0, N, 16, True)
            h_C.copy_(C0, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            e2e2.append(e0.elapsed_time(e1))
        t2ms = sum(ms2) / len(ms2)
        tier2 = {"ms": round(t2ms, 3), "effective_tflops": round(flops / (t2ms * 1e-3) / 1e12, 6),
                 "stages_ms": {k: round(v, 3) for k, v in st.items()},
                 "e2e_ms": round(sum(e2e2) / len(e2e2), 3),
                 "e2e_tflops": round(flops / (sum(e2e2) / len(e2e2) * 1e-3) / 1e12, 6),
                 "h2d_bytes": int(h_rp.numel() * 4 + h_ci.numel() * 4 + h_v.numel() * 2 +
                                  h_B.numel() * 2),
                 "d2h_bytes": int(h_C.numel() * 4), "steps": args.tier2_steps, "warmup": 1,
                 "call": "xspmm::spmm(exec, A_csr, B, C, N, 16, true, &timings) through the C ABI"}
        del B0, C0, Ae, Be, h_rp, h_ci, h_v, h_B, h_C
        torch.cuda.empty_cache()
    barrier()

    # ---- the plan, through the multi-GPU C ABI (xspmm_dist_*): every rank clusters (the result is
    # deterministic), counts the permuted matrix's blocks and keeps only its own block rows ---------
    uid = xd.share_unique_id() if world > 1 else xd.unique_id()
    comm = xd.DistComm(ex, world, rank, uid, timeout_ms=300000)
    e = [ev() for _ in range(3)]
    e[0].record(stream)
    perm = torch.empty(P.M, dtype=torch.int32, device=dev)
    xs.compute_1d_jaccard_clustering(ex, A, 0.5, 16, perm)  # the clustering stage alone
    e[1].record(stream)
    shard = xd.DistPlan(comm, A)  # clustering, permutation, block count, own block rows, plan
    e[2].record(stream)
    torch.cuda.synchronize()
    clustering_ms = rmax(e[0].elapsed_time(e[1]))
    plan_build_ms = rmax(e[1].elapsed_time(e[2]))
    sinfo = shard.info()
    nnzb = sinfo["nnz_blocks_total"]
    B = torch.as_tensor(P.B).to(dev) if rank == 0 else torch.zeros((P.K, N), dtype=torch.float16,
                                                                    device=dev)
    b_bcast_ms = None
    if world > 1:  # the communicator is set up by the first collective: warm it, then time
        w = torch.zeros(1, device=dev)
        dist.all_reduce(w)
        barrier()
        torch.cuda.synchronize()
        b0, b1 = ev(), ev()
        b0.record(stream)
        broadcast_b(B, src=0)
        b1.record(stream)
        torch.cuda.synchronize()
        b_bcast_ms = rmax(b0.elapsed_time(b1))
    C = torch.empty((max(shard.num_rows, 1), N), dtype=torch.float32, device=dev)

    # ---- the timed product (value) ----------------------------------------------------------------
    for _ in range(args.warmup):
        shard.execute(B, C, N)
    torch.cuda.synchronize()
    starts = [ev() for _ in range(args.steps)]
    ends = [ev() for _ in range(args.steps)]
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ex.reset_launch_count()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.fill_(float(i))
        torch.cuda.nvtx.range_push("timed_step")  # ncu --nvtx --nvtx-include timed_step/
        starts[i].record(stream)
        shard.execute(B, C, N)
        ends[i].record(stream)
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    launches = ex.launch_count()
    clocks = sampler.stop()
    ms = rmax(sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps)

    # sampled rows of C against an fp64 product of the host CSR (local row i is clustered row
    # 16*r_p + i, which is original row perm[16*r_p + i])
    rng = np.random.default_rng(1000 + rank)
    nloc = shard.num_rows
    chk = {"rows": 0, "max_rel_guarded": 0.0}
    if nloc > 0:
        li = np.sort(rng.choice(nloc, min(256, nloc), replace=False))
        orig = perm[shard.row_begin + torch.as_tensor(li, device=dev)].cpu().numpy()
        got = C[torch.as_tensor(li, device=dev)].cpu().numpy().astype(np.float64)
        Bh = P.B.astype(np.float64)
        ref = np.zeros_like(got)
        for k, r in enumerate(orig):
            a, b = P.row_ptr[r], P.row_ptr[r + 1]
            ref[k] = P.values[a:b].astype(np.float64) @ Bh[P.col_ind[a:b]]
        rms = float(np.sqrt(np.mean(ref * ref))) or 1.0
        err = float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3 * rms)))
        chk = {"rows": int(len(li)), "max_rel_guarded": err}
    chk_err = rmax(chk["max_rel_guarded"])
    chk_rows = int(rsum(chk["rows"]))

    # ---- end to end: B up (rank 0, pinned) + broadcast, product, local C rows down --------------
    # Every step uploads its B from pinned host memory, runs the product (the library broadcasts
    # B to the other ranks) and downloads its C rows to pinned host memory. Steps are pipelined
    # the way a serving loop double-buffers: step i's download (device -> host) overlaps step
    # i+1's upload (host -> device, the other PCIe direction) and product, on three streams with
    # two device buffers each for B and C. The interval runs from before the first upload to the
    # end of the last download; B (K x N fp16) and C are larger than L2, so no flush is needed.
    h_B = torch.from_numpy(P.B).pin_memory() if rank == 0 else None
    Bs = [B, torch.empty_like(B)]
    Cs = [C, torch.empty_like(C)]
    h_Cs = [torch.empty((max(shard.num_rows, 1), N), dtype=torch.float32).pin_memory()
            for _ in range(2)]
    s_up, s_dn = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_run(nsteps):
        up = [ev() for _ in range(nsteps)]
        comp = [ev() for _ in range(nsteps)]
        dn = [ev() for _ in range(nsteps)]
        t0, t1 = ev(), ev()
        t0.record(stream)
        s_up.wait_event(t0)
        for i in range(nsteps):
            b = i % 2
            with torch.cuda.stream(s_up):
                if i >= 2:
                    s_up.wait_event(comp[i - 2])  # step i-2's product has read B[b]
                if rank == 0:
                    Bs[b].copy_(h_B, non_blocking=True)
                up[i].record(s_up)
            stream.wait_event(up[i])
            if i >= 2:
                stream.wait_event(dn[i - 2])  # step i-2's download has read C[b]
            shard.execute(Bs[b], Cs[b], N, bcast_root=0 if world > 1 else -1)
            comp[i].record(stream)
            with torch.cuda.stream(s_dn):
                s_dn.wait_event(comp[i])
                h_Cs[b].copy_(Cs[b], non_blocking=True)
                dn[i].record(s_dn)
        stream.wait_event(dn[nsteps - 1])
        t1.record(stream)
        t1.synchronize()
        return t0.elapsed_time(t1) / nsteps

    e2e_run(max(args.warmup, 2))
    torch.cuda.synchronize()
    barrier()
    e2e_ms = rmax(e2e_run(args.steps))
    e2e_h2d = int(P.K * N * 2)  # B, once per step (rank 0)
    e2e_d2h = int(rsum(shard.num_rows * N * 4))

    per_rank_blocks = int(sinfo["nnz_blocks"])
    blocks_all = [int(x) for x in ([per_rank_blocks] if world == 1 else
                                   _gather_ints(dist, dev, per_rank_blocks, world))]
    bytes_all = [int(x) for x in ([sinfo["device_bytes"]] if world == 1 else
                                  _gather_ints(dist, dev, int(sinfo["device_bytes"]), world))]
    launches_all = int(rsum(launches))
    shard.close()
    comm.close()

    if rank != 0:
        barrier()
        if world > 1:
            dist.destroy_process_group()
        return
    pk = peaks()
    if tier2 is not None:
        # Bandwidth of the two data-movement stages of that Tier-2 call (algorithmic bytes: each
        # array read once and written once). Permutation: CSR in (row_ptr, 4 B index + 2 B value
        # per nonzero) and out, plus perm. Conversion: the permuted CSR in, the BCSR out (16 x 16
        # fp16 blocks, block column indices, block row pointers).
        perm_b = 2 * (P.nnz * 6 + (P.M + 1) * 4) + P.M * 4
        conv_b = P.nnz * 6 + (P.M + 1) * 4 + nnzb * (512 + 4) + ((P.M + 15) // 16 + 1) * 4
        sm = tier2["stages_ms"]
        tier2["stage_bandwidth"] = {
            k: {"bytes": int(b), "gbs": round(b / (sm[ms] * 1e-3) / 1e9, 1),
                "frac_of_hbm": round(b / (sm[ms] * 1e-3) / 1e9 / pk["hbm_gbs"], 4)}
            for k, ms, b in (("permutation", "permutation_ms", perm_b),
                             ("conversion", "conversion_ms", conv_b)) if sm.get(ms, 0) > 0}
    padded = 2.0 * nnzb * 256 * N
    alg_bytes = P.nnz * (4 + 2) + (P.M + 1) * 4 + P.K * N * 2 + P.M * N * 4
    achieved = alg_bytes / (ms * 1e-3) / 1e9
    plan_ms = plan_build_ms
    out = {
        "metric": METRIC,
        "value": round(flops / (ms * 1e-3) / 1e12, 5),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded generator of the config; no dataset)",
        "config": _config(args, P, label, N, world),
        "clustering_plus_conversion_ms": round(plan_build_ms, 3),
        "plan_ms": {"clustering": round(clustering_ms, 3),
                    "plan_build": round(plan_build_ms, 3),
                    "note": "plan_build = the rank's xspmm_dist_plan_csr call: clustering, "
                            "permutation, block count, its own block rows' BCSR, product set-up "
                            "(max over ranks); clustering = the clustering call alone"},
        "nnzb_after_clustering": nnzb,
        "padded_tflops": round(padded / (ms * 1e-3) / 1e12, 4),
        "padded_frac_of_bf16_peak": round(padded / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 5),
        "amortized_1000": {
            "tflops": round(1000 * flops / ((plan_ms + 1000 * ms) * 1e-3) / 1e12, 5),
            "note": "plan once (clustering, permutation, conversion, shard set-up) + 1000 products"},
        "tier2": tier2,
        "roofline": {"kernel": "Tier-1 product (one plan execute)", "bound": "hbm",
                     "achieved": round(achieved, 2), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 5),
                     "traffic": TRAFFIC.get((label, N, world)),
                     "alg_bytes": int(alg_bytes),
                     "alg_bytes_def": "A as CSR (4 B index + 2 B value per nonzero, row_ptr), "
                                      "B read once, C written once; B's gathers not counted",
                     "peak_source": pk["source"]},
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 5), "unit": "TFLOPS",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": e2e_h2d,
                "d2h_bytes_per_step": e2e_d2h,
                "schedule": "per step: B up (pinned), product, C rows down (pinned); steps "
                            "double-buffered on 3 streams so a step's download overlaps the "
                            "next step's upload and product; inputs larger than L2, no flush"},
        "b_broadcast_ms": None if b_bcast_ms is None else round(b_bcast_ms, 4),
        "per_rank_blocks": blocks_all,
        "per_rank_plan_device_bytes": bytes_all,
        "c_check": {"sampled_rows": chk_rows, "max_rel_guarded": chk_err, "tol": 1e-3,
                    "reference": "fp64 product of the host CSR rows"},
        "gpu_launches": launches_all,
        "wall_s_timed_region": round(wall, 4),
        "clocks": clocks,
    }
    assert chk_err <= 1e-3, chk_err
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args, args.workload, N, args.cpu_budget)
    print(json.dumps(out), flush=True)
    barrier()
    if world > 1:
        dist.destroy_process_group()


def _gather_ints(dist, dev, v, world):
    import torch
    t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
    outs = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
    dist.all_gather(outs, t)
    return [int(x.item()) for x in outs]


def run_reference(args):
    """The reference arm: the reference's own CPU path for this workload on the host cores, on a
    bounded sample (see cpu_baseline): its host code clusters, permutes and converts once, then
    each step is one product (oracle fp64 BCSR SpMM on all cores; the reference has none)."""
    # torchrun sets OMP_NUM_THREADS=1 for its ranks; the arm runs on rank 0 alone and uses every
    # core of the process (set before the oracle's OpenMP runtime is loaded)
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))
    import oracle
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    label, N0, make, make_sample, desc = _workload(args.workload, args.rows_log2)
    N = args.n_cols or N0
    P = make(N)  # the full workload, for the config description only
    S = make_sample(N)
    kind, stages, (brp, bci, bv), _ = _ref_stage_times(S)
    Bf = S.B.astype(np.float32)
    for _ in range(args.warmup):
        oracle.bcsr_spmm_f64(S.M, S.K, N, brp, bci, bv, Bf)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.bcsr_spmm_f64(S.M, S.K, N, brp, bci, bv, Bf)
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    val = 2.0 * S.nnz * N / t / 1e12
    sample = (f"{desc} (M={S.M}, nnz={S.nnz}); step = oracle fp64 BCSR SpMM "
              f"({oracle.num_threads()} OpenMP threads; the reference has no CPU SpMM); "
              "clustering/permutation/conversion = the reference's host code, 1 thread, once")
    out = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(val, 6),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded generator of the config; no dataset)",
        "config": _config(args, P, label, N, world),
        "clustering_plus_conversion_ms": round(stages["clustering_ms"] + stages["permutation_ms"] +
                                               stages["conversion_ms"], 3),
        "stage_ms": {k: round(v, 3) for k, v in stages.items()},
        "cpu_baseline": {"value": round(val, 6), "unit": "TFLOPS", "cores": oracle.num_threads(),
                         "kind": kind, "sample": sample, "cpu_model": _cpu_model(),
                         "nproc": os.cpu_count()},
        "e2e": {"value": round(val, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)

def run_tier1_compare(args):
    """mma.sync vs tcgen05 Tier-1 kernels on the pruned-LLM config (
    4096 x 11008, every 16x16 block present) over the N sweep; one JSON line per (N, kernel)."""
    import torch

    import xspmm_b200 as xs
    from xspmm_b200 import synth

    P = synth.cfg3_pruned_llm(N=16)
    ex = xs.CudaExecutor(0)
    A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    Ab = xs.csr_to_bcsr(ex, A, 16, 16)
    pk = peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    for N in [int(x) for x in args.compare_n.split(",")]:
        B = torch.randn((P.K, N), device="cuda").half()
        C = torch.empty((P.M, N), dtype=torch.float32, device="cuda")
        for kind in args.compare_kernels.split(","):
            ex.set_tier1_kernel(kind)
            plan = xs.SpMMPlan.from_bcsr(Ab)  # per-matrix set-up (tcgen05 tiles) done here

            def timed(fn):
                for _ in range(args.warmup):
                    fn()
                torch.cuda.synchronize()
                ts = []
                for i in range(args.steps):
                    flush.fill_(float(i))
                    s0 = torch.cuda.Event(enable_timing=True)
                    s1 = torch.cuda.Event(enable_timing=True)
                    s0.record()
                    fn()
                    s1.record()
                    torch.cuda.synchronize()
                    ts.append(s0.elapsed_time(s1))
                return sorted(ts)[len(ts) // 2]

            call_ms = timed(lambda: xs.api._tier1(Ab, B, C, N))
            ms = timed(lambda: plan.execute(B, C, N))
            plan.close()
            padded = 2.0 * Ab.num_blocks * 256 * N / (ms * 1e-3) / 1e12
            print(json.dumps({
                "workload": "cfg3_pruned_llm", "N": N, "kernel": kind, "ms": round(ms, 4),
                "call_ms": round(call_ms, 4),
                "effective_tflops": round(2.0 * P.nnz * N / (ms * 1e-3) / 1e12, 2),
                "padded_tflops": round(padded, 2),
                "padded_frac_of_bf16_peak": round(padded / pk["bf16_tflops"], 4),
                "peak_source": pk["source"], "nnzb": Ab.num_blocks, "steps": args.steps,
                "timing": "ms: plan execute (A's set-up done once); call_ms: stateless Tier-1 "
                          "call (set-up every call); median, L2 flushed before every launch"}),
                flush=True)
        ex.set_tier1_kernel("auto")


def run_cluster_compare(args):
    """The clustering call alone (xspmm::compute_1d_jaccard_clustering through the C ABI), one
    JSON line per (workload, path): CUDA events around each call after one warm-up call, tau 0.5,
    w 16, checked equal across the paths of a workload. Workloads: cfg2, cfg3 (full size), cfg4:S
    / cfg5:S (the banded / R-MAT generators at 2^S rows; S omitted = full size); paths: auto, or
    forced through XSPMM_CLUSTER_KERNEL (index, bits, sweep) and XSPMM_CLUSTER_SEED_SETS=0
    (index-nosets)."""
    import torch

    import xspmm_b200 as xs
    from xspmm_b200 import synth

    ex = xs.CudaExecutor(0)
    for wl in args.cluster_workloads.split(","):
        name, _, sc = wl.partition(":")
        if name == "cfg2":
            P = synth.cfg2_hidden_block(N=8)
        elif name == "cfg3":
            P = synth.cfg3_pruned_llm(N=8)
        elif name == "cfg4":
            P = synth.cfg4_banded(n=(1 << int(sc)) if sc else 2_000_000, N=8)
        elif name == "cfg5":
            P = synth.cfg5_rmat(scale=int(sc) if sc else 20, N=8)
        else:
            raise ValueError(wl)
        A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                                   index_dtype=torch.int32)
        first = None
        for path in args.cluster_paths.split(","):
            kind, _, opt = path.partition("-")
            os.environ.pop("XSPMM_CLUSTER_KERNEL", None)
            os.environ["XSPMM_CLUSTER_SEED_SETS"] = "0" if opt == "nosets" else "1"
            if kind != "auto":
                os.environ["XSPMM_CLUSTER_KERNEL"] = kind
            perm = torch.zeros(P.M, dtype=torch.int32, device="cuda")
            try:
                times = []
                for it in range(1 + args.steps):
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    xs.compute_1d_jaccard_clustering(ex, A, 0.5, 16, perm)
                    e1.record()
                    torch.cuda.synchronize()
                    if it > 0:
                        times.append(e0.elapsed_time(e1))
            except xs.XSpMMError as e:
                print(json.dumps({"workload": wl, "M": P.M, "path": path, "unsupported": str(e)}),
                      flush=True)
                continue
            p = perm.cpu().numpy()
            same = None if first is None else bool(np.array_equal(first, p))
            first = p if first is None else first
            print(json.dumps({"workload": wl, "M": P.M, "nnz": P.nnz, "path": path,
                              "ms": round(statistics.median(times), 3),
                              "ms_all": [round(t, 3) for t in times], "same_perm": same}),
                  flush=True)
        os.environ.pop("XSPMM_CLUSTER_KERNEL", None)
        os.environ.pop("XSPMM_CLUSTER_SEED_SETS", None)
        del A
        torch.cuda.empty_cache()


VENDOR_HEADER = ("Pattern,M,K,N,Density(%),NNZ,xSpMM_Total,xSpMM_Clust,xSpMM_Perm,xSpMM_Conv,"
                 "xSpMM_Math,xSpMM_Unperm,Vendor_CSR,Vendor_BSR,Dense_BLAS,dtype,xSpMM_Plan,"
                 "nnzb_before,nnzb_after")


def vendor_patterns(size, densities):
    """The pattern list of the reference's examples/02_spmm_benchmark.cpp:251-280 (generators of
    xspmm_b200.generators, values U[0.1, 1))."""
    from xspmm_b200 import generators as gen
    yield "Banded_bw16", gen.banded(size, 16)
    yield "Arrowhead_w16", gen.arrowhead(size, 16)
    yield "Checkers_b16", gen.checkers(size, size, 16)
    yield "PowerLaw_a2.5", gen.power_law(size, size, 2.5)
    for d in densities:
        tag = f"{d * 100:g}%"
        yield "UpperTri_" + tag, gen.triangular(size, True, d)
        yield "Hessenberg_" + tag, gen.hessenberg(size, True, d)
        yield "BlockDiag_" + tag, gen.block_diagonal(size, 16, d)
        if size <= 4096:  # sampled per upper-triangle entry on the host
            yield "NearSymm_" + tag, gen.near_symmetric(size, d, 0.1)


def run_vendor_compare(args):
    """xSpMM against the vendor libraries on the reference's benchmark patterns (the columns of
    examples/02_spmm_benchmark.cpp:81, plus dtype, the plan-reusing product and block counts).
    Times in ms: xSpMM stage times from SpMMTimings of one Tier-2 call after warm-up (as the
    reference prints them); vendor and plan times averaged over 10 calls after 3 warm-ups with
    CUDA events (the reference's BenchTimer). Vendor CSR = cuSPARSE SpMM through torch.sparse;
    Vendor BSR = torch's 16x16 BSR product (fp32 only), which torch runs with its own Triton
    block kernel rather than cuSPARSE; dense = cuBLAS
    through torch.matmul (TF32 off, as cublasSgemm). N = M = K, B = ones, as the reference."""
    import torch

    import xspmm_b200 as xs

    torch.backends.cuda.matmul.allow_tf32 = False
    dev = "cuda:0"
    ex = xs.CudaExecutor(0)
    sizes = [int(s) for s in args.vendor_sizes.split(",")]
    dens = [float(d) for d in args.vendor_densities.split(",")]
    dtypes = {"fp32": (np.float32, torch.float32), "fp16": (np.float16, torch.float16)}
    print(VENDOR_HEADER, flush=True)

    def avg_ms(fn, iters=10, warm=3):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    for size in sizes:
        for name, (rp, ci, v) in vendor_patterns(size, dens):
            for dname in args.vendor_dtypes.split(","):
                npt, tdt = dtypes[dname]
                M = K = N = size
                nnz = int(rp[-1])
                rp32, ci32 = rp.astype(np.int32), ci.astype(np.int32)
                vals = v.astype(npt)
                A = xs.CSRMatrix.from_host(ex, M, K, rp32, ci32, vals, index_dtype=torch.int32)
                B = torch.ones((K, N), dtype=tdt, device=dev)
                C = torch.zeros((M, N), dtype=torch.float32, device=dev)
                for _ in range(2):
                    xs.spmm(ex, A, B, C, N, 16, True)
                t = xs.SpMMTimings()
                xs.spmm(ex, A, B, C, N, 16, True, t)
                torch.cuda.synchronize()
                plan = xs.SpMMPlan(ex, A, 16, True)
                plan_ms = avg_ms(lambda: plan.execute(B, C, N))
                after = plan.info()["nnz_blocks"]
                plan.close()
                before = xs.csr_to_bcsr(ex, A, 16, 16).num_blocks
                Acsr = torch.sparse_csr_tensor(torch.as_tensor(rp32, device=dev),
                                               torch.as_tensor(ci32, device=dev),
                                               torch.as_tensor(vals, device=dev), size=(M, K))
                row = {"csr": None, "bsr": None, "dense": None}
                try:
                    row["csr"] = avg_ms(lambda: torch.sparse.mm(Acsr, B))
                except Exception:
                    pass
                if dname == "fp32":
                    try:
                        Absr = Acsr.to_sparse_bsr((16, 16)) if M % 16 == 0 else None
                        if Absr is not None:
                            row["bsr"] = avg_ms(lambda: torch.sparse.mm(Absr, B))
                        del Absr
                    except Exception:
                        pass
                try:
                    Ad = Acsr.to_dense()
                    row["dense"] = avg_ms(lambda: torch.matmul(Ad, B))
                    del Ad
                except Exception:
                    pass
                del Acsr

                def f(x):
                    return "" if x is None else f"{x:.3f}"
                print(",".join([name, str(M), str(K), str(N), f"{100.0 * nnz / (M * K):.4f}",
                                str(nnz), f(t.total_pipeline_ms), f(t.clustering_ms),
                                f(t.permutation_ms), f(t.conversion_ms), f(t.spmm_ms),
                                f(t.unpermutation_ms), f(row["csr"]), f(row["bsr"]),
                                f(row["dense"]), dname, f(plan_ms), str(before), str(after)]),
                      flush=True)
                del A, B, C
                torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["xspmm", "reference"], default="xspmm")
    ap.add_argument("--workload", choices=["cfg5", "cfg4", "cfg2"], default="cfg5",
                    help="cfg5: GNN R-MAT 2^20 (the largest single-GPU config); cfg4: banded 2M")
    ap.add_argument("--n-cols", type=int, default=0, help="N (default: the config's)")
    ap.add_argument("--rows-log2", type=int, default=0,
                    help="cfg4/cfg5 at 2^k rows instead of full size (small profiling cases)")
    ap.add_argument("--tier2-steps", type=int, default=2,
                    help="timed one-call Tier-2 pipelines (rank 0), after one warm-up")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tier1-compare", action="store_true",
                    help="mma.sync vs tcgen05 Tier-1 on the pruned-LLM config, N sweep")
    ap.add_argument("--compare-n", default="16,64,256,1024,4096")
    ap.add_argument("--compare-kernels", default="mma,tc")
    ap.add_argument("--vendor-compare", action="store_true",
                    help="CSV: xSpMM vs cuSPARSE CSR/BSR and cuBLAS on the reference's patterns")
    ap.add_argument("--vendor-sizes", default="1024,4096",
                    help="the reference sweeps 1024,2048,4096,8192")
    ap.add_argument("--vendor-densities", default="0.1,0.01,0.001",
                    help="the reference sweeps 0.7,0.5,0.2,0.1,0.01,0.005,0.001")
    ap.add_argument("--vendor-dtypes", default="fp32,fp16")
    ap.add_argument("--cluster-compare", action="store_true",
                    help="time the clustering call per workload and clustering path")
    ap.add_argument("--cluster-workloads", default="cfg2,cfg4:18,cfg5:18")
    ap.add_argument("--cluster-paths", default="auto")
    args = ap.parse_args()
    if args.cluster_compare:
        run_cluster_compare(args)
        return
    if args.vendor_compare:
        run_vendor_compare(args)
        return
    if args.tier1_compare:
        run_tier1_compare(args)
        return
    if args.warmup < 3 and args.impl == "xspmm":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
