"""Benchmark of the xSpMM hot path on B200 (one JSON line on rank 0).

Workload ("hidden-block recovery"): A is 16384 x 16384 built from dense
16x16 blocks at 0.5 % block density, each block 50 % filled with fp16 N(0,1), rows randomly
permuted; B is 16384 x 256 fp16 N(0,1); C fp32; clustering on. Synthetic, seeded (42).

One step = one Tier-2 pipeline call  xspmm::spmm(exec, A_csr, B, C, N, 16, true)  through the C ABI:
clustering -> row permutation -> CSR->BCSR -> Tier-1 SpMM (unpermute fused). Metric: effective
TFLOPS = 2*nnz*N / step time.

  value : inputs resident in HBM, device time (CUDA events on the launching stream) per step,
          L2 flushed (256 MiB write) before every step, outside the timed interval.
  e2e   : the same call with the CSR arrays and B copied from pinned host memory and C copied back
          inside the timed interval.
  tier1 : the Tier-1 SpMM alone on the clustered BCSR (the amortized, plan-reusing use).
  cpu_baseline / --impl reference : the reference's own host code for clustering, permutation and
          conversion (compiled from its sources, oracle/_ref) plus the oracle's OpenMP fp64 SpMM
          (the reference has no CPU SpMM), on this box's host cores.

Multi-GPU (torchrun, N ranks): weak scaling. Each rank owns one block-row stripe of the global A
(a cfg2-shaped 16384-row stripe, seed 42 + rank); B is broadcast from rank 0 with NCCL once per
distinct B (measured, reported as b_broadcast_ms) and each rank writes its own slice of C. The
step has no collective; the time is the max over ranks.
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

METRIC = "SpMM effective TFLOPS (2*nnz*N/s), Tier-2 pipeline with clustering + conversion"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# DRAM bytes (read + write) of one cluster_kernel launch on the cfg2 workload, from the ncu capture
# summarised in profiles/cluster_kernel_cfg2.md (351 KB read, nothing written back).
CLUSTER_TRAFFIC_BYTES = 350976 + 0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        d["source"] = "measured"
        return d
    d = dict(PEAKS_FALLBACK)
    d["source"] = "fallback"
    return d


def make_problem(rank: int, N: int):
    from xspmm_b200 import synth
    return synth.cfg2_hidden_block(seed=42 + rank, N=N)


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
# CPU baseline: the reference's host code + the oracle SpMM
# ------------------------------------------------------------------------------------------------
def cpu_pipeline_once(P):
    import oracle
    t0 = time.perf_counter()
    if oracle.ref_available():
        perm = oracle.ref_cluster(P.row_ptr, P.col_ind, P.M, P.K, 0.5, 16)
        t1 = time.perf_counter()
        prp, pci, pv = oracle.ref_permute(P.row_ptr, P.col_ind, P.values, perm, P.K)
        t2 = time.perf_counter()
        brp, bci, bv = oracle.ref_csr_to_bcsr(prp, pci, pv, P.M, P.K)
        kind = "reference"
    else:
        perm = oracle.cluster_literal(P.row_ptr, P.col_ind, P.M, P.K, 0.5, 16)
        t1 = time.perf_counter()
        prp, pci, pv = oracle.permute_rows(P.row_ptr, P.col_ind, P.values.astype(np.float32), perm)
        t2 = time.perf_counter()
        brp, bci, bv = oracle.csr_to_bcsr(prp, pci, pv, P.M, P.K)
        kind = "port"
    t3 = time.perf_counter()
    Cp = oracle.bcsr_spmm_f64(P.M, P.K, P.N, brp, bci, bv, P.B.astype(np.float32))
    C = oracle.unpermute_dense(Cp, perm)
    t4 = time.perf_counter()
    return kind, {"clustering_s": t1 - t0, "permutation_s": t2 - t1, "conversion_s": t3 - t2,
                  "spmm_unpermute_s": t4 - t3, "total_s": t4 - t0}, C


def cpu_baseline(P, budget_s=12.0, min_runs=1, max_runs=50):
    import oracle
    runs = []
    kind = None
    t_start = time.perf_counter()
    while len(runs) < max_runs and (len(runs) < min_runs or time.perf_counter() - t_start < budget_s):
        kind, t, _ = cpu_pipeline_once(P)
        runs.append(t)
    mean = {k: sum(r[k] for r in runs) / len(runs) for k in runs[0]}
    flops = 2.0 * P.nnz * P.N
    return {
        "value": flops / mean["total_s"] / 1e12,
        "unit": "TFLOPS",
        "cores": oracle.num_threads(),
        "kind": kind,
        "sample": (f"full {P.name} workload x{len(runs)} runs ({time.perf_counter() - t_start:.1f} s); "
                   "clustering/permutation/conversion = reference host code (1 thread), "
                   f"SpMM+unpermute = oracle fp64 restatement ({oracle.num_threads()} OpenMP threads)"),
        "stage_ms": {k[:-2] + "_ms": round(v * 1e3, 3) for k, v in mean.items()},
        "cpu_model": _cpu_model(),
        "nproc": os.cpu_count(),
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
    import torch
    import torch.distributed as dist

    import xspmm_b200 as xs
    from xspmm_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    N = args.n_cols
    P = make_problem(rank, N)
    stream = torch.cuda.current_stream(dev)
    ex = xs.CudaExecutor(local)
    A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    # B: rank 0's matrix, broadcast to every rank (once per distinct B)
    B = torch.as_tensor(make_problem(0, N).B if rank == 0 else np.zeros((P.K, N), np.float16)).to(dev)
    b_bcast_ms = None
    if world > 1:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dist.broadcast(B, src=0)
        e1.record(stream)
        torch.cuda.synchronize()
        b_bcast_ms = e0.elapsed_time(e1)
    C = torch.empty((P.M, N), dtype=torch.float32, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flops = 2.0 * P.nnz * N

    def step(timings=None):
        xs.spmm(ex, A, B, C, N, 16, True, timings)

    # warm-up
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timed region ----
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stage = {k: 0.0 for k in ("clustering_ms", "permutation_ms", "conversion_ms", "spmm_ms",
                              "unpermutation_ms", "total_pipeline_ms")}
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ex.reset_launch_count()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.fill_(float(i))
        starts[i].record(stream)
        t = xs.SpMMTimings()
        step(t)
        ends[i].record(stream)
        for k in stage:
            stage[k] += getattr(t, k)
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    launches = ex.launch_count()
    clocks = sampler.stop()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = sum(step_ms) / len(step_ms)
    stage = {k: v / args.steps for k, v in stage.items()}

    # reference result check on rank 0 happens in the tests; here a cheap finite check
    assert torch.isfinite(C).all().item()

    # ---- Tier-1 alone on a plan (clustering + BCSR built once, the amortized use) ----
    plan = xs.SpMMPlan(ex, A, 16, True)
    for _ in range(args.warmup):
        plan.execute(B, C, N)
    torch.cuda.synchronize()
    t1s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t1e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(float(i))
        t1s[i].record(stream)
        plan.execute(B, C, N)
        t1e[i].record(stream)
    torch.cuda.synchronize()
    t1_ms = sum(s.elapsed_time(e) for s, e in zip(t1s, t1e)) / args.steps
    plan_info = plan.info()
    plan.close()
    nnzb = plan_info["nnz_blocks"]
    nnzb_before = xs.csr_to_bcsr(ex, A, 16, 16).num_blocks

    # ---- e2e through the same call with host buffers ----
    h_rp = torch.from_numpy(P.row_ptr.astype(np.int32)).pin_memory()
    h_ci = torch.from_numpy(P.col_ind.astype(np.int32)).pin_memory()
    h_v = torch.from_numpy(P.values).pin_memory()
    h_B = B.cpu().pin_memory()
    h_C = torch.empty((P.M, N), dtype=torch.float32).pin_memory()
    Ae = xs.CSRMatrix(ex, P.M, P.K, P.nnz, torch.float16, torch.int32)
    Be = torch.empty_like(B)
    bi = (h_rp.numel() * 4 + h_ci.numel() * 4 + h_v.numel() * 2 + h_B.numel() * 2)
    bo = h_C.numel() * 4

    def e2e_step():
        Ae.row_ptr.copy_(h_rp, non_blocking=True)
        Ae.col_ind.copy_(h_ci, non_blocking=True)
        Ae.values.copy_(h_v, non_blocking=True)
        Be.copy_(h_B, non_blocking=True)
        xs.spmm(ex, Ae, Be, C, N, 16, True, None)
        h_C.copy_(C, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    es = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ee = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(float(i))
        es[i].record(stream)
        e2e_step()
        ee[i].record(stream)
        ee[i].synchronize()
    e2e_ms = sum(s.elapsed_time(e) for s, e in zip(es, ee)) / args.steps

    # ---- max over ranks ----
    def rmax(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def rsum(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    ms_max = rmax(ms)
    e2e_max = rmax(e2e_ms)
    t1_max = rmax(t1_ms)
    flops_all = rsum(flops)
    padded_all = rsum(2.0 * nnzb * 256 * N)
    launches_max = int(rmax(float(launches)))
    nnz_all = int(rsum(float(P.nnz)))

    pk = peaks()
    # per-stage algorithmic bytes (int32 indices, fp16 values, fp32 C)
    idx = 4
    M, K = P.M, P.K
    bytes_stage = {
        "clustering_ms": (M + 1) * idx + P.nnz * idx + M * idx,
        "permutation_ms": 2 * ((M + 1) * idx + P.nnz * (idx + 2)) + M * idx,
        "conversion_ms": (M + 1) * idx + P.nnz * (idx + 2) + (M // 16 + 1) * idx + nnzb * (idx + 512),
        "spmm_ms": nnzb * (idx + 512) + (M // 16 + 1) * idx + M * idx + K * N * 2 + M * N * 4,
    }
    stages = {}
    for k, b in bytes_stage.items():
        t = stage[k]
        stages[k.replace("_ms", "")] = {"ms": round(t, 4),
                                         "alg_bytes": int(b),
                                         "achieved_gbs": round(b / (t * 1e-3) / 1e9, 2) if t > 0 else None}
    dom = max(bytes_stage, key=lambda k: stage[k])
    dom_t = stage[dom]
    achieved = bytes_stage[dom] / (dom_t * 1e-3) / 1e9
    roofline = {"kernel": {"clustering_ms": "cluster_greedy (+ pattern/index build)",
                           "permutation_ms": "permute_lengths/scan/copy",
                           "conversion_ms": "bcsr_count/scan/fill",
                           "spmm_ms": "bcsr_spmm_f16_mma"}[dom],
                "bound": "hbm", "achieved": round(achieved, 2),
                "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 5),
                "traffic": CLUSTER_TRAFFIC_BYTES if dom == "clustering_ms" else None,
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                   "cluster_kernel launch on this workload "
                                   "(profiles/cluster_kernel_cfg2.md)") if dom == "clustering_ms" else None,
                "peak_source": pk["source"],
                "note": "dominant stage of the timed step; achieved = algorithmic bytes / stage time; "
                        "latency-bound (one CTA, serial across clusters), so the fraction is small "
                        "by construction"}
    t1_bytes = bytes_stage["spmm_ms"]
    tier1 = {
        "ms": round(t1_max, 4),
        "effective_tflops": round(flops_all / (t1_max * 1e-3) / 1e12, 3),
        "padded_tflops": round(padded_all / (t1_max * 1e-3) / 1e12, 3),
        "padded_frac_of_bf16_peak": round(padded_all / (t1_max * 1e-3) / 1e12 / pk["bf16_tflops"], 5),
        "hbm_gbs": round(t1_bytes / (t1_ms * 1e-3) / 1e9, 2),
        "hbm_frac": round(t1_bytes / (t1_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        "kernel": ("bcsr_spmm_tc (tcgen05/TMEM)" if plan_info["tcgen05_ready"]
                   else "bcsr_spmm_f16_mma (mma.sync m16n8k16)"),
        "timing": "SpMMPlan built once (clustering, permutation, BCSR); execute timed",
    }

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    out = {
        "metric": METRIC,
        "value": round(flops_all / (ms_max * 1e-3) / 1e12, 5),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded generator of the hidden-block config; no dataset)",
        "config": {"workload": "cfg2_hidden_block", "M": P.M, "K": P.K, "N": N,
                   "nnz_per_rank": P.nnz, "nnz_total": nnz_all,
                   "nnzb_before_clustering": nnzb_before, "nnzb_after_clustering": nnzb,
                   "block_density": 0.005, "block_fill": 0.5, "clustering": True,
                   "hw_block": 16, "accumulate": "fp32", "index": "int32",
                   "parallelism": f"block-row stripes, {world} rank(s), B broadcast once",
                   "l2": "flushed before every step (256 MiB write, outside the timed interval)",
                   "seed": 42},
        "pipeline_ms": {k: round(v, 4) for k, v in stage.items()},
        "clustering_plus_conversion_ms": round(stage["clustering_ms"] + stage["conversion_ms"], 4),
        "stages": stages,
        "tier1": tier1,
        "roofline": roofline,
        "e2e": {"value": round(flops_all / (e2e_max * 1e-3) / 1e12, 5), "unit": "TFLOPS",
                "ms_per_step": round(e2e_max, 4), "h2d_bytes_per_step": int(bi),
                "d2h_bytes_per_step": int(bo)},
        "gpu_launches": launches_max,
        "wall_s_timed_region": round(wall, 4),
        "clocks": clocks,
    }
    if b_bcast_ms is not None:
        out["b_broadcast_ms"] = round(b_bcast_ms, 4)
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(P, budget_s=args.cpu_budget)
    print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    P = make_problem(0, args.n_cols)
    for _ in range(args.warmup):
        cpu_pipeline_once(P)
    times = []
    kind = None
    for _ in range(args.steps):
        kind, t, _ = cpu_pipeline_once(P)
        times.append(t)
    mean = {k: sum(r[k] for r in times) / len(times) for k in times[0]}
    import oracle
    flops = 2.0 * P.nnz * P.N
    val = flops / mean["total_s"] / 1e12
    out = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(val, 6),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(mean["total_s"] * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (reference CPU path; fp16 inputs widened exactly)",
        "data": "synthetic (seeded generator of the hidden-block config; no dataset)",
        "config": {"workload": "cfg2_hidden_block", "M": P.M, "K": P.K, "N": P.N, "nnz": P.nnz,
                   "clustering": True, "hw_block": 16, "seed": 42},
        "cpu_baseline": {"value": round(val, 6), "unit": "TFLOPS", "cores": oracle.num_threads(),
                         "kind": kind,
                         "sample": ("full workload per step; clustering/permutation/conversion = "
                                    "reference host code (1 thread), SpMM+unpermute = oracle fp64 "
                                    "restatement (OpenMP) since the reference has no CPU SpMM"),
                         "stage_ms": {k[:-2] + "_ms": round(v * 1e3, 3) for k, v in mean.items()},
                         "cpu_model": _cpu_model(), "nproc": os.cpu_count()},
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


def run_sharded(args):
    """One matrix (cfg4 banded or cfg5 R-MAT at full size) split by block rows over the ranks
    (balanced by nonzero blocks), B broadcast once over NCCL, then the steady-state Tier-1 product
    timed on every rank (max over ranks). Clustering runs once on rank 0 and its permutation is
    broadcast. Strong scaling: the total work is fixed. One JSON line from rank 0."""
    import datetime

    import torch
    import torch.distributed as dist

    import xspmm_b200 as xs
    from xspmm_b200 import synth
    from xspmm_b200.shard import BlockRowShard, broadcast_b, partition_block_rows

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def ev():
        return torch.cuda.Event(enable_timing=True)

    if args.sharded == "cfg4":
        P, N, label = synth.cfg4_banded(N=64), 64, "cfg4_banded_2M"
    else:
        P, N, label = synth.cfg5_rmat(N=128), 128, "cfg5_rmat_2^20"
    ex = xs.CudaExecutor(local)
    A = xs.CSRMatrix.from_host(ex, P.M, P.K, P.row_ptr, P.col_ind, P.values,
                               index_dtype=torch.int32)
    stream = torch.cuda.current_stream(dev)
    # clustering once (rank 0), permutation broadcast
    perm = torch.empty(P.M, dtype=torch.int32, device=dev)
    c0, c1 = ev(), ev()
    barrier()
    c0.record(stream)
    if rank == 0:
        xs.compute_1d_jaccard_clustering(ex, A, 0.5, 16, perm)
    c1.record(stream)
    if world > 1:
        dist.broadcast(perm, src=0)
    torch.cuda.synchronize()
    cluster_ms = c0.elapsed_time(c1)
    v0, v1 = ev(), ev()
    v0.record(stream)
    Ap = xs.apply_permutation(ex, A, perm)
    Ab = xs.csr_to_bcsr(ex, Ap, 16, 16)
    v1.record(stream)
    torch.cuda.synchronize()
    convert_ms = v0.elapsed_time(v1)
    del Ap
    nnzb_before = xs.csr_to_bcsr(ex, A, 16, 16).num_blocks
    row_ptr_host = Ab.row_ptr.cpu().numpy()
    B_full = torch.as_tensor(P.B).to(dev) if rank == 0 else None
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    sizes = [g for g in (1, 2, 4, 8, 16) if g <= world] if args.scaling_sweep else [world]
    for g in sizes:
        # ranks [0, g) form the group; the others wait at the barrier below
        group = dist.new_group(ranks=list(range(g))) if world > 1 and g > 1 else None
        if rank < g:
            bounds = partition_block_rows(row_ptr_host, g)
            shard = BlockRowShard(Ab, int(bounds[rank]), int(bounds[rank + 1]))
            B = B_full.clone() if rank == 0 else torch.zeros(P.B.shape, dtype=torch.float16,
                                                              device=dev)
            if g > 1:  # the group's communicator is set up by its first collective: not timed
                warm = torch.zeros(1, device=dev)
                dist.all_reduce(warm, group=group)
                dist.barrier(group=group)
                torch.cuda.synchronize()
            b0, b1 = ev(), ev()
            b0.record(stream)
            if g > 1:
                broadcast_b(B, src=0, group=group)
            b1.record(stream)
            torch.cuda.synchronize()
            bcast_ms = b0.elapsed_time(b1)
            C = torch.empty((shard.num_rows, N), dtype=torch.float32, device=dev)
            for _ in range(args.warmup):
                shard.execute(B, C, N)
            torch.cuda.synchronize()
            starts = [ev() for _ in range(args.steps)]
            ends = [ev() for _ in range(args.steps)]
            sampler = ClockSampler(local)
            sampler.start()
            time.sleep(0.3)
            if g > 1:
                dist.barrier(group=group)
            torch.cuda.synchronize()
            for i in range(args.steps):
                flush.fill_(float(i))
                starts[i].record(stream)
                shard.execute(B, C, N)
                ends[i].record(stream)
            torch.cuda.synchronize()
            if g > 1:
                dist.barrier(group=group)
            clocks = sampler.stop()
            ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
            assert torch.isfinite(C).all().item()
            ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
            blocks_t = torch.tensor([shard.nnz_blocks], dtype=torch.float64, device=dev)
            if g > 1:
                dist.all_reduce(ms_t, op=dist.ReduceOp.MAX, group=group)
                all_blocks = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(g)]
                dist.all_gather(all_blocks, blocks_t, group=group)
                per_rank_blocks = [int(x.item()) for x in all_blocks]
            else:
                per_rank_blocks = [shard.nnz_blocks]
            shard.close()
            del C, B
            if rank == 0:
                t = ms_t.item()
                pk = peaks()
                eff = 2.0 * P.nnz * N / (t * 1e-3) / 1e12
                padded = 2.0 * Ab.num_blocks * 256 * N / (t * 1e-3) / 1e12
                alg_bytes = (Ab.num_blocks * (512 + 4) + (Ab.num_block_rows + 1) * 4 +
                             P.K * N * 2 + P.M * N * 4)
                print(json.dumps({
                    "metric": "SpMM effective TFLOPS (2*nnz*N/s), Tier-1 block-row sharded, "
                              "B resident",
                    "value": round(eff, 4), "unit": "TFLOPS", "n_gpus": g, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": round(t, 4), "higher_is_better": True,
                    "scaling": "strong", "dtype": "f16", "data": "synthetic (seeded generator)",
                    "config": {"workload": label, "M": P.M, "K": P.K, "N": N, "nnz": P.nnz,
                               "nnzb_before_clustering": nnzb_before, "nnzb": Ab.num_blocks,
                               "partition": "block rows balanced by nonzero blocks",
                               "per_rank_blocks": per_rank_blocks,
                               "l2": "flushed before every step (256 MiB write)"},
                    "padded_tflops": round(padded, 3),
                    "padded_frac_of_bf16_peak": round(padded / pk["bf16_tflops"], 5),
                    "hbm_frac_whole_job": round(alg_bytes / (t * 1e-3) / 1e9 / (pk["hbm_gbs"] * g), 4),
                    "b_broadcast_ms": round(bcast_ms, 4), "clustering_ms": round(cluster_ms, 2),
                    "conversion_ms": round(convert_ms, 3), "clocks": clocks,
                }), flush=True)
        if world > 1:
            dist.barrier()
    if world > 1:
        dist.destroy_process_group()


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
    ap.add_argument("--n-cols", type=int, default=256)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tier1-compare", action="store_true",
                    help="mma.sync vs tcgen05 Tier-1 on the pruned-LLM config, N sweep")
    ap.add_argument("--compare-n", default="16,64,256,1024,4096")
    ap.add_argument("--compare-kernels", default="mma,tc")
    ap.add_argument("--sharded", choices=["cfg4", "cfg5"],
                    help="one full-size matrix split by block rows over the ranks (Tier-1)")
    ap.add_argument("--scaling-sweep", action="store_true",
                    help="with --sharded: also time the first 1, 2, 4, ... ranks of the launch")
    ap.add_argument("--vendor-compare", action="store_true",
                    help="CSV: xSpMM vs cuSPARSE CSR/BSR and cuBLAS on the reference's patterns")
    ap.add_argument("--vendor-sizes", default="1024,4096",
                    help="the reference sweeps 1024,2048,4096,8192")
    ap.add_argument("--vendor-densities", default="0.1,0.01,0.001",
                    help="the reference sweeps 0.7,0.5,0.2,0.1,0.01,0.005,0.001")
    ap.add_argument("--vendor-dtypes", default="fp32,fp16")
    args = ap.parse_args()
    if args.vendor_compare:
        run_vendor_compare(args)
        return
    if args.tier1_compare:
        run_tier1_compare(args)
        return
    if args.sharded:
        if args.warmup < 3:
            args.warmup = 3
        run_sharded(args)
        return
    if args.warmup < 3 and args.impl == "xspmm":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
