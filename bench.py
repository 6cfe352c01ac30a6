#!/usr/bin/env python
"""MARS B200 benchmark: exact retrieval top-K (cosine x decay x importance).

Workload (the headline metric: queries/s + p99 at N=1M, D=768, K=10, HBM GB/s
vs peak):
  * corpus N = 1,000,000 rows x D = 768 fp32, i.i.d. Gaussian rows divided by
    (||v|| + 1e-8), timestamps U[0, 600] s, importance U[0, 1], 4 modalities;
    seeded synthetic data (no dataset is involved);
  * a step is 16 concurrent queries, each the exact top-K = 10 of
    dot x exp(-lambda * age) x importance over all N rows, lambda = 0.01,
    answered by mars_query_batch_topk (an fp16 tensor-core short list with a
    proven error margin, then an exact fp32 rescore: the results are those of
    the fp32 fused scan bit for bit, which the run checks);
  * N GPUs (`--shard replicas`, the default): the 1M-row corpus (4.6 GB with
    its fp16 copy) fits every GPU, so every GPU holds it and answers its own
    16 queries per step, with no data-path collective (weak scaling: 16 N
    queries per step).  `--shard rows`: the corpus is row-sharded (strong
    scaling), every GPU answers the same queries on its shard, and the
    per-query local top-K lists are all-gathered over NCCL and merged on
    every GPU.

`value` is queries/s with queries and corpus resident in HBM, timed with CUDA
events on the query stream (max over ranks).  `e2e` goes through the public
API with host buffers: queries copied host->device and results device->host
inside the timed region.  `latency_us` is the single-query p50/p99 of
mars_query (host in, host out).  `fused_scan` reports the fp32 fused scan
kernel, one query per launch, against the HBM roofline.  `--impl reference`
times the CPU implementation of the same path (the oracle port) on the host
cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "cuda-multimodal-memory_b200"), os.path.join(ROOT, "oracle"),
           os.path.join(ROOT, "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np

FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mars", "reference"], default="mars")
    ap.add_argument("--n", type=int, default=1_000_000)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--queries-per-step", type=int, default=16)
    ap.add_argument("--lam", type=float, default=0.01)
    ap.add_argument("--ts-max", type=float, default=600.0)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=10.0)
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--queries", type=int, default=10000)
    ap.add_argument("--shard", choices=["replicas", "rows"], default="replicas",
                    help="headline on several GPUs: replicas (every GPU holds the whole corpus and answers "
                         "its own queries; weak scaling) or rows (the corpus row-sharded, every GPU answers "
                         "the same queries on its shard, NCCL all-gather + merge; strong scaling)")
    ap.add_argument("--workload", choices=["scan", "c0", "c1", "c2", "c3", "c4"], default="scan",
                    help="scan: the headline (default); c0: single-query latency at N=2400 "
                         "with BFS depth 1; c1: streaming loop (append 10 rows + query per frame)")
    ap.add_argument("--frames", type=int, default=10000)
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def metric_name(a):
    return (f"queries/s (exact top-K of cosine*exp(-lambda*age)*importance over all rows, "
            f"N={a.n}, D={a.dim}, K={a.k})")


def config_dict(a, world):
    rows = world > 1 and a.shard == "rows"
    per_gpu = a.n // world if rows else a.n
    return {
        "workload": f"retrieval N={a.n} D={a.dim} K={a.k}: {a.queries_per_step} concurrent queries "
                    f"per step, each the exact top-K over all rows (mars_query_batch_topk: "
                    f"fp16 tensor-core short list + exact fp32 rescore; results bit-identical "
                    f"to the fp32 fused scan)",
        "n_rows": a.n, "dim": a.dim, "top_k": a.k, "queries_per_step": a.queries_per_step,
        "lambda": a.lam, "importance": True, "gpus": world,
        "parallelism": (f"row-shard x{world} + NCCL all-gather + merge" if rows else
                        (f"replicas x{world}: every GPU holds all {a.n} rows and answers its own "
                         f"{a.queries_per_step} queries per step, no data-path collective" if world > 1
                         else "one GPU")),
        "l2": "inputs larger than L2: each step streams the fp16 rows, "
              f"{per_gpu * ((a.dim + 7) // 8 * 16 + 8) / 1e9:.3f} GB per GPU (L2 126 MB)",
    }


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic():
    """dram bytes per candidates-pass launch from the committed ncu summary (or None)."""
    p = os.path.join(ROOT, "profiles", "batch_gemm_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return None


# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names[1:], parts[5:9]):
                if v.lower() in ("active", "0x1", "1", "yes"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
def run_reference(a):
    """CPU implementation of the same path (oracle port), rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle as O
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_rows(0, a.n, a.dim, seed=a.seed, ts_max=a.ts_max)
    c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    Q = datagen.queries(64, a.dim, seed=a.seed + 1)
    threads = os.cpu_count() or 1
    for w in range(a.warmup):
        O.scan_topk_fast(c, Q[w % 64], a.ts_max, a.lam, a.k, use_importance=True, n_threads=threads)
    t0 = time.perf_counter()
    for s in range(a.steps):
        O.scan_topk_fast(c, Q[s % 64], a.ts_max, a.lam, a.k, use_importance=True, n_threads=threads)
    dt = time.perf_counter() - t0
    v = a.steps / dt
    line = {
        "impl": "reference", "metric": metric_name(a), "value": v, "unit": "queries/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": dt / a.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian corpus)", "config": config_dict(a, 1),
        "cpu_baseline": {"value": v, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"each step = 1 query scanned over all {a.n} rows "
                                   f"(oracle/mars_oracle.c orc_scan_topk_fast, {threads} threads)"},
        "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def cpu_baseline(a, E, mod, ts, imp, Qh):
    import oracle as O
    c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    O.scan_topk_fast(c, Qh[0], a.ts_max, a.lam, a.k, use_importance=True, n_threads=threads)
    t1 = time.perf_counter() - t0
    n = int(max(2, min(32, math.ceil(a.cpu_budget_s / max(t1, 1e-3)))))
    answers = []
    t0 = time.perf_counter()
    for i in range(n):
        answers.append(O.scan_topk_fast(c, Qh[i % Qh.shape[0]], a.ts_max, a.lam, a.k, use_importance=True,
                                        n_threads=threads))
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{n} queries, each scanning all {a.n} rows (same corpus, same K/lambda), "
                      f"oracle/mars_oracle.c orc_scan_topk_fast with {threads} OpenMP threads"}, answers


def compare_with_oracle(gpu_ids, gpu_vals, answers):
    """Tie-aware comparison of the GPU answers of queries 0.. with the oracle's
    (ids identical wherever scores are separated by more than 1e-5 relative)."""
    from _util import assert_ranked_equivalent
    try:
        for i, (oi, ov) in enumerate(answers):
            assert_ranked_equivalent(gpu_ids[i], gpu_vals[i], oi, ov, what=f"query {i}")
        return True
    except AssertionError:
        return False


def run_mars(a):
    import torch
    import mars_b200 as mb
    from mars_b200 import datagen

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        from datetime import timedelta
        dist = dist_mod
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    # rows: shard r holds rows [r N / G, (r + 1) N / G) and answers every
    # query; replicas: every rank holds all rows and answers its own queries
    sharded = world > 1 and a.shard == "rows"
    lo, hi = (a.n * rank // world, a.n * (rank + 1) // world) if sharded else (0, a.n)
    n_local = hi - lo
    E, mod, ts, imp = datagen.gaussian_rows(lo, hi, a.dim, seed=a.seed, ts_max=a.ts_max)
    Qh = datagen.queries(64, a.dim, seed=a.seed + 1 + (0 if sharded else 1000 * rank))
    store = mb.Store(n_local, a.dim, device=local)
    store.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(n_local, a.dim, max_k=a.k, device=local)
    K, Q = a.k, a.queries_per_step
    bc = mb.BatchContext(n_local, a.dim, max_batch=Q, max_k=K, device=local)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))
    torch.cuda.set_stream(stream)
    Qd = torch.from_numpy(Qh).cuda()
    ids = torch.empty((Q, K), dtype=torch.int32, device="cuda")
    vals = torch.empty((Q, K), dtype=torch.float32, device="cuda")
    if sharded:
        gids = torch.empty((world, Q, K), dtype=torch.int32, device="cuda")
        gvals = torch.empty((world, Q, K), dtype=torch.float32, device="cuda")
        mids = torch.empty((Q, K), dtype=torch.int32, device="cuda")
        mvals = torch.empty((Q, K), dtype=torch.float32, device="cuda")
    n_ev = a.steps + a.warmup
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]

    def batch(q, out_ids, out_vals):
        bc.query_batch_topk(store, q, Q, a.ts_max, a.lam, K, out_ids, out_vals, use_importance=True,
                            row_offset=lo, stream=ctx.stream)

    def step(i):
        # one step: Q concurrent queries, each the exact top-K of the fused
        # score over every row of the shard (mars_query_batch_topk: fp16
        # tensor-core short list, exact fp32 rescore)
        base = (i * Q) % (Qd.shape[0] - Q + 1)
        ev_a[i].record(stream)
        batch(Qd[base:base + Q], ids, vals)
        if sharded:
            dist.all_gather_into_tensor(gids, ids)
            dist.all_gather_into_tensor(gvals, vals)
            ctx.topk_merge_batch(gids, gvals, world, K, Q, mids, mvals, stream=ctx.stream)
        ev_b[i].record(stream)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for w in range(a.warmup):
        step(a.steps + w)
    barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    barrier()
    t_start.record(stream)
    for s in range(a.steps):
        step(s)
    t_end.record(stream)
    barrier()
    clocks = sampler.stop() if sampler else None
    elapsed_ms = t_start.elapsed_time(t_end)
    step_ms = [ev_a[i].elapsed_time(ev_b[i]) for i in range(a.steps)]
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())

    # ---- outside the timed region ------------------------------------------
    # the dominant kernel (the candidates pass) timed by the library's CUDA
    # events on the call's stream
    gemm_ms, bstats = [], None
    for j in range(10):
        batch(Qd[:Q], ids, vals)
        bstats = bc.last_stats()
        gemm_ms.append(bstats["gemm_ms"])
    # exactness: the step's answers against the fp32 fused scan, bit for bit
    ref_ids = torch.empty_like(ids)
    ref_vals = torch.empty_like(vals)
    exact = True
    for base in (0, 16, 48):
        q = Qd[base:base + Q]
        batch(q, ids, vals)
        ctx.scan_topk_multi(store, q, Q, a.ts_max, a.lam, K, ref_ids, ref_vals, use_importance=True,
                            row_offset=lo, stream=ctx.stream)
        torch.cuda.synchronize()
        exact = exact and torch.equal(ids, ref_ids) and torch.equal(vals.view(torch.int32),
                                                                    ref_vals.view(torch.int32))
    if world > 1:
        t = torch.tensor([1 if exact else 0], dtype=torch.int32, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        exact = bool(t.item())
    # the step's answers for queries 0..31 (two steps), compared with the
    # oracle's answers on the same queries (computed by the CPU baseline)
    ans_ids, ans_vals = [], []
    for base in (0, Q):
        batch(Qd[base:base + Q], ids, vals)
        torch.cuda.synchronize()
        ans_ids.append(ids.cpu().numpy().copy())
        ans_vals.append(vals.cpu().numpy().copy())
    ans_ids, ans_vals = np.concatenate(ans_ids), np.concatenate(ans_vals)

    # the fused scan: one query per launch (the HBM-bound kernel), the
    # multi-query launch of the step's queries, and its fp16-filtered form
    def timed(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        out = []
        for _ in range(reps):
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            out.append(e0.elapsed_time(e1))
        return out
    scan_ms = timed(lambda: ctx.scan_topk(store, Qd[0], a.ts_max, a.lam, K, ids[0], vals[0],
                                          use_importance=True, row_offset=lo, stream=ctx.stream), 64)
    multi_ms = timed(lambda: ctx.scan_topk_multi(store, Qd[:Q], Q, a.ts_max, a.lam, K, ids, vals,
                                                 use_importance=True, row_offset=lo, stream=ctx.stream), 8)
    f16_ms = timed(lambda: ctx.scan_topk_f16(store, Qd[:Q], Q, a.ts_max, a.lam, K, ids, vals,
                                             use_importance=True, row_offset=lo, stream=ctx.stream), 8)

    # ---- end to end through the public API with host buffers --------------
    # A serving loop: every step copies its queries host -> device, answers
    # them and copies the ids and scores device -> host into one of two pinned
    # buffers; the host then waits for the previous step's results and reads
    # them, so the GPU is not idle while the host issues the next step.  The
    # device buffers are reused in stream order.
    Qpin = torch.from_numpy(Qh).pin_memory()
    qbuf = torch.empty((Q, a.dim), dtype=torch.float32, device="cuda")
    out_ids = [torch.empty((Q, K), dtype=torch.int32).pin_memory() for _ in range(2)]
    out_vals = [torch.empty((Q, K), dtype=torch.float32).pin_memory() for _ in range(2)]
    out_cnt = [torch.empty(Q, dtype=torch.int32).pin_memory() for _ in range(2)]
    cnt = torch.empty(Q, dtype=torch.int32, device="cuda")
    mcnt = torch.empty(Q, dtype=torch.int32, device="cuda")
    done = [torch.cuda.Event() for _ in range(2)]
    res_ids, res_vals = (mids, mvals) if sharded else (ids, vals)
    checksum = 0
    e2e_valid = True
    barrier()
    t0 = time.perf_counter()
    for s in range(a.steps + 1):
        if s < a.steps:
            b = s % 2
            base = (s * Q) % (64 - Q + 1)
            qbuf.copy_(Qpin[base:base + Q], non_blocking=True)
            bc.query_batch_topk(store, qbuf, Q, a.ts_max, a.lam, K, ids, vals, cnt, use_importance=True,
                                row_offset=lo, stream=ctx.stream)
            if sharded:
                dist.all_gather_into_tensor(gids, ids)
                dist.all_gather_into_tensor(gvals, vals)
                ctx.topk_merge_batch(gids, gvals, world, K, Q, mids, mvals, mcnt, stream=ctx.stream)
            out_ids[b].copy_(res_ids, non_blocking=True)
            out_vals[b].copy_(res_vals, non_blocking=True)
            out_cnt[b].copy_(mcnt if sharded else cnt, non_blocking=True)
            done[b].record(stream)
        if s > 0:   # the previous step's results, read and checked on the host
            p = (s - 1) % 2
            done[p].synchronize()
            e2e_valid = e2e_valid and bool((out_cnt[p] == K).all())
            checksum += int(out_ids[p][0, 0])
    dt = time.perf_counter() - t0
    bc.last_stats()      # raises if the last step's pipeline reported an error
    if world > 1:
        t = torch.tensor([dt], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    q_all = Q * (1 if sharded else world)   # queries answered per step by the whole job
    e2e = {"value": a.steps * q_all / dt, "unit": "queries/s",
           "h2d_bytes_per_step": Q * a.dim * 4, "d2h_bytes_per_step": Q * K * 8 + Q * 4,
           "every_step_valid": e2e_valid,
           "path": "pinned H2D of the step's queries, mars_query_batch_topk"
                   + (" per shard, NCCL all-gather, mars_topk_merge_batch" if sharded else
                      (" on every replica" if world > 1 else ""))
                   + ", D2H of the top-K ids, scores and counts into one of two pinned buffers; the host "
                     "waits for and reads each step's results (checking every count) while the next step "
                     "runs"}
    latency = None
    if world == 1:
        # single-query latency through mars_query (host query in, host results out)
        cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=0, time_decay_lambda=a.lam, use_importance=True)
        for i in range(3):
            ctx.query(store, Qh[i], a.ts_max, cfg)
        lat = []
        for j in range(256):
            c0 = time.perf_counter()
            ctx.query(store, Qh[j % 64], a.ts_max, cfg)
            lat.append(time.perf_counter() - c0)
        latency = {"path": "mars_query (C ABI), one query, host in / host out, N=%d" % n_local,
                   "p50_us": float(np.percentile(lat, 50) * 1e6),
                   "p99_us": float(np.percentile(lat, 99) * 1e6)}

    if rank == 0:
        peak, peak_kind = measured_peak()
        pitch16 = (a.dim + 7) // 8 * 8
        # small batches (path 3) read each row once; the 128-query tiles once
        # per query tile; rows carry a timestamp and an importance (4 + 4 B)
        small = bool(bstats and bstats.get("path") == 3)
        qtiles = 1 if small else (Q + 127) // 128
        gemm_bytes = qtiles * n_local * (pitch16 * 2 + 8)
        # the fused pass also streams its sampled 128-row tiles a second time:
        # reported apart, not counted as algorithmic bytes
        overhead_bytes = bstats.get("sample_tiles", 0) * 128 * (pitch16 * 2 + 8) if small else 0
        mean_gemm = statistics.mean(gemm_ms)
        achieved = gemm_bytes / (mean_gemm * 1e-3) / 1e9
        tr = committed_traffic()
        traffic = None
        if tr and tr.get("n_rows") and tr.get("dram_bytes"):
            traffic = tr["dram_bytes"] * n_local / tr["n_rows"]
        scan_bytes = n_local * (a.dim * 4 + 4 + 4)
        scan_med = float(np.median(scan_ms))
        qps = a.steps * q_all / (elapsed_ms * 1e-3)
        line = {
            "metric": metric_name(a), "value": qps, "unit": "queries/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": elapsed_ms / a.steps,
            "higher_is_better": True, "scaling": "strong" if sharded or world == 1 else "weak",
            "vs_baseline": None,
            "dtype": "f32 results (exact; fp16 tensor-core short list, fp32 rescore)",
            "data": "synthetic (seeded Gaussian corpus and queries)",
            "config": config_dict(a, world),
            "exact_vs_fp32_scan": exact,
            "latency_us": latency,
            "step_ms_p50": float(np.percentile(step_ms, 50)),
            "step_ms_p99": float(np.percentile(step_ms, 99)),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": ("batch::gemm_small_kernel<kFused> (sample, thresholds and candidates in one "
                                    f"cooperative launch, 128 rows x {Q} queries per tile)" if small else
                                    "batch::gemm_kernel<kCandidates> (the candidates pass)"),
                         "kernel_ms": mean_gemm,
                         "algorithmic_bytes_per_launch": gemm_bytes,
                         "overhead_bytes_per_launch": overhead_bytes,
                         "bytes_note": "fp16 rows (pitch %d halves) plus a timestamp and an importance "
                                       "per row, once per query tile (one tile at B <= 64)" % pitch16},
            "batch_stats": bstats,
            "fused_scan": {
                "note": "the fp32 fused scan (score x decay x importance -> top-K), event-timed "
                        "outside the timed region",
                "single_query_kernel_ms_p50": scan_med,
                "single_query_kernel_ms_p99": float(np.percentile(scan_ms, 99)),
                "single_query_hbm_gbs": scan_bytes / (scan_med * 1e-3) / 1e9,
                "single_query_hbm_frac": scan_bytes / (scan_med * 1e-3) / 1e9 / peak,
                "multi_query_launch_qps": Q / (float(np.median(multi_ms)) * 1e-3),
                "f16_filtered_launch_qps": Q / (float(np.median(f16_ms)) * 1e-3)},
            "e2e": e2e,
            # per step and GPU: query prep, the fused sample + threshold +
            # candidates pass (three launches on the 128-query tiles), rescore,
            # device rescan (+ the merge when sharded); all GPUs
            "gpu_launches": a.steps * world * ((4 if small else 6) + (1 if sharded else 0)),
            "clocks": clocks,
        }
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"], answers = cpu_baseline(a, E, mod, ts, imp, Qh)
            n_cmp = min(len(answers), ans_ids.shape[0])
            line["exact_vs_oracle"] = compare_with_oracle(ans_ids, ans_vals, answers[:n_cmp])
            line["oracle_checked_queries"] = n_cmp
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
def _pct(xs, p):
    return float(np.percentile(np.asarray(xs), p))


def run_latency(a):
    """c0 / c1: single-query latency through the public API (host query in,
    host results out), one GPU.  c0: N = 2,400, lambda = 0.5, K = 10, BFS
    depth 1 over 4 random cross-modal bridges per node.  c1: start with
    N = 10,000 (same generator); every 1 ms frame appends 10 rows stamped with
    the frame time (normalised on the device) and 2 bridge edges per new row,
    then queries with lambda = 1.0, K = 10, depth 1; latency and freshness
    (share of the top-K stamped within the last 100 ms) over all frames."""
    import torch
    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen

    D, K = a.dim, 10
    if a.workload == "c0":
        N0, lam, frames, per = 2400, 0.5, a.frames, 0
    else:
        N0, lam, frames, per = 10000, 1.0, a.frames, 10
    E, mod, ts, imp = datagen.gaussian_corpus(N0, D, seed=a.seed, n_mod=4, ts_max=10.0)
    ro, ci = datagen.random_bridges(mod, 4, seed=7)
    cap = N0 + frames * per
    rng = np.random.default_rng(a.seed + 3)
    Q = datagen.queries(256, D, seed=0x5EED0000)
    cfg_kw = dict(top_k=K, bfs_max_hops=1, time_decay_lambda=lam, bfs_score_decay=0.5)

    if a.impl == "reference":
        oc = O.Corpus(E=E, ts=ts, mod=mod, row_offsets=ro, col_indices=ci)
        lat = []
        for f in range(min(frames, 200)):
            t0 = time.perf_counter()
            O.query(oc, Q[f % 256], 10.0, top_k=K, bfs_max_hops=1, lam=lam, bfs_score_decay=0.5,
                    dot_order=O.DOT_FAST)
            lat.append(time.perf_counter() - t0)
        v = len(lat) / sum(lat)
        print(json.dumps({"impl": "reference", "workload": a.workload, "metric": "queries/s",
                          "value": v, "unit": "queries/s", "p50_us": _pct(lat, 50) * 1e6,
                          "p99_us": _pct(lat, 99) * 1e6,
                          "cpu_baseline": {"value": v, "unit": "queries/s", "cores": 1,
                                           "kind": "port", "sample": f"{len(lat)} queries, "
                                           "oracle orc_query single thread (corpus fixed)"}}))
        return

    slack = 64 if per else 0
    store = mb.Store(cap, D, edge_slack=slack)
    slack_used = np.zeros(cap, np.int32)
    store.upload(E, mod, ts, None, ro, ci)
    ctx = mb.QueryContext(cap, D, max_k=K)
    cfg = mb.RetrievalConfig(**cfg_kw)
    for i in range(20):
        ctx.query(store, Q[i], 10.0, cfg)
    torch.cuda.synchronize()
    q_lat, a_lat, fresh = [], [], []
    ts_host = np.zeros(cap, np.float32)
    ts_host[:N0] = ts
    t_base = 10.0
    t_all0 = time.perf_counter()
    for f in range(frames):
        t_now = t_base + f * 1e-3
        if per:
            raw = rng.standard_normal((per, D)).astype(np.float32)
            m = rng.integers(0, 4, per).astype(np.int32)
            t0 = time.perf_counter()
            first = store.append(raw, m, np.full(per, t_now, np.float32), normalize=True)
            ts_host[first:first + per] = np.float32(t_now)
            # one bridge per new row to a random older row that still has a
            # free neighbour slot (both directions)
            src = np.arange(first, first + per, dtype=np.int32)
            dst = rng.integers(0, first, per).astype(np.int32)
            for i in range(per):
                while slack_used[dst[i]] >= slack:
                    dst[i] = rng.integers(0, first)
                slack_used[dst[i]] += 1
                slack_used[src[i]] += 1
            store.append_edges(np.concatenate([src, dst]), np.concatenate([dst, src]))
            a_lat.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        res = ctx.query(store, Q[f % 256], t_now, cfg)
        q_lat.append(time.perf_counter() - t0)
        if per:
            fresh.append(float(np.mean(ts_host[res["node_id"]] >= np.float32(t_now - 0.1)))
                         if len(res) else 0.0)
    total = time.perf_counter() - t_all0
    line = {"workload": a.workload, "metric": "single-query latency (mars_query, host in/out)",
            "n_start": N0, "n_end": N0 + frames * per, "frames": frames, "dim": D, "top_k": K,
            "lambda": lam, "bfs_max_hops": 1,
            "query_p50_us": _pct(q_lat, 50) * 1e6, "query_p99_us": _pct(q_lat, 99) * 1e6,
            "query_max_us": float(np.max(q_lat) * 1e6),
            "queries_per_s": frames / sum(q_lat)}
    if per:
        line.update({"append_p50_us": _pct(a_lat, 50) * 1e6, "append_p99_us": _pct(a_lat, 99) * 1e6,
                     "freshness_mean": float(np.mean(fresh)),
                     "frames_per_s_incl_append": frames / total})
    print(json.dumps(line), flush=True)


def run_batch(a):
    """c2: batched queries on the tensor cores.  N = 1M rows (row-sharded over
    the ranks), B = 1024 queries per step, K = 100, lambda = 0.01, t_q = 600,
    importance on.  A step is one mars_query_batch_topk per rank (+ NCCL
    all-gather of the [B][K] lists and mars_topk_merge_batch when sharded)."""
    import torch
    import mars_b200 as mb
    from mars_b200 import datagen

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        from datetime import timedelta
        dist = dist_mod
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    K, B, D = (a.k if a.k != 10 else 100), a.batch, a.dim
    lo, hi = a.n * rank // world, a.n * (rank + 1) // world
    E, mod, ts, imp = datagen.gaussian_rows(lo, hi, D, seed=a.seed, ts_max=a.ts_max)
    store = mb.Store(hi - lo, D, device=local)
    store.upload(E, mod, ts, imp)
    del E
    bc = mb.BatchContext(hi - lo, D, max_batch=B, max_k=K, device=local)
    ctx = mb.QueryContext(hi - lo, D, max_k=K, device=local)
    Qh = datagen.queries(B, D, seed=a.seed + 1)
    Qd = torch.from_numpy(Qh).cuda()
    ids = torch.empty((B, K), dtype=torch.int32, device="cuda")
    vals = torch.empty((B, K), dtype=torch.float32, device="cuda")
    if world > 1:
        gids = torch.empty((world, B, K), dtype=torch.int32, device="cuda")
        gvals = torch.empty((world, B, K), dtype=torch.float32, device="cuda")
        mids = torch.empty((B, K), dtype=torch.int32, device="cuda")
        mvals = torch.empty((B, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))
    torch.cuda.set_stream(stream)

    def step():
        bc.query_batch_topk(store, Qd, B, a.ts_max, a.lam, K, ids, vals, use_importance=True,
                            row_offset=lo, stream=ctx.stream)
        if world > 1:
            dist.all_gather_into_tensor(gids, ids)
            dist.all_gather_into_tensor(gvals, vals)
            ctx.topk_merge_batch(gids, gvals, world, K, B, mids, mvals, stream=ctx.stream)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()        # after the sampler started: no rank waits inside the timed region
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(a.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    stats = bc.last_stats()
    # phase breakdown (outside the timed region): batch alone, exchange alone
    phases = {}
    for name, fn in (("batch_ms", lambda: bc.query_batch_topk(store, Qd, B, a.ts_max, a.lam, K, ids, vals,
                                                              use_importance=True, row_offset=lo,
                                                              stream=ctx.stream)),
                     ("exchange_merge_ms", (lambda: (dist.all_gather_into_tensor(gids, ids),
                                                     dist.all_gather_into_tensor(gvals, vals),
                                                     ctx.topk_merge_batch(gids, gvals, world, K, B, mids, mvals,
                                                                          stream=ctx.stream)))
                      if world > 1 else None)):
        if fn is None:
            continue
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        phases[name] = (time.perf_counter() - t0) / 3 * 1e3
    if rank == 0:
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except Exception:
            pass
        flops = 2.0 * B * a.n * D
        per_batch_s = ms * 1e-3 / a.steps
        achieved = flops / per_batch_s / 1e12 / world
        bf16 = float(peaks.get("bf16_tflops", 1590.0))
        line = {"workload": "c2", "metric": f"queries/s (batched top-K, N={a.n}, D={D}, B={B}, K={K})",
                "value": B * a.steps / (ms * 1e-3), "unit": "queries/s", "n_gpus": world,
                "steps": a.steps, "ms_per_step": ms / a.steps, "scaling": "strong",
                "roofline": {"bound": "tensor", "achieved": achieved, "unit": "TFLOP/s per GPU",
                             "operands": {2: "fp16 (kind::f16)", 1: "tf32 (kind::tf32)"}.get(
                                 stats.get("path"), "scan"),
                             # fp16 runs at the bf16 rate; TF32 at half of it
                             "peak": bf16 if stats.get("path") == 2 else bf16 / 2,
                             "peak_kind": ("measured bf16 GEMM" if "bf16_tflops" in peaks else "fallback")
                                          + (" (same rate as fp16)" if stats.get("path") == 2 else " / 2 (TF32)"),
                             "frac": achieved / (bf16 if stats.get("path") == 2 else bf16 / 2),
                             "flops_per_batch": flops},
                "batch_stats_rank0": stats, "phases_rank0_wall": phases, "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _init_dist(local, world):
    """NCCL process group for torchrun launches (None on one GPU)."""
    if world <= 1:
        return None
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return dist


def _sharded_graph(mb, st, N, deg, deg_cross, n_mod, rank, world, dist):
    """cmng_build split by row blocks: rank r builds rows [r*N/G, (r+1)*N/G)
    against the whole (replicated) store, then one NCCL all-gather of the
    equal-sized padded blocks gives every rank the full N x deg graph.
    Returns (graph, device ms of the build + gather, max over ranks)."""
    import torch
    lo, hi = N * rank // world, N * (rank + 1) // world
    rows_max = (N + world - 1) // world
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize()
    e0.record()
    if world == 1:
        nb = torch.empty((N, deg), dtype=torch.int32, device="cuda")
        mb.cmng_build_rows(st, 0, N, deg, deg_cross, n_mod, nb)
    else:
        block = torch.full((rows_max, deg), -1, dtype=torch.int32, device="cuda")
        mb.cmng_build_rows(st, lo, hi - lo, deg, deg_cross, n_mod, block)
        allb = torch.empty((world * rows_max, deg), dtype=torch.int32, device="cuda")
        dist.all_gather_into_tensor(allb, block)
        nb = torch.cat([allb[r * rows_max: r * rows_max + (N * (r + 1) // world - N * r // world)]
                        for r in range(world)])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return nb, ms


def run_knn_build(a):
    """c3: cmng_build of an exact out-degree-32 kNN graph.  N = 100,000 rows
    (100 isotropic Gaussian clusters, centres N(0,1), sigma 0.3, normalised),
    degree 32, no bridges.  A step is one full build (tensor-core kNN with
    exact rescoring + neighbour selection), device-timed.  Under torchrun
    every rank holds the whole corpus and builds one row block; an NCCL
    all-gather of the blocks completes the step (strong scaling)."""
    import torch
    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen

    rank, world, local = dist_env()
    N = a.n if a.n != 1_000_000 else 100_000
    D, deg = a.dim, 32
    E, mod, ts, _ = datagen.cluster_corpus(N, D, 100, 0.3, seed=a.seed, n_mod=4, ts_max=10.0)
    if a.impl == "reference":
        if rank != 0:
            return
        c = O.Corpus(E=E, ts=ts, mod=mod)
        rows = np.arange(0, N, max(1, N // 200), dtype=np.int32)
        t0 = time.perf_counter()
        O.knn(c, rows, 2 * deg, dot_order=O.DOT_FAST)
        dt = time.perf_counter() - t0
        full = dt * N / rows.shape[0]
        print(json.dumps({"impl": "reference", "workload": "c3", "metric": "cmng_build ms", "value": full * 1e3,
                          "unit": "ms", "higher_is_better": False,
                          "cpu_baseline": {"value": full * 1e3, "unit": "ms", "cores": os.cpu_count(),
                                           "kind": "port", "sample": f"exact kNN of {rows.shape[0]} rows "
                                           f"against all {N}, extrapolated x{N / rows.shape[0]:.0f}"}}))
        return
    torch.cuda.set_device(local)
    dist = _init_dist(local, world)
    st = mb.Store(N, D, device=local)
    st.upload(E, mod, ts)
    for _ in range(max(1, a.warmup)):
        nb, _ = _sharded_graph(mb, st, N, deg, 0, 4, rank, world, dist)
    times = []
    for _ in range(a.steps):
        nb, ms = _sharded_graph(mb, st, N, deg, 0, 4, rank, world, dist)
        times.append(ms)
    if rank == 0:
        # spot check of the gathered graph against the exact oracle kNN
        rows = np.arange(0, N, N // 64, dtype=np.int32)
        rid, _ = O.knn(O.Corpus(E=E, ts=ts, mod=mod), rows, 2 * deg)
        ref = O.cmng_select(rid, mod, rows, deg, 0, 4)
        exact = bool(np.array_equal(nb.cpu().numpy()[rows], ref))
        ms = statistics.median(times)
        flops = 2.0 * N * N * D
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except Exception:
            pass
        bf16 = float(peaks.get("bf16_tflops", 1590.0))
        print(json.dumps({"workload": "c3", "metric": f"cmng_build ms (N={N}, D={D}, degree {deg})",
                          "value": ms, "unit": "ms", "higher_is_better": False, "n_gpus": world,
                          "steps": a.steps, "scaling": "strong",
                          "parallelism": f"row blocks x{world}" + (" + NCCL all-gather" if world > 1 else ""),
                          "tflops_effective": flops / (ms * 1e-3) / 1e12,
                          "roofline": {"bound": "tensor", "flops_per_build": flops,
                                       "frac_of_tf32_nominal_per_gpu":
                                           flops / world / (ms * 1e-3) / 1e12 / (bf16 / 2)},
                          "spot_check_rows": int(rows.shape[0]), "neighbours_bit_exact": exact}),
              flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_cmng_bfs(a):
    """c4: cmng_search + cross-modal BFS.  N = 1,000,000 rows from a 1,000
    cluster mixture (sigma 0.3, 4 modalities, normalised); graph = degree-32
    kNN + 4 cross-modal bridges (degree 36, built once, untimed); 10,000
    queries, beam 64, K = 10, lambda = 0.05, BFS depth 2.  Under torchrun:
    replicas (every rank holds the corpus; the graph is built by row blocks
    and all-gathered), the queries split across ranks, and an NCCL
    all-gather of the per-rank results ends each step."""
    import torch
    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen

    rank, world, local = dist_env()
    N, D, deg, K, nq = a.n, a.dim, 36, 10, a.queries
    if a.impl == "reference" and rank != 0:
        return
    torch.cuda.set_device(local)
    E, mod, ts, _ = datagen.cluster_corpus(N, D, 1000, 0.3, seed=a.seed, n_mod=4, ts_max=10.0)
    Q = datagen.queries(nq, D, seed=a.seed + 5)
    dist = _init_dist(local, world) if a.impl != "reference" else None
    st = mb.Store(N, D, device=local)
    st.upload(E, mod, ts)
    if a.impl == "reference":   # rank 0 alone: the graph is built locally
        nb, build_ms = _sharded_graph(mb, st, N, deg, 4, 4, 0, 1, None)
    else:
        nb, build_ms = _sharded_graph(mb, st, N, deg, 4, 4, rank, world, dist)
    if a.impl == "reference":
        nbh = nb.cpu().numpy()
        c = O.Corpus(E=E, ts=ts, mod=mod, fixed_nbrs=nbh)
        sample = min(nq, 50)
        t0 = time.perf_counter()
        for q in range(sample):
            res, _ = O.cmng_search(c, nbh, Q[q], 10.0, K=K, beam_width=64, max_iterations=64, lam=0.05,
                                   dot_order=O.DOT_FAST)
            O.bfs(c, res["node_id"], res["score"], None, 2, 0.5, q=Q[q], t_q=10.0, lam=0.05,
                  dot_order=O.DOT_FAST)
        dt = time.perf_counter() - t0
        v = sample / dt
        print(json.dumps({"impl": "reference", "workload": "c4", "metric": "queries/s", "value": v,
                          "unit": "queries/s",
                          "cpu_baseline": {"value": v, "unit": "queries/s", "cores": 1, "kind": "port",
                                           "sample": f"{sample} queries, oracle beam search + BFS, 1 thread"}}))
        return
    q0, q1 = nq * rank // world, nq * (rank + 1) // world
    nql = q1 - q0
    qmax = (nq + world - 1) // world
    Qd = torch.from_numpy(np.ascontiguousarray(Q[q0:q1])).cuda()
    cfg = mb.CmngConfig(K=K, beam_width=64, max_iterations=64, time_decay_lambda=0.05)
    ctx = mb.CmngContext(qmax, K, deg, 2, N, device=local)
    ids = torch.full((qmax, K), -1, dtype=torch.int32, device="cuda")
    sc = torch.zeros((qmax, K), dtype=torch.float32, device="cuda")
    cnt = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    vis = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    bits = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    bscored = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    if world > 1:
        all_ids = torch.empty((world * qmax, K), dtype=torch.int32, device="cuda")
        all_sc = torch.empty((world * qmax, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()       # a real stream: NULL would mean the store's own stream
    torch.cuda.set_stream(stream)

    def step():
        ctx.search_bfs(st, nb, deg, Qd, nql, 10.0, cfg, 2, 0.5, ids, sc, cnt, d_visited=vis,
                       stream=stream.cuda_stream)
        if world > 1:
            dist.all_gather_into_tensor(all_ids, ids)
            dist.all_gather_into_tensor(all_sc, sc)

    for _ in range(max(1, a.warmup)):
        step()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(a.steps):
        step()
    e1.record(stream)
    for _ in range(a.steps):
        mb.cmng_search_batch(st, nb, deg, Qd, nql, 10.0, cfg, ids, sc, cnt, d_iters=bits,
                             d_scored=bscored, stream=stream.cuda_stream)
    e2.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    ms_beam = e1.elapsed_time(e2) / a.steps
    if world > 1:
        t = torch.tensor([ms, ms_beam], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_beam = float(t[0].item()), float(t[1].item())
    rows_bfs = float(vis[:nql].double().mean().item())
    rows_beam = float(bscored[:nql].double().mean().item())
    # rows read per query: beam-scored rows + the BFS levels >= 1 (seeds are beam rows)
    bytes_q = (rows_beam + rows_bfs) * D * 4
    peak, _ = measured_peak()
    achieved = bytes_q * nql / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({"workload": "c4", "metric": f"queries/s (cmng_search + BFS depth 2, N={N}, K={K})",
                          "value": nq / (ms * 1e-3), "unit": "queries/s", "n_gpus": world,
                          "scaling": "strong", "ms_per_batch": ms,
                          "parallelism": f"replicas x{world}, queries split" +
                                         (" + NCCL all-gather of results" if world > 1 else ""),
                          "beam_only_queries_per_s": nq / (ms_beam * 1e-3), "graph_build_ms": build_ms,
                          "mean_rows_scored_beam": rows_beam, "mean_nodes_visited_bfs": rows_bfs,
                          "mean_iterations": float(bits[:nql].double().mean().item()),
                          "roofline": {"bound": "hbm", "achieved_per_gpu": achieved, "peak": peak,
                                       "unit": "GB/s", "frac": achieved / peak,
                                       "note": "row gathers: (beam-scored + BFS-visited rows) x D x 4 bytes"}}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    a = parse_args()
    if a.workload == "c3":
        run_knn_build(a)
    elif a.workload == "c4":
        run_cmng_bfs(a)
    elif a.workload == "c2":
        run_batch(a)
    elif a.workload in ("c0", "c1"):
        run_latency(a)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_mars(a)


if __name__ == "__main__":
    main()
