#!/usr/bin/env python
"""MARS B200 benchmark: exact retrieval top-K (cosine x decay x importance).

Workload (the headline metric: queries/s + p99 at N=1M, D=768, K=10, HBM GB/s
vs peak):
  * corpus N = 1,000,000 rows x D = 768 fp32, i.i.d. Gaussian rows divided by
    (||v|| + 1e-8), timestamps U[0, 600] s, importance U[0, 1], 4 modalities;
    seeded synthetic data (no dataset is involved);
  * a step is 64 concurrent queries (`--queries-per-step`), each the exact
    top-K = 10 of dot x exp(-lambda * age) x importance over all N rows,
    lambda = 0.01, answered by mars_query_batch_topk (an fp16 tensor-core
    short list with a proven error margin, then an exact fp32 rescore: the
    results are those of the fp32 fused scan bit for bit, which the run
    checks, and the oracle's, which the run checks on 32 queries); 64 is the
    most the small-batch tiles hold, so a step stays one pass over the rows
    (the line's `batch_sweep_per_gpu` has the step at 16 / 32 / 48 / 128 /
    256);
  * N GPUs (`--shard replicas`, the default): the 1M-row corpus (4.6 GB with
    its fp16 copy) fits every GPU, so every GPU holds it and answers its own
    64 queries per step, with no data-path collective (weak scaling: 64 N
    queries per step).  `--shard rows`: the corpus is row-sharded (strong
    scaling), every GPU answers the same queries on its shard, and the
    per-query local top-K lists are all-gathered over NCCL and merged on
    every GPU.  The line's `configs` carries every config of the family
    (c0-c4), c2 row-sharded through the library's own NCCL path.

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
    ap.add_argument("--queries-per-step", type=int, default=64,
                    help="concurrent queries answered by one step (one mars_query_batch_topk call); 64 is the "
                         "most the small-batch tensor-core tiles hold, so the step stays one pass over the rows")
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
                    help="scan: the headline (default; its line also carries every config under "
                         "`configs`); c0: single-query latency at N=2400 with BFS depth 1; c1: streaming "
                         "loop (append 10 rows + query per frame); c2: batched top-K B=1024 K=100, rows "
                         "sharded; c3: kNN-graph build; c4: graph search + BFS")
    ap.add_argument("--frames", type=int, default=10000)
    ap.add_argument("--c4-n", type=int, default=1_000_000, help="rows of the c4 corpus")
    ap.add_argument("--skip-configs", default="",
                    help="comma-separated configs (c0..c4) left out of the default run's `configs`")
    ap.add_argument("--no-configs", action="store_true", help="the headline only")
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
    n_pool = max(256, 2 * a.queries_per_step)    # query pool the steps cycle through (and the sweep's batches)
    Qh = datagen.queries(n_pool, a.dim, seed=a.seed + 1 + (0 if sharded else 1000 * rank))
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
    for base in sorted({0, Q // 2, n_pool - Q}):
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

    # the same step with fewer or more concurrent queries (device time per
    # step, 20 steps each, outside the timed region): how the step's cost
    # grows with the batch (above 64 queries the 128 x 256 tiles: one pass
    # over the rows per 128 queries)
    sweep = {}
    if not sharded:
        for Bs in (16, 32, 48, 128, 256):
            if Bs == Q:
                continue
            bcs = mb.BatchContext(n_local, a.dim, max_batch=Bs, max_k=K, device=local)
            i2 = torch.empty((Bs, K), dtype=torch.int32, device="cuda")
            v2 = torch.empty((Bs, K), dtype=torch.float32, device="cuda")
            for _ in range(3):
                bcs.query_batch_topk(store, Qd[:Bs], Bs, a.ts_max, a.lam, K, i2, v2, use_importance=True,
                                     row_offset=lo, stream=ctx.stream)
            t_ms = timed(lambda: [bcs.query_batch_topk(store, Qd[:Bs], Bs, a.ts_max, a.lam, K, i2, v2,
                                                       use_importance=True, row_offset=lo, stream=ctx.stream)
                                  for _ in range(20)], 1)[0] / 20
            sweep[str(Bs)] = {"ms_per_step": t_ms, "queries_per_s": Bs / (t_ms * 1e-3)}
            bcs.close()

    # ---- end to end through the public API with host buffers --------------
    # A serving loop: every step copies its queries host -> device, answers
    # them and copies the ids, scores and counts device -> host into one of
    # two pinned buffers; the host waits for the previous step's results and
    # reads them, so the GPU is not idle while the host issues the next step.
    # The copies run on their own stream: step s + 1's queries travel while
    # step s is answered, and step s's results while step s + 1 is; the
    # device buffers (two of each) are reused in event order.
    Qpin = torch.from_numpy(Qh).pin_memory()
    cstream = torch.cuda.Stream(device=torch.device("cuda", local))
    qbufs = [torch.empty((Q, a.dim), dtype=torch.float32, device="cuda") for _ in range(2)]
    # one packed result buffer per step (ids | scores | counts): one D2H copy
    ress = [torch.empty(2 * Q * K + Q, dtype=torch.int32, device="cuda") for _ in range(2)]
    outs = [torch.empty(2 * Q * K + Q, dtype=torch.int32).pin_memory() for _ in range(2)]
    outs_np = [o.numpy() for o in outs]
    q_in = [torch.cuda.Event() for _ in range(2)]       # a step's queries are on the device
    answered = [torch.cuda.Event() for _ in range(2)]   # a step's results are in its device buffer
    done = [torch.cuda.Event() for _ in range(2)]       # ... and in its pinned host buffer
    checksum = 0
    e2e_valid = True

    def h2d(step):
        base = (step * Q) % (n_pool - Q + 1)
        with torch.cuda.stream(cstream):
            qbufs[step % 2].copy_(Qpin[base:base + Q], non_blocking=True)
            q_in[step % 2].record(cstream)

    barrier()
    t0 = time.perf_counter()
    h2d(0)
    for s in range(a.steps + 1):
        if s < a.steps:
            b = s % 2
            res = ress[b]
            r_ids = res[:Q * K].view(Q, K)
            r_vals = res[Q * K:2 * Q * K].view(torch.float32).view(Q, K)
            r_cnt = res[2 * Q * K:]
            stream.wait_event(q_in[b])
            if sharded:
                bc.query_batch_topk(store, qbufs[b], Q, a.ts_max, a.lam, K, ids, vals, use_importance=True,
                                    row_offset=lo, stream=ctx.stream)
                dist.all_gather_into_tensor(gids, ids)
                dist.all_gather_into_tensor(gvals, vals)
                ctx.topk_merge_batch(gids, gvals, world, K, Q, r_ids, r_vals, r_cnt, stream=ctx.stream)
            else:
                bc.query_batch_topk(store, qbufs[b], Q, a.ts_max, a.lam, K, r_ids, r_vals, r_cnt,
                                    use_importance=True, row_offset=lo, stream=ctx.stream)
            answered[b].record(stream)
            if s + 1 < a.steps:
                # the next step's queries, into the buffer step s - 1 read
                # (answered: the copy stream waited for it before its D2H)
                h2d(s + 1)
            cstream.wait_event(answered[b])
            with torch.cuda.stream(cstream):
                outs[b].copy_(res, non_blocking=True)
                done[b].record(cstream)
        if s > 0:   # the previous step's results, read and checked on the host
            p = (s - 1) % 2
            done[p].synchronize()
            e2e_valid = e2e_valid and bool(outs_np[p][2 * Q * K:].min() == K)
            checksum += int(outs_np[p][0])
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    bc.last_stats()      # raises if the last step's pipeline reported an error
    if world > 1:
        t = torch.tensor([dt], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    q_all = Q * (1 if sharded else world)   # queries answered per step by the whole job
    e2e = {"value": a.steps * q_all / dt, "unit": "queries/s",
           "h2d_bytes_per_step": Q * a.dim * 4, "d2h_bytes_per_step": (2 * Q * K + Q) * 4,
           "every_step_valid": e2e_valid,
           "path": "pinned H2D of the step's queries, mars_query_batch_topk"
                   + (" per shard, NCCL all-gather, mars_topk_merge_batch" if sharded else
                      (" on every replica" if world > 1 else ""))
                   + ", one packed D2H of the top-K ids, scores and counts into one of two pinned buffers "
                     "(both copies on a copy stream, overlapped with the neighbouring steps' compute); the "
                     "host waits for and reads each step's results (checking every count) while the next "
                     "step runs"}
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

    # every config of the family (c2-c4 on all ranks, c0/c1 on one GPU)
    configs = None
    if not a.no_configs and not sharded:
        env = {"rank": rank, "world": world, "local": local, "dist": dist, "rows": (E, mod, ts, imp),
               "store": store}
        configs = run_configs(a, env)
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
            "batch_sweep_per_gpu": sweep,
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
        if configs is not None:
            line["configs"] = configs
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
# The configurations of the workload family (c0-c4).  Each function runs on
# every rank (collectives in the same order on all of them) and returns the
# config's record on rank 0 (None elsewhere).  The default run embeds them in
# the headline line under "configs"; `--workload cX` prints one of them.
def _pct(xs, p):
    return float(np.percentile(np.asarray(xs), p))


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


def _tensor_peaks():
    """(sustained, burst, kind): the measured bf16 GEMM rates (fp16 runs at
    the same rate), else the fallback figures."""
    p = _peaks()
    if "bf16_tflops" in p:
        return float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), float(p["bf16_tflops"]), "measured"
    return 1400.0, 1590.0, "fallback"


def _max_over_ranks(dist, x):
    if dist is None:
        return x
    import torch
    t = torch.tensor([float(x)], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _all_true(dist, ok):
    if dist is None:
        return bool(ok)
    import torch
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def _barrier(dist):
    import torch
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize()


def _init_dist(local, world):
    """NCCL process group for torchrun launches (None on one GPU)."""
    if world <= 1:
        return None
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return dist


def cfg_latency(a, which):
    """c0 / c1: single-query latency through the public API (host query in,
    host results out), one GPU.  c0: N = 2,400, lambda = 0.5, K = 10, BFS
    depth 1 over 4 random cross-modal bridges per node.  c1: start with
    N = 10,000 (same generator); every 1 ms frame appends 10 rows stamped with
    the frame time (normalised on the device) and 2 bridge edges per new row,
    then queries with lambda = 1.0, K = 10, depth 1; latency and freshness
    (share of the top-K stamped within the last 100 ms) over all frames.
    Parity: the answers of sampled frames against the oracle on the same
    corpus and graph (c1: the store read back, the CSR plus appended edges)."""
    import torch
    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen
    from _util import assert_ranked_equivalent

    D, K = a.dim, 10
    frames = a.frames
    if which == "c0":
        N0, lam, per = 2400, 0.5, 0
    else:
        N0, lam, per = 10000, 1.0, 10
    E, mod, ts, imp = datagen.gaussian_corpus(N0, D, seed=a.seed, n_mod=4, ts_max=10.0)
    ro, ci = datagen.random_bridges(mod, 4, seed=7)
    cap = N0 + frames * per
    rng = np.random.default_rng(a.seed + 3)
    Q = datagen.queries(256, D, seed=0x5EED0000)
    cfg_kw = dict(top_k=K, bfs_max_hops=1, time_decay_lambda=lam, bfs_score_decay=0.5)
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
    extra_src, extra_dst = [], []
    check_frames = set(range(0, frames, max(1, frames // 8))) | {frames - 1}
    answers = {}
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
            s2, d2 = np.concatenate([src, dst]), np.concatenate([dst, src])
            store.append_edges(s2, d2)
            a_lat.append(time.perf_counter() - t0)
            extra_src.append(s2)
            extra_dst.append(d2)
        t0 = time.perf_counter()
        res = ctx.query(store, Q[f % 256], t_now, cfg)
        q_lat.append(time.perf_counter() - t0)
        if f in check_frames:
            answers[f] = (res.copy(), store.num_nodes if per else N0)
        if per:
            fresh.append(float(np.mean(ts_host[res["node_id"]] >= np.float32(t_now - 0.1)))
                         if len(res) else 0.0)
    total = time.perf_counter() - t_all0
    # parity of the sampled frames: the oracle on the corpus as it was then
    n_end = store.num_nodes
    if per:
        Eh, modh, tsh, _ = store.read(0, n_end)
        es = np.concatenate(extra_src) if extra_src else np.zeros(0, np.int32)
        ed = np.concatenate(extra_dst) if extra_dst else np.zeros(0, np.int32)
    exact = True
    for f, (res, n_f) in sorted(answers.items()):
        if per:
            # CSR over the first n_f rows: the uploaded graph plus the bridges appended by then
            keep = (es < n_f) & (ed < n_f)
            adj = [[] for _ in range(n_f)]
            for u in range(N0):
                adj[u].extend(ci[ro[u]:ro[u + 1]].tolist())
            for u, v in zip(es[keep].tolist(), ed[keep].tolist()):
                adj[u].append(v)
            ro_f = np.zeros(n_f + 1, np.int32)
            ro_f[1:] = np.cumsum([len(x) for x in adj])
            ci_f = np.asarray([v for x in adj for v in x], np.int32)
            oc = O.Corpus(E=Eh[:n_f], ts=tsh[:n_f], mod=modh[:n_f], row_offsets=ro_f, col_indices=ci_f)
        else:
            oc = O.Corpus(E=E, ts=ts, mod=mod, row_offsets=ro, col_indices=ci)
        ref = O.query(oc, Q[f % 256], t_base + f * 1e-3, top_k=K, bfs_max_hops=1, lam=lam, bfs_score_decay=0.5)
        try:
            assert_ranked_equivalent(res["node_id"], res["score"], ref["node_id"], ref["score"], res["hops"],
                                     ref["hops"], what=f"frame {f}")
        except AssertionError:
            exact = False
    # CPU baseline: the oracle port answering the same queries on the final
    # corpus, one thread (the reference's only CPU path is NumPy)
    oc = O.Corpus(E=E, ts=ts, mod=mod, row_offsets=ro, col_indices=ci)
    lat = []
    for f in range(64):
        t0 = time.perf_counter()
        O.query(oc, Q[f % 256], 10.0, top_k=K, bfs_max_hops=1, lam=lam, bfs_score_decay=0.5, dot_order=O.DOT_FAST)
        lat.append(time.perf_counter() - t0)
    rec = {"workload": which, "metric": "single-query latency (mars_query, host in/out)",
           "n_start": N0, "n_end": n_end, "frames": frames, "dim": D, "top_k": K,
           "lambda": lam, "bfs_max_hops": 1,
           "query_p50_us": _pct(q_lat, 50) * 1e6, "query_p99_us": _pct(q_lat, 99) * 1e6,
           "query_max_us": float(np.max(q_lat) * 1e6), "queries_per_s": frames / sum(q_lat),
           "oracle_checked_frames": len(answers), "exact_vs_oracle": exact,
           "cpu_baseline": {"value": len(lat) / sum(lat), "unit": "queries/s", "cores": 1, "kind": "port",
                            "sample": f"{len(lat)} queries over the starting {N0}-row corpus, oracle orc_query "
                                      "(fast dot order) on one thread",
                            "p50_us": _pct(lat, 50) * 1e6}}
    if per:
        rec.update({"append_p50_us": _pct(a_lat, 50) * 1e6, "append_p99_us": _pct(a_lat, 99) * 1e6,
                    "freshness_mean": float(np.mean(fresh)),
                    "frames_per_s_incl_append": frames / total})
    return rec


def cfg_c2(a, env):
    """c2: batched top-K over N = 1M rows (the headline's corpus), B = 1024
    queries per step, K = 100, lambda = 0.01, importance on, row-sharded over
    the ranks: one mars_shard_query_batch_topk per step and rank (the
    library's NCCL: bound all-reduce between the rescore passes, one
    all-gather of packed keys, merge).  Strong scaling (N fixed)."""
    import torch
    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen
    from _util import assert_ranked_equivalent
    rank, world, local, dist = env["rank"], env["world"], env["local"], env["dist"]
    B, K, D, N = a.batch, 100, a.dim, a.n
    lo, hi = N * rank // world, N * (rank + 1) // world
    E, mod, ts, imp = env["rows"]            # every row (the headline holds them all)
    full = env["store"]
    if world == 1:
        st = full
    else:
        st = mb.Store(hi - lo, D, device=local)
        st.upload(E[lo:hi], mod[lo:hi], ts[lo:hi], imp[lo:hi])
    bc = mb.BatchContext(hi - lo, D, max_batch=B, max_k=K, device=local)
    uid = [mb.shard_unique_id() if rank == 0 else None]
    if dist is not None:
        dist.broadcast_object_list(uid, src=0)
    comm = mb.ShardComm(local, rank, world, uid[0], max_batch=B, max_k=K)
    Qh = datagen.queries(B, D, seed=a.seed + 7)
    Qd = torch.from_numpy(Qh).cuda()
    stream = torch.cuda.Stream()
    res = torch.empty(2 * B * K + B, dtype=torch.int32, device="cuda")   # ids | scores | counts
    ids, vals, cnt = res[:B * K].view(B, K), res[B * K:2 * B * K].view(torch.float32).view(B, K), res[2 * B * K:]

    def step(q):
        comm.query_batch_topk(st, bc, q, B, a.ts_max, a.lam, K, ids, vals, cnt, use_importance=True,
                              row_offset=lo, stream=stream.cuda_stream)

    for _ in range(max(3, a.warmup)):
        step(Qd)
    steps = max(5, min(a.steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(dist)
    e0.record(stream)
    for _ in range(steps):
        step(Qd)
    e1.record(stream)
    _barrier(dist)
    ms = _max_over_ranks(dist, e0.elapsed_time(e1) / steps)
    comm.set_timing(True)
    step(Qd)
    phases = comm.last_times()
    comm.set_timing(False)
    stats = bc.last_stats()
    gemm_ms = _max_over_ranks(dist, stats["gemm_ms"])
    phases = {k: _max_over_ranks(dist, v) for k, v in phases.items()}
    ans = res.cpu().numpy()
    a_ids, a_vals = ans[:B * K].reshape(B, K), ans[B * K:2 * B * K].view(np.float32).reshape(B, K)
    valid = bool(np.all(ans[2 * B * K:] == K))

    # end to end: host queries in (pinned), one packed result copy out, both
    # copies on a copy stream with two device buffers each (the next batch's
    # queries and the previous batch's results travel while a batch runs)
    Qpin = torch.from_numpy(Qh).pin_memory()
    cstream = torch.cuda.Stream()
    qbufs = [torch.empty((B, D), dtype=torch.float32, device="cuda") for _ in range(2)]
    ress = [torch.empty(2 * B * K + B, dtype=torch.int32, device="cuda") for _ in range(2)]
    outs = [torch.empty(2 * B * K + B, dtype=torch.int32).pin_memory() for _ in range(2)]
    q_in = [torch.cuda.Event() for _ in range(2)]
    answered = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    e2e_valid = True

    def h2d(b):
        with torch.cuda.stream(cstream):
            qbufs[b].copy_(Qpin, non_blocking=True)
            q_in[b].record(cstream)

    _barrier(dist)
    t0 = time.perf_counter()
    h2d(0)
    for s in range(steps + 1):
        if s < steps:
            b = s % 2
            r = ress[b]
            stream.wait_event(q_in[b])
            comm.query_batch_topk(st, bc, qbufs[b], B, a.ts_max, a.lam, K, r[:B * K].view(B, K),
                                  r[B * K:2 * B * K].view(torch.float32).view(B, K), r[2 * B * K:],
                                  use_importance=True, row_offset=lo, stream=stream.cuda_stream)
            answered[b].record(stream)
            if s + 1 < steps:
                h2d((s + 1) % 2)
            cstream.wait_event(answered[b])
            with torch.cuda.stream(cstream):
                outs[b].copy_(r, non_blocking=True)
                done[b].record(cstream)
        if s > 0:
            p = (s - 1) % 2
            done[p].synchronize()
            e2e_valid = e2e_valid and bool(np.all(outs[p].numpy()[2 * B * K:] == K))
    torch.cuda.synchronize()
    dt = _max_over_ranks(dist, time.perf_counter() - t0)

    # exactness: the merged answer equals one GPU's answer over all rows (bit
    # for bit) and the oracle's (tie-aware) on sampled queries
    exact_single = None
    exact_oracle = None
    cpu = None
    if rank == 0:
        bcf = mb.BatchContext(N, D, max_batch=B, max_k=K, device=local)
        fi = torch.empty((B, K), dtype=torch.int32, device="cuda")
        fv = torch.empty((B, K), dtype=torch.float32, device="cuda")
        bcf.query_batch_topk(full, Qd, B, a.ts_max, a.lam, K, fi, fv, use_importance=True, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        exact_single = bool(np.array_equal(fi.cpu().numpy(), a_ids) and
                            np.array_equal(fv.cpu().numpy().view(np.int32), a_vals.view(np.int32)))
        bcf.close()
        corpus = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
        threads = os.cpu_count() or 1
        sample = 8
        oi, ov = O.query_batch_topk(corpus, Qh[:4], a.ts_max, a.lam, K, use_importance=True)
        try:
            for q in range(4):
                assert_ranked_equivalent(a_ids[q], a_vals[q], oi[q], ov[q], what=f"c2 query {q}")
            exact_oracle = True
        except AssertionError:
            exact_oracle = False
        if world == 1:
            t1 = time.perf_counter()
            for q in range(sample):
                O.scan_topk_fast(corpus, Qh[q], a.ts_max, a.lam, K, use_importance=True, n_threads=threads)
            cdt = time.perf_counter() - t1
            cpu = {"value": sample / cdt, "unit": "queries/s", "cores": threads, "kind": "port",
                   "sample": f"{sample} of the {B} queries, each scanning all {N} rows (K = {K}), "
                             f"oracle orc_scan_topk_fast with {threads} OpenMP threads; queries/s of the "
                             f"sample stands for the batch ({B // sample}x the sample's work)"}
    exact_all = _all_true(dist, valid and (exact_single is not False))
    sus, burst, kind = _tensor_peaks()
    achieved = 2.0 * B * (hi - lo) * D / (gemm_ms * 1e-3) / 1e12
    comm.close()
    del bc
    if world > 1:
        st.close()
    if rank != 0:
        return None
    return {"workload": "c2", "metric": f"queries/s (batched exact top-K, N={N}, D={D}, B={B}, K={K})",
            "value": B / (ms * 1e-3), "unit": "queries/s", "n_gpus": world, "steps": steps,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "parallelism": (f"rows sharded x{world}: mars_shard_query_batch_topk (inside the library: NCCL "
                            f"all-gathers of the sampled bounds, of the per-query count / bound records and of "
                            f"the packed keys, then the merge)" if world > 1
                            else "one GPU (mars_shard_query_batch_topk, world 1)"),
            "phases_ms_max_over_ranks": phases,
            "exact_vs_single_gpu": exact_single, "exact_vs_oracle": exact_oracle,
            "oracle_checked_queries": 4, "all_results_valid": exact_all,
            "e2e": {"value": steps * B / dt, "unit": "queries/s", "h2d_bytes_per_step": B * D * 4,
                    "d2h_bytes_per_step": (2 * B * K + B) * 4, "every_step_valid": e2e_valid,
                    "path": "pinned H2D of the batch, mars_shard_query_batch_topk, one packed D2H of ids, "
                            "scores and counts (both copies on a copy stream, overlapped with the neighbouring "
                            "batches); the host checks each step's counts while the next runs"},
            "roofline": {"bound": "tensor", "kernel": "batch::gemm_kernel<kCandidates, fp16> (128 queries x "
                                                      "256 rows per tcgen05 tile)",
                         "kernel_ms": gemm_ms, "achieved": achieved, "unit": "TFLOP/s",
                         "peak": sus, "frac": achieved / sus, "peak_kind": f"{kind} bf16 GEMM, sustained",
                         "frac_of_burst": achieved / burst,
                         "flops_per_launch": 2.0 * B * (hi - lo) * D,
                         "step_tflops_per_gpu": 2.0 * B * N * D / world / (ms * 1e-3) / 1e12},
            "batch_stats_rank0": stats, "cpu_baseline": cpu}


def _sharded_graph(mb, st, N, deg, deg_cross, n_mod, rank, world, dist):
    """cmng_build split by row blocks: rank r builds rows [r*N/G, (r+1)*N/G)
    against the whole (replicated) store, then one NCCL all-gather of the
    equal-sized padded blocks gives every rank the full N x deg graph.
    Returns (graph, device ms of the build + gather, max over ranks)."""
    import torch
    lo, hi = N * rank // world, N * (rank + 1) // world
    rows_max = (N + world - 1) // world
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(dist)
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
    return nb, _max_over_ranks(dist, e0.elapsed_time(e1))


def cfg_c3(a, env):
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
    rank, world, local, dist = env["rank"], env["world"], env["local"], env["dist"]
    N, D, deg = 100_000, a.dim, 32
    E, mod, ts, _ = datagen.cluster_corpus(N, D, 100, 0.3, seed=a.seed, n_mod=4, ts_max=10.0)
    st = mb.Store(N, D, device=local)
    st.upload(E, mod, ts)
    nb, _ = _sharded_graph(mb, st, N, deg, 0, 4, rank, world, dist)
    times = []
    for _ in range(3):
        nb, ms = _sharded_graph(mb, st, N, deg, 0, 4, rank, world, dist)
        times.append(ms)
    rec = None
    if rank == 0:
        # bit-exact check of sampled rows against the oracle's exact kNN
        rows = np.arange(0, N, N // 128, dtype=np.int32)
        c = O.Corpus(E=E, ts=ts, mod=mod)
        rid, _ = O.knn(c, rows, 2 * deg)
        ref = O.cmng_select(rid, mod, rows, deg, 0, 4)
        exact = bool(np.array_equal(nb.cpu().numpy()[rows], ref))
        threads = os.cpu_count() or 1
        crow = np.arange(0, N, N // 256, dtype=np.int32)
        t0 = time.perf_counter()
        O.knn(c, crow, 2 * deg, dot_order=O.DOT_FAST, n_threads=threads)
        cdt = (time.perf_counter() - t0) * N / crow.shape[0]
        ms = statistics.median(times)
        flops = 2.0 * N * N * D
        sus, burst, kind = _tensor_peaks()
        ach = flops / world / (ms * 1e-3) / 1e12
        rec = {"workload": "c3", "metric": f"cmng_build ms (N={N}, D={D}, degree {deg})", "value": ms, "unit": "ms",
               "higher_is_better": False, "n_gpus": world, "steps": len(times), "scaling": "strong",
               "parallelism": f"row blocks x{world}" + (" + NCCL all-gather" if world > 1 else ""),
               "tflops_effective": flops / (ms * 1e-3) / 1e12,
               "roofline": {"bound": "tensor", "flops_per_build": flops, "achieved_per_gpu": ach, "unit": "TFLOP/s",
                            "peak": sus, "frac": ach / sus, "peak_kind": f"{kind} bf16 GEMM, sustained",
                            "frac_of_burst": ach / burst},
               "oracle_checked_rows": int(rows.shape[0]), "neighbours_bit_exact": exact,
               "cpu_baseline": {"value": cdt * 1e3, "unit": "ms", "cores": threads, "kind": "port",
                                "sample": f"exact kNN of {crow.shape[0]} rows against all {N} (oracle orc_knn, fast "
                                          f"dot order, {threads} threads), extrapolated x{N // crow.shape[0]}"}}
    st.close()
    return rec


def cfg_c4(a, env):
    """c4: cmng_search + cross-modal BFS.  N = 1,000,000 rows from a 1,000
    cluster mixture (sigma 0.3, 4 modalities, normalised); graph = degree-32
    kNN + 4 cross-modal bridges (degree 36, built by row blocks, untimed);
    10,000 queries, beam 64, K = 10, lambda = 0.05, BFS depth 2.  Under
    torchrun: replicas (every rank holds the corpus and the graph), the
    queries split across ranks, an NCCL all-gather of the per-rank results
    ends each step."""
    import torch
    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen
    from _util import assert_ranked_equivalent
    rank, world, local, dist = env["rank"], env["world"], env["local"], env["dist"]
    N, D, deg, K, nq = a.c4_n, a.dim, 36, 10, a.queries
    E, mod, ts, _ = datagen.cluster_corpus(N, D, 1000, 0.3, seed=a.seed, n_mod=4, ts_max=10.0)
    Q = datagen.queries(nq, D, seed=a.seed + 5)
    st = mb.Store(N, D, device=local)
    st.upload(E, mod, ts)
    nb, build_ms = _sharded_graph(mb, st, N, deg, 4, 4, rank, world, dist)
    q0, q1 = nq * rank // world, nq * (rank + 1) // world
    nql = q1 - q0
    qmax = (nq + world - 1) // world
    Qd = torch.from_numpy(np.ascontiguousarray(Q[q0:q1])).cuda()
    cfg = mb.CmngConfig(K=K, beam_width=64, max_iterations=64, time_decay_lambda=0.05)
    ctx = mb.CmngContext(qmax, K, deg, 2, N, device=local)
    ids = torch.full((qmax, K), -1, dtype=torch.int32, device="cuda")
    sc = torch.zeros((qmax, K), dtype=torch.float32, device="cuda")
    hp = torch.zeros((qmax, K), dtype=torch.int32, device="cuda")
    cnt = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    vis = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    iters = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    scored = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    bids = torch.zeros((qmax, K), dtype=torch.int32, device="cuda")     # beam-only outputs
    bsc = torch.zeros((qmax, K), dtype=torch.float32, device="cuda")
    bcnt = torch.zeros(qmax, dtype=torch.int32, device="cuda")
    if world > 1:
        all_ids = torch.empty((world * qmax, K), dtype=torch.int32, device="cuda")
        all_sc = torch.empty((world * qmax, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def step():
        ctx.search_bfs(st, nb, deg, Qd, nql, 10.0, cfg, 2, 0.5, ids, sc, cnt, d_hops=hp, d_visited=vis,
                       stream=stream.cuda_stream)
        if world > 1:
            with torch.cuda.stream(stream):
                dist.all_gather_into_tensor(all_ids, ids)
                dist.all_gather_into_tensor(all_sc, sc)

    step()
    steps = 10
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    _barrier(dist)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    for _ in range(steps):
        mb.cmng_search_batch(st, nb, deg, Qd, nql, 10.0, cfg, bids, bsc, bcnt, d_iters=iters, d_scored=scored,
                             stream=stream.cuda_stream)
    e2.record(stream)
    _barrier(dist)
    clocks = sampler.stop() if sampler else None
    ms_local = e0.elapsed_time(e1) / steps
    ms = _max_over_ranks(dist, ms_local)
    ms_fastest = -_max_over_ranks(dist, -ms_local)     # the fastest rank (load balance across ranks)
    ms_beam = _max_over_ranks(dist, e1.elapsed_time(e2) / steps)
    rows_bfs = float(vis[:nql].double().mean().item())
    rows_beam = float(scored[:nql].double().mean().item())
    bytes_q = (rows_beam + rows_bfs) * D * 4
    rec = None
    if rank == 0:
        nbh = nb.cpu().numpy()
        oc = O.Corpus(E=E, ts=ts, mod=mod, fixed_nbrs=nbh)
        gi, gs, gh, gc = ids.cpu().numpy(), sc.cpu().numpy(), hp.cpu().numpy(), cnt.cpu().numpy()
        exact = True
        n_check = 8
        for q in range(n_check):
            beam, _ = O.cmng_search(oc, nbh, Q[q0 + q], 10.0, K=K, beam_width=64, max_iterations=64, lam=0.05)
            visited = O.bfs(oc, beam["node_id"], beam["score"], None, 2, 0.5, q=Q[q0 + q], t_q=10.0, lam=0.05)
            ref = O.finalize(visited, K)
            n = int(gc[q])
            try:
                assert n == ref.shape[0]
                assert_ranked_equivalent(gi[q, :n], gs[q, :n], ref["node_id"], ref["score"], gh[q, :n], ref["hops"],
                                         rtol=2e-6, what=f"c4 query {q}")
            except AssertionError:
                exact = False
        sample = 16
        t0 = time.perf_counter()
        for q in range(sample):
            beam, _ = O.cmng_search(oc, nbh, Q[q], 10.0, K=K, beam_width=64, max_iterations=64, lam=0.05,
                                    dot_order=O.DOT_FAST)
            O.bfs(oc, beam["node_id"], beam["score"], None, 2, 0.5, q=Q[q], t_q=10.0, lam=0.05, dot_order=O.DOT_FAST)
        cdt = time.perf_counter() - t0
        peak, peak_kind = measured_peak()
        achieved = bytes_q * nql / (ms * 1e-3) / 1e9
        rec = {"workload": "c4", "metric": f"queries/s (cmng_search + BFS depth 2, N={N}, K={K})",
               "value": nq / (ms * 1e-3), "unit": "queries/s", "n_gpus": world, "steps": steps, "scaling": "strong",
               "ms_per_batch": ms, "ms_per_batch_fastest_rank": ms_fastest, "queries_per_batch": nq,
               "clocks": clocks,
               "parallelism": f"replicas x{world}, queries split" + (" + NCCL all-gather of results" if world > 1 else ""),
               "beam_only_queries_per_s": nq / (ms_beam * 1e-3), "graph_build_ms": build_ms,
               "mean_rows_scored_beam": rows_beam, "mean_nodes_visited_bfs": rows_bfs,
               "oracle_checked_queries": n_check, "exact_vs_oracle": exact,
               "roofline": {"bound": "hbm", "achieved_per_gpu": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak, "peak_kind": peak_kind,
                            "bytes_per_query": bytes_q,
                            "note": "measured row gathers per query: (beam-scored + BFS-visited rows) x D x 4 bytes"},
               "cpu_baseline": {"value": sample / cdt, "unit": "queries/s", "cores": 1, "kind": "port",
                                "sample": f"{sample} queries, oracle beam search + BFS (fast dot order), one thread, "
                                          "on the same graph"}}
    st.close()
    return rec


def run_configs(a, env):
    """Every config of the family, in the same order on every rank."""
    out = {}
    import gc
    for name, fn in (("c2", cfg_c2), ("c3", cfg_c3), ("c4", cfg_c4)):
        if name in a.skip_configs:
            continue
        t0 = time.perf_counter()
        rec = fn(a, env)
        gc.collect()
        if rec is not None:
            rec["setup_and_run_s"] = time.perf_counter() - t0
            out[name] = rec
    if env["world"] == 1:
        for name in ("c0", "c1"):
            if name in a.skip_configs:
                continue
            t0 = time.perf_counter()
            out[name] = cfg_latency(a, name)
            out[name]["setup_and_run_s"] = time.perf_counter() - t0
    return out


def run_workload(a):
    """`--workload cX`: one config's record as its own JSON line."""
    import torch
    rank, world, local = dist_env()
    if a.workload in ("c0", "c1"):
        if rank == 0:
            print(json.dumps(cfg_latency(a, a.workload)), flush=True)
        return
    torch.cuda.set_device(local)
    dist = _init_dist(local, world)
    env = {"rank": rank, "world": world, "local": local, "dist": dist}
    if a.workload == "c2":
        import mars_b200 as mb
        from mars_b200 import datagen
        E, mod, ts, imp = datagen.gaussian_rows(0, a.n, a.dim, seed=a.seed, ts_max=a.ts_max)
        st = mb.Store(a.n, a.dim, device=local)
        st.upload(E, mod, ts, imp)
        env.update({"rows": (E, mod, ts, imp), "store": st})
        rec = cfg_c2(a, env)
    elif a.workload == "c3":
        rec = cfg_c3(a, env)
    else:
        rec = cfg_c4(a, env)
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_workload(a):
    """`--impl reference --workload cX`: the CPU implementation of config X
    (the oracle port) on the host cores, rank 0 only."""
    rank, _, _ = dist_env()
    if rank != 0:
        return
    import oracle as O
    from mars_b200 import datagen
    if a.workload in ("c0", "c1"):
        D, K = a.dim, 10
        N0, lam = (2400, 0.5) if a.workload == "c0" else (10000, 1.0)
        E, mod, ts, imp = datagen.gaussian_corpus(N0, D, seed=a.seed, n_mod=4, ts_max=10.0)
        ro, ci = datagen.random_bridges(mod, 4, seed=7)
        Q = datagen.queries(256, D, seed=0x5EED0000)
        oc = O.Corpus(E=E, ts=ts, mod=mod, row_offsets=ro, col_indices=ci)
        lat = []
        for f in range(min(a.frames, 200)):
            t0 = time.perf_counter()
            O.query(oc, Q[f % 256], 10.0, top_k=K, bfs_max_hops=1, lam=lam, bfs_score_decay=0.5,
                    dot_order=O.DOT_FAST)
            lat.append(time.perf_counter() - t0)
        v = len(lat) / sum(lat)
        rec = {"impl": "reference", "workload": a.workload, "metric": "queries/s", "value": v, "unit": "queries/s",
               "p50_us": _pct(lat, 50) * 1e6, "p99_us": _pct(lat, 99) * 1e6,
               "cpu_baseline": {"value": v, "unit": "queries/s", "cores": 1, "kind": "port",
                                "sample": f"{len(lat)} queries, oracle orc_query single thread (corpus fixed)"}}
    elif a.workload == "c3":
        N, deg = 100_000, 32
        E, mod, ts, _ = datagen.cluster_corpus(N, a.dim, 100, 0.3, seed=a.seed, n_mod=4, ts_max=10.0)
        c = O.Corpus(E=E, ts=ts, mod=mod)
        rows = np.arange(0, N, max(1, N // 200), dtype=np.int32)
        t0 = time.perf_counter()
        O.knn(c, rows, 2 * deg, dot_order=O.DOT_FAST)
        full = (time.perf_counter() - t0) * N / rows.shape[0]
        rec = {"impl": "reference", "workload": "c3", "metric": "cmng_build ms", "value": full * 1e3, "unit": "ms",
               "higher_is_better": False,
               "cpu_baseline": {"value": full * 1e3, "unit": "ms", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"exact kNN of {rows.shape[0]} rows against all {N}, extrapolated "
                                          f"x{N / rows.shape[0]:.0f}"}}
    elif a.workload == "c2":
        B, K = a.batch, 100
        E, mod, ts, imp = datagen.gaussian_rows(0, a.n, a.dim, seed=a.seed, ts_max=a.ts_max)
        c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
        Qh = datagen.queries(B, a.dim, seed=a.seed + 7)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        for q in range(8):
            O.scan_topk_fast(c, Qh[q], a.ts_max, a.lam, K, use_importance=True, n_threads=threads)
        v = 8 / (time.perf_counter() - t0)
        rec = {"impl": "reference", "workload": "c2", "metric": "queries/s", "value": v, "unit": "queries/s",
               "cpu_baseline": {"value": v, "unit": "queries/s", "cores": threads, "kind": "port",
                                "sample": f"8 of the {B} queries over all {a.n} rows, K = {K}"}}
    else:
        print(json.dumps({"impl": "reference", "workload": a.workload,
                          "unavailable": "the c4 reference arm runs inside the GPU run (it needs the GPU-built graph)"}))
        return
    print(json.dumps(rec), flush=True)


def main():
    a = parse_args()
    a.skip_configs = set(x for x in a.skip_configs.split(",") if x) if isinstance(a.skip_configs, str) else set()
    if a.workload != "scan":
        if a.impl == "reference":
            run_reference_workload(a)
        else:
            run_workload(a)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_mars(a)


if __name__ == "__main__":
    main()
