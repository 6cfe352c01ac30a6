"""One rank of the row-sharded batched top-K check, launched by
tests/test_gpu_shard.py under torchrun (one process per GPU).

Rank r holds rows [r N / G, (r + 1) N / G) of a seeded corpus in its own
store and answers the same queries through mars_shard_query_batch_topk
(NCCL owned by the library).  Rank 0 also builds the whole corpus on its GPU
and answers the queries with the single-GPU mars_query_batch_topk; it writes
whether every rank's merged answer equals that, bit for bit, and whether the
answers match the CPU oracle on a few queries.
"""
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "cuda-multimodal-memory_b200"), os.path.join(ROOT, "oracle"),
          os.path.join(ROOT, "tests")):
    sys.path.insert(0, p)


def main():
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen
    from _util import assert_ranked_equivalent

    out_path = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    N, D = 300_000, 768
    lo, hi = N * rank // world, N * (rank + 1) // world
    Ef, modf, tsf, impf = datagen.gaussian_rows(0, N, D, seed=5, ts_max=600.0)
    E, mod, ts, imp = Ef[lo:hi], modf[lo:hi], tsf[lo:hi], impf[lo:hi]
    st = mb.Store(hi - lo, D, device=local)
    st.upload(E, mod, ts, imp)
    ro, ci = datagen.random_bridges(modf, 4, seed=7)      # the global graph, replicated
    uid = [mb.shard_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    cases = [(16, 10), (200, 100), (64, 256)]
    comm = mb.ShardComm(local, rank, world, uid[0], max_batch=256, max_k=256)
    bc = mb.BatchContext(hi - lo, D, max_batch=256, max_k=256, device=local)
    Qh = datagen.queries(256, D, seed=6)
    Qd = torch.from_numpy(Qh).cuda()
    got = {}
    for B, K in cases:
        ids = torch.full((B, K), -7, dtype=torch.int32, device="cuda")
        vals = torch.zeros((B, K), dtype=torch.float32, device="cuda")
        cnt = torch.zeros(B, dtype=torch.int32, device="cuda")
        comm.query_batch_topk(st, bc, Qd[:B], B, 600.0, 0.01, K, ids, vals, cnt, use_importance=True,
                              row_offset=lo)
        torch.cuda.synchronize()
        got[(B, K)] = (ids.cpu().numpy(), vals.cpu().numpy(), cnt.cpu().numpy())
    # every rank's merged answer must be the same: gather them to rank 0
    same = True
    for (B, K), (i, v, c) in got.items():
        t = torch.from_numpy(np.concatenate([i.ravel(), v.view(np.int32).ravel(), c])).cuda()
        lst = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(lst, t)
        same = same and all(torch.equal(lst[0], x) for x in lst)
    # sharded query + BFS (mars_shard_query) over the replicated global graph
    qctx = mb.QueryContext(hi - lo, D, max_k=64, device=local)
    d_ro, d_ci = torch.from_numpy(ro).cuda(), torch.from_numpy(ci).cuda()
    bfs_cases = [(0, 10, -1), (1, 10, -1), (2, 10, 1), (2, 32, -1)]
    bfs_got = {}
    for hops, K, filt in bfs_cases:
        cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=hops, time_decay_lambda=0.01, bfs_score_decay=0.5,
                                 modality_filter=filt, use_importance=True)
        bfs_got[(hops, K, filt)] = [comm.query(st, qctx, d_ro, d_ci, N, Qh[q], 600.0, cfg, row_offset=lo)
                                    for q in range(4)]
    for (hops, K, filt), res in bfs_got.items():
        flat = np.full((len(res), 4, K), -9, np.int32)     # fixed size on every rank
        for i, r in enumerate(res):
            n = len(r)
            flat[i, :, :n] = np.stack([r["node_id"], r["score"].view(np.int32), r["modality"], r["hops"]])
        flat = flat.ravel()
        t = torch.from_numpy(flat).cuda()
        lst = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(lst, t)
        same = same and all(torch.equal(lst[0], x) for x in lst)
    report = {"world": world, "ranks_agree": bool(same)}
    if rank == 0:
        full = mb.Store(N, D, device=local)
        full.upload(Ef, modf, tsf, impf, ro, ci)
        fctx = mb.QueryContext(N, D, max_k=64, device=local)
        bfs_exact = True
        for (hops, K, filt), res in bfs_got.items():
            cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=hops, time_decay_lambda=0.01, bfs_score_decay=0.5,
                                     modality_filter=filt, use_importance=True)
            for q in range(4):
                ref = fctx.query(full, Qh[q], 600.0, cfg)
                g = res[q]
                bfs_exact = bfs_exact and len(g) == len(ref) and np.array_equal(g["node_id"], ref["node_id"]) and \
                    np.array_equal(g["score"].view(np.int32), ref["score"].view(np.int32)) and \
                    np.array_equal(g["hops"], ref["hops"]) and np.array_equal(g["modality"], ref["modality"])
        report["bfs_equal_to_single_gpu"] = bool(bfs_exact)
        bcf = mb.BatchContext(N, D, max_batch=256, max_k=256, device=local)
        exact, oracle_ok = True, True
        corpus = O.Corpus(E=Ef, ts=tsf, mod=modf, imp=impf)
        for B, K in cases:
            ids = torch.empty((B, K), dtype=torch.int32, device="cuda")
            vals = torch.empty((B, K), dtype=torch.float32, device="cuda")
            cnt = torch.zeros(B, dtype=torch.int32, device="cuda")
            bcf.query_batch_topk(full, Qd[:B], B, 600.0, 0.01, K, ids, vals, cnt, use_importance=True)
            torch.cuda.synchronize()
            gi, gv, gc = got[(B, K)]
            exact = exact and np.array_equal(gi, ids.cpu().numpy()) and \
                np.array_equal(gv.view(np.int32), vals.cpu().numpy().view(np.int32)) and \
                np.array_equal(gc, cnt.cpu().numpy())
            oi, ov = O.query_batch_topk(corpus, Qh[:2], 600.0, 0.01, K, use_importance=True)
            try:
                for b in range(2):
                    assert_ranked_equivalent(gi[b], gv[b], oi[b], ov[b], what=f"B={B} K={K} query {b}")
            except AssertionError:
                oracle_ok = False
        report.update({"equal_to_single_gpu": bool(exact), "oracle_ok": bool(oracle_ok)})
        with open(out_path, "w") as f:
            json.dump(report, f)
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
