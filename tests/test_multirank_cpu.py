"""Host-side logic of the row-sharded path with world_size 2 on CPU (gloo).

Each rank builds its shard with mars_b200.datagen.gaussian_rows, computes the
shard's top-K with the oracle (standing in for mars_scan_topk on the GPU),
offsets ids by the shard start, all-gathers the [Q][K] lists into the
rank-major [world][Q][K] layout that mars_topk_merge_batch reads, and merges.
The merged lists must equal the single-process top-K over the whole corpus.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

N, D, K, Q = 3001, 64, 7, 5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _merge_rank_major(gids, gvals, world, Qn, K):
    """CPU statement of mars_topk_merge_batch: list l of query q at (l*Q+q)*K."""
    out_i = np.full((Qn, K), -1, np.int32)
    out_v = np.full((Qn, K), -np.inf, np.float32)
    for q in range(Qn):
        cand = []
        for l in range(world):
            for k in range(K):
                i = int(gids[l, q, k])
                if i >= 0:
                    cand.append((-float(gvals[l, q, k]), i))
        cand.sort()
        for j, (nv, i) in enumerate(cand[:K]):
            out_i[q, j] = i
            out_v[q, j] = -nv
    return out_i, out_v


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cuda-multimodal-memory_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle as O
    from mars_b200 import datagen
    lo, hi = N * rank // world, N * (rank + 1) // world
    E, mod, ts, imp = datagen.gaussian_rows(lo, hi, D, seed=9, ts_max=600.0)
    Qm = datagen.queries(Q, D, seed=10)
    c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    ids = np.full((Q, K), -1, np.int32)
    vals = np.full((Q, K), -np.inf, np.float32)
    for q in range(Q):
        s = O.fused_scores(c, Qm[q], 600.0, 0.01, use_importance=True)
        i, v = O.topk(s, mod, -1, K)
        ids[q, :len(i)] = i + lo        # global ids
        vals[q, :len(v)] = v
    # gloo has no all_gather_into_tensor; the stacked list is the same
    # rank-major [world][Q][K] layout NCCL's all_gather_into_tensor produces
    gl_i = [torch.empty((Q, K), dtype=torch.int32) for _ in range(world)]
    gl_v = [torch.empty((Q, K), dtype=torch.float32) for _ in range(world)]
    dist.all_gather(gl_i, torch.from_numpy(ids))
    dist.all_gather(gl_v, torch.from_numpy(vals))
    gids = torch.stack(gl_i).numpy()
    gvals = torch.stack(gl_v).numpy()
    mi, mv = _merge_rank_major(gids, gvals, world, Q, K)
    if rank == 0:
        np.savez(out_path, ids=mi, vals=mv)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_topk_merge_equals_whole_corpus(tmp_path, world):
    out = str(tmp_path / "merged.npz")
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, join=True,
                       start_method="spawn")
    z = np.load(out)
    import oracle as O
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_rows(0, N, D, seed=9, ts_max=600.0)
    Qm = datagen.queries(Q, D, seed=10)
    c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    for q in range(Q):
        s = O.fused_scores(c, Qm[q], 600.0, 0.01, use_importance=True)
        i, v = O.topk(s, mod, -1, K)
        assert np.array_equal(z["ids"][q], i)
        assert np.array_equal(z["vals"][q], v)


def test_shards_union_equals_whole_corpus():
    from mars_b200 import datagen
    full = datagen.gaussian_rows(0, 70_000, 16, seed=3)
    for world in (2, 3, 8):
        parts = [datagen.gaussian_rows(70_000 * r // world, 70_000 * (r + 1) // world, 16, seed=3)
                 for r in range(world)]
        for k in range(4):
            assert np.array_equal(np.concatenate([p[k] for p in parts]), full[k])


# ---------------------------------------------------------------------------
# Row-block kNN-graph build (bench.py _sharded_graph): rank r builds rows
# [r*N/G, (r+1)*N/G) against all rows, pads its block to ceil(N/G) rows and
# all-gathers; trimming the padding reproduces the whole graph.
NG, DG, DEG = 301, 32, 6


def _graph_worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cuda-multimodal-memory_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle as O
    from mars_b200 import datagen
    E, mod, ts, _ = datagen.cluster_corpus(NG, DG, 7, 0.3, seed=4, n_mod=4, ts_max=10.0)
    lo, hi = NG * rank // world, NG * (rank + 1) // world
    rows_max = (NG + world - 1) // world
    rows = np.arange(lo, hi, dtype=np.int32)
    rid, _ = O.knn(O.Corpus(E=E, ts=ts, mod=mod), rows, 2 * DEG)
    block = np.full((rows_max, DEG), -1, np.int32)
    block[:hi - lo] = O.cmng_select(rid, mod, rows, DEG, 2, 4)
    got = [torch.empty((rows_max, DEG), dtype=torch.int32) for _ in range(world)]
    dist.all_gather(got, torch.from_numpy(block))
    allb = torch.cat(got)
    nb = torch.cat([allb[r * rows_max: r * rows_max + (NG * (r + 1) // world - NG * r // world)]
                    for r in range(world)])
    if rank == 0:
        np.save(out_path, nb.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_block_graph_equals_whole_graph(tmp_path, world):
    out = str(tmp_path / "graph.npy")
    mp.start_processes(_graph_worker, args=(world, _free_port(), out), nprocs=world, join=True,
                       start_method="spawn")
    got = np.load(out)
    import oracle as O
    from mars_b200 import datagen
    E, mod, ts, _ = datagen.cluster_corpus(NG, DG, 7, 0.3, seed=4, n_mod=4, ts_max=10.0)
    rows = np.arange(NG, dtype=np.int32)
    rid, _ = O.knn(O.Corpus(E=E, ts=ts, mod=mod), rows, 2 * DEG)
    assert np.array_equal(got, O.cmng_select(rid, mod, rows, DEG, 2, 4))


def test_query_split_covers_every_query_once():
    for nq in (1, 7, 10000, 10001):
        for world in (1, 2, 3, 8):
            seen = np.concatenate([np.arange(nq * r // world, nq * (r + 1) // world) for r in range(world)])
            assert np.array_equal(seen, np.arange(nq))
            assert max(nq * (r + 1) // world - nq * r // world for r in range(world)) <= (nq + world - 1) // world


# ---------------------------------------------------------------------------
# Row shards with a shared short-list threshold and a shared pruning bound
# (mars_shard_query_batch_topk), restated on the CPU with approximate scores
# = exact + noise within a stated margin (lower / upper bounds = approx -+
# margin):
#  1. every rank sends its 16 best sampled lower bounds per query and its
#     (sampled rows, rows); one all-gather; every rank takes the same
#     threshold theta = the j-th largest of the union, j = ceil(mu + 5 sqrt(mu)
#     + 3), mu = K x sampled rows / rows over all ranks;
#  2. candidates: rows whose upper bound reaches theta;
#  3. per query a record (count of candidates with lower bound >= theta, K-th
#     and ceil(K / world)-th largest candidate lower bound, -inf where fewer)
#     and a failure flag; one all-gather;
#  4. the counts over all ranks certify every rank's short list (>= K);
#     the bound max(theta, largest K-th, smallest ceil(K / world)-th) is a
#     lower bound of the global K-th score, so only candidates whose upper
#     bound reaches it are rescored exactly; an uncertified query is scanned
#     exactly on every rank;
#  5. local top-K as 64-bit rank keys (score, then id), one all-gather, a
#     per-query selection.  A rank that flags a failure makes every rank's
#     answer invalid (count -1).
NS, DS, KS, QS, MARGIN, SAMPLE_STRIDE, JMAX = 4001, 32, 9, 6, 2e-3, 7, 16


def _f2key(v):
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    return np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)


def _rank_keys(ids, vals):
    k = (_f2key(vals) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids.astype(np.int64).astype(np.uint64))
    return np.where(ids >= 0, k, np.uint64(0)).astype(np.uint64)


def _key_decode(k):
    hi = (k >> np.uint64(32)).astype(np.uint32)
    u = np.where(hi & 0x80000000, hi & 0x7FFFFFFF, ~hi).astype(np.uint32)
    ids = (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64).astype(np.int32)
    return ids, u.view(np.float32)


def _kth(v, k):
    v = np.sort(np.asarray(v, np.float32))[::-1]
    return np.float32(v[k - 1]) if v.size >= k else np.float32(-np.inf)


def _bound_worker(rank, world, port, out_path, fail_rank, theta_shift):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import math
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cuda-multimodal-memory_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle as O
    from mars_b200 import datagen
    lo, hi = NS * rank // world, NS * (rank + 1) // world
    E, mod, ts, imp = datagen.gaussian_rows(lo, hi, DS, seed=21, ts_max=600.0)
    Qm = datagen.queries(QS, DS, seed=22)
    c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    rng = np.random.default_rng(100 + rank)
    exact = np.stack([O.fused_scores(c, Qm[q], 600.0, 0.01, use_importance=True) for q in range(QS)])
    approx = exact + rng.uniform(-MARGIN, MARGIN, exact.shape).astype(np.float32)
    lob, hib = approx - MARGIN, approx + MARGIN
    n = hi - lo
    # 1. the threshold record: 16 best sampled lower bounds, sampled rows, rows
    samp = np.arange(0, n, SAMPLE_STRIDE)
    top = np.full((QS, JMAX), -np.inf, np.float32)
    for q in range(QS):
        v = np.sort(lob[q, samp])[::-1][:JMAX]
        top[q, :v.size] = v
    rec = torch.from_numpy(np.concatenate([top.ravel(), [samp.size, n]]).astype(np.float64))
    got = [torch.empty_like(rec) for _ in range(world)]
    dist.all_gather(got, rec)
    recs = torch.stack(got).numpy()
    srows, rows = recs[:, -2].sum(), recs[:, -1].sum()
    mu = KS * srows / rows
    j = max(1, min(JMAX, int(math.ceil(mu + 5.0 * math.sqrt(mu) + 3.0))))
    union = recs[:, :-2].reshape(world, QS, JMAX)
    theta = np.array([_kth(union[:, q, :].ravel(), j) for q in range(QS)], np.float32) + np.float32(theta_shift)
    # 2-3. candidates and the bound record
    m = (KS + world - 1) // world
    cand = [np.nonzero(hib[q] >= theta[q])[0] for q in range(QS)]
    cnt = np.array([(lob[q, cand[q]] >= theta[q]).sum() for q in range(QS)], np.float64)
    kth = np.array([_kth(lob[q, cand[q]], KS) for q in range(QS)], np.float64)
    mth = np.array([_kth(lob[q, cand[q]], m) for q in range(QS)], np.float64)
    flag = 1.0 if rank == fail_rank else 0.0
    rec2 = torch.from_numpy(np.concatenate([cnt, kth, mth, [flag]]))
    got2 = [torch.empty_like(rec2) for _ in range(world)]
    dist.all_gather(got2, rec2)
    r2 = torch.stack(got2).numpy()
    failed = r2[:, -1].max()
    total = r2[:, :QS].sum(axis=0)
    bound = np.maximum(np.maximum(r2[:, QS:2 * QS].max(axis=0), r2[:, 2 * QS:3 * QS].min(axis=0)), theta)
    # 4. exact scores of the rows that can still place (all rows when uncertified)
    ids = np.full((QS, KS), -1, np.int32)
    vals = np.full((QS, KS), -np.inf, np.float32)
    kept, uncertified = 0, 0
    for q in range(QS):
        if total[q] >= KS:
            rowsq = cand[q][hib[q, cand[q]] >= np.float32(bound[q])]
        else:
            rowsq = np.arange(n)
            uncertified += 1
        kept += rowsq.size
        order = sorted(rowsq.tolist(), key=lambda r: (-float(exact[q, r]), r))[:KS]
        ids[q, :len(order)] = np.asarray(order, np.int32) + lo
        vals[q, :len(order)] = exact[q, order]
    # 5. keys, all-gather, merge
    keys = torch.from_numpy(_rank_keys(ids, vals).view(np.int64))
    got3 = [torch.empty_like(keys) for _ in range(world)]
    dist.all_gather(got3, keys)
    allk = torch.stack(got3).numpy().view(np.uint64)           # [world][Q][K]
    out_i = np.full((QS, KS), -1, np.int32)
    out_v = np.full((QS, KS), -np.inf, np.float32)
    outc = np.zeros(QS, np.int32)
    for q in range(QS):
        if failed > 0:
            outc[q] = -1
            continue
        k = np.sort(allk[:, q, :].ravel())[::-1]
        k = k[k != 0][:KS]
        out_i[q, :k.size], out_v[q, :k.size] = _key_decode(k)
        outc[q] = k.size
    stats = torch.tensor([kept, uncertified, sum(x.size for x in cand)], dtype=torch.int64)
    dist.all_reduce(stats)
    if rank == 0:
        np.savez(out_path, ids=out_i, vals=out_v, cnt=outc, kept=int(stats[0]), uncertified=int(stats[1]),
                 cand=int(stats[2]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,fail_rank,theta_shift", [(2, -1, 0.0), (3, -1, 0.0), (4, -1, 0.0), (2, 1, 0.0),
                                                         (3, -1, 10.0)])
def test_shared_threshold_shards_equal_whole_corpus(tmp_path, world, fail_rank, theta_shift):
    out = str(tmp_path / "bound.npz")
    mp.start_processes(_bound_worker, args=(world, _free_port(), out, fail_rank, theta_shift), nprocs=world,
                       join=True, start_method="spawn")
    z = np.load(out)
    if fail_rank >= 0:
        assert np.all(z["cnt"] == -1) and np.all(z["ids"] == -1)
        return
    import oracle as O
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_rows(0, NS, DS, seed=21, ts_max=600.0)
    Qm = datagen.queries(QS, DS, seed=22)
    c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    for q in range(QS):
        s = O.fused_scores(c, Qm[q], 600.0, 0.01, use_importance=True)
        i, v = O.topk(s, mod, -1, KS)
        assert np.array_equal(z["ids"][q], i)
        assert np.array_equal(z["vals"][q], v)
        assert z["cnt"][q] == KS
    if theta_shift > 0:
        # a threshold above every score certifies nothing: every query is
        # answered by the exact scans, still exactly
        assert z["uncertified"] == world * QS
        return
    assert z["uncertified"] == 0
    # the shared threshold and bound prune: far fewer rows than world x K per
    # query are rescored, and the shards together short-list about what one
    # corpus-wide sample would
    assert z["kept"] < world * KS * QS
    assert z["cand"] < 40 * KS * QS


# ---------------------------------------------------------------------------
# Sharded query with BFS (mars_shard_query): every rank holds a row shard and
# the whole graph; the seeds are the merged local top-K; every rank expands
# each level itself over the graph (the level sorted by id), each node's own
# score comes from the rank that holds its row through an all-reduce (max,
# -inf elsewhere), and a node scores fmaxf(best parent * decay, own * 0.8).
# The answer must be the single-process oracle query's.
NB, DB, KB = 2001, 32, 8


def _bfs_worker(rank, world, port, out_path, hops, filt):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cuda-multimodal-memory_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle as O
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_rows(0, NB, DB, seed=31, ts_max=10.0)
    ro, ci = datagen.random_bridges(mod, 3, seed=7)
    lo, hi = NB * rank // world, NB * (rank + 1) // world
    shard = O.Corpus(E=E[lo:hi], ts=ts[lo:hi], mod=mod[lo:hi], imp=imp[lo:hi])
    q = datagen.queries(1, DB, seed=32)[0]
    own_local = O.fused_scores(shard, q, 10.0, 0.5, modality_filter=filt, use_importance=True)
    li, lv = O.topk(own_local, mod[lo:hi], filt, KB)
    keys = np.zeros(KB, np.uint64)
    keys[:len(li)] = _rank_keys(li.astype(np.int32) + lo, lv)
    got = [torch.empty(KB, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(got, torch.from_numpy(keys.view(np.int64)))
    allk = np.sort(torch.cat(got).numpy().view(np.uint64))[::-1]
    allk = allk[allk != 0][:KB]
    seed_ids, seed_vals = _key_decode(allk)
    score = {int(i): np.float32(v) for i, v in zip(seed_ids, seed_vals)}
    hop_of = {int(i): 0 for i in seed_ids}
    frontier = [int(i) for i in seed_ids]
    decay = np.float32(0.5)
    for h in range(1, hops + 1):
        best = {}
        for p in frontier:
            for v in ci[ro[p]:ro[p + 1]].tolist():
                if v in score:
                    continue
                c = np.float32(score[p] * decay)
                best[v] = max(best.get(v, np.float32(-np.inf)), c)
        level = sorted(best)
        own = np.full(len(level), -np.inf, np.float32)
        for j, v in enumerate(level):
            if lo <= v < hi:
                own[j] = own_local[v - lo]
        t = torch.from_numpy(own)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        for j, v in enumerate(level):
            score[v] = np.float32(max(best[v], np.float32(t[j].item()) * np.float32(0.8)))
            hop_of[v] = h
        frontier = level
    final = sorted(score, key=lambda v: (-float(score[v]), v))[:KB]
    if rank == 0:
        np.savez(out_path, ids=np.asarray(final, np.int32),
                 vals=np.asarray([score[v] for v in final], np.float32),
                 hops=np.asarray([hop_of[v] for v in final], np.int32))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,hops,filt", [(2, 1, -1), (3, 2, -1), (2, 2, 1)])
def test_sharded_bfs_query_equals_single_process_query(tmp_path, world, hops, filt):
    out = str(tmp_path / "sbfs.npz")
    mp.start_processes(_bfs_worker, args=(world, _free_port(), out, hops, filt), nprocs=world, join=True,
                       start_method="spawn")
    z = np.load(out)
    import oracle as O
    from mars_b200 import datagen
    from _util import assert_ranked_equivalent
    E, mod, ts, imp = datagen.gaussian_rows(0, NB, DB, seed=31, ts_max=10.0)
    ro, ci = datagen.random_bridges(mod, 3, seed=7)
    q = datagen.queries(1, DB, seed=32)[0]
    ref = O.query(O.Corpus(E=E, ts=ts, mod=mod, imp=imp, row_offsets=ro, col_indices=ci), q, 10.0, top_k=KB,
                  bfs_max_hops=hops, lam=0.5, bfs_score_decay=0.5, modality_filter=filt, use_importance=True)
    assert_ranked_equivalent(z["ids"], z["vals"], ref["node_id"], ref["score"], z["hops"], ref["hops"],
                             rtol=0, atol=0, what="sharded BFS")
