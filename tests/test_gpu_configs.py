"""Parity at the configurations' own shapes (the other GPU tests use smaller
corpora).

* c3 shape: N = 100,000 rows, D = 768, a 100-cluster mixture (sigma 0.3),
  out-degree 32, no bridges: the kNN-graph build's neighbour lists of
  sampled rows equal the oracle's exact kNN + selection bit for bit.
* c4-like shape: N = 200,000 rows from a 200-cluster mixture, 4
  modalities, degree 32 + 4 cross-modal bridges (36): sampled neighbour
  lists bit-exact against the oracle; beam search (width 64, 64 iterations)
  + BFS depth 2 answers of sampled queries equal the oracle's beam search +
  canonical BFS on the same graph.
* c2 shape: B = 1024 queries, K = 100 over N = 400,000 rows: the batched
  tensor-core path equals the per-query fp32 scans bit for bit, and sampled
  queries equal the oracle.
"""
import numpy as np
import pytest

import oracle as O
from _util import assert_ranked_equivalent

pytestmark = pytest.mark.gpu


def _graph(mb, torch, E, mod, ts, deg, cross):
    N, D = E.shape
    st = mb.Store(N, D)
    st.upload(E, mod, ts)
    nb = torch.empty((N, deg), dtype=torch.int32, device="cuda")
    mb.cmng_build(st, deg, cross, 4, nb)
    torch.cuda.synchronize()
    return st, nb


def test_c3_shape_knn_graph_bit_exact_on_sampled_rows():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    N, D, deg = 100_000, 768, 32
    E, mod, ts, _ = datagen.cluster_corpus(N, D, 100, 0.3, seed=42, n_mod=4, ts_max=10.0)
    st, nb = _graph(mb, torch, E, mod, ts, deg, 0)
    rows = np.arange(7, N, N // 300, dtype=np.int32)
    rid, _ = O.knn(O.Corpus(E=E, ts=ts, mod=mod), rows, 2 * deg)
    ref = O.cmng_select(rid, mod, rows, deg, 0, 4)
    got = nb.cpu().numpy()[rows]
    assert np.array_equal(got, ref), f"{int((got != ref).any(axis=1).sum())} of {rows.shape[0]} rows differ"


def test_c4_shape_graph_and_search_bfs_match_oracle():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    N, D, deg, K, hops = 200_000, 768, 36, 10, 2
    E, mod, ts, _ = datagen.cluster_corpus(N, D, 200, 0.3, seed=7, n_mod=4, ts_max=10.0)
    st, nb = _graph(mb, torch, E, mod, ts, deg, 4)
    nbh = nb.cpu().numpy()
    rows = np.arange(3, N, N // 200, dtype=np.int32)
    oc = O.Corpus(E=E, ts=ts, mod=mod, fixed_nbrs=nbh)
    rid, _ = O.knn(oc, rows, 2 * deg)
    assert np.array_equal(nbh[rows], O.cmng_select(rid, mod, rows, deg, 4, 4))

    nq = 64
    Q = datagen.queries(nq, D, seed=8)
    Q[:32] = E[np.arange(32) * 997] + 0.05 * Q[:32]      # half the queries near stored rows
    Qd = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    cfg = mb.CmngConfig(K=K, beam_width=64, max_iterations=64, time_decay_lambda=0.05)
    ctx = mb.CmngContext(nq, K, deg, hops, N)
    ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    hp = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    cnt = torch.empty(nq, dtype=torch.int32, device="cuda")
    vis = torch.empty(nq, dtype=torch.int32, device="cuda")
    ctx.search_bfs(st, nb, deg, Qd, nq, 10.0, cfg, hops, 0.5, ids, sc, cnt, d_hops=hp, d_visited=vis)
    torch.cuda.synchronize()
    gi, gs, gh, gc, gv = (t.cpu().numpy() for t in (ids, sc, hp, cnt, vis))
    for q in range(0, nq, 2):
        beam, _ = O.cmng_search(oc, nbh, Q[q], 10.0, K=K, beam_width=64, max_iterations=64, lam=0.05)
        visited = O.bfs(oc, beam["node_id"], beam["score"], None, hops, 0.5, q=Q[q], t_q=10.0, lam=0.05)
        assert int(gv[q]) == visited.shape[0], f"query {q}: visited {gv[q]} vs {visited.shape[0]}"
        ref = O.finalize(visited, K)
        n = int(gc[q])
        assert n == ref.shape[0]
        assert_ranked_equivalent(gi[q, :n], gs[q, :n], ref["node_id"], ref["score"], gh[q, :n], ref["hops"],
                                 rtol=2e-6, what=f"query {q}")


def test_c2_shape_batch_equals_scans_and_oracle():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    N, D, B, K = 400_000, 768, 1024, 100
    E, mod, ts, imp = datagen.gaussian_rows(0, N, D, seed=17, ts_max=600.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    Qh = datagen.queries(B, D, seed=18)
    Qd = torch.from_numpy(Qh).cuda()
    bc = mb.BatchContext(N, D, max_batch=B, max_k=K)
    ctx = mb.QueryContext(N, D, max_k=K)
    ids = torch.empty((B, K), dtype=torch.int32, device="cuda")
    vals = torch.empty((B, K), dtype=torch.float32, device="cuda")
    bc.query_batch_topk(st, Qd, B, 600.0, 0.01, K, ids, vals, use_importance=True)
    stats = bc.last_stats()
    assert stats["path"] == 2
    rids = torch.empty((B, K), dtype=torch.int32, device="cuda")
    rvals = torch.empty((B, K), dtype=torch.float32, device="cuda")
    for b0 in range(0, B, 64):
        ctx.scan_topk_multi(st, Qd[b0:b0 + 64], 64, 600.0, 0.01, K, rids[b0:b0 + 64], rvals[b0:b0 + 64],
                            use_importance=True)
    torch.cuda.synchronize()
    assert torch.equal(ids, rids)
    assert torch.equal(vals.view(torch.int32), rvals.view(torch.int32))
    oi, ov = O.query_batch_topk(O.Corpus(E=E, ts=ts, mod=mod, imp=imp), Qh[:6], 600.0, 0.01, K,
                                use_importance=True)
    gi, gv = ids.cpu().numpy(), vals.cpu().numpy()
    for q in range(6):
        assert_ranked_equivalent(gi[q], gv[q], oi[q], ov[q], what=f"query {q}")
