"""GPU parity of the fused scan, BFS and the whole query pipeline against the
CPU oracle.  All calls go through the C ABI (mars_b200 -> libmars_b200.so).

Bars:
  * the fused dot product is bit-exact (canonical order on both sides;
    lambda = 0 makes the decay weight exactly 1);
  * fused scores with decay agree to 1e-6 relative (__expf on the device,
    expf on the host);
  * top-K / query results agree up to near-ties (tests/_util.py);
  * given identical per-row scores, the BFS output is bit-exact.
"""
import json
import os

import numpy as np
import pytest

import oracle as O
from _util import assert_ranked_equivalent, assert_topk_matches_scores, close, load_golden

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def mb():
    import mars_b200
    return mars_b200


def make_corpus(N, D, seed=0, graph=True, importance=True, n_mod=4, ts_max=10.0):
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=seed, n_mod=n_mod, ts_max=ts_max,
                                              importance=importance)
    ro = ci = None
    if graph:
        ro, ci = datagen.random_bridges(mod, 4, seed=seed + 1)
    return E, mod, ts, imp, ro, ci


def build(mb, E, mod, ts, imp, ro, ci, capacity=None, slack=0, max_k=128):
    N, D = E.shape
    st = mb.Store(capacity or max(N, 1), D, edge_slack=slack)
    st.upload(E, mod, ts, imp, ro, ci)
    ctx = mb.QueryContext(capacity or max(N, 1), D, max_k=max_k)
    return st, ctx


def oracle_corpus(E, mod, ts, imp, ro, ci, extra=None, extra_cnt=None):
    return O.Corpus(E=E, ts=ts, mod=mod, imp=imp, row_offsets=ro, col_indices=ci,
                    extra_nbrs=extra, extra_cnt=extra_cnt)


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---------------------------------------------------------------------------
@pytest.mark.parametrize("D", [768, 64, 100, 1024, 98])
def test_fused_dot_bit_exact(torch_mod, mb, D):
    torch = torch_mod
    E, mod, ts, imp, _, _ = make_corpus(3001, D, seed=D, graph=False)
    st, ctx = build(mb, E, mod, ts, imp, None, None)
    q = np.random.default_rng(1).standard_normal(D).astype(np.float32)
    qp = np.zeros((D + 3) // 4 * 4, np.float32)
    qp[:D] = q
    out = torch.empty(E.shape[0], dtype=torch.float32, device="cuda")
    if D % 4:
        with pytest.raises(mb.MarsError):
            ctx.debug_fused_scores(st, dev(torch, qp), 5.0, 0.0, out)
        return
    ctx.debug_fused_scores(st, dev(torch, qp), 5.0, 0.0, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ref = O.fused_scores(oracle_corpus(E, mod, ts, imp, None, None), q, 5.0, 0.0)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("use_imp", [False, True])
@pytest.mark.parametrize("filt", [-1, 2])
def test_fused_scores_with_decay(torch_mod, mb, use_imp, filt):
    torch = torch_mod
    E, mod, ts, imp, _, _ = make_corpus(4099, 768, seed=3, graph=False)
    st, ctx = build(mb, E, mod, ts, imp, None, None)
    q = np.random.default_rng(2).standard_normal(768).astype(np.float32)
    out = torch.empty(E.shape[0], dtype=torch.float32, device="cuda")
    ctx.debug_fused_scores(st, dev(torch, q), 10.0, 0.5, out, modality_filter=filt,
                           use_importance=use_imp)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ref = O.fused_scores(oracle_corpus(E, mod, ts, imp, None, None), q, 10.0, 0.5,
                         modality_filter=filt, use_importance=use_imp)
    assert np.all(close(got, ref, rtol=1e-6, atol=1e-9))
    if filt >= 0:
        assert np.all(got[mod != filt] == -np.finfo(np.float32).max)


@pytest.mark.parametrize("K", [1, 10, 31, 32, 33, 64, 100, 128])
def test_scan_topk_matches_oracle(torch_mod, mb, K):
    torch = torch_mod
    E, mod, ts, imp, _, _ = make_corpus(20011, 768, seed=K, graph=False)
    st, ctx = build(mb, E, mod, ts, imp, None, None)
    q = np.random.default_rng(K).standard_normal(768).astype(np.float32)
    ids = torch.empty(K, dtype=torch.int32, device="cuda")
    vals = torch.empty(K, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.scan_topk(st, dev(torch, q), 10.0, 0.5, K, ids, vals, cnt, use_importance=True)
    torch.cuda.synchronize()
    assert int(cnt.item()) == K
    ref = O.fused_scores(oracle_corpus(E, mod, ts, imp, None, None), q, 10.0, 0.5,
                         use_importance=True)
    assert_topk_matches_scores(ids.cpu().numpy(), vals.cpu().numpy(), ref, what=f"K={K}")


@pytest.mark.parametrize("N,K", [(1, 10), (5, 10), (31, 32), (33, 64), (100, 128), (257, 7)])
def test_scan_topk_small_and_ragged(torch_mod, mb, N, K):
    torch = torch_mod
    E, mod, ts, imp, _, _ = make_corpus(N, 768, seed=N, graph=False)
    st, ctx = build(mb, E, mod, ts, imp, None, None)
    q = np.random.default_rng(N).standard_normal(768).astype(np.float32)
    ids = torch.empty(K, dtype=torch.int32, device="cuda")
    vals = torch.empty(K, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.scan_topk(st, dev(torch, q), 10.0, 0.5, K, ids, vals, cnt)
    torch.cuda.synchronize()
    n = int(cnt.item())
    assert n == min(N, K)
    ids_h, vals_h = ids.cpu().numpy(), vals.cpu().numpy()
    assert np.all(ids_h[n:] == -1) and np.all(np.isneginf(vals_h[n:]))
    ref = O.fused_scores(oracle_corpus(E, mod, ts, imp, None, None), q, 10.0, 0.5)
    assert_topk_matches_scores(ids_h[:n], vals_h[:n], ref, what=f"N={N} K={K}")


def test_scan_modality_filter_fewer_rows_than_k(torch_mod, mb):
    torch = torch_mod
    E, mod, ts, imp, _, _ = make_corpus(300, 768, seed=9, graph=False)
    mod[:] = 0
    mod[[5, 77, 123]] = 3
    st, ctx = build(mb, E, mod, ts, imp, None, None)
    q = np.random.default_rng(9).standard_normal(768).astype(np.float32)
    ids = torch.empty(10, dtype=torch.int32, device="cuda")
    vals = torch.empty(10, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.scan_topk(st, dev(torch, q), 10.0, 0.5, 10, ids, vals, cnt, modality_filter=3)
    torch.cuda.synchronize()
    assert int(cnt.item()) == 3
    assert set(ids.cpu().numpy()[:3].tolist()) == {5, 77, 123}


# ---------------------------------------------------------------------------
@pytest.mark.parametrize("hops", [0, 1, 2, 3])
@pytest.mark.parametrize("K", [10, 50])
def test_query_pipeline_matches_oracle(torch_mod, mb, hops, K):
    E, mod, ts, imp, ro, ci = make_corpus(6007, 768, seed=11 + hops)
    st, ctx = build(mb, E, mod, ts, imp, ro, ci)
    oc = oracle_corpus(E, mod, ts, imp, ro, ci)
    rng = np.random.default_rng(5)
    for qi in range(3):
        q = rng.standard_normal(768).astype(np.float32)
        q /= np.linalg.norm(q)
        cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=hops, time_decay_lambda=0.5,
                                 bfs_score_decay=0.5, use_importance=bool(qi % 2))
        got = ctx.query(st, q, 10.0, cfg)
        ref = O.query(oc, q, 10.0, top_k=K, bfs_max_hops=hops, lam=0.5, bfs_score_decay=0.5,
                      use_importance=bool(qi % 2))
        assert_ranked_equivalent(got["node_id"], got["score"], ref["node_id"], ref["score"],
                                 got["hops"], ref["hops"], what=f"hops={hops} q{qi}")
        assert np.array_equal(got["modality"], mod[got["node_id"]])


@pytest.mark.parametrize("hops", [1, 2, 3])
def test_bfs_bit_exact_given_scores(torch_mod, mb, hops):
    """With the device's own per-row scores as input, the oracle BFS +
    finalize reproduces the device result bit for bit."""
    torch = torch_mod
    E, mod, ts, imp, ro, ci = make_corpus(5003, 768, seed=21 + hops)
    st, ctx = build(mb, E, mod, ts, imp, ro, ci)
    oc = oracle_corpus(E, mod, ts, imp, ro, ci)
    q = np.random.default_rng(hops).standard_normal(768).astype(np.float32)
    K = 16
    out = torch.empty(E.shape[0], dtype=torch.float32, device="cuda")
    ctx.debug_fused_scores(st, dev(torch, q), 10.0, 0.3, out, use_importance=True)
    torch.cuda.synchronize()
    final = out.cpu().numpy()
    cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=hops, time_decay_lambda=0.3,
                             bfs_score_decay=0.5, use_importance=True)
    got, stats = ctx.query(st, q, 10.0, cfg, with_stats=True)
    ids, vals = O.topk(final, mod, -1, K)
    visited = O.bfs(oc, ids, vals, final, hops, 0.5)
    assert stats["nodes_visited"] == visited.shape[0]
    ref = O.finalize(visited, K)
    assert np.array_equal(got["node_id"], ref["node_id"])
    assert np.array_equal(got["hops"], ref["hops"])
    assert np.array_equal(got["score"].view(np.uint32), ref["score"].view(np.uint32))


def test_graph_replay_equals_direct_launch(torch_mod, mb):
    E, mod, ts, imp, ro, ci = make_corpus(4000, 768, seed=31)
    st, ctx = build(mb, E, mod, ts, imp, ro, ci)
    ctx2 = mb.QueryContext(4000, 768, max_k=64, use_graph=False)
    rng = np.random.default_rng(7)
    cfg = mb.RetrievalConfig(top_k=10, bfs_max_hops=2, time_decay_lambda=0.5)
    for _ in range(20):   # many epochs on the same context
        q = rng.standard_normal(768).astype(np.float32)
        a = ctx.query(st, q, 10.0, cfg)
        b = ctx2.query(st, q, 10.0, cfg)
        c = mb.query_once(st, q, 10.0, cfg)
        assert a.tobytes() == b.tobytes() == c.tobytes()


@pytest.mark.parametrize("name", ["pipeline_d64", "pipeline_d768"])
def test_gpu_matches_reference_golden(torch_mod, mb, name):
    z = load_golden(os.path.join(HERE, "golden", f"{name}.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    E, mods, ts = z["emb"], z["mods"], z["ts"]
    st, ctx = build(mb, E, mods, ts, None, z["row_off"], z["col_idx"])
    for di, (lam, qts) in enumerate(meta["decays"]):
        for k in meta["top_ks"]:
            for h in (0, 1):
                tag = f"d{di}_k{k}_h{h}"
                for qi in range(z["queries"].shape[0]):
                    cfg = mb.RetrievalConfig(top_k=k, bfs_max_hops=h, time_decay_lambda=lam,
                                             bfs_score_decay=0.5)
                    got = ctx.query(st, z["queries"][qi], qts, cfg)
                    assert_ranked_equivalent(got["node_id"], got["score"], z["ids_" + tag][qi],
                                             z["scores_" + tag][qi], got["hops"],
                                             z["hops_" + tag][qi], what=f"{name} {tag} q{qi}")


def test_errors_are_reported_not_fatal(torch_mod, mb):
    E, mod, ts, imp, ro, ci = make_corpus(100, 64, seed=1)
    st, ctx = build(mb, E, mod, ts, imp, ro, ci, max_k=16)
    with pytest.raises(mb.MarsError) as e:
        ctx.query(st, E[0], 1.0, mb.RetrievalConfig(top_k=17))
    assert e.value.status == mb.MARS_ERR_INVALID
    with pytest.raises(mb.MarsError) as e:
        ctx.query(st, E[0], 1.0, mb.RetrievalConfig(top_k=4, bfs_max_hops=15))
    assert e.value.status == mb.MARS_ERR_INVALID
    small = mb.QueryContext(50, 64, max_k=16)
    with pytest.raises(mb.MarsError) as e:
        small.query(st, E[0], 1.0, mb.RetrievalConfig(top_k=4))
    assert e.value.status == mb.MARS_ERR_CAPACITY
    # still usable afterwards
    r = ctx.query(st, E[0], 1.0, mb.RetrievalConfig(top_k=4, bfs_max_hops=0))
    assert r["node_id"][0] == 0


@pytest.mark.parametrize("N,K,nq", [(100003, 10, 16), (5000, 64, 9), (77, 100, 3), (250000, 1, 40)])
def test_scan_topk_multi_equals_single_scans(torch_mod, mb, N, K, nq):
    """mars_scan_topk_multi: the queries of one launch give exactly the
    results of separate mars_scan_topk calls (ids, score bits, counts)."""
    torch = torch_mod
    from mars_b200 import datagen
    D = 768
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=N % 97, ts_max=10.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=max(K, 10))
    Q = torch.from_numpy(datagen.queries(nq, D, seed=K)).cuda()
    ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    vals = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    cnt = torch.empty(nq, dtype=torch.int32, device="cuda")
    for rep in range(2):   # tickets and counters re-armed between launches
        ctx.scan_topk_multi(st, Q, nq, 10.0, 0.3, K, ids, vals, cnt, use_importance=True, row_offset=7)
        torch.cuda.synchronize()
        for i in range(nq):
            i1 = torch.empty(K, dtype=torch.int32, device="cuda")
            v1 = torch.empty(K, dtype=torch.float32, device="cuda")
            c1 = torch.empty(1, dtype=torch.int32, device="cuda")
            ctx.scan_topk(st, Q[i], 10.0, 0.3, K, i1, v1, c1, use_importance=True, row_offset=7)
            torch.cuda.synchronize()
            assert int(cnt[i].item()) == int(c1.item())
            assert np.array_equal(ids[i].cpu().numpy(), i1.cpu().numpy()), (rep, i)
            assert np.array_equal(vals[i].cpu().numpy().view(np.uint32), v1.cpu().numpy().view(np.uint32))
