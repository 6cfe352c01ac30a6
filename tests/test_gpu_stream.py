"""Streaming insert (in place, no rebuild) and sharded top-K merge on the GPU,
checked against the oracle over the same grown corpus."""
import numpy as np
import pytest

import oracle as O
from _util import assert_ranked_equivalent, assert_topk_matches_scores

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def mb():
    import mars_b200
    return mars_b200


def test_append_normalizes_bit_exact(torch_mod, mb):
    rng = np.random.default_rng(0)
    D = 768
    st = mb.Store(64, D)
    raw = (rng.standard_normal((10, D)) * 3.0).astype(np.float32)
    first = st.append(raw, np.arange(10) % 4, np.linspace(0, 1, 10), normalize=True)
    assert first == 0 and st.num_nodes == 10
    E, mod, ts, imp = st.read()
    for i in range(10):
        assert np.array_equal(E[i].view(np.uint32), O.l2_normalize(raw[i]).view(np.uint32))
    assert np.all(imp == 1.0)
    # without normalisation rows are stored as given
    st.append(raw[:2], [1, 2], [5.0, 6.0], normalize=False)
    E2, _, _, _ = st.read(10, 2)
    assert np.array_equal(E2, raw[:2])


def test_append_capacity_error(torch_mod, mb):
    st = mb.Store(8, 16)
    st.append(np.ones((8, 16), np.float32), np.zeros(8), np.zeros(8))
    with pytest.raises(mb.MarsError) as e:
        st.append(np.ones((1, 16), np.float32), [0], [0.0])
    assert e.value.status == mb.MARS_ERR_CAPACITY
    assert st.num_nodes == 8


def test_streaming_loop_matches_oracle(torch_mod, mb):
    """Config-1 shape at small scale: start corpus, then frames of
    (append 10 normalised rows stamped now, query); no re-upload."""
    from mars_b200 import datagen
    D, N0, frames, per = 768, 3000, 40, 10
    E0, mod0, ts0, _ = datagen.gaussian_corpus(N0, D, seed=5, importance=False)
    ro, ci = datagen.random_bridges(mod0, 4, seed=6)
    cap = N0 + frames * per
    st = mb.Store(cap, D, edge_slack=8)
    st.upload(E0, mod0, ts0, None, ro, ci)
    ctx = mb.QueryContext(cap, D, max_k=10)
    rng = np.random.default_rng(8)
    E_all, mod_all, ts_all = [E0], [mod0], [ts0]
    ex = np.full((cap, 8), -1, np.int32)
    exc = np.zeros(cap, np.int32)
    for f in range(frames):
        t_now = 10.0 + f * 1e-3
        raw = rng.standard_normal((per, D)).astype(np.float32)
        m = rng.integers(0, 4, per).astype(np.int32)
        first = st.append(raw, m, np.full(per, t_now, np.float32), normalize=True)
        # bridge every new node to one older node of another modality (both ways)
        src, dst = [], []
        for i in range(per):
            u = first + i
            v = int(rng.integers(0, first))
            src += [u, v]
            dst += [v, u]
        if f % 2 == 0:
            st.append_edges(src, dst)
            for a, b in zip(src, dst):
                ex[a, exc[a]] = b
                exc[a] += 1
        E_all.append(np.stack([O.l2_normalize(r) for r in raw]))
        mod_all.append(m)
        ts_all.append(np.full(per, t_now, np.float32))
        q = rng.standard_normal(D).astype(np.float32)
        q /= np.linalg.norm(q)
        cfg = mb.RetrievalConfig(top_k=10, bfs_max_hops=1, time_decay_lambda=1.0)
        got = ctx.query(st, q, t_now, cfg)
        n = first + per
        oc = O.Corpus(E=np.concatenate(E_all), ts=np.concatenate(ts_all),
                      mod=np.concatenate(mod_all), row_offsets=np.concatenate(
                          [ro, np.full(n - N0, ro[-1], np.int32)]),
                      col_indices=ci, extra_nbrs=ex[:n], extra_cnt=exc[:n])
        ref = O.query(oc, q, t_now, top_k=10, bfs_max_hops=1, lam=1.0)
        assert_ranked_equivalent(got["node_id"], got["score"], ref["node_id"], ref["score"],
                                 got["hops"], ref["hops"], what=f"frame {f}")


def test_edge_slack_exhaustion_is_atomic(torch_mod, mb):
    st = mb.Store(16, 8, edge_slack=2)
    st.append(np.eye(8, dtype=np.float32).repeat(2, axis=0)[:16], np.zeros(16), np.zeros(16))
    st.append_edges([0, 0], [1, 2])
    with pytest.raises(mb.MarsError) as e:
        st.append_edges([3, 0], [4, 5])
    assert e.value.status == mb.MARS_ERR_CAPACITY
    st.append_edges([3], [4])   # node 3 still had room: nothing was written before


@pytest.mark.parametrize("shards", [2, 3, 4])
def test_sharded_scan_merge_equals_single(torch_mod, mb, shards):
    torch = torch_mod
    from mars_b200 import datagen
    N, D, K = 30011, 768, 100
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=shards)
    q = datagen.queries(1, D, seed=shards)[0]
    qd = torch.from_numpy(q).cuda()
    bounds = [N * s // shards for s in range(shards + 1)]
    ids = torch.empty(shards * K, dtype=torch.int32, device="cuda")
    vals = torch.empty(shards * K, dtype=torch.float32, device="cuda")
    keep = []
    for s in range(shards):
        lo, hi = bounds[s], bounds[s + 1]
        st = mb.Store(hi - lo, D)
        st.upload(E[lo:hi], mod[lo:hi], ts[lo:hi], imp[lo:hi])
        ctx = mb.QueryContext(hi - lo, D, max_k=K)
        ctx.scan_topk(st, qd, 600.0, 0.01, K, ids[s * K:(s + 1) * K], vals[s * K:(s + 1) * K],
                      use_importance=True, row_offset=lo)
        torch.cuda.synchronize()
        keep.append((st, ctx))
    mids = torch.empty(K, dtype=torch.int32, device="cuda")
    mvals = torch.empty(K, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    keep[0][1].topk_merge(ids, vals, shards, K, mids, mvals, cnt)
    torch.cuda.synchronize()
    # single-store reference on the GPU and the oracle
    st1 = mb.Store(N, D)
    st1.upload(E, mod, ts, imp)
    ctx1 = mb.QueryContext(N, D, max_k=K)
    i1 = torch.empty(K, dtype=torch.int32, device="cuda")
    v1 = torch.empty(K, dtype=torch.float32, device="cuda")
    ctx1.scan_topk(st1, qd, 600.0, 0.01, K, i1, v1, use_importance=True)
    torch.cuda.synchronize()
    assert int(cnt.item()) == K
    assert np.array_equal(mids.cpu().numpy(), i1.cpu().numpy())
    assert np.array_equal(mvals.cpu().numpy().view(np.uint32), v1.cpu().numpy().view(np.uint32))
    ref = O.fused_scores(O.Corpus(E=E, ts=ts, mod=mod, imp=imp), q, 600.0, 0.01,
                         use_importance=True)
    assert_topk_matches_scores(mids.cpu().numpy(), mvals.cpu().numpy(), ref)


@pytest.mark.parametrize("n_lists,K,Q", [(8, 100, 64), (2, 10, 5), (3, 256, 4), (40, 100, 3), (1, 1, 7)])
def test_topk_merge_batch_against_numpy(torch_mod, mb, n_lists, K, Q):
    """mars_topk_merge_batch on rank-major [n_lists][Q][K] ranked lists, with
    tied scores, short lists (-1 padding) and, for 40 x 100 entries, more
    entries than the one-CTA selection holds (the list-by-list path)."""
    torch = torch_mod
    rng = np.random.default_rng(n_lists * 1000 + K)
    ids = np.full((n_lists, Q, K), -1, np.int32)
    vals = np.full((n_lists, Q, K), -np.inf, np.float32)
    for l in range(n_lists):
        for q in range(Q):
            n = K if (l + q) % 3 else K // 2            # some short lists
            s = np.round(rng.standard_normal(n), 1).astype(np.float32)   # many ties
            i = (rng.permutation(100000)[:n] * n_lists + l).astype(np.int32)   # unique across lists
            o = np.lexsort((i, -s))
            ids[l, q, :n], vals[l, q, :n] = i[o], s[o]
    ctx = mb.QueryContext(16, 8, max_k=256)
    di, dv = torch.from_numpy(ids).cuda(), torch.from_numpy(vals).cuda()
    mi = torch.empty((Q, K), dtype=torch.int32, device="cuda")
    mv = torch.empty((Q, K), dtype=torch.float32, device="cuda")
    mc = torch.empty(Q, dtype=torch.int32, device="cuda")
    ctx.topk_merge_batch(di, dv, n_lists, K, Q, mi, mv, mc)
    torch.cuda.synchronize()
    for q in range(Q):
        valid = ids[:, q, :] >= 0
        ai, av = ids[:, q, :][valid], vals[:, q, :][valid]
        o = np.lexsort((ai, -av))[:K]
        n = o.shape[0]
        assert int(mc[q].item()) == n
        assert np.array_equal(mi[q, :n].cpu().numpy(), ai[o])
        assert np.array_equal(mv[q, :n].cpu().numpy(), av[o])
        assert np.all(mi[q, n:].cpu().numpy() == -1)


def test_tombstone_delete_matches_reference_rule(torch_mod, mb):
    """mars_store_delete zeroes the row and sets its timestamp to -1 (the
    reference's engine_server DELETE); queries then equal the oracle on a
    corpus edited the same way, BFS included (edges stay)."""
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(3000, 768, seed=77, ts_max=10.0)
    ro, ci = datagen.random_bridges(mod, 4, seed=78)
    st = mb.Store(3200, 768, edge_slack=4)
    st.upload(E, mod, ts, imp, ro, ci)
    rows, m2, t2, w2 = datagen.gaussian_corpus(50, 768, seed=79, ts_max=10.0)
    first = st.append(rows, m2, t2, w2, normalize=False)
    E = np.concatenate([E, rows]); mod = np.concatenate([mod, m2])
    ts = np.concatenate([ts, t2]); imp = np.concatenate([imp, w2])
    ctx = mb.QueryContext(3200, 768, max_k=64)
    q = E[first + 3] + E[17]                     # close to rows that get deleted
    cfg = mb.RetrievalConfig(top_k=20, bfs_max_hops=1, time_decay_lambda=0.1, use_importance=True)
    before = ctx.query(st, q, 10.0, cfg)
    dead = np.array([17, first + 3, 5000, -1, int(before["node_id"][2])], np.int32)   # two ignored
    st.delete(dead)
    for u in dead:
        if 0 <= u < E.shape[0]:
            E[u] = 0.0
            ts[u] = -1.0
    got = ctx.query(st, q, 10.0, cfg)
    ctx.set_fused(False)
    got_pipe = ctx.query(st, q, 10.0, cfg)
    assert got.tobytes() == got_pipe.tobytes()
    # the oracle's CSR covers every row: appended rows have no edges
    ro_all = np.concatenate([ro, np.full(E.shape[0] - (ro.shape[0] - 1), ro[-1], ro.dtype)])
    oc = O.Corpus(E=E, ts=ts, mod=mod, imp=imp, row_offsets=ro_all, col_indices=ci)
    ref = O.query(oc, q, 10.0, top_k=20, bfs_max_hops=1, lam=0.1, bfs_score_decay=0.5, use_importance=True)
    assert_ranked_equivalent(got["node_id"], got["score"], ref["node_id"], ref["score"], got["hops"],
                             ref["hops"], what="after delete")
    Er, mr, tr, ir = st.read(0, E.shape[0])
    assert np.array_equal(Er[17], np.zeros(768, np.float32)) and tr[17] == -1.0
    assert np.array_equal(tr, ts)
