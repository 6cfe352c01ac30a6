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
