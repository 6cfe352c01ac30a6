"""mars_scan_topk_f16 (csrc/mars_scan16.cu): the fused scan top-K streamed
from the store's fp16 copy with an exact fp32 rescore of the rows the fp16
bound cannot rule out.

Its results must be those of mars_scan_topk_multi bit for bit (same ids,
same score bits, same counts): the fp16 pass only filters.  That scan is
itself checked against the oracle in test_gpu_query.py; a small case here is
also checked against the oracle directly.
"""
import numpy as np
import pytest

import oracle as O
from _util import assert_ranked_equivalent

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


def run_both(torch, ctx, st, Q, K, **kw):
    nq = Q.shape[0]
    out = []
    for fn in (ctx.scan_topk_f16, ctx.scan_topk_multi):
        ids = torch.full((nq, K), -7, dtype=torch.int32, device="cuda")
        vals = torch.zeros((nq, K), dtype=torch.float32, device="cuda")
        cnt = torch.full((nq,), -7, dtype=torch.int32, device="cuda")
        fn(st, Q, nq, kw.get("t_q", 10.0), kw.get("lam", 0.3), K, ids, vals, cnt,
           modality_filter=kw.get("modality_filter", -1), use_importance=kw.get("use_importance", False),
           row_offset=kw.get("row_offset", 0))
        torch.cuda.synchronize()
        out.append((ids.cpu().numpy(), vals.cpu().numpy(), cnt.cpu().numpy()))
    return out


def assert_same(a, b, what):
    (ia, va, ca), (ib, vb, cb) = a, b
    assert np.array_equal(ca, cb), f"{what}: counts {ca} != {cb}"
    assert np.array_equal(ia, ib), f"{what}: ids differ"
    assert np.array_equal(va.view(np.uint32), vb.view(np.uint32)), f"{what}: score bits differ"


@pytest.mark.parametrize("N,D", [(1, 768), (37, 768), (10007, 768), (125000, 768), (1000000, 768),
                                 (20000, 1024), (30001, 100), (5000, 4), (40000, 64)])
def test_f16_scan_equals_fp32_scan(torch_mod, mb, N, D):
    torch = torch_mod
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=N % 1009 + D, ts_max=10.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=64)
    nq = 20
    Q = torch.from_numpy(datagen.queries(nq, D, seed=D + 1)).cuda()
    for i, K in enumerate((1, 10, 33, 64)):
        kw = dict(use_importance=bool(i % 2), modality_filter=(i % 4) - 1 if i >= 2 else -1,
                  row_offset=3 * i, lam=0.1 * i)
        a, b = run_both(torch, ctx, st, Q, K, **kw)
        assert_same(a, b, f"N={N} D={D} K={K}")
    # ordinary data never overflows the candidate list
    if N >= 1000:
        assert ctx.f16_reruns() == 0


def test_f16_scan_signed_importance_and_clustered_rows(torch_mod, mb):
    """Negative importance flips the bound; clustered rows put many scores
    near the K-th one (many candidates to rescore)."""
    torch = torch_mod
    from mars_b200 import datagen
    N, D = 200000, 768
    E, mod, ts = datagen.cluster_corpus(N, D, n_clusters=16, sigma=0.05, seed=5)[:3]
    imp = np.random.default_rng(6).uniform(-1.0, 1.0, N).astype(np.float32)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=64)
    Q = torch.from_numpy(E[:16] + 0.01 * datagen.queries(16, D, seed=9)).cuda().contiguous()
    for K in (1, 10, 64):
        for use_imp in (False, True):
            a, b = run_both(torch, ctx, st, Q, K, use_importance=use_imp, lam=0.05)
            assert_same(a, b, f"clustered K={K} imp={use_imp}")


def test_f16_scan_matches_oracle(torch_mod, mb):
    torch = torch_mod
    from mars_b200 import datagen
    N, D = 6000, 768
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=77, ts_max=10.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=64)
    oc = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    qs = datagen.queries(4, D, seed=3)
    Q = torch.from_numpy(qs).cuda()
    K = 10
    ids = torch.empty((4, K), dtype=torch.int32, device="cuda")
    vals = torch.empty((4, K), dtype=torch.float32, device="cuda")
    ctx.scan_topk_f16(st, Q, 4, 10.0, 0.5, K, ids, vals, use_importance=True)
    torch.cuda.synchronize()
    for i in range(4):
        ref = O.query(oc, qs[i], 10.0, top_k=K, bfs_max_hops=0, lam=0.5, use_importance=True)
        assert_ranked_equivalent(ids[i].cpu().numpy(), vals[i].cpu().numpy(), ref["node_id"], ref["score"],
                                 what=f"query {i}")


def test_f16_scan_overflow_is_answered_by_the_fp32_scan(torch_mod, mb):
    """Every row identical: all upper bounds reach the K-th lower bound, the
    candidate list overflows and the host re-runs each query in fp32."""
    torch = torch_mod
    N, D = 100000, 64
    E = np.tile(np.random.default_rng(0).standard_normal((1, D)).astype(np.float32), (N, 1))
    st = mb.Store(N, D)
    st.upload(E, np.zeros(N, np.int32), np.zeros(N, np.float32), None)
    ctx = mb.QueryContext(N, D, max_k=64)
    Q = torch.from_numpy(np.random.default_rng(1).standard_normal((3, D)).astype(np.float32)).cuda()
    a, b = run_both(torch, ctx, st, Q, 10, lam=0.0)
    assert_same(a, b, "ties")
    assert np.array_equal(a[0][0], np.arange(10, dtype=np.int32))
    assert ctx.f16_reruns() == 3


def test_f16_scan_out_of_range_rows_use_the_fp32_scan(torch_mod, mb):
    """Components beyond the fp16 range: the call runs the fp32 scan."""
    torch = torch_mod
    from mars_b200 import datagen
    N, D = 5000, 128
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=2, ts_max=10.0)
    E = E * 1.0e6
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=64)
    Q = torch.from_numpy(datagen.queries(5, D, seed=4)).cuda()
    a, b = run_both(torch, ctx, st, Q, 16)
    assert_same(a, b, "out of range")
    assert ctx.f16_reruns() == 0


def test_f16_copy_follows_appends_and_deletes(torch_mod, mb):
    torch = torch_mod
    from mars_b200 import datagen
    N0, D = 50000, 768
    E, mod, ts, imp = datagen.gaussian_corpus(N0, D, seed=11, ts_max=10.0)
    st = mb.Store(N0 + 4000, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N0 + 4000, D, max_k=64)
    rng = np.random.default_rng(12)
    for step in range(4):
        rows, m, t, w = datagen.gaussian_corpus(1000, D, seed=200 + step, ts_max=10.0)
        first = st.append(rows, m, t + 5.0, w, normalize=True)
        qs = rows[:8] + 0.05 * rng.standard_normal((8, D)).astype(np.float32)
        Q = torch.from_numpy(qs).cuda()
        a, b = run_both(torch, ctx, st, Q, 10, t_q=15.0)
        assert_same(a, b, f"append {step}")
        # the best rows are the new ones: delete them and ask again
        st.delete(np.unique(a[0][:, :3].ravel()))
        a, b = run_both(torch, ctx, st, Q, 10, t_q=15.0)
        assert_same(a, b, f"delete {step}")
        assert first >= N0


def test_f16_scan_falls_back_for_large_k_and_odd_dim(torch_mod, mb):
    """K > 64 runs the fp32 scan; a dimension that is not a multiple of 4 is
    refused exactly as mars_scan_topk_multi refuses it."""
    torch = torch_mod
    from mars_b200 import datagen
    N = 3000
    E, mod, ts, imp = datagen.gaussian_corpus(N, 768, seed=1, ts_max=10.0)
    st = mb.Store(N, 768)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, 768, max_k=128)
    Q = torch.from_numpy(datagen.queries(3, 768, seed=1)).cuda()
    a, b = run_both(torch, ctx, st, Q, 100)
    assert_same(a, b, "K=100")
    E2, mod2, ts2, imp2 = datagen.gaussian_corpus(N, 99, seed=2, ts_max=10.0)
    st2 = mb.Store(N, 99)
    st2.upload(E2, mod2, ts2, imp2)
    ctx2 = mb.QueryContext(N, 99, max_k=16)
    Q2 = torch.zeros((3, 100), dtype=torch.float32, device="cuda")
    ids = torch.empty((3, 10), dtype=torch.int32, device="cuda")
    vals = torch.empty((3, 10), dtype=torch.float32, device="cuda")
    for fn in (ctx2.scan_topk_f16, ctx2.scan_topk_multi):
        with pytest.raises(mb.MarsError) as e:
            fn(st2, Q2, 3, 10.0, 0.3, 10, ids, vals)
        assert e.value.status == mb.MARS_ERR_UNSUPPORTED


def test_mars_query_uses_the_f16_scan_for_large_hop_free_queries(torch_mod, mb):
    """mars_query with no BFS hops over >= 2^18 rows streams the fp16 copy:
    the results (ids, score bits, modalities, hops) equal the fp32 pipeline's."""
    torch = torch_mod
    from mars_b200 import datagen
    N, D = 300_000, 768
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=31, ts_max=10.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    fast = mb.QueryContext(N, D, max_k=64)
    pipe = mb.QueryContext(N, D, max_k=64, use_fused=False)
    rng = np.random.default_rng(5)
    for i, K in enumerate((1, 10, 33, 64)):
        q = rng.standard_normal(D).astype(np.float32)
        cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=0, time_decay_lambda=0.2 * i,
                                 use_importance=bool(i % 2), modality_filter=(i % 3) - 1)
        a = fast.query(st, q, 10.0, cfg)
        b = pipe.query(st, q, 10.0, cfg)
        assert a.tobytes() == b.tobytes(), K
        # a device-resident query takes the same route
        c = fast.query(st, torch.from_numpy(q).cuda(), 10.0, cfg)
        assert c.tobytes() == b.tobytes(), K
    assert fast.f16_reruns() == 0
    assert fast.path_counts()[0] == 8


def test_mars_query_f16_overflow_falls_back(torch_mod, mb):
    """Every row identical: the fp16 candidate list overflows and mars_query
    answers with the fp32 single-launch kernel (same results)."""
    N, D = 300_000, 64
    E = np.tile(np.random.default_rng(0).standard_normal((1, D)).astype(np.float32), (N, 1))
    st = mb.Store(N, D)
    st.upload(E, np.zeros(N, np.int32), np.zeros(N, np.float32), None)
    fast = mb.QueryContext(N, D, max_k=16)
    pipe = mb.QueryContext(N, D, max_k=16, use_fused=False)
    q = np.random.default_rng(1).standard_normal(D).astype(np.float32)
    cfg = mb.RetrievalConfig(top_k=10, bfs_max_hops=0, time_decay_lambda=0.0)
    a = fast.query(st, q, 0.0, cfg)
    assert a.tobytes() == pipe.query(st, q, 0.0, cfg).tobytes()
    assert np.array_equal(a["node_id"], np.arange(10))
    assert fast.f16_reruns() == 1
