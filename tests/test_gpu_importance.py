"""Importance update and novelty, the store-side companions of the query.

* mars_importance_update restates update_importance
  (src/memory_cuda.cu:1179-1224): every row's importance is multiplied by
  (1 - decay_rate), then each listed id gets min(importance + boost,
  max_importance), once per occurrence (ids outside [0, N) are skipped).
  The check below restates that rule in float32 numpy, applying the boosts
  one after another; the device applies the same function once per
  occurrence in some order, which gives the same bits.
* mars_novelty restates compute_novelty (src/memory_cuda.cu:1232-1290): the
  largest dot(E_i, q) over the rows.  It is the fused scan with K = 1 and a
  weight of exactly 1, so it equals the largest canonical dot product of the
  oracle bit for bit.
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


def restated_update(imp, ids, boost, decay, max_imp):
    out = (imp.astype(np.float32) * (np.float32(1.0) - np.float32(decay))).astype(np.float32)
    for u in ids:
        if 0 <= u < out.shape[0]:
            out[u] = np.float32(min(np.float32(out[u] + np.float32(boost)), np.float32(max_imp)))
    return out


def test_importance_update_matches_the_restated_rule(torch_mod, mb):
    torch = torch_mod
    from mars_b200 import datagen
    N, D = 5000, 64
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=3, ts_max=10.0)
    st = mb.Store(N + 100, D)
    st.upload(E, mod, ts, imp)
    rng = np.random.default_rng(4)
    expect = imp.astype(np.float32)
    for step, (boost, decay, max_imp) in enumerate(((0.1, 0.001, 5.0), (0.75, 0.05, 1.2), (2.0, 0.0, 3.0))):
        ids = rng.integers(0, N, 300).astype(np.int32)
        ids[:20] = ids[20:40]                       # repeated ids: boosted once per occurrence
        ids[40:43] = np.array([-1, N, N + 50])      # outside the store: skipped
        d_ids = torch.from_numpy(ids).cuda()
        st.importance_update(d_ids, ids.shape[0], boost=boost, decay_rate=decay, max_importance=max_imp)
        torch.cuda.synchronize()
        expect = restated_update(expect, ids, boost, decay, max_imp)
        got = st.read(0, N)[3]
        assert np.array_equal(got.view(np.uint32), expect.view(np.uint32)), f"step {step}"


def test_importance_fill_and_query_after_update(torch_mod, mb):
    """The fused scan's importance term reads the updated values."""
    torch = torch_mod
    from mars_b200 import datagen
    N, D = 20000, 768
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=8, ts_max=10.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    st.importance_fill(0.5)
    assert np.all(st.read(0, N)[3] == np.float32(0.5))
    ids = np.arange(0, N, 7, dtype=np.int32)
    st.importance_update(torch.from_numpy(ids).cuda(), ids.shape[0], boost=1.0, decay_rate=0.1,
                         max_importance=1.3)
    torch.cuda.synchronize()
    imp_now = st.read(0, N)[3]
    ctx = mb.QueryContext(N, D, max_k=16)
    oc = O.Corpus(E=E, ts=ts, mod=mod, imp=imp_now)
    q = datagen.queries(1, D, seed=9)[0]
    K = 10
    dq = torch.from_numpy(q).cuda()
    ids_d = torch.empty(K, dtype=torch.int32, device="cuda")
    vals_d = torch.empty(K, dtype=torch.float32, device="cuda")
    ctx.scan_topk(st, dq, 10.0, 0.2, K, ids_d, vals_d, use_importance=True)
    torch.cuda.synchronize()
    ref = O.query(oc, q, 10.0, top_k=K, bfs_max_hops=0, lam=0.2, use_importance=True)
    # the oracle's decay uses the C library's expf: ranked equivalence within
    # the tests' tolerance, as for every scan
    assert_ranked_equivalent(ids_d.cpu().numpy(), vals_d.cpu().numpy(), ref["node_id"], ref["score"],
                             what="after update")


@pytest.mark.parametrize("N,D", [(1, 768), (3000, 64), (50000, 768)])
def test_novelty_is_the_largest_dot_product(torch_mod, mb, N, D):
    torch = torch_mod
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=N + D, ts_max=10.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=8)
    oc = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    d_max = torch.empty(1, dtype=torch.float32, device="cuda")
    for i, q in enumerate(datagen.queries(4, D, seed=D)):
        ctx.novelty(st, torch.from_numpy(q).cuda(), d_max)
        torch.cuda.synchronize()
        ref = np.float32(O.fused_scores(oc, q, 0.0, 0.0).max())
        assert d_max.cpu().numpy().view(np.uint32)[0] == np.array([ref]).view(np.uint32)[0], i
    # a stored row as the query: its own dot product is the largest
    ctx.novelty(st, torch.from_numpy(E[N // 2].copy()).cuda(), d_max)
    torch.cuda.synchronize()
    assert d_max.item() == pytest.approx(1.0, abs=1e-5)
