"""mars_scan_topk_noalloc: the fused scan for callers that may not allocate
GPU memory (a process whose whole device budget is reserved up front, or a
host that forbids the library from growing its footprint).

It reads the caller's own device arrays and keeps its working memory in a
library-owned device array, so this test gives it plain tensors and checks
that two calls in a row -- the second finding the array as the first left it
-- return what the regular entry point (mars_scan_topk through a store and a
query context) returns for the same inputs, and what the CPU oracle returns.
The cases reach the scratch's row counter (corpora large enough for the
dynamic row hand-out, on both calls), its 512-block cap (small D, K <= 32)
and its own count word (no d_count).  This file is collected last so that a
run stopping at the first failure has run every other test already.
"""
import numpy as np
import pytest

from _util import assert_ranked_equivalent

pytestmark = pytest.mark.gpu


def test_noalloc_scan_matches_regular_entry_point_twice():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen

    N, D = 40_009, 768
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=321, ts_max=600.0)
    Q = datagen.queries(2, D, seed=77)
    Ed, tsd, impd, modd = (torch.from_numpy(a).cuda() for a in (E, ts, imp, mod))
    Qd = torch.from_numpy(Q).cuda()

    store = mb.Store(N, D)
    store.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=mb.NOALLOC_MAX_K)

    # two calls in a row with different K, query and filter: the second one
    # runs on the scratch exactly as the first left it
    for call, (K, filt) in enumerate([(100, -1), (10, 2)]):
        ref_ids = torch.empty(K, dtype=torch.int32, device="cuda")
        ref_vals = torch.empty(K, dtype=torch.float32, device="cuda")
        ref_cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        ctx.scan_topk(store, Qd[call], 600.0, 0.01, K, ref_ids, ref_vals, ref_cnt,
                      modality_filter=filt, use_importance=True)
        torch.cuda.synchronize()

        ids = torch.full((K,), -7, dtype=torch.int32, device="cuda")
        vals = torch.zeros(K, dtype=torch.float32, device="cuda")
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        mb.scan_topk_noalloc(Ed, D, tsd, impd, modd, N, D, Qd[call], 600.0, 0.01, K, ids, vals,
                             cnt, modality_filter=filt, use_importance=True)
        torch.cuda.synchronize()

        assert int(cnt.item()) == int(ref_cnt.item()) == K
        assert_ranked_equivalent(ids.cpu().numpy(), vals.cpu().numpy(), ref_ids.cpu().numpy(),
                                 ref_vals.cpu().numpy(), what=f"call {call}")
        # same kernel and arithmetic: in fact identical
        assert np.array_equal(ids.cpu().numpy(), ref_ids.cpu().numpy())


def test_noalloc_rejects_k_beyond_its_scratch():
    import torch

    import mars_b200 as mb

    D = 64
    E = torch.zeros((8, D), dtype=torch.float32, device="cuda")
    ts = torch.zeros(8, dtype=torch.float32, device="cuda")
    q = torch.zeros(D, dtype=torch.float32, device="cuda")
    K = mb.NOALLOC_MAX_K + 1
    ids = torch.empty(K, dtype=torch.int32, device="cuda")
    vals = torch.empty(K, dtype=torch.float32, device="cuda")
    with pytest.raises(mb.MarsError) as e:
        mb.scan_topk_noalloc(E, D, ts, None, None, 8, D, q, 0.0, 0.0, K, ids, vals)
    assert e.value.status == mb.MARS_ERR_CAPACITY
    assert "K must be in" in str(e.value)


@pytest.mark.parametrize("N,D,calls", [
    # dynamic row hand-out (n >= 32 x the launch's warps) on both calls
    (150_000, 768, [(100, -1, True), (10, 1, True)]),
    # D = 64, K = 8: the grid is capped at the scratch's 512 blocks; the
    # second call passes no d_count (the scratch's own count word)
    (200_000, 64, [(8, -1, True), (8, 3, False)]),
])
def test_noalloc_large_and_capped_cases_match_regular_and_oracle(N, D, calls):
    import torch

    import mars_b200 as mb
    import oracle as O
    from mars_b200 import datagen

    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=4242 + D, ts_max=600.0)
    Q = datagen.queries(len(calls), D, seed=99 + D)
    Ed, tsd, impd, modd = (torch.from_numpy(a).cuda() for a in (E, ts, imp, mod))
    Qd = torch.from_numpy(Q).cuda()
    store = mb.Store(N, D)
    store.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=mb.NOALLOC_MAX_K)
    corpus = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)

    for call, (K, filt, with_count) in enumerate(calls):
        ref_ids = torch.empty(K, dtype=torch.int32, device="cuda")
        ref_vals = torch.empty(K, dtype=torch.float32, device="cuda")
        ctx.scan_topk(store, Qd[call], 600.0, 0.01, K, ref_ids, ref_vals, modality_filter=filt,
                      use_importance=True)
        ids = torch.full((K,), -7, dtype=torch.int32, device="cuda")
        vals = torch.zeros(K, dtype=torch.float32, device="cuda")
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda") if with_count else None
        mb.scan_topk_noalloc(Ed, D, tsd, impd, modd, N, D, Qd[call], 600.0, 0.01, K, ids, vals, cnt,
                             modality_filter=filt, use_importance=True)
        torch.cuda.synchronize()
        if with_count:
            assert int(cnt.item()) == K
        got_ids, got_vals = ids.cpu().numpy(), vals.cpu().numpy()
        # the same kernel as the regular entry point: identical bits
        assert np.array_equal(got_ids, ref_ids.cpu().numpy()), f"call {call}"
        assert np.array_equal(got_vals.view(np.int32), ref_vals.cpu().numpy().view(np.int32)), f"call {call}"
        # and the oracle's answer (canonical dot; expf against __expf: tie-aware)
        o_ids, o_vals = O.query_batch_topk(corpus, Q[call:call + 1], 600.0, 0.01, K, modality_filter=filt,
                                           use_importance=True)
        assert_ranked_equivalent(got_ids, got_vals, o_ids[0], o_vals[0], what=f"oracle call {call}")
