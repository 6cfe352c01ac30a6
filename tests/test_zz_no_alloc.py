"""mars_scan_topk_noalloc: the fused scan for callers that may not allocate
GPU memory (a process whose whole device budget is reserved up front, or a
host that forbids the library from growing its footprint).

It reads the caller's own device arrays and keeps its working memory in a
library-owned device array, so this test gives it plain tensors and checks
that two calls in a row -- the second finding the array as the first left it
-- return what the regular entry point (mars_scan_topk through a store and a
query context) returns for the same inputs.  This file is collected last so
that a run stopping at the first failure has run every other test already.
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
    ctx = mb.QueryContext(N, D, max_k=mb.MAX_TOP_K)

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
    K = mb.MAX_TOP_K + 1
    ids = torch.empty(K, dtype=torch.int32, device="cuda")
    vals = torch.empty(K, dtype=torch.float32, device="cuda")
    with pytest.raises(mb.MarsError) as e:
        mb.scan_topk_noalloc(E, D, ts, None, None, 8, D, q, 0.0, 0.0, K, ids, vals)
    assert e.value.status == mb.MARS_ERR_CAPACITY
    assert "K must be in" in str(e.value)
