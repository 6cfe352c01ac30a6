"""Allocation failures, made on the host side without any GPU fault: a
store, a batch context or a search context larger than the device cannot be
allocated (cudaMalloc answers out of memory), and the library must

* refuse it with MARS_ERR_OOM and a message naming the allocation,
* free whatever it had already allocated for that object (the device's free
  memory returns to where it was), and
* stay usable: the next store, batch context and query work, and their
  answers are exact (equal to the CPU oracle)."""
import numpy as np
import pytest

import oracle as O
from _util import assert_ranked_equivalent

pytestmark = pytest.mark.gpu


def _free_bytes():
    import torch
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]


def test_oversized_objects_are_refused_and_leave_the_device_usable():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    N, D, K = 20_000, 768, 10
    # warm up the context and the library's first-use allocations
    st0 = mb.Store(1024, D)
    st0.close()
    base = _free_bytes()

    # 2e9 rows x 768 floats = 6 TB: the first allocation fails
    with pytest.raises(mb.MarsError) as e:
        mb.Store(2_000_000_000, D)
    assert e.value.status == mb.MARS_ERR_OOM
    # 4M queries x 4,096 candidate records of 16 B = 268 GB: the smaller
    # buffers before it were allocated, then freed again
    with pytest.raises(mb.MarsError) as e:
        mb.BatchContext(N, D, max_batch=4_000_000, max_k=K)
    assert e.value.status == mb.MARS_ERR_OOM
    assert "candidates" in str(e.value) or "out of memory" in str(e.value).lower()
    with pytest.raises(mb.MarsError) as e:
        mb.CmngContext(2_000_000_000, 256, 36, 2, 1_000_000)   # 2 TB of seed lists
    assert e.value.status == mb.MARS_ERR_OOM
    after = _free_bytes()
    assert abs(after - base) < 64 << 20, (base, after)

    # the device and the library still work, exactly
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=61, ts_max=600.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    B = 16
    bc = mb.BatchContext(N, D, max_batch=B, max_k=K)
    Q = datagen.queries(B, D, seed=62)
    Qd = torch.from_numpy(Q).cuda()
    ids = torch.empty((B, K), dtype=torch.int32, device="cuda")
    vals = torch.empty((B, K), dtype=torch.float32, device="cuda")
    bc.query_batch_topk(st, Qd, B, 600.0, 0.01, K, ids, vals, use_importance=True)
    torch.cuda.synchronize()
    c = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    for q in range(4):
        s = O.fused_scores(c, Q[q], 600.0, 0.01, use_importance=True)
        oi, ov = O.topk(s, mod, -1, K)
        assert_ranked_equivalent(ids[q].cpu().numpy(), vals[q].cpu().numpy(), oi, ov, what=f"query {q}")
    bc.close()
    st.close()
