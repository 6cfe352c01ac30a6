"""Row-sharded batched top-K over several shards on ONE GPU
(mars_shard_emulate_query_batch_topk).

Every shard runs the same pipeline as mars_shard_query_batch_topk under
NCCL: the short-list threshold shared by all shards (taken from every
shard's sampled bounds), the per-query count / bound records between the
rescore passes, packed keys and the merge.  Only the all-gathers are device
copies between the shards' buffers.  The merged answer must equal
mars_query_batch_topk over the whole corpus on one store, bit for bit:

* 2, 3, 4 and 8 shards, even and uneven, on the 128 x 256 tiles (B > 64:
  the shared threshold, certified by the counts over all shards);
* the small-batch tiles (B <= 64: each shard keeps its own threshold and
  certifies itself);
* K = 256 (exact per-query scans on every shard, neutral records);
* a shard too small for the tensor-core path next to large ones;
* a modality filter without importance;
* a shard whose bounded device wait gives up: every merged answer of that
  call is invalid, and the calls after it recover.

With the shared threshold the shards together short-list about as many
candidates as one store does, not `world` times as many.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N, D = 150_000, 768


@pytest.fixture(scope="module")
def corpus():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=51, ts_max=600.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    Qd = torch.from_numpy(datagen.queries(256, D, seed=52)).cuda()
    yield E, mod, ts, imp, st, Qd
    st.close()


def _bounds(sizes):
    b = [0]
    for s in sizes:
        b.append(b[-1] + s)
    assert b[-1] == N
    return b


def _shards(corpus, sizes):
    import mars_b200 as mb
    E, mod, ts, imp, _, _ = corpus
    b = _bounds(sizes)
    stores, ctxs = [], []
    for r in range(len(sizes)):
        lo, hi = b[r], b[r + 1]
        s = mb.Store(hi - lo, D)
        s.upload(E[lo:hi], mod[lo:hi], ts[lo:hi], imp[lo:hi])
        stores.append(s)
        ctxs.append(mb.BatchContext(hi - lo, D, max_batch=256, max_k=256))
    return stores, ctxs, b[:-1]


def _run(fn, B, K):
    import torch
    ids = torch.full((B, K), -7, dtype=torch.int32, device="cuda")
    vals = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    cnt = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    fn(ids, vals, cnt)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), vals.cpu().numpy(), cnt.cpu().numpy()


def _even(world):
    return [N * (r + 1) // world - N * r // world for r in range(world)]


CASES = [
    # (shard sizes, B, K, modality filter, importance)
    (_even(2), 200, 100, -1, True),
    ([40_000, 70_000, 40_000], 256, 100, -1, True),
    (_even(4), 128, 10, -1, True),
    (_even(8), 256, 100, -1, True),
    (_even(8), 16, 10, -1, True),
    ([60_000, 90_000], 64, 64, -1, True),
    (_even(2), 64, 256, -1, True),
    ([74_500, 500, 75_000], 200, 50, -1, True),
    (_even(3), 130, 20, 2, False),
]


@pytest.mark.parametrize("sizes,B,K,filt,use_imp", CASES)
def test_emulated_shards_equal_one_store(corpus, sizes, B, K, filt, use_imp):
    import mars_b200 as mb
    E, mod, ts, imp, st, Qd = corpus
    bc = mb.BatchContext(N, D, max_batch=256, max_k=256)
    ref = _run(lambda i, v, c: bc.query_batch_topk(st, Qd[:B], B, 600.0, 0.01, K, i, v, c, modality_filter=filt,
                                                   use_importance=use_imp), B, K)
    one = bc.last_stats()
    stores, ctxs, offs = _shards(corpus, sizes)
    try:
        got = _run(lambda i, v, c: mb.shard_emulate_query_batch_topk(stores, ctxs, offs, Qd[:B], B, 600.0, 0.01, K,
                                                                     i, v, c, modality_filter=filt,
                                                                     use_importance=use_imp), B, K)
        assert np.array_equal(got[2], ref[2])
        assert np.array_equal(got[0], ref[0])
        assert np.array_equal(got[1].view(np.int32), ref[1].view(np.int32))
        if B > 64 and K < 256 and min(sizes) >= 10_000:
            # the shared threshold: the shards short-list about what one store does
            cand = sum(c.last_stats()["candidates"] for c in ctxs)
            assert cand <= 1.5 * one["candidates"] + 100 * B, (cand, one["candidates"])
        # a second call on the same shards is still exact (records and
        # thresholds are rewritten every call)
        again = _run(lambda i, v, c: mb.shard_emulate_query_batch_topk(stores, ctxs, offs, Qd[:B], B, 600.0, 0.01,
                                                                       K, i, v, c, modality_filter=filt,
                                                                       use_importance=use_imp), B, K)
        assert np.array_equal(again[0], ref[0]) and np.array_equal(again[2], ref[2])
    finally:
        for s in stores:
            s.close()


def test_failed_shard_invalidates_every_answer(corpus):
    """A shard whose bounded device wait gives up (the batch context's test
    hook) flags its bound record: the merged answers of that call are all
    invalid (counts -1); the failing shard reports the timeout on its next
    call, whose answers are invalid too (it joins the exchanges with neutral
    records), and the call after that is exact again."""
    import mars_b200 as mb
    E, mod, ts, imp, st, Qd = corpus
    B, K = 16, 10
    bc = mb.BatchContext(N, D, max_batch=256, max_k=256)
    ref = _run(lambda i, v, c: bc.query_batch_topk(st, Qd[:B], B, 600.0, 0.01, K, i, v, c, use_importance=True),
               B, K)
    stores, ctxs, offs = _shards(corpus, _even(3))
    try:
        call = lambda i, v, c: mb.shard_emulate_query_batch_topk(stores, ctxs, offs, Qd[:B], B, 600.0, 0.01, K, i,
                                                                  v, c, use_importance=True)
        ctxs[1].debug_wait(4096, 1)        # shard 1's grid-wide wait cannot end
        ids, vals, cnt = _run(call, B, K)
        assert np.all(cnt == -1) and np.all(ids == -1) and np.all(np.isneginf(vals))
        with pytest.raises(mb.MarsError) as e:
            _run(call, B, K)
        assert e.value.status == mb.MARS_ERR_TIMEOUT
        got = _run(call, B, K)
        assert np.array_equal(got[0], ref[0]) and np.array_equal(got[2], ref[2])
        assert np.array_equal(got[1].view(np.int32), ref[1].view(np.int32))
    finally:
        for s in stores:
            s.close()
