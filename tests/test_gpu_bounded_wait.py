"""The bounded grid-wide wait of the single-launch small-batch path gives up
cleanly.

The fused launch's epilogue warps meet on a grid-wide arrival counter.  The
test hook mars_batch_ctx_debug_wait makes the next call wait for one arrival
that no CTA makes (a counter that nothing raises far enough), with a short
poll limit.  No GPU fault is involved: the wait runs out, records its status
word and the kernel carries on.  The test checks that

* the failed call's results are not served (counts -1, ids -1, scores -inf);
* its status reaches the host as MARS_ERR_TIMEOUT, through
  mars_batch_last_stats or through the next call;
* the call after that is bit-identical to the per-query exact scans (the
  grid counter was reset once the stream was idle).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N, D, B, K = 200_000, 768, 16, 10


@pytest.fixture(scope="module")
def setup():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=11, ts_max=600.0)
    Q = datagen.queries(B, D, seed=12)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    ctx = mb.QueryContext(N, D, max_k=K)
    Qd = torch.from_numpy(Q).cuda()
    rids = torch.empty((B, K), dtype=torch.int32, device="cuda")
    rvals = torch.empty((B, K), dtype=torch.float32, device="cuda")
    ctx.scan_topk_multi(st, Qd, B, 600.0, 0.01, K, rids, rvals, use_importance=True)
    torch.cuda.synchronize()
    return st, Qd, rids.cpu().numpy(), rvals.cpu().numpy()


def _call(bc, st, Qd):
    import torch
    ids = torch.full((B, K), -7, dtype=torch.int32, device="cuda")
    vals = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    cnt = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    bc.query_batch_topk(st, Qd, B, 600.0, 0.01, K, ids, vals, cnt, use_importance=True)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), vals.cpu().numpy(), cnt.cpu().numpy()


def _assert_exact(got, rids, rvals):
    ids, vals, cnt = got
    assert np.all(cnt == K)
    assert np.array_equal(ids, rids)
    assert np.array_equal(vals.view(np.uint32), rvals.view(np.uint32))


def test_wait_gives_up_results_invalid_status_timeout_then_recovers(setup):
    import mars_b200 as mb
    st, Qd, rids, rvals = setup
    bc = mb.BatchContext(N, D, max_batch=B, max_k=K)
    _assert_exact(_call(bc, st, Qd), rids, rvals)
    assert bc.last_stats()["path"] == 3

    # 4096 polls of >= 128 ns: the wait gives up within milliseconds
    bc.debug_wait(4096, 1)
    ids, vals, cnt = _call(bc, st, Qd)
    assert np.all(cnt == -1), cnt
    assert np.all(ids == -1)
    assert np.all(np.isneginf(vals))
    with pytest.raises(mb.MarsError) as e:
        bc.last_stats()
    assert e.value.status == mb.MARS_ERR_TIMEOUT
    assert "gave up" in str(e.value)

    # the hook held for one call only; the counter was reset
    _assert_exact(_call(bc, st, Qd), rids, rvals)
    bc.last_stats()


def test_timeout_reported_by_the_next_call(setup):
    import mars_b200 as mb
    st, Qd, rids, rvals = setup
    bc = mb.BatchContext(N, D, max_batch=B, max_k=K)
    bc.debug_wait(4096, 1)
    ids, _, cnt = _call(bc, st, Qd)       # synchronised: its status copy has landed
    assert np.all(cnt == -1) and np.all(ids == -1)
    with pytest.raises(mb.MarsError) as e:
        _call(bc, st, Qd)                 # returns the previous call's status, runs nothing
    assert e.value.status == mb.MARS_ERR_TIMEOUT
    _assert_exact(_call(bc, st, Qd), rids, rvals)
    # three launches instead of the cooperative one: no grid-wide wait, the
    # hook's extra arrivals are never waited for
    bc.set_single_launch(False)
    bc.debug_wait(4096, 1)
    _assert_exact(_call(bc, st, Qd), rids, rvals)
    bc.last_stats()
