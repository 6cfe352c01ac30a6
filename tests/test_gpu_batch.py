"""Batched top-K on the tensor cores (mars_query_batch_topk) against the
exact single-query scan: because every short-listed row is rescored with the
scan's own arithmetic and incomplete short lists fall back to the scan, the
batched results must equal per-query mars_scan_topk bit for bit."""
import numpy as np
import pytest

import oracle as O
from _util import assert_topk_matches_scores

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


def _run(torch, N, D, B, K, filt=-1, use_imp=True, lam=0.01, t_q=600.0, seed=0, check_oracle=2,
         tf32_only=False, scale_row=None, scale_query=None, single_launch=True):
    import mars_b200 as mb
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=seed, ts_max=600.0)
    Q = datagen.queries(B, D, seed=seed + 1)
    pitch = (D + 3) // 4 * 4
    if scale_row is not None:            # a row beyond the fp16 range
        E[scale_row[0]] *= scale_row[1]
    if scale_query is not None:          # a query beyond the fp16 range
        Q[scale_query[0]] *= scale_query[1]
    Qp = np.zeros((B, pitch), np.float32)
    Qp[:, :D] = Q
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    bc = mb.BatchContext(N, D, max_batch=B, max_k=K)
    if tf32_only:
        bc.set_precision(True)
    bc.set_single_launch(single_launch)
    ctx = mb.QueryContext(N, D, max_k=K)
    Qd = torch.from_numpy(Qp).cuda()
    ids = torch.full((B, K), -7, dtype=torch.int32, device="cuda")
    vals = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    cnt = torch.zeros(B, dtype=torch.int32, device="cuda")
    bc.query_batch_topk(st, Qd, B, t_q, lam, K, ids, vals, cnt, modality_filter=filt,
                        use_importance=use_imp)
    torch.cuda.synchronize()
    stats = bc.last_stats()
    # per-query exact scans
    rids = torch.empty((B, K), dtype=torch.int32, device="cuda")
    rvals = torch.empty((B, K), dtype=torch.float32, device="cuda")
    rcnt = torch.zeros(B, dtype=torch.int32, device="cuda")
    for b in range(B):
        ctx.scan_topk(st, Qd[b], t_q, lam, K, rids[b], rvals[b], rcnt[b:b + 1], modality_filter=filt,
                      use_importance=use_imp)
    torch.cuda.synchronize()
    assert np.array_equal(cnt.cpu().numpy(), rcnt.cpu().numpy())
    assert np.array_equal(ids.cpu().numpy(), rids.cpu().numpy())
    assert np.array_equal(vals.cpu().numpy().view(np.uint32), rvals.cpu().numpy().view(np.uint32))
    oc = O.Corpus(E=E, ts=ts, mod=mod, imp=imp)
    for b in range(min(check_oracle, B)):
        ref = O.fused_scores(oc, Q[b], t_q, lam, modality_filter=filt, use_importance=use_imp)
        n = int(cnt[b].item())
        elig = None if filt < 0 else (mod == filt)
        assert_topk_matches_scores(ids[b, :n].cpu().numpy(), vals[b, :n].cpu().numpy(), ref, elig)
    return stats


def test_batch_small_smoke(torch_mod):
    stats = _run(torch_mod, N=8192, D=768, B=128, K=10)
    assert stats["path"] == 2


@pytest.mark.parametrize("tf32_only", [False, True])
@pytest.mark.parametrize("N,D,B,K", [(100_003, 768, 200, 100), (60_000, 768, 256, 10),
                                     (50_000, 64, 130, 32), (40_000, 100, 64, 50),
                                     # B >= 256: the three-kernel rescore, at D = 1024 and D = 100
                                     (30_011, 1024, 300, 64), (20_000, 100, 512, 32)])
def test_batch_matches_single_query_scans(torch_mod, N, D, B, K, tf32_only):
    """fp16 operands (default) and TF32 operands give the same results."""
    stats = _run(torch_mod, N, D, B, K, seed=N % 97, tf32_only=tf32_only)
    assert stats["path"] == (1 if tf32_only else (3 if B <= 64 else 2))
    assert stats["fallbacks"] <= max(2, B // 50), stats


def test_batch_with_modality_filter(torch_mod):
    stats = _run(torch_mod, 70_000, 768, 128, 20, filt=2, seed=5)
    assert stats["path"] == 2


def test_batch_out_of_fp16_range(torch_mod):
    """A row beyond the fp16 range covered by the error margin moves the
    batch to TF32 operands; a query beyond it is rescanned exactly on the
    device.  Results unchanged either way."""
    stats = _run(torch_mod, 30_000, 768, 64, 10, seed=8, scale_row=(123, 1e6))
    assert stats["path"] == 1
    stats = _run(torch_mod, 30_000, 768, 64, 10, seed=9, scale_query=(5, 1e6))
    assert stats["path"] == 3 and stats["fallbacks"] >= 1, stats
    stats = _run(torch_mod, 30_000, 768, 100, 10, seed=10, scale_query=(70, 1e6))
    assert stats["path"] == 2 and stats["fallbacks"] >= 1, stats


def test_batch_device_rescans_ties(torch_mod):
    """Every row identical: no short list can be proven complete, so every
    query is rescanned on the device; the answer is the K smallest ids."""
    import mars_b200 as mb
    torch = torch_mod
    N, D, B, K = 50_000, 64, 8, 10
    E = np.tile(np.random.default_rng(0).standard_normal((1, D)).astype(np.float32), (N, 1))
    st = mb.Store(N, D)
    st.upload(E, np.zeros(N, np.int32), np.zeros(N, np.float32), None)
    bc = mb.BatchContext(N, D, max_batch=B, max_k=K)
    Q = torch.from_numpy(np.random.default_rng(1).standard_normal((B, D)).astype(np.float32)).cuda()
    ids = torch.full((B, K), -7, dtype=torch.int32, device="cuda")
    vals = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    bc.query_batch_topk(st, Q, B, 0.0, 0.0, K, ids, vals)
    stats = bc.last_stats()
    assert stats["fallbacks"] == B, stats
    assert np.array_equal(ids.cpu().numpy(), np.tile(np.arange(K, dtype=np.int32), (B, 1)))


def test_batch_fp16_copy_follows_appends_and_deletes(torch_mod):
    """The store's fp16 copy is extended after appends and rebuilt after a
    delete: batched results keep matching the exact scans."""
    import mars_b200 as mb
    from mars_b200 import datagen
    torch = torch_mod
    N0, D, B, K = 20_000, 768, 64, 10
    E, mod, ts, imp = datagen.gaussian_corpus(N0, D, seed=21, ts_max=600.0)
    st = mb.Store(N0 + 5000, D)
    st.upload(E, mod, ts, imp)
    bc = mb.BatchContext(N0 + 5000, D, max_batch=B, max_k=K)
    ctx = mb.QueryContext(N0 + 5000, D, max_k=K)
    Q = torch.from_numpy(datagen.queries(B, D, seed=22)).cuda()

    def check():
        ids = torch.empty((B, K), dtype=torch.int32, device="cuda")
        vals = torch.empty((B, K), dtype=torch.float32, device="cuda")
        bc.query_batch_topk(st, Q, B, 600.0, 0.01, K, ids, vals, use_importance=True)
        torch.cuda.synchronize()
        assert bc.last_stats()["path"] == 3      # B = 64: the small-batch tiles
        for b in range(0, B, 7):
            i1 = torch.empty(K, dtype=torch.int32, device="cuda")
            v1 = torch.empty(K, dtype=torch.float32, device="cuda")
            ctx.scan_topk(st, Q[b], 600.0, 0.01, K, i1, v1, use_importance=True)
            torch.cuda.synchronize()
            assert np.array_equal(ids[b].cpu().numpy(), i1.cpu().numpy())
            assert np.array_equal(vals[b].cpu().numpy().view(np.uint32), v1.cpu().numpy().view(np.uint32))
        return ids

    check()
    # rows close to the queries appended: they must reach the fp16 copy
    rows = Q[:40].cpu().numpy() * 3.0
    st.append(rows, np.zeros(40, np.int32), np.full(40, 600.0, np.float32), np.ones(40, np.float32),
              normalize=False)
    ids = check()
    assert int(ids[0, 0].item()) >= N0
    st.delete(ids[:, 0].cpu().numpy())
    check()


@pytest.mark.parametrize("B", [1, 5, 16, 17, 48, 64])
@pytest.mark.parametrize("K", [3, 10, 64])
def test_batch_small_batches(torch_mod, B, K):
    """B <= 64 on fp16 operands: 128-row x B-query tiles with the queries
    resident in shared memory (gemm_small_kernel); results equal the scans."""
    stats = _run(torch_mod, 100_003, 768, B, K, seed=B * 7 + K, check_oracle=1)
    assert stats["path"] == 3
    assert stats["fallbacks"] == 0, stats


@pytest.mark.parametrize("B,K", [(5, 10), (16, 64), (64, 3)])
def test_batch_small_batches_three_launches(torch_mod, B, K):
    """The small-batch sample, thresholds and candidates as three launches
    (devices without cooperative launch) give the scans' results too."""
    stats = _run(torch_mod, 200_003, 768, B, K, seed=B + K, check_oracle=1, single_launch=False)
    assert stats["path"] == 3
    assert stats["fallbacks"] == 0, stats


@pytest.mark.parametrize("N,D,B,K,filt", [(60_001, 1024, 33, 10, -1), (30_000, 100, 16, 25, 1),
                                          (20_000, 64, 64, 100, -1), (1_000_000, 768, 16, 10, 2)])
def test_batch_small_batches_shapes(torch_mod, N, D, B, K, filt):
    stats = _run(torch_mod, N, D, B, K, filt=filt, seed=N % 101, check_oracle=1)
    assert stats["path"] == 3
    assert stats["fallbacks"] == 0, stats


def test_batch_small_corpus_uses_scans(torch_mod):
    stats = _run(torch_mod, 500, 768, 16, 10, seed=3)
    assert stats["path"] == 0
