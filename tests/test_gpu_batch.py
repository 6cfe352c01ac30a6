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


def _run(torch, N, D, B, K, filt=-1, use_imp=True, lam=0.01, t_q=600.0, seed=0, check_oracle=2):
    import mars_b200 as mb
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=seed, ts_max=600.0)
    Q = datagen.queries(B, D, seed=seed + 1)
    pitch = (D + 3) // 4 * 4
    Qp = np.zeros((B, pitch), np.float32)
    Qp[:, :D] = Q
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    bc = mb.BatchContext(N, D, max_batch=B, max_k=K)
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
    assert stats["path"] == 1


@pytest.mark.parametrize("N,D,B,K", [(100_003, 768, 200, 100), (60_000, 768, 256, 10),
                                     (50_000, 64, 130, 32), (40_000, 100, 64, 50)])
def test_batch_matches_single_query_scans(torch_mod, N, D, B, K):
    stats = _run(torch_mod, N, D, B, K, seed=N % 97)
    assert stats["path"] == 1
    assert stats["fallbacks"] <= max(2, B // 50), stats


def test_batch_with_modality_filter(torch_mod):
    stats = _run(torch_mod, 70_000, 768, 128, 20, filt=2, seed=5)
    assert stats["path"] == 1


def test_batch_small_corpus_uses_scans(torch_mod):
    stats = _run(torch_mod, 500, 768, 16, 10, seed=3)
    assert stats["path"] == 0
