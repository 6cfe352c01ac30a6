"""Comparison helpers shared by the parity tests.

Scores are fp32 and the reference's summation order (cuBLAS SGEMV / NumPy
BLAS) is unspecified, so result lists are compared tie-aware: ids must agree
exactly wherever the scores are separated by more than the tolerance, and
inside a group of scores closer than the tolerance only the count and the
score values have to agree.
"""
from __future__ import annotations

import numpy as np

# Relative score tolerance stated by the build target (1e-5) plus an absolute
# floor for scores near zero.
RTOL = 1e-5
ATOL = 1e-7


def close(a, b, rtol=RTOL, atol=ATOL) -> np.ndarray:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b) <= atol + rtol * np.maximum(np.abs(a), np.abs(b))


def assert_ranked_equivalent(ids_a, scores_a, ids_b, scores_b, hops_a=None, hops_b=None,
                             rtol=RTOL, atol=ATOL, what=""):
    """Two ranked (score-descending) result lists describe the same answer."""
    ids_a = np.asarray(ids_a)
    ids_b = np.asarray(ids_b)
    scores_a = np.asarray(scores_a, np.float64)
    scores_b = np.asarray(scores_b, np.float64)
    assert ids_a.shape == ids_b.shape, f"{what}: lengths {ids_a.shape} vs {ids_b.shape}"
    if ids_a.size == 0:
        return
    assert np.all(close(scores_a, scores_b, rtol, atol)), \
        f"{what}: scores differ\n{scores_a}\n{scores_b}"
    kth = min(scores_a[-1], scores_b[-1])
    tol = atol + rtol * abs(kth)
    sure_a = set(ids_a[scores_a > kth + tol].tolist())
    sure_b = set(ids_b[scores_b > kth + tol].tolist())
    assert sure_a == sure_b, f"{what}: id sets differ above the boundary\n{ids_a}\n{ids_b}"
    # inside groups of near-equal scores the order is free; outside it is fixed
    pos_b = {int(i): k for k, i in enumerate(ids_b.tolist())}
    for k, i in enumerate(ids_a.tolist()):
        if i in pos_b:
            k2 = pos_b[i]
            assert close(scores_a[k], scores_b[k2], rtol, atol), \
                f"{what}: id {i} scores {scores_a[k]} vs {scores_b[k2]}"
            if hops_a is not None and hops_b is not None:
                assert int(hops_a[k]) == int(hops_b[k2]), f"{what}: id {i} hops differ"


def assert_topk_matches_scores(ids, vals, all_scores, eligible=None, rtol=RTOL, atol=ATOL,
                               what=""):
    """ids/vals (descending) are a valid top-K of all_scores up to near-ties."""
    ids = np.asarray(ids)
    vals = np.asarray(vals, np.float64)
    s = np.asarray(all_scores, np.float64)
    if eligible is not None:
        s = np.where(eligible, s, -np.inf)
    K = ids.shape[0]
    order = np.lexsort((np.arange(s.shape[0]), -s))
    ref_ids = order[:K]
    ref_vals = s[ref_ids]
    assert len(set(ids.tolist())) == K, f"{what}: duplicate ids {ids}"
    assert np.all(np.diff(vals) <= 0), f"{what}: not descending {vals}"
    assert np.all(close(vals, s[ids], rtol, atol)), f"{what}: returned scores disagree"
    assert_ranked_equivalent(ids, vals, ref_ids, ref_vals, rtol=rtol, atol=atol, what=what)


def assert_bfs_set_valued(oracle_mod, corpus, q, t_q, lam, K, hops, decay, ref_ids, ref_scores,
                          ref_hops, ours_scores=None, use_importance=False, rtol=RTOL, atol=ATOL,
                          what=""):
    """Check a reference BFS answer whose parent choice is racy (first claimer
    wins, src/memory_cuda.cu:505-512): every returned node must be visited at
    the same hop as in the canonical BFS, and its score must equal
    fmaxf(parent * decay, own * 0.8) for SOME parent one level closer.  The
    canonical (best-parent) answer dominates: its k-th score is >= the
    reference's."""
    O = oracle_mod
    final = O.fused_scores(corpus, q, t_q, lam, use_importance=use_importance)
    ids, vals = O.topk(final, corpus.mod, -1, K)
    visited = O.bfs(corpus, ids, vals, final, hops, decay)
    vmap = {int(v["node_id"]): v for v in visited}
    ro, ci = corpus.row_offsets, corpus.col_indices
    for nid, s, h in zip(np.asarray(ref_ids).tolist(), np.asarray(ref_scores).tolist(),
                         np.asarray(ref_hops).tolist()):
        assert nid in vmap, f"{what}: reference returned an unvisited node {nid}"
        assert int(vmap[nid]["hops"]) == h, f"{what}: node {nid} hop differs"
        if h == 0:
            assert close(s, vmap[nid]["score"], rtol, atol), f"{what}: seed {nid} score"
            continue
        nbrs = ci[ro[nid]:ro[nid + 1]]
        possible = [max(np.float32(vmap[int(p)]["score"]) * np.float32(decay),
                        np.float32(final[nid]) * np.float32(0.8))
                    for p in nbrs if int(p) in vmap and int(vmap[int(p)]["hops"]) == h - 1]
        assert any(close(s, p, rtol, atol) for p in possible), \
            f"{what}: node {nid} score {s} not reachable from any parent {possible}"
    if ours_scores is not None and len(ours_scores) and len(ref_scores):
        assert float(ours_scores[-1]) >= float(ref_scores[-1]) - atol - rtol * abs(ref_scores[-1])


def load_golden(path: str):
    """np.load of a golden fixture after checking its SHA-256 against the
    MANIFEST.sha256 beside it: a fixture that was truncated, corrupted or
    replaced is refused (ValueError) instead of silently pinning the oracle
    to wrong vectors."""
    import hashlib
    import os
    folder, name = os.path.split(path)
    want = None
    with open(os.path.join(folder, "MANIFEST.sha256")) as f:
        for line in f:
            parts = line.split()
            if len(parts) == 2 and parts[1] == name:
                want = parts[0]
    if want is None:
        raise ValueError(f"{name}: not listed in MANIFEST.sha256")
    with open(path, "rb") as f:
        got = hashlib.sha256(f.read()).hexdigest()
    if got != want:
        raise ValueError(f"{name}: SHA-256 {got} does not match the manifest ({want})")
    return np.load(path)

