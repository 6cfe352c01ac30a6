"""Pin the CPU oracle against the reference's own outputs.

The golden vectors were produced by the reference's NumPy pipeline
(scripts/bench_cpu.py:91-146) by tests/golden/make_golden.py.  Depth 0 and 1
must agree up to near-ties.  At depth 2 the reference resolves a node reached
from several parents by frontier order (first claimer), the oracle by the best
parent; there the set of visited ids and hops must agree and every reference
score must be one of the values some parent could have produced.
"""
import json
import os

import numpy as np
import pytest

import oracle as O
from _util import assert_ranked_equivalent, close, load_golden

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = ["pipeline_d64", "pipeline_d768"]


def _load(name):
    z = load_golden(os.path.join(HERE, "golden", f"{name}.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    corpus = O.Corpus(E=z["emb"], ts=z["ts"], mod=z["mods"], row_offsets=z["row_off"],
                      col_indices=z["col_idx"])
    return z, meta, corpus


def test_corrupt_or_unlisted_fixture_is_refused(tmp_path):
    """A fixture whose bytes changed (one flipped byte) or that the manifest
    does not list is refused before any test reads it."""
    import shutil
    src = os.path.join(HERE, "golden")
    shutil.copy(os.path.join(src, "MANIFEST.sha256"), tmp_path / "MANIFEST.sha256")
    shutil.copy(os.path.join(src, "pipeline_d64.npz"), tmp_path / "pipeline_d64.npz")
    load_golden(str(tmp_path / "pipeline_d64.npz"))           # intact: loads
    raw = bytearray((tmp_path / "pipeline_d64.npz").read_bytes())
    raw[len(raw) // 2] ^= 0x01
    (tmp_path / "pipeline_d64.npz").write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="does not match"):
        load_golden(str(tmp_path / "pipeline_d64.npz"))
    shutil.copy(os.path.join(src, "pipeline_d64.npz"), tmp_path / "other.npz")
    with pytest.raises(ValueError, match="not listed"):
        load_golden(str(tmp_path / "other.npz"))


@pytest.mark.parametrize("name", CASES)
def test_golden_csr_is_valid(name):
    z, meta, c = _load(name)
    ro, ci = z["row_off"], z["col_idx"]
    N = meta["N"]
    assert ro.shape == (N + 1,) and ro[0] == 0 and ro[-1] == ci.shape[0]
    assert np.all(np.diff(ro) >= 0) and np.all((ci >= 0) & (ci < N))


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("dot_order", [O.DOT_CANONICAL, O.DOT_F64, O.DOT_REF_BLOCK256])
def test_oracle_matches_reference_pipeline(name, dot_order):
    z, meta, c = _load(name)
    n_checked = 0
    for di, (lam, qts) in enumerate(meta["decays"]):
        for k in meta["top_ks"]:
            for h in meta["hops"]:
                tag = f"d{di}_k{k}_h{h}"
                for qi in range(z["queries"].shape[0]):
                    r = O.query(c, z["queries"][qi], qts, top_k=k, bfs_max_hops=h, lam=lam,
                                bfs_score_decay=meta["bfs_score_decay"], dot_order=dot_order)
                    gi, gs, gh = z["ids_" + tag][qi], z["scores_" + tag][qi], z["hops_" + tag][qi]
                    if h <= 1:
                        assert_ranked_equivalent(r["node_id"], r["score"], gi, gs, r["hops"], gh,
                                                 what=f"{name} {tag} q{qi}")
                    else:
                        _check_depth2(c, z, qi, qts, lam, k, r, gi, gs, gh, meta, dot_order)
                    n_checked += 1
    assert n_checked == len(meta["decays"]) * len(meta["top_ks"]) * len(meta["hops"]) * 6


def _check_depth2(c, z, qi, qts, lam, k, r, gi, gs, gh, meta, dot_order):
    """Set-valued check: the reference score of every returned node must equal
    max(parent*decay, final*0.8) for SOME parent one hop closer."""
    q = z["queries"][qi]
    final = O.fused_scores(c, q, qts, lam, dot_order=dot_order)
    ids, vals = O.topk(final, c.mod, -1, k)
    visited = O.bfs(c, ids, vals, final, 2, meta["bfs_score_decay"])
    vmap = {int(v["node_id"]): v for v in visited}
    ro, ci = z["row_off"], z["col_idx"]
    for nid, s, h in zip(gi.tolist(), gs.tolist(), gh.tolist()):
        assert nid in vmap, f"reference returned an unvisited node {nid}"
        assert int(vmap[nid]["hops"]) == h
        if h == 0:
            assert close(s, vmap[nid]["score"])
            continue
        nbrs = ci[ro[nid]:ro[nid + 1]]
        possible = [max(np.float32(vmap[int(p)]["score"]) * np.float32(0.5),
                        np.float32(final[nid]) * np.float32(0.8))
                    for p in nbrs if int(p) in vmap and int(vmap[int(p)]["hops"]) == h - 1]
        assert any(close(s, p) for p in possible), f"node {nid}: {s} not in {possible}"
    # the canonical answer dominates: its k-th score is >= the reference's
    assert r["score"][-1] >= gs[-1] - 1e-6


def test_dot_orders_agree_within_tolerance():
    rng = np.random.default_rng(3)
    for D in (4, 64, 96, 100, 768, 1030):
        a = rng.standard_normal(D).astype(np.float32)
        b = rng.standard_normal(D).astype(np.float32)
        exact = float(np.dot(a.astype(np.float64), b.astype(np.float64)))
        for order in (O.DOT_CANONICAL, O.DOT_SEQ, O.DOT_F64, O.DOT_REF_BLOCK256, O.DOT_REF_WARP,
                      O.DOT_FAST):
            v = O.dot(a, b, order)
            assert abs(v - exact) <= 1e-5 * np.sqrt(D) * np.linalg.norm(a) * np.linalg.norm(b)


def test_l2_normalize_matches_engine_server_rule():
    rng = np.random.default_rng(5)
    v = rng.standard_normal(768).astype(np.float32)
    got = O.l2_normalize(v)
    # src/engine_server.cu:165-171: sequential fp32 sum of squares
    norm = np.float32(0.0)
    for x in v:
        norm = np.float32(norm + np.float32(x * x))
    norm = np.float32(np.sqrt(norm)) + np.float32(1e-8)
    assert np.array_equal(got, (v / norm).astype(np.float32))


def test_reference_host_tests_pass():
    """The reference's own host tests (tests/test_memory_graph.cpp) on its
    corpus / NSN generator, built from its sources into oracle/_ref."""
    import subprocess
    exe = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "ref_host_tests")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "0 failed" in r.stdout, r.stdout[-1000:]
