"""The reference's own tools, compiled from their unchanged sources against
this library (oracle/Makefile.ref), next to the same tools on the
reference's GPU path.

* engine_server (src/engine_server.cu): the JSON-line server that is the
  reference's insert caller.  One command script -- ADD rows, DELETE some,
  QUERY, ADD more (the server re-uploads), QUERY again, STATS, SHUTDOWN --
  goes to both servers.  Every QUERY answer of the drop-in server must equal
  the reference server's (tie-aware; the reference's default kernels are
  exact for K <= 8 and BFS depth <= 1, so those are the queries compared),
  and hop-free answers with larger K must equal the CPU oracle's on the
  corpus the server holds (rows normalised by the server's own rule).
* latency_bench (src/latency_bench.cu): a short run of both harnesses;
  the drop-in one prints the same JSON report (same keys, same config).

Skipped when oracle/_ref has not been built (it needs the reference
checkout at build time).
"""
import json
import os
import subprocess

import numpy as np
import pytest

from _util import assert_ranked_equivalent

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")


def _bin(name):
    p = os.path.join(REF, name)
    if not os.path.exists(p):
        pytest.skip(f"oracle/_ref/{name} not built")
    return p


def _emb(v):
    return "[" + ",".join(f"{x:.9g}" for x in v) + "]"   # 9 digits: float32 round-trips exactly


def _script(D, seed=3):
    rng = np.random.default_rng(seed)
    n1, n2 = 1500, 300
    raw = rng.standard_normal((n1 + n2, D)).astype(np.float32)
    mod = rng.integers(0, 3, n1 + n2).astype(np.int32)    # the reference's graph builder knows 3 modalities
    ts = rng.uniform(0.0, 100.0, n1 + n2).astype(np.float32)
    cmds, queries = [], []

    def add(i):
        cmds.append(json.dumps({"cmd": "ADD", "id": int(i), "modality": int(mod[i]), "timestamp": float(ts[i])})[:-1]
                    + f', "embedding": {_emb(raw[i])}}}')

    def query(K, hops, filt, q):
        queries.append((len(cmds), K, hops, filt, q))
        cmds.append(json.dumps({"cmd": "QUERY", "top_k": K, "bfs_max_hops": hops, "modality_filter": filt,
                                "timestamp": 100.0})[:-1] + f', "embedding": {_emb(q)}}}')

    for i in range(n1):
        add(i)
    deleted = rng.choice(n1, 25, replace=False)
    for i in deleted:
        cmds.append(json.dumps({"cmd": "DELETE", "id": int(i)}))
    qs = rng.standard_normal((16, D)).astype(np.float32)
    for j in range(8):
        query([5, 8][j % 2], j % 2, [-1, 2][(j // 2) % 2], qs[j])
    query(20, 0, -1, qs[8])
    query(40, 0, 1, qs[9])
    cmds.append(json.dumps({"cmd": "STATS"}))
    for i in range(n1, n1 + n2):
        add(i)
    for j in range(10, 16):
        query([8, 5][j % 2], j % 2, -1, qs[j])
    query(32, 0, -1, qs[10])
    cmds.append(json.dumps({"cmd": "STATS"}))
    cmds.append(json.dumps({"cmd": "SHUTDOWN"}))
    return "\n".join(cmds) + "\n", queries, raw, mod, ts, deleted


def _run(binary, D, text):
    r = subprocess.run([binary, "--dim", str(D)], input=text, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.strip()]


def _server_rows(raw, ts, deleted, n):
    """The server's corpus: add_node's normalisation (sequential fp32 sum of
    squares, sqrt + 1e-8, one division per component), tombstones zeroed."""
    x = raw[:n]
    norm2 = np.cumsum(x * x, axis=1, dtype=np.float32)[:, -1]    # sequential, like the server's loop
    E = x / (np.sqrt(norm2, dtype=np.float32) + np.float32(1e-8))[:, None]
    ts = ts[:n].copy()
    E[deleted] = 0.0
    ts[deleted] = -1.0
    return E.astype(np.float32), ts


def test_engine_server_dropin_matches_reference_server_and_oracle():
    import oracle as O
    D = 128
    text, queries, raw, mod, ts, deleted = _script(D)
    ours = _run(_bin("dropin_engine_server"), D, text)
    ref = _run(_bin("ref_engine_server"), D, text)
    assert len(ours) == len(ref) == len(text.splitlines())
    compared = 0
    for (pos, K, hops, filt, q) in queries:
        a, b = ours[pos]["results"], ref[pos]["results"]
        ga = (np.array([r["id"] for r in a]), np.array([r["score"] for r in a]), np.array([r["hops"] for r in a]))
        assert all(r["modality"] == mod[r["id"]] for r in a)
        if K <= 8:
            gb = (np.array([r["id"] for r in b]), np.array([r["score"] for r in b]), np.array([r["hops"] for r in b]))
            # scores travel as %.6f text: compare within that rounding
            assert_ranked_equivalent(ga[0], ga[1], gb[0], gb[1], ga[2], gb[2], rtol=1e-5, atol=2e-6,
                                     what=f"command {pos}")
            compared += 1
        if hops == 0:
            n = 1500 if pos < 1600 else 1800
            E, tsn = _server_rows(raw, ts, deleted, n)
            # the server passes the query through as given (no normalisation)
            oi, ov = O.scan_topk_fast(O.Corpus(E=E, ts=tsn, mod=mod[:n]), q, 100.0, 1e-8, K, modality_filter=filt)
            assert_ranked_equivalent(ga[0], ga[1], oi, ov, rtol=1e-5, atol=2e-6, what=f"oracle command {pos}")
    assert compared >= 12
    stats = [r for r in ours if "n" in r]
    assert [s["n"] for s in stats] == [1500, 1800]
    assert [s["n"] for s in stats] == [s["n"] for s in ref if "n" in s]
    assert [s["edges"] for s in stats] == [s["edges"] for s in ref if "n" in s]


def test_latency_bench_dropin_reports_the_reference_schema():
    args = ["1000", "5.0", "300", "2400"]
    outs = {}
    for name in ("dropin_latency_bench", "ref_latency_bench"):
        r = subprocess.run([_bin(name)] + args, capture_output=True, text=True, timeout=600)
        assert r.returncode in (0, 1), r.stderr[-2000:]     # 1: p99 above the budget
        outs[name] = json.loads(r.stdout)

    def keys(d, prefix=""):
        out = set()
        for k, v in d.items():
            out.add(prefix + k)
            if isinstance(v, dict):
                out |= keys(v, prefix + k + ".")
        return out

    a, b = outs["dropin_latency_bench"], outs["ref_latency_bench"]
    assert keys(a) == keys(b)
    assert a["config"] == b["config"]
    assert a["tool"] == b["tool"] == "cuda-multimodal-memory-latency-bench"
    for o in (a, b):
        w = o["wall_latency_ms"]
        assert 0 < w["p50"] <= w["p99"] <= w["max"]
    assert a["deadline"]["deadline_misses"] <= b["deadline"]["deadline_misses"] + 3
