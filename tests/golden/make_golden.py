"""Generate golden vectors from the reference's own CPU pipeline.

The reference ships a NumPy mirror of its four CUDA stages,
``scripts/bench_cpu.py`` (``build_graph`` :18-33, ``build_nsn_edges`` :36-88,
``pipeline`` :91-146).  This script imports that module from a checkout of the
reference, runs it on small seeded corpora and stores inputs and outputs as
``.npz`` fixtures next to this file.  The fixtures are committed; the tests
read only them, so neither the tests nor the GPU box need the reference.

Run (in a container that has the reference checkout):

    python tests/golden/make_golden.py --ref /path/to/cuda-multimodal-memory
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, n_text, n_audio, n_image, dim, corpus seed)
CASES = [
    ("pipeline_d64", 300, 150, 150, 64, 42),
    ("pipeline_d768", 100, 50, 50, 768, 7),
]
N_QUERIES = 6
TOP_KS = (5, 10)
HOPS = (0, 1, 2)
# (lambda, query timestamp): the reference's default 1e-8 over U[0, 1e7]
# timestamps is almost no decay; 2e-7 decays the oldest rows to exp(-2).
DECAYS = ((1e-8, 1e7), (2e-7, 1e7))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MARS_REFERENCE_ROOT"),
                    help="root of the reference checkout (or MARS_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set MARS_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, os.path.join(args.ref, "scripts"))
    import bench_cpu  # the reference's own module

    for name, nt, na, ni, dim, seed in CASES:
        emb, mods, ts, N = bench_cpu.build_graph(nt, na, ni, dim, seed=seed)
        row_off, col_idx = bench_cpu.build_nsn_edges(N, mods)
        rng = np.random.default_rng(1000 + seed)
        queries = np.zeros((N_QUERIES, dim), np.float32)
        for i in range(N_QUERIES):
            q = rng.normal(0, 1, size=dim).astype(np.float32)
            q /= (np.linalg.norm(q) + 1e-8)      # as bench_cpu.py:172-173
            queries[i] = q
        out = dict(emb=emb, mods=mods.astype(np.int32), ts=ts.astype(np.float32),
                   row_off=row_off.astype(np.int32), col_idx=col_idx.astype(np.int32),
                   queries=queries)
        meta = dict(case=name, N=int(N), dim=dim, seed=seed, top_ks=TOP_KS, hops=HOPS,
                    decays=DECAYS, bfs_score_decay=0.5,
                    source="scripts/bench_cpu.py:pipeline (reference), imported unchanged")
        for di, (lam, qts) in enumerate(DECAYS):
            for k in TOP_KS:
                for h in HOPS:
                    ids = np.full((N_QUERIES, k), -1, np.int32)
                    sc = np.zeros((N_QUERIES, k), np.float32)
                    md = np.full((N_QUERIES, k), -1, np.int32)
                    hp = np.full((N_QUERIES, k), -1, np.int32)
                    for qi in range(N_QUERIES):
                        res, _, _ = bench_cpu.pipeline(emb, mods, ts, row_off, col_idx,
                                                       queries[qi], qts, top_k=k, bfs_hops=h,
                                                       lam=lam, decay=0.5)
                        for j, (nid, s, m, hh) in enumerate(res):
                            ids[qi, j], sc[qi, j], md[qi, j], hp[qi, j] = nid, s, m, hh
                    tag = f"d{di}_k{k}_h{h}"
                    out[f"ids_{tag}"] = ids
                    out[f"scores_{tag}"] = sc
                    out[f"mods_{tag}"] = md
                    out[f"hops_{tag}"] = hp
        out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        print(f"wrote {path}  N={N} dim={dim} edges={len(col_idx)}")
    # the checksums the tests verify before they read a fixture
    import hashlib
    lines = []
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            with open(os.path.join(HERE, f), "rb") as fh:
                lines.append(f"{hashlib.sha256(fh.read()).hexdigest()}  {f}")
    with open(os.path.join(HERE, "MANIFEST.sha256"), "w") as fh:
        fh.write("\n".join(lines) + "\n")


if __name__ == "__main__":
    main()
