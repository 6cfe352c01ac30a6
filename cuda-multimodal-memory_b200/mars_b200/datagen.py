"""Seeded synthetic corpora with the shapes and distributions of the
benchmark configurations (host-side numpy; nothing here runs on the GPU).

* gaussian_corpus: i.i.d. N(0,1) rows divided by (||v|| + 1e-8) -- the
  reference's normalisation rule (src/memory_graph.cpp:48-50) -- with
  modality uniform over `n_mod` classes, timestamps U[0, ts_max] and
  importance U[0, 1].
* cluster_corpus: points = centre + sigma * N(0,1) around `n_clusters`
  N(0,1) centres, then normalised (kNN-build and graph-search configs).
* random_bridges: every node gets `n_bridges` random edges to nodes of a
  different modality; the graph is made symmetric, rows sorted (CSR).
* queries: N(0,1) vectors normalised the same way.
"""
from __future__ import annotations

import numpy as np


def _normalize_rows(X: np.ndarray) -> np.ndarray:
    X = np.ascontiguousarray(X, dtype=np.float32)
    chunk = 1 << 16
    for s in range(0, X.shape[0], chunk):
        blk = X[s:s + chunk]
        nrm = np.sqrt(np.einsum("ij,ij->i", blk, blk, dtype=np.float32)).astype(np.float32)
        blk /= (nrm + np.float32(1e-8))[:, None]
    return X


def gaussian_corpus(N: int, D: int, seed: int = 42, n_mod: int = 4, ts_max: float = 10.0,
                    importance: bool = True):
    rng = np.random.default_rng(seed)
    E = np.empty((N, D), np.float32)
    chunk = 1 << 16
    for s in range(0, N, chunk):
        e = min(N, s + chunk)
        E[s:e] = rng.standard_normal((e - s, D), dtype=np.float32)
    E = _normalize_rows(E)
    mod = rng.integers(0, n_mod, size=N, dtype=np.int32)
    ts = rng.uniform(0.0, ts_max, size=N).astype(np.float32)
    imp = rng.uniform(0.0, 1.0, size=N).astype(np.float32) if importance else None
    return E, mod, ts, imp


ROW_CHUNK = 1 << 16


def gaussian_rows(lo: int, hi: int, D: int, seed: int = 42, n_mod: int = 4,
                  ts_max: float = 10.0):
    """Rows [lo, hi) of a corpus defined chunk by chunk (chunk c of ROW_CHUNK
    rows is drawn from its own generator seeded (seed, c)), so any row range
    -- e.g. one GPU's shard -- is identical to the same rows of the whole
    corpus.  Returns E (normalised), modality, timestamp, importance."""
    n = hi - lo
    E = np.empty((n, D), np.float32)
    mod = np.empty(n, np.int32)
    ts = np.empty(n, np.float32)
    imp = np.empty(n, np.float32)
    c0, c1 = lo // ROW_CHUNK, (hi - 1) // ROW_CHUNK if hi > lo else lo // ROW_CHUNK - 1
    for c in range(c0, c1 + 1):
        rng = np.random.default_rng([seed, c])
        base = c * ROW_CHUNK
        m = ROW_CHUNK
        e = rng.standard_normal((m, D), dtype=np.float32)
        md = rng.integers(0, n_mod, size=m, dtype=np.int32)
        t = rng.uniform(0.0, ts_max, size=m).astype(np.float32)
        im = rng.uniform(0.0, 1.0, size=m).astype(np.float32)
        a, b = max(lo, base), min(hi, base + m)
        E[a - lo:b - lo] = e[a - base:b - base]
        mod[a - lo:b - lo] = md[a - base:b - base]
        ts[a - lo:b - lo] = t[a - base:b - base]
        imp[a - lo:b - lo] = im[a - base:b - base]
    return _normalize_rows(E), mod, ts, imp


def cluster_corpus(N: int, D: int, n_clusters: int, sigma: float, seed: int = 42,
                   n_mod: int = 4, ts_max: float = 10.0):
    rng = np.random.default_rng(seed)
    centres = rng.standard_normal((n_clusters, D), dtype=np.float32)
    lab = rng.integers(0, n_clusters, size=N)
    E = np.empty((N, D), np.float32)
    chunk = 1 << 16
    for s in range(0, N, chunk):
        e = min(N, s + chunk)
        E[s:e] = centres[lab[s:e]] + np.float32(sigma) * rng.standard_normal((e - s, D),
                                                                             dtype=np.float32)
    E = _normalize_rows(E)
    mod = rng.integers(0, n_mod, size=N, dtype=np.int32)
    ts = rng.uniform(0.0, ts_max, size=N).astype(np.float32)
    return E, mod, ts, lab.astype(np.int32)


def queries(B: int, D: int, seed: int = 0x5EED0000):
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((B, D), dtype=np.float32)
    return _normalize_rows(Q)


def random_bridges(mod: np.ndarray, n_bridges: int = 4, seed: int = 7):
    """Symmetric CSR: each node links to n_bridges random nodes of other modalities."""
    rng = np.random.default_rng(seed)
    mod = np.asarray(mod, np.int32)
    N = mod.shape[0]
    n_mod = int(mod.max()) + 1 if N else 0
    pools = [np.flatnonzero(mod == m).astype(np.int64) for m in range(n_mod)]
    src = np.repeat(np.arange(N, dtype=np.int64), n_bridges)
    # choose a different modality uniformly, then a uniform node of it
    shift = rng.integers(1, max(n_mod, 2), size=src.shape[0])
    tm = (mod[src] + shift) % max(n_mod, 1)
    dst = np.empty_like(src)
    for m in range(n_mod):
        sel = np.flatnonzero(tm == m)
        if pools[m].shape[0] == 0 or sel.shape[0] == 0:
            dst[sel] = -1
            continue
        dst[sel] = pools[m][rng.integers(0, pools[m].shape[0], size=sel.shape[0])]
    ok = (dst >= 0) & (dst != src)
    a = np.concatenate([src[ok], dst[ok]])
    b = np.concatenate([dst[ok], src[ok]])
    key = np.unique(a * N + b)
    a = (key // N).astype(np.int32)
    b = (key % N).astype(np.int32)
    row_offsets = np.zeros(N + 1, np.int32)
    np.add.at(row_offsets, a.astype(np.int64) + 1, 1)
    row_offsets = np.cumsum(row_offsets, dtype=np.int64).astype(np.int32)
    return row_offsets, b
