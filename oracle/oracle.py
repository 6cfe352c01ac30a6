"""ctypes binding of the CPU oracle (oracle/libmars_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py for the CPU baseline and the reference arm.  The
product library never imports this module.

Every wrapper takes numpy arrays; see mars_oracle.h for the reference
file:line each C function restates.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmars_oracle.so")

DOT_CANONICAL = 0
DOT_SEQ = 1
DOT_F64 = 2
DOT_REF_BLOCK256 = 3
DOT_REF_WARP = 4
DOT_FAST = 5

FLT_MAX = float(np.finfo(np.float32).max)


class _Corpus(C.Structure):
    _fields_ = [
        ("N", C.c_int32), ("D", C.c_int32), ("pitch", C.c_int64),
        ("E", C.c_void_p), ("ts", C.c_void_p), ("imp", C.c_void_p), ("mod", C.c_void_p),
        ("row_offsets", C.c_void_p), ("col_indices", C.c_void_p),
        ("extra_nbrs", C.c_void_p), ("extra_cnt", C.c_void_p), ("extra_stride", C.c_int32),
        ("fixed_nbrs", C.c_void_p), ("fixed_degree", C.c_int32),
    ]


class _Config(C.Structure):
    _fields_ = [
        ("top_k", C.c_int32), ("bfs_max_hops", C.c_int32), ("lambda_", C.c_float),
        ("bfs_score_decay", C.c_float), ("modality_filter", C.c_int32),
        ("use_importance", C.c_int32), ("dot_order", C.c_int32),
    ]


class Result(C.Structure):
    _fields_ = [("node_id", C.c_int32), ("score", C.c_float),
                ("modality", C.c_int32), ("hops", C.c_int32)]


class _ScoreParams(C.Structure):
    _fields_ = [("q", C.c_void_p), ("t_q", C.c_float), ("lambda_", C.c_float),
                ("modality_filter", C.c_int32), ("use_importance", C.c_int32),
                ("dot_order", C.c_int32)]


class _CmngConfig(C.Structure):
    _fields_ = [("K", C.c_int32), ("beam_width", C.c_int32), ("max_iterations", C.c_int32),
                ("num_parents", C.c_int32), ("lambda_", C.c_float), ("dot_order", C.c_int32)]


class _CmngStats(C.Structure):
    _fields_ = [("iterations", C.c_int32), ("rows_scored", C.c_int32)]


RESULT_DTYPE = np.dtype([("node_id", "<i4"), ("score", "<f4"), ("modality", "<i4"), ("hops", "<i4")])

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"oracle library missing: {_LIB_PATH} (run make -C oracle)")
        L = C.CDLL(_LIB_PATH)
        L.orc_dot.restype = C.c_float
        L.orc_dot.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32]
        L.orc_l2_normalize.argtypes = [C.c_void_p, C.c_int32]
        L.orc_fused_scores.argtypes = [C.c_void_p, C.c_void_p, C.c_float, C.c_float, C.c_int32,
                                       C.c_int32, C.c_int32, C.c_void_p]
        L.orc_topk.restype = C.c_int32
        L.orc_topk.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                               C.c_void_p, C.c_void_p]
        L.orc_bfs.restype = C.c_int32
        L.orc_bfs.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p,
                              C.c_void_p, C.c_int32, C.c_float, C.c_void_p, C.c_int32]
        L.orc_finalize.restype = C.c_int32
        L.orc_finalize.argtypes = [C.c_void_p, C.c_int32, C.c_int32]
        L.orc_query.restype = C.c_int32
        L.orc_query.argtypes = [C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p]
        L.orc_query_batch_topk.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_float, C.c_float,
                                           C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                           C.c_void_p, C.c_void_p]
        L.orc_scan_topk_fast.restype = C.c_int32
        L.orc_scan_topk_fast.argtypes = [C.c_void_p, C.c_void_p, C.c_float, C.c_float, C.c_int32,
                                         C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]
        L.orc_knn.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                              C.c_void_p, C.c_void_p]
        L.orc_cmng_select.argtypes = [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p,
                                      C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p]
        L.orc_cmng_search.restype = C.c_int32
        L.orc_cmng_search.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_float,
                                      C.c_void_p, C.c_void_p, C.c_void_p]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


@dataclass
class Corpus:
    """Host corpus; arrays are kept alive by this object."""
    E: np.ndarray                    # N x pitch float32 (pitch >= D)
    ts: np.ndarray                   # N float32
    mod: np.ndarray                  # N int32
    imp: np.ndarray | None = None    # N float32
    row_offsets: np.ndarray | None = None
    col_indices: np.ndarray | None = None
    extra_nbrs: np.ndarray | None = None
    extra_cnt: np.ndarray | None = None
    fixed_nbrs: np.ndarray | None = None
    D: int | None = None

    def __post_init__(self):
        self.E = np.ascontiguousarray(self.E, dtype=np.float32)
        self.ts = np.ascontiguousarray(self.ts, dtype=np.float32)
        self.mod = np.ascontiguousarray(self.mod, dtype=np.int32)
        if self.imp is not None:
            self.imp = np.ascontiguousarray(self.imp, dtype=np.float32)
        for name in ("row_offsets", "col_indices", "extra_nbrs", "extra_cnt", "fixed_nbrs"):
            v = getattr(self, name)
            if v is not None:
                setattr(self, name, np.ascontiguousarray(v, dtype=np.int32))
        if self.D is None:
            self.D = self.E.shape[1]
        # the C restatement indexes these arrays by row without checks
        N = self.E.shape[0]
        if self.row_offsets is not None:
            if self.row_offsets.shape[0] != N + 1 or self.col_indices is None:
                raise ValueError(f"row_offsets needs N + 1 = {N + 1} entries and col_indices")
            if self.col_indices.shape[0] < int(self.row_offsets[-1]):
                raise ValueError("col_indices shorter than row_offsets[-1]")
        for name in ("ts", "mod", "imp", "extra_cnt", "fixed_nbrs", "extra_nbrs"):
            v = getattr(self, name)
            if v is not None and v.shape[0] != N:
                raise ValueError(f"{name} needs {N} rows, has {v.shape[0]}")

    def struct(self) -> _Corpus:
        s = _Corpus()
        s.N = self.E.shape[0]
        s.D = self.D
        s.pitch = self.E.shape[1]
        s.E, s.ts, s.imp, s.mod = _p(self.E), _p(self.ts), _p(self.imp), _p(self.mod)
        s.row_offsets, s.col_indices = _p(self.row_offsets), _p(self.col_indices)
        s.extra_nbrs, s.extra_cnt = _p(self.extra_nbrs), _p(self.extra_cnt)
        s.extra_stride = 0 if self.extra_nbrs is None else self.extra_nbrs.shape[1]
        s.fixed_nbrs = _p(self.fixed_nbrs)
        s.fixed_degree = 0 if self.fixed_nbrs is None else self.fixed_nbrs.shape[1]
        return s


def dot(a, b, order=DOT_CANONICAL) -> float:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return float(lib().orc_dot(_p(a), _p(b), a.shape[0], order))


def l2_normalize(v) -> np.ndarray:
    v = np.array(v, dtype=np.float32, copy=True)
    lib().orc_l2_normalize(_p(v), v.shape[0])
    return v


def fused_scores(c: Corpus, q, t_q, lam, modality_filter=-1, use_importance=False,
                 dot_order=DOT_CANONICAL) -> np.ndarray:
    q = _pad_query(q, c)
    out = np.empty(c.E.shape[0], dtype=np.float32)
    s = c.struct()
    lib().orc_fused_scores(C.byref(s), _p(q), t_q, lam, modality_filter, int(use_importance),
                           dot_order, _p(out))
    return out


def topk(scores, mod, modality_filter, K):
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    mod = np.ascontiguousarray(mod, dtype=np.int32)
    ids = np.full(K, -1, np.int32)
    vals = np.full(K, -FLT_MAX, np.float32)
    n = lib().orc_topk(_p(scores), _p(mod), modality_filter, scores.shape[0], K, _p(ids), _p(vals))
    return ids[:n], vals[:n]


def bfs(c: Corpus, seed_ids, seed_vals, final_scores, hops, decay, q=None, t_q=0.0, lam=0.0,
        modality_filter=-1, use_importance=False, dot_order=DOT_CANONICAL):
    seed_ids = np.ascontiguousarray(seed_ids, dtype=np.int32)
    seed_vals = np.ascontiguousarray(seed_vals, dtype=np.float32)
    N = c.E.shape[0]
    out = np.zeros(N, dtype=RESULT_DTYPE)
    s = c.struct()
    sp = None
    qq = None
    if final_scores is not None:
        final_scores = np.ascontiguousarray(final_scores, dtype=np.float32)
    else:
        qq = _pad_query(q, c)
        sp = _ScoreParams(_p(qq), t_q, lam, modality_filter, int(use_importance), dot_order)
    n = lib().orc_bfs(C.byref(s), _p(seed_ids), _p(seed_vals), seed_ids.shape[0],
                      _p(final_scores), None if sp is None else C.byref(sp), hops, decay,
                      _p(out), N)
    if n < 0:
        raise RuntimeError("orc_bfs overflow")
    return out[:n]


def finalize(visited, K):
    v = np.ascontiguousarray(visited.copy(), dtype=RESULT_DTYPE)
    n = lib().orc_finalize(_p(v), v.shape[0], K)
    return v[:n]


def query(c: Corpus, q, t_q, top_k=10, bfs_max_hops=2, lam=1e-8, bfs_score_decay=0.5,
          modality_filter=-1, use_importance=False, dot_order=DOT_CANONICAL):
    q = _pad_query(q, c)
    cfg = _Config(top_k, bfs_max_hops, lam, bfs_score_decay, modality_filter,
                  int(use_importance), dot_order)
    out = np.zeros(max(top_k, 1), dtype=RESULT_DTYPE)
    s = c.struct()
    n = lib().orc_query(C.byref(s), _p(q), t_q, C.byref(cfg), _p(out))
    return out[:n]


def query_batch_topk(c: Corpus, Q, t_q, lam, K, modality_filter=-1, use_importance=False,
                     dot_order=DOT_CANONICAL, n_threads=0):
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    if Q.shape[1] != c.E.shape[1]:
        Qp = np.zeros((Q.shape[0], c.E.shape[1]), np.float32)
        Qp[:, :Q.shape[1]] = Q
        Q = Qp
    B = Q.shape[0]
    ids = np.full((B, K), -1, np.int32)
    vals = np.full((B, K), -FLT_MAX, np.float32)
    s = c.struct()
    lib().orc_query_batch_topk(C.byref(s), _p(Q), B, t_q, lam, modality_filter,
                               int(use_importance), K, dot_order, n_threads, _p(ids), _p(vals))
    return ids, vals


def scan_topk_fast(c: Corpus, q, t_q, lam, K, modality_filter=-1, use_importance=False,
                   n_threads=0):
    q = _pad_query(q, c)
    ids = np.full(K, -1, np.int32)
    vals = np.full(K, -FLT_MAX, np.float32)
    s = c.struct()
    n = lib().orc_scan_topk_fast(C.byref(s), _p(q), t_q, lam, modality_filter,
                                 int(use_importance), K, n_threads, _p(ids), _p(vals))
    return ids[:n], vals[:n]


def knn(c: Corpus, rows, k, dot_order=DOT_CANONICAL, n_threads=0):
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    ids = np.full((rows.shape[0], k), -1, np.int32)
    vals = np.full((rows.shape[0], k), -1e30, np.float32)
    s = c.struct()
    lib().orc_knn(C.byref(s), _p(rows), rows.shape[0], k, dot_order, n_threads, _p(ids), _p(vals))
    return ids, vals


def cmng_select(knn_ids, mod, rows, degree, degree_cross, num_modalities=3):
    knn_ids = np.ascontiguousarray(knn_ids, dtype=np.int32)
    mod = np.ascontiguousarray(mod, dtype=np.int32)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    out = np.full((rows.shape[0], degree), -1, np.int32)
    lib().orc_cmng_select(_p(knn_ids), knn_ids.shape[1], _p(mod), mod.shape[0], _p(rows),
                          rows.shape[0], degree, degree_cross, num_modalities, _p(out))
    return out


def cmng_search(c: Corpus, neighbors, q, t_q, K=10, beam_width=128, max_iterations=64,
                num_parents=1, lam=1e-8, dot_order=DOT_CANONICAL):
    neighbors = np.ascontiguousarray(neighbors, dtype=np.int32)
    q = _pad_query(q, c)
    cfg = _CmngConfig(K, beam_width, max_iterations, num_parents, lam, dot_order)
    out = np.zeros(max(K, 1), dtype=RESULT_DTYPE)
    st = _CmngStats()
    s = c.struct()
    n = lib().orc_cmng_search(C.byref(s), _p(neighbors), neighbors.shape[1], _p(q), t_q,
                              C.byref(cfg), _p(out), C.byref(st))
    return out[:n], {"iterations": st.iterations, "rows_scored": st.rows_scored}


def _pad_query(q, c: Corpus):
    q = np.ascontiguousarray(q, dtype=np.float32)
    if q.shape[0] < c.E.shape[1]:
        qp = np.zeros(c.E.shape[1], np.float32)
        qp[:q.shape[0]] = q
        q = qp
    return q
