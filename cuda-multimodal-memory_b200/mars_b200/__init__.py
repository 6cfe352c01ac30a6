"""Python binding of the MARS B200 C ABI (include/mars_b200.h).

A thin ctypes layer for tests, benchmarks and Python callers.  All compute
runs in lib/libmars_b200.so; importing this module fails loudly when that
library has not been built, and there is no CPU fallback.

Device buffers may be passed as torch tensors (their data_ptr is used) or as
raw integer addresses.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "lib", "libmars_b200.so")

MARS_OK = 0
MARS_ERR_INVALID = 1
MARS_ERR_CUDA = 2
MARS_ERR_OOM = 3
MARS_ERR_CAPACITY = 4
MARS_ERR_UNSUPPORTED = 5
MARS_ERR_TIMEOUT = 6
MARS_ERR_NO_DEVICE = 7
MARS_ERR_DEVICE = 8
MAX_TOP_K = 256          # MARS_MAX_TOP_K
NOALLOC_MAX_K = 128      # MARS_NOALLOC_MAX_K: K limit of scan_topk_noalloc
MAX_BFS_HOPS = 14

RESULT_DTYPE = np.dtype([("node_id", "<i4"), ("score", "<f4"), ("modality", "<i4"),
                         ("hops", "<i4")])


class MarsError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[{status}] {msg}")
        self.status = status


class RetrievalConfig(C.Structure):
    """mars_retrieval_config (RetrievalConfig, include/memory_cuda.cuh:92-99)."""
    _fields_ = [("top_k", C.c_int32), ("bfs_max_hops", C.c_int32),
                ("time_decay_lambda", C.c_float), ("bfs_score_decay", C.c_float),
                ("modality_filter", C.c_int32), ("use_importance", C.c_int32)]

    def __init__(self, top_k=10, bfs_max_hops=2, time_decay_lambda=1e-8, bfs_score_decay=0.5,
                 modality_filter=-1, use_importance=False):
        super().__init__(top_k, bfs_max_hops, time_decay_lambda, bfs_score_decay,
                         modality_filter, int(use_importance))


class RetrievalStats(C.Structure):
    _fields_ = [("gpu_ms_similarity", C.c_float), ("gpu_ms_topk", C.c_float),
                ("gpu_ms_bfs", C.c_float), ("gpu_ms_rerank", C.c_float),
                ("gpu_ms_total", C.c_float), ("nodes_scanned", C.c_int32),
                ("bfs_waves", C.c_int32), ("nodes_visited", C.c_int32)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class StoreInfo(C.Structure):
    _fields_ = [("device", C.c_int32), ("num_nodes", C.c_int32), ("capacity", C.c_int32),
                ("embedding_dim", C.c_int32), ("row_pitch", C.c_int32), ("num_edges", C.c_int32),
                ("csr_nodes", C.c_int32), ("edge_slack", C.c_int32),
                ("d_embeddings", C.c_void_p), ("d_modalities", C.c_void_p),
                ("d_timestamps", C.c_void_p), ("d_importance", C.c_void_p),
                ("d_row_offsets", C.c_void_p), ("d_col_indices", C.c_void_p),
                ("d_num_nodes", C.c_void_p)]


class BatchStats(C.Structure):
    _fields_ = [("path", C.c_int32), ("fallbacks", C.c_int32), ("candidates", C.c_int64),
                ("max_candidates", C.c_int32), ("sample_tiles", C.c_int32),
                ("sample_rank", C.c_int32), ("rescored", C.c_int64), ("gemm_ms", C.c_float)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class CmngConfig(C.Structure):
    """mars_cmng_config (CMNGSearchConfig, include/cmng.cuh:54-62)."""
    _fields_ = [("K", C.c_int32), ("beam_width", C.c_int32), ("max_iterations", C.c_int32),
                ("num_parents", C.c_int32), ("time_decay_lambda", C.c_float),
                ("modality_filter", C.c_int32), ("use_fp16", C.c_int32)]

    def __init__(self, K=10, beam_width=128, max_iterations=64, num_parents=1,
                 time_decay_lambda=1e-8, modality_filter=-1, use_fp16=False):
        super().__init__(K, beam_width, max_iterations, num_parents, time_decay_lambda,
                         modality_filter, int(use_fp16))


_VP = C.c_void_p
_I32 = C.c_int32
_F32 = C.c_float

# name -> argtypes (all return int status unless listed in _RESTYPE)
_SIGS = {
    "mars_store_create": [_I32, _I32, _I32, _I32, C.POINTER(_VP)],
    "mars_store_upload": [_VP, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _I32],
    "mars_store_append": [_VP, _I32, _VP, _VP, _VP, _VP, _I32, C.POINTER(_I32)],
    "mars_store_append_edges": [_VP, _I32, _VP, _VP],
    "mars_store_delete": [_VP, _I32, _VP],
    "mars_store_set_importance": [_VP, _I32, _I32, _VP],
    "mars_store_info_get": [_VP, C.POINTER(StoreInfo)],
    "mars_importance_fill": [_VP, _F32],
    "mars_importance_update": [_VP, _VP, _I32, _F32, _F32, _F32, _VP],
    "mars_novelty": [_VP, _VP, _VP, _VP, _VP],
    "mars_store_read": [_VP, _I32, _I32, _VP, _VP, _VP, _VP],
    "mars_store_destroy": [_VP],
    "mars_query_ctx_create": [_I32, _I32, _I32, _I32, C.POINTER(_VP)],
    "mars_query_ctx_destroy": [_VP],
    "mars_query_ctx_use_graph": [_VP, _I32],
    "mars_query_ctx_use_fused": [_VP, _I32],
    "mars_query_ctx_path_counts": [_VP, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)],
    "mars_query": [_VP, _VP, _VP, _F32, C.POINTER(RetrievalConfig), _VP, C.POINTER(_I32),
                   C.POINTER(RetrievalStats)],
    "mars_query_device": [_VP, _VP, _VP, _F32, C.POINTER(RetrievalConfig), _VP, _VP, _VP],
    "mars_query_once": [_VP, _VP, _F32, C.POINTER(RetrievalConfig), _VP, C.POINTER(_I32),
                        C.POINTER(RetrievalStats)],
    "mars_scan_topk": [_VP, _VP, _VP, _F32, _F32, _I32, _I32, _I32, _I32, _VP, _VP, _VP, _VP],
    "mars_scan_topk_multi": [_VP, _VP, _VP, _I32, _I32, _F32, _F32, _I32, _I32, _I32, _I32, _VP, _VP, _VP,
                             _VP],
    "mars_scan_topk_f16": [_VP, _VP, _VP, _I32, _I32, _F32, _F32, _I32, _I32, _I32, _I32, _VP, _VP, _VP, _VP],
    "mars_query_ctx_f16_stats": [_VP, _VP, _VP, _VP],
    "mars_topk_merge": [_VP, _VP, _VP, _I32, _I32, _VP, _VP, _VP, _VP],
    "mars_topk_merge_batch": [_VP, _VP, _VP, _I32, _I32, _I32, _VP, _VP, _VP, _VP],
    "mars_debug_fused_scores": [_VP, _VP, _VP, _F32, _F32, _I32, _I32, _VP, _VP],
    "mars_batch_ctx_create": [_I32, _I32, _I32, _I32, _I32, C.POINTER(_VP)],
    "mars_batch_ctx_destroy": [_VP],
    "mars_batch_ctx_set_precision": [_VP, _I32],
    "mars_batch_ctx_set_single_launch": [_VP, _I32],
    "mars_query_batch_topk": [_VP, _VP, _VP, _I32, _I32, _F32, _F32, _I32, _I32, _I32, _I32, _VP,
                              _VP, _VP, _VP],
    "mars_batch_last_stats": [_VP, C.POINTER(BatchStats)],
    "mars_batch_ctx_debug_wait": [_VP, C.c_uint32, _I32],
    "mars_shard_unique_id": [_VP],
    "mars_shard_comm_create": [_I32, _I32, _I32, _VP, _I32, _I32, C.POINTER(_VP)],
    "mars_shard_comm_create_timeout": [_I32, _I32, _I32, _VP, _I32, _I32, _I32, C.POINTER(_VP)],
    "mars_shard_comm_destroy": [_VP],
    "mars_shard_comm_status": [_VP],
    "mars_shard_comm_abort": [_VP],
    "mars_shard_comm_set_timing": [_VP, _I32],
    "mars_shard_comm_set_exchange_at_world1": [_VP, _I32],
    "mars_shard_last_times": [_VP, C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_float)],
    "mars_shard_query": [_VP, _VP, _VP, _VP, _VP, _I32, _VP, _F32, C.POINTER(RetrievalConfig), _I32, _VP,
                         C.POINTER(_I32)],
    "mars_shard_query_batch_topk": [_VP, _VP, _VP, _VP, _I32, _I32, _F32, _F32, _I32, _I32, _I32, _I32,
                                    _VP, _VP, _VP, _VP],
    "mars_shard_emulate_query_batch_topk": [_I32, _VP, _VP, _VP, _VP, _I32, _I32, _F32, _F32, _I32, _I32, _I32,
                                            _VP, _VP, _VP],
    "mars_cmng_build": [_VP, _I32, _I32, _I32, _VP, C.POINTER(C.c_float)],
    "mars_cmng_build_rows": [_VP, _I32, _I32, _I32, _I32, _I32, _VP, C.POINTER(C.c_float)],
    "mars_cmng_knn": [_VP, _I32, _VP, _VP, _VP],
    "mars_cmng_search_batch": [_VP, _VP, _I32, _VP, _I32, _I32, _F32, C.POINTER(CmngConfig), _VP,
                               _VP, _VP, _VP, _VP, _VP, _VP],
    "mars_cmng_ctx_create": [_I32, _I32, _I32, _I32, _I32, _I32, C.POINTER(_VP)],
    "mars_cmng_ctx_destroy": [_VP],
    "mars_cmng_ctx_set_bfs_smem_nodes": [_VP, _I32],
    "mars_cmng_search_bfs_batch": [_VP, _VP, _VP, _I32, _VP, _I32, _I32, _F32, C.POINTER(CmngConfig),
                                   _I32, _F32, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _VP],
    "mars_scan_topk_noalloc": [_VP, _I32, _VP, _VP, _VP, _I32, _I32, _VP, _F32, _F32, _I32, _I32,
                               _I32, _I32, _VP, _VP, _VP, _VP],
}
_RESTYPE = {"mars_last_error": C.c_char_p, "mars_status_string": C.c_char_p,
            "mars_abi_version": C.c_int, "mars_query_ctx_stream": C.c_void_p}

_lib = None


def lib() -> C.CDLL:
    """Load lib/libmars_b200.so (raises if it is missing: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"MARS B200 library not built: {LIB_PATH} "
                              "(run `make -C cuda-multimodal-memory_b200`)")
        L = C.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = C.c_int
        for name, rt in _RESTYPE.items():
            getattr(L, name).restype = rt
        L.mars_status_string.argtypes = [C.c_int]
        L.mars_query_ctx_stream.argtypes = [_VP]
        _lib = L
    return _lib


def exported_symbols():
    return sorted(list(_SIGS) + list(_RESTYPE))


def _check(status: int):
    if status != MARS_OK:
        raise MarsError(status, lib().mars_last_error().decode())


def _ptr(x):
    """Device/host address of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    raise TypeError(f"cannot take the address of {type(x)}")


def _host(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


_STREAM_LEGACY = 1   # cudaStreamLegacy: the legacy default stream, named explicitly


def _cuda_tensors(arrays):
    return [a for a in arrays if getattr(a, "is_cuda", False)]


def _stream(stream, *arrays):
    """The stream a device call runs on.  An explicit stream is used as given.
    Without one, a call that reads or writes torch CUDA tensors runs on
    torch's current stream of their device, so it follows the work that made
    its inputs and precedes the work that reads its outputs, as a torch op
    would (cudaStreamLegacy names torch's default stream, since NULL means
    the library object's own stream).  Otherwise NULL."""
    if stream is not None:
        return stream
    t = _cuda_tensors(arrays)
    if not t:
        return None
    import torch
    h = torch.cuda.current_stream(t[0].device).cuda_stream
    return h if h != 0 else _STREAM_LEGACY


def _settle(*arrays):
    """Store writes run on the store's own stream and return when done: torch
    CUDA inputs must be complete before the library reads them."""
    t = _cuda_tensors(arrays)
    if t:
        import torch
        torch.cuda.current_stream(t[0].device).synchronize()


class Store:
    """Device store (DeviceMemoryGraph) with in-place streaming append."""

    def __init__(self, capacity: int, dim: int, device: int = 0, edge_slack: int = 0):
        h = C.c_void_p()
        _check(lib().mars_store_create(device, capacity, dim, edge_slack, C.byref(h)))
        self.handle = h
        self.device = device
        self.dim = dim
        self._keep = []

    def upload(self, E, modalities, timestamps, importance=None, row_offsets=None,
               col_indices=None):
        """E etc. may be numpy arrays (host) or torch tensors (host or device)."""
        keep = []

        def prep(a, dt):
            if a is None:
                return None
            if isinstance(a, np.ndarray) or not hasattr(a, "data_ptr"):
                a = _host(a, dt)
            keep.append(a)
            return _ptr(a)
        n = int(E.shape[0])
        ne = 0 if col_indices is None else int(col_indices.shape[0])
        _settle(E, modalities, timestamps, importance, row_offsets, col_indices)
        _check(lib().mars_store_upload(self.handle, n, prep(E, np.float32),
                                       prep(modalities, np.int32), prep(timestamps, np.float32),
                                       prep(importance, np.float32),
                                       prep(row_offsets, np.int32), prep(col_indices, np.int32),
                                       ne))

    def append(self, E, modalities, timestamps, importance=None, normalize=True) -> int:
        E = _host(E, np.float32) if not hasattr(E, "data_ptr") else E
        mod = _host(modalities, np.int32) if not hasattr(modalities, "data_ptr") else modalities
        ts = _host(timestamps, np.float32) if not hasattr(timestamps, "data_ptr") else timestamps
        imp = importance
        if imp is not None and not hasattr(imp, "data_ptr"):
            imp = _host(imp, np.float32)
        first = C.c_int32()
        _settle(E, mod, ts, imp)
        _check(lib().mars_store_append(self.handle, int(E.shape[0]), _ptr(E), _ptr(mod), _ptr(ts),
                                       _ptr(imp), int(normalize), C.byref(first)))
        return first.value

    def append_edges(self, src, dst):
        src = _host(src, np.int32)
        dst = _host(dst, np.int32)
        _check(lib().mars_store_append_edges(self.handle, src.shape[0], _ptr(src), _ptr(dst)))

    def delete(self, ids):
        """Tombstone rows: zero embedding, timestamp -1 (engine_server DELETE)."""
        a = _host(ids, np.int32)
        _check(lib().mars_store_delete(self.handle, int(a.shape[0]), a.ctypes.data))

    def set_importance(self, first, importance):
        imp = importance if hasattr(importance, "data_ptr") else _host(importance, np.float32)
        _settle(imp)
        _check(lib().mars_store_set_importance(self.handle, first, int(imp.shape[0]), _ptr(imp)))

    def read(self, first=0, n=None):
        """Rows [first, first+n) back on the host: (E, modalities, ts, importance)."""
        if n is None:
            n = self.num_nodes - first
        E = np.empty((n, self.dim), np.float32)
        mod = np.empty(n, np.int32)
        ts = np.empty(n, np.float32)
        imp = np.empty(n, np.float32)
        _check(lib().mars_store_read(self.handle, first, n, _ptr(E), _ptr(mod), _ptr(ts), _ptr(imp)))
        return E, mod, ts, imp

    def importance_fill(self, value=1.0):
        _check(lib().mars_importance_fill(self.handle, float(value)))

    def importance_update(self, d_ids, n, boost=0.1, decay_rate=0.001, max_importance=5.0,
                          stream=None):
        _check(lib().mars_importance_update(self.handle, _ptr(d_ids), n, boost, decay_rate,
                                            max_importance, _stream(stream, d_ids)))

    def info(self) -> StoreInfo:
        i = StoreInfo()
        _check(lib().mars_store_info_get(self.handle, C.byref(i)))
        return i

    @property
    def num_nodes(self) -> int:
        return self.info().num_nodes

    def close(self):
        if getattr(self, "handle", None):
            lib().mars_store_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QueryContext:
    """Query scratch (QueryContext) bound to a device."""

    def __init__(self, max_nodes: int, dim: int, max_k: int = 64, device: int = 0,
                 use_graph: bool = True, use_fused: bool = True):
        h = C.c_void_p()
        _check(lib().mars_query_ctx_create(device, max_nodes, dim, max_k, C.byref(h)))
        self.handle = h
        self.device = device
        self.dim = dim
        if not use_graph:
            _check(lib().mars_query_ctx_use_graph(self.handle, 0))
        if not use_fused:
            _check(lib().mars_query_ctx_use_fused(self.handle, 0))

    def set_fused(self, enable: bool) -> None:
        """Single-launch mars_query (True) or the multi-kernel pipeline (False)."""
        _check(lib().mars_query_ctx_use_fused(self.handle, int(bool(enable))))

    def path_counts(self) -> tuple[int, int]:
        """(queries answered by the single launch, of those re-run by the pipeline)."""
        f, r = C.c_uint64(), C.c_uint64()
        _check(lib().mars_query_ctx_path_counts(self.handle, C.byref(f), C.byref(r)))
        return f.value, r.value

    def f16_stats(self) -> dict:
        """scan_topk_f16's filter: re-runs on the fp32 scan (context life), largest
        candidate list and rescored-row count of one query in the last call."""
        r, mc, ms = C.c_uint64(), C.c_int32(), C.c_int32()
        _check(lib().mars_query_ctx_f16_stats(self.handle, C.byref(r), C.byref(mc), C.byref(ms)))
        return {"reruns": r.value, "max_candidates": mc.value, "max_survivors": ms.value}

    def f16_reruns(self) -> int:
        """Queries of scan_topk_f16 answered again by the fp32 scan (candidate overflow)."""
        return self.f16_stats()["reruns"]

    @property
    def stream(self) -> int:
        return lib().mars_query_ctx_stream(self.handle)

    def query(self, store: Store, q, t_q: float, cfg: RetrievalConfig | None = None,
              with_stats: bool = False):
        """query_memory_fast: host (numpy) or device (torch) query -> numpy results."""
        cfg = cfg or RetrievalConfig()
        qa = q if hasattr(q, "data_ptr") else _host(q, np.float32)
        out = np.zeros(max(cfg.top_k, 1), dtype=RESULT_DTYPE)
        n = C.c_int32()
        st = RetrievalStats()
        _check(lib().mars_query(store.handle, self.handle, _ptr(qa), float(t_q), C.byref(cfg),
                                out.ctypes.data, C.byref(n),
                                C.byref(st) if with_stats else None))
        res = out[:n.value]
        return (res, st.as_dict()) if with_stats else res

    def query_device(self, store: Store, d_query, t_q, cfg, d_out, d_count, stream=None):
        _check(lib().mars_query_device(store.handle, self.handle, _ptr(d_query), float(t_q),
                                       C.byref(cfg), _ptr(d_out), _ptr(d_count),
                                       _stream(stream, d_query, d_out, d_count)))

    def scan_topk(self, store: Store, d_query, t_q, lam, K, d_ids, d_vals, d_count=None,
                  modality_filter=-1, use_importance=False, row_offset=0, stream=None):
        _check(lib().mars_scan_topk(store.handle, self.handle, _ptr(d_query), float(t_q),
                                    float(lam), modality_filter, int(use_importance), K,
                                    row_offset, _ptr(d_ids), _ptr(d_vals), _ptr(d_count),
                                    _stream(stream, d_query, d_ids, d_vals, d_count)))

    def scan_topk_multi(self, store: Store, d_queries, nq, t_q, lam, K, d_ids, d_vals, d_counts=None,
                        modality_filter=-1, use_importance=False, row_offset=0, stream=None, query_pitch=None):
        """nq fused scans in one launch; d_queries: [nq][pitch] float32 on the device."""
        pitch = query_pitch if query_pitch is not None else (d_queries.stride(0) if hasattr(d_queries, "stride")
                                                             else store.dim)
        _check(lib().mars_scan_topk_multi(store.handle, self.handle, _ptr(d_queries), int(pitch), int(nq),
                                          float(t_q), float(lam), modality_filter, int(use_importance), K,
                                          row_offset, _ptr(d_ids), _ptr(d_vals), _ptr(d_counts),
                                          _stream(stream, d_queries, d_ids, d_vals, d_counts)))

    def scan_topk_f16(self, store: Store, d_queries, nq, t_q, lam, K, d_ids, d_vals, d_counts=None,
                      modality_filter=-1, use_importance=False, row_offset=0, stream=None, query_pitch=None):
        """scan_topk_multi's results from the store's fp16 copy (exact: fp16 only filters)."""
        pitch = query_pitch if query_pitch is not None else (d_queries.stride(0) if hasattr(d_queries, "stride")
                                                             else store.dim)
        _check(lib().mars_scan_topk_f16(store.handle, self.handle, _ptr(d_queries), int(pitch), int(nq),
                                        float(t_q), float(lam), modality_filter, int(use_importance), K,
                                        row_offset, _ptr(d_ids), _ptr(d_vals), _ptr(d_counts),
                                        _stream(stream, d_queries, d_ids, d_vals, d_counts)))

    def topk_merge(self, d_ids_in, d_vals_in, n_lists, K, d_ids_out, d_vals_out, d_count=None,
                   stream=None):
        _check(lib().mars_topk_merge(self.handle, _ptr(d_ids_in), _ptr(d_vals_in), n_lists, K,
                                     _ptr(d_ids_out), _ptr(d_vals_out), _ptr(d_count),
                                     _stream(stream, d_ids_in, d_vals_in, d_ids_out, d_vals_out, d_count)))

    def topk_merge_batch(self, d_ids_in, d_vals_in, n_lists, K, Q, d_ids_out, d_vals_out,
                         d_counts=None, stream=None):
        _check(lib().mars_topk_merge_batch(self.handle, _ptr(d_ids_in), _ptr(d_vals_in), n_lists,
                                           K, Q, _ptr(d_ids_out), _ptr(d_vals_out),
                                           _ptr(d_counts),
                                           _stream(stream, d_ids_in, d_vals_in, d_ids_out, d_vals_out, d_counts)))

    def novelty(self, store: Store, d_query, d_max, stream=None):
        _check(lib().mars_novelty(store.handle, self.handle, _ptr(d_query), _ptr(d_max),
        _stream(stream, d_query, d_max)))

    def debug_fused_scores(self, store: Store, d_query, t_q, lam, d_out, modality_filter=-1,
                           use_importance=False, stream=None):
        _check(lib().mars_debug_fused_scores(store.handle, self.handle, _ptr(d_query), float(t_q),
                                             float(lam), modality_filter, int(use_importance),
                                             _ptr(d_out), _stream(stream, d_query, d_out)))

    def close(self):
        if getattr(self, "handle", None):
            lib().mars_query_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchContext:
    """Scratch for batched top-K on the tensor cores (mars_query_batch_topk)."""

    def __init__(self, max_nodes: int, dim: int, max_batch: int, max_k: int = 128, device: int = 0):
        h = C.c_void_p()
        _check(lib().mars_batch_ctx_create(device, max_nodes, dim, max_batch, max_k, C.byref(h)))
        self.handle = h

    def set_precision(self, tf32_only: bool) -> None:
        """TF32 operands always (True) or fp16 when in range (False, the default)."""
        _check(lib().mars_batch_ctx_set_precision(self.handle, int(bool(tf32_only))))

    def set_single_launch(self, enable: bool) -> None:
        """Small batches: sample, thresholds and candidates as one cooperative launch (default) or three."""
        _check(lib().mars_batch_ctx_set_single_launch(self.handle, int(bool(enable))))

    def query_batch_topk(self, store: Store, d_queries, B, t_q, lam, K, d_ids, d_vals, d_counts=None,
                         modality_filter=-1, use_importance=False, row_offset=0, query_pitch=None,
                         stream=None):
        pitch = query_pitch if query_pitch is not None else (store.dim + 3) // 4 * 4
        _check(lib().mars_query_batch_topk(store.handle, self.handle, _ptr(d_queries), pitch, B,
                                           float(t_q), float(lam), modality_filter,
                                           int(use_importance), K, row_offset, _ptr(d_ids),
                                           _ptr(d_vals), _ptr(d_counts),
                                           _stream(stream, d_queries, d_ids, d_vals, d_counts)))

    def last_stats(self):
        st = BatchStats()
        _check(lib().mars_batch_last_stats(self.handle, C.byref(st)))
        return st.as_dict()

    def debug_wait(self, spin_limit: int, extra_arrivals: int) -> None:
        """Test hook: bound the grid-wide arrival wait to spin_limit polls and make
        the next call wait for extra_arrivals arrivals that never come."""
        _check(lib().mars_batch_ctx_debug_wait(self.handle, int(spin_limit), int(extra_arrivals)))

    def close(self):
        if getattr(self, "handle", None):
            lib().mars_batch_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


SHARD_ID_BYTES = 128


def shard_unique_id() -> bytes:
    """A fresh NCCL unique id (make it on rank 0 and give it to every rank)."""
    buf = C.create_string_buffer(SHARD_ID_BYTES)
    _check(lib().mars_shard_unique_id(buf))
    return buf.raw


class ShardComm:
    """Row-shard communicator (one per rank and GPU; NCCL owned by the library)."""

    def __init__(self, device: int, rank: int, world: int, unique_id: bytes, max_batch: int, max_k: int,
                 timeout_ms: int = None):
        """timeout_ms: deadline of NCCL's set-up work (creation, first use,
        teardown); None: the library's default, 0: none."""
        assert len(unique_id) == SHARD_ID_BYTES
        h = C.c_void_p()
        buf = C.create_string_buffer(unique_id, SHARD_ID_BYTES)
        if timeout_ms is None:
            _check(lib().mars_shard_comm_create(device, rank, world, buf, max_batch, max_k, C.byref(h)))
        else:
            _check(lib().mars_shard_comm_create_timeout(device, rank, world, buf, max_batch, max_k,
                                                        int(timeout_ms), C.byref(h)))
        self.handle = h
        self.rank, self.world = rank, world

    def query_batch_topk(self, store: Store, bc: "BatchContext", d_queries, B, t_q, lam, K, d_ids, d_vals,
                         d_counts=None, modality_filter=-1, use_importance=False, row_offset=0,
                         query_pitch=None, stream=None):
        """The global top-K of every query over all ranks' shards (collective)."""
        pitch = query_pitch if query_pitch is not None else (store.dim + 3) // 4 * 4
        _check(lib().mars_shard_query_batch_topk(store.handle, bc.handle, self.handle, _ptr(d_queries), pitch, B,
                                                 float(t_q), float(lam), modality_filter, int(use_importance),
                                                 K, row_offset, _ptr(d_ids), _ptr(d_vals), _ptr(d_counts),
                                                 _stream(stream, d_queries, d_ids, d_vals, d_counts)))

    def query(self, store: Store, ctx: "QueryContext", d_row_offsets, d_col_indices, n_global, q, t_q,
              cfg: RetrievalConfig, row_offset=0):
        """query_memory_fast over all ranks' shards with BFS over the replicated
        global CSR (collective); numpy results on every rank."""
        qa = q if hasattr(q, "data_ptr") else _host(q, np.float32)
        out = np.zeros(max(cfg.top_k, 1), dtype=RESULT_DTYPE)
        n = C.c_int32()
        _check(lib().mars_shard_query(store.handle, ctx.handle, self.handle, _ptr(d_row_offsets),
                                      _ptr(d_col_indices), int(n_global), _ptr(qa), float(t_q), C.byref(cfg),
                                      int(row_offset), out.ctypes.data, C.byref(n)))
        return out[:n.value]

    def set_timing(self, enable: bool) -> None:
        _check(lib().mars_shard_comm_set_timing(self.handle, int(bool(enable))))

    def set_exchange_at_world1(self, enable: bool) -> None:
        """Test hook: one rank runs the whole exchange protocol (records, NCCL
        all-gathers, merge) instead of the single-store pipeline."""
        _check(lib().mars_shard_comm_set_exchange_at_world1(self.handle, int(bool(enable))))

    def last_times(self) -> dict:
        a, b, m = C.c_float(), C.c_float(), C.c_float()
        _check(lib().mars_shard_last_times(self.handle, C.byref(a), C.byref(b), C.byref(m)))
        return {"local_ms": a.value, "gather_ms": b.value, "merge_ms": m.value}

    def status(self) -> None:
        _check(lib().mars_shard_comm_status(self.handle))

    def abort(self) -> None:
        _check(lib().mars_shard_comm_abort(self.handle))

    def close(self):
        if getattr(self, "handle", None):
            lib().mars_shard_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard_emulate_query_batch_topk(stores, contexts, row_offsets, d_queries, B, t_q, lam, K, d_ids, d_vals,
                                   d_counts, modality_filter=-1, use_importance=False, query_pitch=None):
    """Test hook: the sharded batched top-K over len(stores) row shards that
    all live on this GPU (each shard's pipeline on its own thread and its
    context's stream, the all-gathers done as device copies); blocks until
    the merged answer is written."""
    w = len(stores)
    assert len(contexts) == w and len(row_offsets) == w
    hs = (C.c_void_p * w)(*[s.handle.value for s in stores])
    hc = (C.c_void_p * w)(*[c.handle.value for c in contexts])
    offs = (C.c_int32 * w)(*[int(o) for o in row_offsets])
    pitch = query_pitch if query_pitch is not None else (stores[0].dim + 3) // 4 * 4
    _check(lib().mars_shard_emulate_query_batch_topk(w, hs, hc, offs, _ptr(d_queries), pitch, B, float(t_q),
                                                     float(lam), modality_filter, int(use_importance), K,
                                                     _ptr(d_ids), _ptr(d_vals), _ptr(d_counts)))


def cmng_build(store: Store, degree, degree_cross, num_modalities, d_neighbors) -> float:
    """build_cmng over the store's rows into d_neighbors (N x degree, device)."""
    ms = C.c_float()
    _check(lib().mars_cmng_build(store.handle, degree, degree_cross, num_modalities,
                                 _ptr(d_neighbors), C.byref(ms)))
    return ms.value


def cmng_build_rows(store: Store, first, count, degree, degree_cross, num_modalities,
                    d_neighbors) -> float:
    """Neighbour lists of rows first .. first+count-1 into d_neighbors (count x degree)."""
    ms = C.c_float()
    _check(lib().mars_cmng_build_rows(store.handle, first, count, degree, degree_cross, num_modalities,
                                      _ptr(d_neighbors), C.byref(ms)))
    return ms.value


def cmng_knn(store: Store, k, d_ids, d_vals, d_counts=None):
    _check(lib().mars_cmng_knn(store.handle, k, _ptr(d_ids), _ptr(d_vals), _ptr(d_counts)))


def cmng_search_batch(store: Store, d_neighbors, degree, d_queries, nq, t_q, cfg: CmngConfig,
                      d_ids, d_scores, d_counts, d_mods=None, d_iters=None, d_scored=None,
                      query_pitch=None, stream=None):
    pitch = query_pitch if query_pitch is not None else (store.dim + 3) // 4 * 4
    _check(lib().mars_cmng_search_batch(store.handle, _ptr(d_neighbors), degree, _ptr(d_queries),
                                        pitch, nq, float(t_q), C.byref(cfg), _ptr(d_ids),
                                        _ptr(d_scores), _ptr(d_mods), _ptr(d_counts),
                                        _ptr(d_iters), _ptr(d_scored),
                                        _stream(stream, d_neighbors, d_queries, d_ids, d_scores, d_mods, d_counts, d_iters, d_scored)))


class CmngContext:
    """Scratch for cmng_search + BFS batches (mars_cmng_search_bfs_batch)."""

    def __init__(self, max_queries, K, degree, bfs_hops, max_nodes, device=0):
        h = C.c_void_p()
        _check(lib().mars_cmng_ctx_create(device, max_queries, K, degree, bfs_hops, max_nodes,
                                          C.byref(h)))
        self.handle = h

    def set_bfs_smem_nodes(self, max_nodes: int) -> None:
        """Visited nodes per query the shared-memory BFS holds (<= 2048; 0: global tables only)."""
        _check(lib().mars_cmng_ctx_set_bfs_smem_nodes(self.handle, int(max_nodes)))

    def search_bfs(self, store: Store, d_neighbors, degree, d_queries, nq, t_q, cfg: CmngConfig,
                   bfs_hops, bfs_score_decay, d_ids, d_scores, d_counts, d_mods=None, d_hops=None,
                   d_visited=None, use_importance=False, query_pitch=None, stream=None):
        pitch = query_pitch if query_pitch is not None else (store.dim + 3) // 4 * 4
        _check(lib().mars_cmng_search_bfs_batch(store.handle, self.handle, _ptr(d_neighbors), degree,
                                                _ptr(d_queries), pitch, nq, float(t_q), C.byref(cfg),
                                                bfs_hops, float(bfs_score_decay),
                                                int(use_importance), _ptr(d_ids), _ptr(d_scores),
                                                _ptr(d_mods), _ptr(d_hops), _ptr(d_counts),
                                                _ptr(d_visited),
                                                _stream(stream, d_neighbors, d_queries, d_ids, d_scores, d_mods, d_hops, d_counts, d_visited)))

    def close(self):
        if getattr(self, "handle", None):
            lib().mars_cmng_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def scan_topk_noalloc(d_embeddings, row_pitch, d_timestamps, d_importance, d_modalities, n, dim,
                      d_query, t_q, lam, K, d_ids, d_vals, d_count=None, modality_filter=-1,
                      use_importance=False, row_offset=0, stream=None):
    """mars_scan_topk_noalloc: the fused scan over caller-owned device arrays
    for callers that may not allocate GPU memory (no store, no context)."""
    _check(lib().mars_scan_topk_noalloc(_ptr(d_embeddings), row_pitch, _ptr(d_timestamps),
                                        _ptr(d_importance), _ptr(d_modalities), n, dim,
                                        _ptr(d_query), float(t_q), float(lam), modality_filter,
                                        int(use_importance), K, row_offset, _ptr(d_ids),
                                        _ptr(d_vals), _ptr(d_count),
                                        _stream(stream, d_embeddings, d_timestamps, d_importance, d_modalities, d_query, d_ids, d_vals, d_count)))


def query_once(store: Store, q, t_q, cfg: RetrievalConfig | None = None):
    """query_memory (no persistent context)."""
    cfg = cfg or RetrievalConfig()
    qa = _host(q, np.float32)
    out = np.zeros(max(cfg.top_k, 1), dtype=RESULT_DTYPE)
    n = C.c_int32()
    _check(lib().mars_query_once(store.handle, _ptr(qa), float(t_q), C.byref(cfg),
                                 out.ctypes.data, C.byref(n), None))
    return out[:n.value]
