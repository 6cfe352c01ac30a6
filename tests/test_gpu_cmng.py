"""CMNG on the GPU: the kNN lists and the built graph against the oracle's
exact kNN + neighbour selection (bit-exact, ties by id), the beam search
against the oracle's step-by-step restatement of the reference kernel (same
warp dot order: identical beams), and both against the reference's own GPU
code when oracle/_ref is built."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
from _util import assert_ranked_equivalent

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libmars_ref_gpu.so")


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def clustered():
    from mars_b200 import datagen
    N, D = 6000, 768
    E, mod, ts, lab = datagen.cluster_corpus(N, D, 60, 0.3, seed=11, n_mod=4, ts_max=10.0)
    return E, mod, ts


def _store(mb, E, mod, ts):
    st = mb.Store(E.shape[0], E.shape[1])
    st.upload(E, mod, ts)
    return st


@pytest.mark.parametrize("k", [32, 64, 128])
def test_knn_lists_bit_exact(torch_mod, clustered, k):
    import mars_b200 as mb
    torch = torch_mod
    E, mod, ts = clustered
    N = E.shape[0]
    st = _store(mb, E, mod, ts)
    ids = torch.empty((N, k), dtype=torch.int32, device="cuda")
    vals = torch.empty((N, k), dtype=torch.float32, device="cuda")
    mb.cmng_knn(st, k, ids, vals)
    torch.cuda.synchronize()
    rows = np.arange(0, N, 37, dtype=np.int32)
    rid, rv = O.knn(O.Corpus(E=E, ts=ts, mod=mod), rows, k)
    got_i = ids.cpu().numpy()[rows]
    got_v = vals.cpu().numpy()[rows]
    assert np.array_equal(got_i, rid)
    assert np.array_equal(got_v.view(np.uint32), rv.view(np.uint32))


@pytest.mark.parametrize("degree,degree_cross,nmod", [(32, 0, 4), (36, 4, 4), (64, 4, 3)])
def test_cmng_build_matches_oracle(torch_mod, clustered, degree, degree_cross, nmod):
    import mars_b200 as mb
    torch = torch_mod
    E, mod, ts = clustered
    N = E.shape[0]
    st = _store(mb, E, mod, ts)
    nb = torch.empty((N, degree), dtype=torch.int32, device="cuda")
    ms = mb.cmng_build(st, degree, degree_cross, nmod, nb)
    torch.cuda.synchronize()
    assert ms > 0
    rows = np.arange(0, N, 53, dtype=np.int32)
    k_init = 2 * degree
    rid, _ = O.knn(O.Corpus(E=E, ts=ts, mod=mod), rows, k_init)
    ref = O.cmng_select(rid, mod, rows, degree, degree_cross, nmod)
    assert np.array_equal(nb.cpu().numpy()[rows], ref)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_row_block_builds_equal_the_whole_build(torch_mod, clustered, world):
    """The sharded build: row blocks [r*N/G, (r+1)*N/G) built separately
    (as G GPUs each holding the whole store would) and concatenated equal the
    single build bit for bit."""
    import mars_b200 as mb
    torch = torch_mod
    E, mod, ts = clustered
    N, degree = E.shape[0], 36
    st = _store(mb, E, mod, ts)
    whole = torch.empty((N, degree), dtype=torch.int32, device="cuda")
    mb.cmng_build(st, degree, 4, 4, whole)
    parts = []
    for r in range(world):
        lo, hi = N * r // world, N * (r + 1) // world
        part = torch.empty((hi - lo, degree), dtype=torch.int32, device="cuda")
        mb.cmng_build_rows(st, lo, hi - lo, degree, 4, 4, part)
        parts.append(part)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts), whole)
    with pytest.raises(mb.MarsError):
        mb.cmng_build_rows(st, N - 10, 11, degree, 4, 4, whole)


def _graph(mb, torch, E, mod, ts, degree=32):
    st = _store(mb, E, mod, ts)
    nb = torch.empty((E.shape[0], degree), dtype=torch.int32, device="cuda")
    mb.cmng_build(st, degree, 0, 4, nb)
    torch.cuda.synchronize()
    return st, nb


@pytest.mark.parametrize("beam,iters,K", [(64, 64, 10), (128, 32, 20), (16, 100, 16), (8, 5, 10)])
def test_cmng_search_matches_oracle(torch_mod, clustered, beam, iters, K):
    import mars_b200 as mb
    from mars_b200 import datagen
    torch = torch_mod
    E, mod, ts = clustered
    st, nb = _graph(mb, torch, E, mod, ts)
    nbh = nb.cpu().numpy()
    nq = 24
    Q = datagen.queries(nq, E.shape[1], seed=beam + iters)
    Q[: nq // 2] = E[np.arange(nq // 2) * 97] + 0.05 * Q[: nq // 2]   # some queries near clusters
    Qd = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    cnt = torch.empty(nq, dtype=torch.int32, device="cuda")
    its = torch.empty(nq, dtype=torch.int32, device="cuda")
    scored = torch.empty(nq, dtype=torch.int32, device="cuda")
    cfg = mb.CmngConfig(K=K, beam_width=beam, max_iterations=iters, time_decay_lambda=0.05)
    mb.cmng_search_batch(st, nb, 32, Qd, nq, 10.0, cfg, ids, sc, cnt, d_iters=its, d_scored=scored)
    torch.cuda.synchronize()
    c = O.Corpus(E=E, ts=ts, mod=mod)
    for q in range(nq):
        res, stats = O.cmng_search(c, nbh, Q[q], 10.0, K=K, beam_width=beam, max_iterations=iters,
                                   lam=0.05, dot_order=O.DOT_REF_WARP)
        n = int(cnt[q].item())
        assert n == len(res)
        assert int(its[q].item()) == stats["iterations"]
        assert int(scored[q].item()) == stats["rows_scored"]
        assert_ranked_equivalent(ids[q, :n].cpu().numpy(), sc[q, :n].cpu().numpy(),
                                 res["node_id"], res["score"], rtol=2e-6, what=f"q{q}")


def test_cmng_search_matches_reference_kernel(torch_mod, clustered):
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref not built")
    import mars_b200 as mb
    from mars_b200 import datagen
    torch = torch_mod
    E, mod, ts = clustered
    st, nb = _graph(mb, torch, E, mod, ts)
    nbh = np.ascontiguousarray(nb.cpu().numpy())
    nq, K, beam, iters = 16, 10, 64, 64
    Q = datagen.queries(nq, E.shape[1], seed=4)
    L = C.CDLL(REF_LIB)
    P = C.c_void_p
    L.ref_cmng_search.argtypes = [P, P, P, C.c_int32, C.c_int32, P, C.c_int32, P, C.c_int32,
                                  C.c_float, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                                  P, P, P, P]
    rid = np.full((nq, K), -1, np.int32)
    rsc = np.zeros((nq, K), np.float32)
    rcnt = np.zeros(nq, np.int32)
    L.ref_cmng_search(E.ctypes.data, mod.ctypes.data, ts.ctypes.data, E.shape[0], E.shape[1],
                      nbh.ctypes.data, 32, Q.ctypes.data, nq, 10.0, K, beam, iters, 1, 0.05,
                      rid.ctypes.data, rsc.ctypes.data, rcnt.ctypes.data, None)
    Qd = torch.from_numpy(Q).cuda()
    ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    cnt = torch.empty(nq, dtype=torch.int32, device="cuda")
    mb.cmng_search_batch(st, nb, 32, Qd, nq, 10.0,
                         mb.CmngConfig(K=K, beam_width=beam, max_iterations=iters, time_decay_lambda=0.05),
                         ids, sc, cnt)
    torch.cuda.synchronize()
    for q in range(nq):
        n = int(cnt[q].item())
        assert n == rcnt[q]
        assert np.array_equal(ids[q, :n].cpu().numpy(), rid[q, :n])
        assert np.array_equal(sc[q, :n].cpu().numpy().view(np.uint32), rsc[q, :n].view(np.uint32))


@pytest.mark.parametrize("hops", [0, 1, 2])
def test_cmng_search_bfs_matches_oracle(torch_mod, clustered, hops):
    """Beam search then the canonical BFS over the CMNG adjacency: with the
    device's beam as seeds, the oracle's BFS gives the same answer (the own
    scores differ only by __expf vs expf, so ranks are compared tie-aware)."""
    import mars_b200 as mb
    from mars_b200 import datagen
    torch = torch_mod
    E, mod, ts = clustered
    N, D = E.shape
    deg = 36
    st = _store(mb, E, mod, ts)
    nb = torch.empty((N, deg), dtype=torch.int32, device="cuda")
    mb.cmng_build(st, deg, 4, 4, nb)
    nbh = nb.cpu().numpy()
    nq, K = 20, 10
    Q = datagen.queries(nq, D, seed=50 + hops)
    Q[:8] = E[np.arange(8) * 311] + 0.05 * Q[:8]
    Qd = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    cfg = mb.CmngConfig(K=K, beam_width=64, max_iterations=64, time_decay_lambda=0.05)
    ctx = mb.CmngContext(nq, K, deg, hops, N)
    ids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    hp = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    cnt = torch.empty(nq, dtype=torch.int32, device="cuda")
    vis = torch.empty(nq, dtype=torch.int32, device="cuda")
    ctx.search_bfs(st, nb, deg, Qd, nq, 10.0, cfg, hops, 0.5, ids, sc, cnt, d_hops=hp, d_visited=vis)
    # beam results alone, as the BFS seeds
    bids = torch.empty((nq, K), dtype=torch.int32, device="cuda")
    bsc = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    bcnt = torch.empty(nq, dtype=torch.int32, device="cuda")
    mb.cmng_search_batch(st, nb, deg, Qd, nq, 10.0, cfg, bids, bsc, bcnt)
    torch.cuda.synchronize()
    oc = O.Corpus(E=E, ts=ts, mod=mod, fixed_nbrs=nbh)
    for q in range(nq):
        n0 = int(bcnt[q].item())
        visited = O.bfs(oc, bids[q, :n0].cpu().numpy(), bsc[q, :n0].cpu().numpy(), None, hops, 0.5,
                        q=Q[q], t_q=10.0, lam=0.05)
        assert int(vis[q].item()) == visited.shape[0]
        ref = O.finalize(visited, K)
        n = int(cnt[q].item())
        assert n == ref.shape[0]
        assert_ranked_equivalent(ids[q, :n].cpu().numpy(), sc[q, :n].cpu().numpy(), ref["node_id"],
                                 ref["score"], hp[q, :n].cpu().numpy(), ref["hops"], rtol=2e-6,
                                 what=f"q{q}")


@pytest.mark.parametrize("hops,K", [(1, 10), (2, 10), (2, 64), (3, 16)])
def test_bfs_shared_tables_equal_global_tables(torch_mod, clustered, hops, K):
    """The BFS with its visited set in shared memory (the default), the
    global-table kernel alone, and a shared-table limit so small that every
    query is handed to the global kernel, give the same answers bit for bit
    (ids, scores, hops, counts, visited)."""
    import mars_b200 as mb
    from mars_b200 import datagen
    torch = torch_mod
    E, mod, ts = clustered
    N, D = E.shape
    deg = 36
    st = _store(mb, E, mod, ts)
    nb = torch.empty((N, deg), dtype=torch.int32, device="cuda")
    mb.cmng_build(st, deg, 4, 4, nb)
    nq = 300
    Q = datagen.queries(nq, D, seed=70 + hops)
    Q[:100] = E[np.arange(100) * 53] + 0.05 * Q[:100]
    Qd = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    cfg = mb.CmngConfig(K=K, beam_width=64, max_iterations=64, time_decay_lambda=0.05)
    ctx = mb.CmngContext(nq, K, deg, hops, N)

    def run(limit):
        ctx.set_bfs_smem_nodes(limit)
        out = [torch.full((nq, K), -9, dtype=torch.int32, device="cuda"),
               torch.zeros((nq, K), dtype=torch.float32, device="cuda"),
               torch.full((nq, K), -9, dtype=torch.int32, device="cuda"),
               torch.full((nq,), -9, dtype=torch.int32, device="cuda"),
               torch.full((nq,), -9, dtype=torch.int32, device="cuda")]
        ctx.search_bfs(st, nb, deg, Qd, nq, 10.0, cfg, hops, 0.5, out[0], out[1], out[3], d_hops=out[2],
                       d_visited=out[4], use_importance=True)
        torch.cuda.synchronize()
        return [o.cpu().numpy() for o in out]

    shared = run(2048)
    glob = run(0)
    redo = run(16)            # more than 16 visited nodes: every query goes to the global kernel
    again = run(2048)
    for other in (glob, redo, again):
        assert np.array_equal(shared[3], other[3])
        assert np.array_equal(shared[4], other[4])
        assert np.array_equal(shared[0], other[0])
        assert np.array_equal(shared[1].view(np.int32), other[1].view(np.int32))
        assert np.array_equal(shared[2], other[2])
    assert shared[4].max() > 16
