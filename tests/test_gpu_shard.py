"""Row-sharded batched top-K (mars_shard_query_batch_topk) with the NCCL
communicator owned by the library.

* One rank on one GPU (world 1, real NCCL): the call equals
  mars_query_batch_topk on the same store bit for bit, for the small-batch
  tiles (B <= 64), the 128 x 256 tiles and K = 256, with a row offset --
  both as one rank answers by default (the single-store pipeline) and with
  the whole exchange protocol forced (records, NCCL all-gathers, merge).
* A bounded device wait that gives up on a rank (the batch context's test
  hook) marks that call's merged results invalid (counts -1) and the call
  after it is exact again.
* mars_shard_query (top-K seeds merged over NCCL, then BFS over a replicated
  global graph with each level's own scores exchanged) on one rank equals
  mars_query bit for bit, hops 0-3, with and without a modality filter.
* Two ranks on two GPUs (tests/shard_worker.py under torchrun, when two GPUs
  are visible): every rank's merged answer is the same, equals the single-GPU
  answer over the whole corpus bit for bit (batched top-K and the sharded BFS
  query), and matches the CPU oracle.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def env():
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    N, D = 150_000, 768
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=31, ts_max=600.0)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp)
    comm = mb.ShardComm(0, 0, 1, mb.shard_unique_id(), max_batch=256, max_k=256)
    Qd = torch.from_numpy(datagen.queries(256, D, seed=32)).cuda()
    yield st, comm, Qd, N, D
    comm.close()


def _answers(fn, B, K):
    import torch
    ids = torch.full((B, K), -7, dtype=torch.int32, device="cuda")
    vals = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    cnt = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    fn(ids, vals, cnt)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), vals.cpu().numpy(), cnt.cpu().numpy()


@pytest.mark.parametrize("full", [False, True])
@pytest.mark.parametrize("B,K", [(16, 10), (200, 100), (64, 256)])
def test_world1_equals_unsharded_call(env, B, K, full):
    import mars_b200 as mb
    st, comm, Qd, N, D = env
    comm.set_exchange_at_world1(full)
    bc = mb.BatchContext(N, D, max_batch=256, max_k=256)
    off = 1_000_000
    ref = _answers(lambda i, v, c: bc.query_batch_topk(st, Qd[:B], B, 600.0, 0.01, K, i, v, c, use_importance=True,
                                                       row_offset=off), B, K)
    got = _answers(lambda i, v, c: comm.query_batch_topk(st, bc, Qd[:B], B, 600.0, 0.01, K, i, v, c,
                                                         use_importance=True, row_offset=off), B, K)
    assert np.array_equal(got[2], ref[2])
    assert np.array_equal(got[0], ref[0])
    assert np.array_equal(got[1].view(np.int32), ref[1].view(np.int32))
    comm.set_timing(True)
    _answers(lambda i, v, c: comm.query_batch_topk(st, bc, Qd[:B], B, 600.0, 0.01, K, i, v, c,
                                                   use_importance=True, row_offset=off), B, K)
    t = comm.last_times()
    comm.set_timing(False)
    assert t["local_ms"] > 0 and t["gather_ms"] >= 0 and t["merge_ms"] >= 0
    if full:
        assert t["merge_ms"] > 0
    comm.status()
    comm.set_exchange_at_world1(False)


@pytest.mark.parametrize("full", [False, True])
def test_failed_rank_invalidates_merged_results(env, full):
    import mars_b200 as mb
    st, comm, Qd, N, D = env
    comm.set_exchange_at_world1(full)
    B, K = 16, 10
    bc = mb.BatchContext(N, D, max_batch=256, max_k=256)
    ref = _answers(lambda i, v, c: bc.query_batch_topk(st, Qd[:B], B, 600.0, 0.01, K, i, v, c,
                                                       use_importance=True), B, K)
    bc.debug_wait(4096, 1)          # this call's grid-wide wait cannot end
    ids, vals, cnt = _answers(lambda i, v, c: comm.query_batch_topk(st, bc, Qd[:B], B, 600.0, 0.01, K, i, v, c,
                                                                    use_importance=True), B, K)
    assert np.all(cnt == -1) and np.all(ids == -1) and np.all(np.isneginf(vals))
    # the failing rank reports the timeout on its next call (which joins the
    # collectives with neutral data, so its results are invalid too) ...
    with pytest.raises(mb.MarsError) as e:
        _answers(lambda i, v, c: comm.query_batch_topk(st, bc, Qd[:B], B, 600.0, 0.01, K, i, v, c,
                                                       use_importance=True), B, K)
    assert e.value.status == mb.MARS_ERR_TIMEOUT
    # ... and the one after is exact again
    got = _answers(lambda i, v, c: comm.query_batch_topk(st, bc, Qd[:B], B, 600.0, 0.01, K, i, v, c,
                                                         use_importance=True), B, K)
    assert np.array_equal(got[0], ref[0]) and np.array_equal(got[2], ref[2])
    comm.set_exchange_at_world1(False)


def test_two_ranks_on_two_gpus(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = str(tmp_path / "shard.json")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29517",
           os.path.join(ROOT, "tests", "shard_worker.py"), out]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rep = json.load(open(out))
    assert rep["world"] == 2
    assert rep["ranks_agree"] and rep["equal_to_single_gpu"] and rep["oracle_ok"], rep
    assert rep["bfs_equal_to_single_gpu"], rep


@pytest.mark.parametrize("hops,K,filt", [(0, 10, -1), (1, 10, -1), (2, 10, 2), (3, 16, -1), (2, 64, -1)])
def test_world1_sharded_bfs_query_equals_mars_query(hops, K, filt):
    """mars_shard_query (seeds merged over NCCL, own scores of each BFS
    level exchanged by all-reduce) on one rank equals mars_query over the
    same rows and graph, bit for bit."""
    import torch

    import mars_b200 as mb
    from mars_b200 import datagen
    N, D = 60_000, 768
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=41, n_mod=4, ts_max=10.0)
    ro, ci = datagen.random_bridges(mod, 4, seed=7)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp, ro, ci)
    ctx = mb.QueryContext(N, D, max_k=64)
    comm = mb.ShardComm(0, 0, 1, mb.shard_unique_id(), max_batch=4, max_k=64)
    d_ro, d_ci = torch.from_numpy(ro).cuda(), torch.from_numpy(ci).cuda()
    cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=hops, time_decay_lambda=0.5, bfs_score_decay=0.5,
                             modality_filter=filt, use_importance=True)
    Q = datagen.queries(6, D, seed=42)
    for q in range(Q.shape[0]):
        ref = ctx.query(st, Q[q], 10.0, cfg)
        got = comm.query(st, ctx, d_ro, d_ci, N, Q[q], 10.0, cfg, row_offset=0)
        assert len(got) == len(ref)
        assert np.array_equal(got["node_id"], ref["node_id"]), (q, got, ref)
        assert np.array_equal(got["score"].view(np.int32), ref["score"].view(np.int32))
        assert np.array_equal(got["hops"], ref["hops"])
        assert np.array_equal(got["modality"], ref["modality"])
    comm.close()


def test_rank_that_never_joins_ends_creation_with_timeout():
    """A communicator of two ranks of which only rank 0 ever calls create:
    the non-blocking creation is polled against its deadline (3 s) and ends
    with MARS_ERR_TIMEOUT (the half-made communicator aborted) instead of
    waiting for ever; the same process then makes a working communicator.
    It runs in a child process with a hard time limit of its own; nothing of
    it runs on the GPU beyond NCCL's start-up."""
    import mars_b200 as mb
    code = "\n".join([
        "import sys, time",
        f"sys.path.insert(0, {os.path.join(ROOT, 'cuda-multimodal-memory_b200')!r})",
        "import mars_b200 as mb",
        "uid = mb.shard_unique_id()",
        "t0 = time.time()",
        "try:",
        "    mb.ShardComm(0, 0, 2, uid, max_batch=4, max_k=8, timeout_ms=3000)",
        "    print('created')",
        "except mb.MarsError as e:",
        "    print('status', e.status, 'elapsed', round(time.time() - t0, 1))",
        "c = mb.ShardComm(0, 0, 1, mb.shard_unique_id(), max_batch=4, max_k=8, timeout_ms=60000)",
        "c.status()",
        "c.close()",
        "print('ok')",
    ])
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", code], capture_output=True, text=True,
                       env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    words = r.stdout.split()
    assert "status" in words, r.stdout
    assert int(words[words.index("status") + 1]) == mb.MARS_ERR_TIMEOUT, r.stdout
    assert float(words[words.index("elapsed") + 1]) < 60.0, r.stdout
    assert words[-1] == "ok", r.stdout
