"""Entry points around the query that the other GPU tests do not reach:
mars_query_device (device query in, device results out, asynchronous on a
stream), mars_store_set_importance and mars_store_info_get."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def mb():
    import mars_b200
    return mars_b200


def corpus(N, D, seed):
    from mars_b200 import datagen
    E, mod, ts, imp = datagen.gaussian_corpus(N, D, seed=seed, n_mod=4, ts_max=10.0)
    ro, ci = datagen.random_bridges(mod, 4, seed=seed + 1)
    return E, mod, ts, imp, ro, ci


@pytest.mark.parametrize("hops", [0, 1, 2])
def test_query_device_equals_host_query(torch_mod, mb, hops):
    """The device-resident form of mars_query gives the host form's results
    byte for byte, on a stream of the caller's, back to back."""
    torch = torch_mod
    N, D = 8000, 768
    E, mod, ts, imp, ro, ci = corpus(N, D, seed=50 + hops)
    st = mb.Store(N, D)
    st.upload(E, mod, ts, imp, ro, ci)
    ctx = mb.QueryContext(N, D, max_k=32)
    s = torch.cuda.Stream()
    rng = np.random.default_rng(hops)
    for K in (5, 10, 32):
        cfg = mb.RetrievalConfig(top_k=K, bfs_max_hops=hops, time_decay_lambda=0.3, bfs_score_decay=0.5,
                                 use_importance=True)
        q = rng.standard_normal(D).astype(np.float32)
        host = ctx.query(st, q, 10.0, cfg)
        d_out = torch.zeros((K, 4), dtype=torch.int32, device="cuda")   # mars_query_result rows
        d_cnt = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        with torch.cuda.stream(s):
            dq = torch.from_numpy(q).cuda()
            ctx.query_device(st, dq, 10.0, cfg, d_out, d_cnt, stream=s.cuda_stream)
        s.synchronize()
        n = int(d_cnt.item())
        dev = np.frombuffer(d_out.cpu().numpy().tobytes(), dtype=mb.RESULT_DTYPE)[:n]
        assert n == len(host), (K, n, len(host))
        assert dev.tobytes() == host.tobytes(), K


def test_set_importance_and_info(torch_mod, mb):
    torch = torch_mod
    N, D = 3000, 100
    E, mod, ts, imp, ro, ci = corpus(N, D, seed=7)
    st = mb.Store(N + 500, D, edge_slack=4)
    st.upload(E, mod, ts, imp, ro, ci)
    info = st.info()
    assert info.num_nodes == N and info.capacity == N + 500 and info.embedding_dim == D
    assert info.row_pitch == 100 and info.num_edges == ci.shape[0] and info.csr_nodes == N
    assert info.edge_slack == 4 and info.d_embeddings and info.d_importance and info.d_num_nodes
    # host values, then device values, into a slice of rows
    new = np.linspace(0.1, 2.0, 200).astype(np.float32)
    st.set_importance(1000, new)
    assert np.array_equal(st.read(1000, 200)[3], new)
    dnew = torch.from_numpy(new[::-1].copy()).cuda()
    st.set_importance(2000, dnew)
    assert np.array_equal(st.read(2000, 200)[3], new[::-1])
    assert np.array_equal(st.read(0, 1000)[3], imp[:1000].astype(np.float32))
    # the scan's importance term sees them: a row given a large importance wins
    st.set_importance(2500, np.array([1000.0], np.float32))
    ctx = mb.QueryContext(N + 500, D, max_k=8)
    res = ctx.query(st, E[2500], 10.0,
                    mb.RetrievalConfig(top_k=1, bfs_max_hops=0, time_decay_lambda=0.0, use_importance=True))
    assert int(res["node_id"][0]) == 2500
    assert float(res["score"][0]) == pytest.approx(1000.0, rel=1e-4)
