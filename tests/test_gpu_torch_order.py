"""Torch CUDA tensors passed to the Python API are ordered like torch ops:
store writes wait for the torch work that made their inputs, and device
calls without an explicit stream run on torch's current stream, after the
work that made their inputs and before the work that reads their outputs."""
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


def test_upload_and_scans_follow_torch_work(torch_mod, mb):
    torch = torch_mod
    N, D = 400000, 768
    st = mb.Store(N + 64, D)
    g = torch.Generator(device="cuda").manual_seed(0)
    E = torch.randn(N, D, device="cuda", generator=g)
    E = E / E.norm(dim=1, keepdim=True)          # queued on torch's stream when upload is called
    mod = torch.zeros(N, dtype=torch.int32, device="cuda")
    ts = torch.zeros(N, device="cuda")
    st.upload(E, mod, ts, None)
    rows = st.read(N - 1000, 1000)[0]
    assert np.array_equal(rows, E[N - 1000:].cpu().numpy())
    extra = torch.randn(64, D, device="cuda", generator=g) * 3.0
    first = st.append(extra, torch.ones(64, dtype=torch.int32, device="cuda"), torch.zeros(64, device="cuda"),
                      normalize=False)
    assert first == N
    assert np.array_equal(st.read(N, 64)[0], extra.cpu().numpy())

    ctx = mb.QueryContext(N + 64, D, max_k=16)
    idx = torch.arange(0, 16 * 997, 997, device="cuda")
    for scan in (ctx.scan_topk_multi, ctx.scan_topk_f16):
        Q = (E[idx] * 2.0).contiguous()               # made on torch's stream
        ids = torch.full((16, 10), -1, dtype=torch.int32, device="cuda")
        vals = torch.empty((16, 10), device="cuda")
        scan(st, Q, 16, 0.0, 0.0, 10, ids, vals, modality_filter=0)
        best = ids[:, 0].cpu()                        # read on torch's stream, no explicit synchronize
        assert torch.equal(best, idx.to(torch.int32).cpu())
