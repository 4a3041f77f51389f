"""The per-hop operator (fg_hop_fwd / fg_hop_bwd, flyguy_b200.fly_cuda.HopCuda) against the reference's HopCuda math
(flyguy/fly_cuda.py:25-54, 78-115) restated in float64 numpy: forward, weight and state gradients, fp32 and the 16-bit
mode, on a CSR with duplicate connections and empty rows and a batch that is not a multiple of 128."""
import numpy as np
import pytest

from conftest import rel
from flyguy_b200 import native

TOL = 1e-5


def _graph(n_src=300, n_rows=200, E=3000, seed=5):
    rng = np.random.default_rng(seed)
    rows = np.sort(rng.integers(0, n_rows - 20, E))            # the last 20 rows have no connections
    col = rng.integers(0, n_src, E)
    col[:50] = col[0]                                          # duplicates (mathematically a sum)
    o = np.lexsort((col, rows))
    rows, col = rows[o], col[o]
    crow = np.concatenate([[0], np.cumsum(np.bincount(rows, minlength=n_rows))]).astype(np.int64)
    t = np.lexsort((rows, col))                                # by source, as fly.py:110-115
    tcrow = np.concatenate([[0], np.cumsum(np.bincount(col, minlength=n_src))]).astype(np.int64)
    w = rng.normal(0, 0.3, E).astype(np.float32)
    return dict(rows=rows, col=col.astype(np.int32), crow=crow, tcol=rows[t].astype(np.int32), tcrow=tcrow,
                tperm=t.astype(np.int64), w=w, n_src=n_src, n_rows=n_rows)


def _dense(g):
    A = np.zeros((g["n_rows"], g["n_src"]))
    np.add.at(A, (g["rows"], g["col"]), g["w"].astype(np.float64))
    return A


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float64)


@pytest.mark.gpu
@pytest.mark.parametrize("half", [False, True])
def test_hop_operator_matches_reference_math(half, cuda):
    import torch
    from flyguy_b200.fly_cuda import HopCuda
    g = _graph()
    B = 96
    rng = np.random.default_rng(9)
    h = np.maximum(rng.normal(0, 1, (g["n_src"], B)), 0).astype(np.float32)
    gz = rng.normal(0, 1e-3, (g["n_rows"], B)).astype(np.float32)
    T = {k: torch.as_tensor(g[k]).cuda() for k in ("crow", "col", "tcrow", "tcol", "tperm")}
    w = torch.as_tensor(g["w"]).cuda().requires_grad_(True)
    ht = torch.as_tensor(h).cuda().requires_grad_(True)
    out = HopCuda.apply(w, ht, T["crow"], T["col"], T["tcrow"], T["tcol"], T["tperm"], half)
    out.backward(torch.as_tensor(gz).cuda())
    A = _dense(g)
    hs = _f16(h) if half else h.astype(np.float64)
    assert rel(out.detach().cpu().numpy(), A @ hs) < TOL
    scale = max(float(np.abs(gz).max()), 1e-30)
    gzs = _f16(gz / scale) * scale if half else gz.astype(np.float64)
    want_gw = np.einsum("eb,eb->e", gzs[g["rows"]], hs[g["col"]])
    assert rel(w.grad.cpu().numpy(), want_gw) < TOL
    assert rel(ht.grad.cpu().numpy(), A.T @ gzs) < TOL


@pytest.mark.gpu
def test_hop_operator_autograd_matches_torch_sparse_hop(cuda):
    """Through a loss: the gradients of HopCuda equal torch autograd of the reference's _Hop formulation
    (flyguy/fly.py:51-72) computed densely in float64."""
    import torch
    from flyguy_b200.fly_cuda import HopCuda
    g = _graph(seed=7)
    B = 128
    h = np.random.default_rng(3).normal(0, 1, (g["n_src"], B)).astype(np.float32)
    T = {k: torch.as_tensor(g[k]).cuda() for k in ("crow", "col", "tcrow", "tcol", "tperm")}
    w = torch.as_tensor(g["w"]).cuda().requires_grad_(True)
    ht = torch.as_tensor(h).cuda().requires_grad_(True)
    z = HopCuda.apply(w, ht, T["crow"], T["col"], T["tcrow"], T["tcol"], T["tperm"], False)
    (torch.relu(z) ** 2).sum().backward()
    w64 = torch.as_tensor(g["w"], dtype=torch.float64).requires_grad_(True)
    h64 = torch.as_tensor(h, dtype=torch.float64).requires_grad_(True)
    A = torch.zeros(g["n_rows"], g["n_src"], dtype=torch.float64).index_put(
        (torch.as_tensor(g["rows"]), torch.as_tensor(g["col"].astype(np.int64))), w64, accumulate=True)
    (torch.relu(A @ h64) ** 2).sum().backward()
    assert rel(z.detach().cpu().numpy(), (A @ h64).detach().numpy()) < TOL
    assert rel(w.grad.cpu().numpy(), w64.grad.numpy()) < TOL
    assert rel(ht.grad.cpu().numpy(), h64.grad.numpy()) < TOL


@pytest.mark.gpu
def test_hop_operator_refuses_misaligned_states(cuda):
    import torch
    g = _graph()
    T = {k: torch.as_tensor(g[k]).cuda() for k in ("crow", "col")}
    w = torch.as_tensor(g["w"]).cuda()
    buf = torch.zeros(g["n_src"] * 64 + 1, device="cuda")
    out = torch.empty(g["n_rows"], 64, device="cuda")
    L = native.lib()
    rc = L.fg_hop_fwd(w.data_ptr(), buf.data_ptr() + 4, T["crow"].data_ptr(), T["col"].data_ptr(), g["n_rows"],
                      g["n_src"], 64, 0, out.data_ptr(), None)
    assert rc == -1 and "aligned" in L.fg_hop_last_error().decode()
