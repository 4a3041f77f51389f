"""fg_kl_loss_noalloc - the loss entry point for callers that cannot allocate device memory (a trainer embedded in a
host application that only passes pointers into memory it reserved up front). Collected last on purpose, so that a
failure here cannot hide any other test. It must pass alone in a fresh process and after the other tests: the
entry point's one-time set-up happens on its first call on a device."""
import numpy as np
import pytest

from conftest import load_case, rel
from flyguy_b200 import native

pytestmark = pytest.mark.gpu


def test_noalloc_loss_matches_the_fused_teaching_step(cuda):
    import torch
    s, P, d = load_case("syn_small")
    B, A = len(d["obs"]), s["n_act"]
    h = native.Handle(s, B)
    h.set_params(P)
    obs = torch.as_tensor(d["obs"]).cuda()
    teacher = torch.as_tensor(d["teacher"]).cuda()
    it = float(d["inv_temp"])
    logits = torch.empty(B, A, device="cuda")
    h.zero_grad()
    kl, agree = h.teach(obs, teacher, it, logits=logits)            # the existing entry point (fg_teach)
    G_ref = [g.cpu().numpy() for g in h.get(4)]
    for _ in range(2):                                               # two calls in a row share the fixed scratch
        dl = torch.full((B, A), float("nan"), device="cuda")
        stats = torch.full((2,), float("nan"), device="cuda")
        native.kl_loss_noalloc(logits, teacher, it, dl, stats)
        torch.cuda.synchronize()
        st = stats.cpu().numpy()
        assert abs(st[0] - kl) <= 1e-5 * max(1.0, abs(kl))
        assert st[1] == agree
        assert rel(dl.cpu().numpy(), d["dlogits"]) < 1e-5
        h.zero_grad()                                                # its gradient through the existing backward
        h.forward(obs)
        h.backward(dl)
        G = [g.cpu().numpy() for g in h.get(4)]
        for i in range(7):
            assert rel(G[i], G_ref[i]) < 1e-4, i


def test_noalloc_loss_refuses_batches_beyond_its_scratch(cuda):
    import torch
    x = torch.zeros(65537, 2, device="cuda")
    with pytest.raises(native.FlyguyError, match="65536"):
        native.kl_loss_noalloc(x, x, 1.0, x, torch.zeros(2, device="cuda"))
