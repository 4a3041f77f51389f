"""The reference-facing host API on the GPU: FlyActor (autograd through the library into the parameters' .grad) and
NativeFlyActor + NativeAdam (gradient kept in the library, pieces of max_batch, Adam in the library, weights pulled
back) against the reference's golden outputs - the checks of flyguy/native/core_check.py as tests."""
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_case, rel

sys.path.insert(0, str(GOLDEN))
from make_golden import toy_connectome  # noqa: E402

from flyguy_b200.fly import FlyActor  # noqa: E402
from flyguy_b200.fly_native import NativeFlyActor, grad_arrays  # noqa: E402
from flyguy_b200.netfile import structure_of_actor  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def toy(tmp_path_factory):
    d = tmp_path_factory.mktemp("toy")
    toy_connectome(d / "wide.npz", 700, 90, 40, 6000, seed=1)
    return d / "wide.npz"


def _load(actor, P):
    """The golden weights into an actor (W in play through the in-play map)."""
    wmap = torch.as_tensor(structure_of_actor(actor)["wmap"])
    with torch.no_grad():
        actor.w[wmap] = torch.as_tensor(P[0])
        for p, v in ((actor.gain, P[1]), (actor.theta, P[2]), (actor.in_w, P[3]), (actor.in_b, P[4]),
                     (actor.out.weight, P[5]), (actor.out.bias, P[6])):
            p.copy_(torch.as_tensor(v).view_as(p))
    return wmap


def _kl(logits, teacher, it):
    lp = torch.log_softmax(logits, -1)
    pt = torch.softmax(teacher * it, -1)
    return (pt * (torch.log_softmax(teacher * it, -1) - lp)).sum(-1).mean()


def test_flyactor_autograd_matches_reference(toy, cuda):
    _, P, d = load_case("toy_wide_h3")
    f = FlyActor(toy, 517, 90, hops=3, fan=8)
    wmap = _load(f, P).cuda()
    f = f.cuda()
    obs, teacher = torch.as_tensor(d["obs"]).cuda(), torch.as_tensor(d["teacher"]).cuda()
    logits = f(obs)
    assert rel(logits.detach().cpu().numpy(), d["logits"]) < 1e-5
    loss = _kl(logits, teacher, float(d["inv_temp"]))
    loss.backward()
    assert abs(loss.item() - float(d["loss"])) < 1e-5 * max(1, abs(float(d["loss"])))
    got = [f.w.grad[wmap], f.gain.grad, f.theta.grad, f.in_w.grad, f.in_b.grad, f.out.weight.grad.reshape(-1),
           f.out.bias.grad]
    for i in range(7):
        assert rel(got[i].cpu().numpy(), d[f"G{i}"]) < 1e-4, i
    out_of_play = torch.ones_like(f.w, dtype=torch.bool)
    out_of_play[wmap] = False
    assert float(f.w.grad[out_of_play].abs().max()) == 0.0 if out_of_play.any() else True
    # a torch optimiser step changes the weights; the next forward sees them (pushed by version)
    opt = torch.optim.Adam(f.parameters(), lr=1e-3)
    opt.step()
    with torch.no_grad():
        after = f(obs)
    assert not torch.equal(after, logits.detach())


def test_native_actor_pieces_and_adam(toy, cuda):
    """core_check.py as a test: one piece vs pieces of max_batch give the same gradient; one Adam step at 1e-3 moves
    strengths and neurons by the expected amounts; strengths out of play stay; optimiser state round-trips."""
    _, P, d = load_case("toy_wide_h3")
    B = len(d["obs"])
    obs, teacher = torch.as_tensor(d["obs"]).cuda(), torch.as_tensor(d["teacher"]).cuda()
    grads = {}
    for mb in (128, 32):                                    # one piece; three pieces of 32
        f = NativeFlyActor(toy, 517, 90, hops=3, fan=8, max_batch=mb)
        wmap = _load(f, P)
        f = f.cuda()
        opt = f.native_adam(1e-3, 0.0)
        opt.zero_grad()
        logits = f(obs)
        assert logits.shape == (B, 90)
        _kl(logits, teacher, float(d["inv_temp"])).backward()
        grads[mb] = grad_arrays(f)
        assert f.w.grad is None                              # the gradient stays in the library
        for i in range(7):
            assert rel(grads[mb][i], d[f"G{i}"]) < 1e-4, (mb, i)
    before = [t.detach().clone() for t in (f.w, f.gain, f.out.weight)]
    opt.step()
    moved = [float((a.detach() - b).abs().max()) for a, b in zip((f.w, f.gain, f.out.weight), before)]
    out_of_play = torch.ones(f.w.numel(), dtype=torch.bool, device="cuda")
    out_of_play[wmap.cuda()] = False
    still = float((f.w.detach() - before[0])[out_of_play].abs().max()) if out_of_play.any() else 0.0
    assert 5e-4 < moved[0] < 2e-3 and 1e-4 < moved[1] < 6e-4 and still == 0.0, (moved, still)
    sd = opt.state_dict()
    assert sd["adam_t"] == 1 and len(sd["m"]) == 7
    opt.load_state_dict(sd)
    with torch.no_grad():
        again = f(obs)
    assert torch.isfinite(again).all()


def test_flyactor_16bit_inference(toy, cuda):
    _, P, d = load_case("toy_wide_h3")
    f = FlyActor(toy, 517, 90, hops=3, fan=8)
    _load(f, P)
    f = f.cuda()
    f.kernel = "cuda16"
    with torch.no_grad():
        got = f(torch.as_tensor(d["obs"]).cuda()).cpu().numpy()
    assert rel(got, d["logits"]) < 1e-2


def test_teach_trainer_learns_and_saves(tmp_path, cuda):
    """flyguy/teach.py's loop on the library: a student network distils a teacher (a different random fly network)
    from a FLYD file; the running average gets closer to the teacher and is saved as a checkpoint that loads back."""
    import argparse
    from flyguy_b200.model import load_actor, save_actor
    from flyguy_b200.teach import train, write_moments
    toy_connectome(tmp_path / "g.npz", 700, 90, 40, 6000, seed=1)
    cfg = {"fly_graph": str(tmp_path / "g.npz"), "fly_hops": 3, "fly_fan": 8, "fly_kernel": "torch"}
    torch.manual_seed(5)
    t = FlyActor(tmp_path / "g.npz", 517, 90, hops=3, fan=8)
    with torch.no_grad():
        t.w.abs_().mul_(2.0)
        t.out.weight.normal_(0, 0.3)
        t.theta.fill_(-2.5)
    save_actor(tmp_path / "teacher.pt", t, cfg, 0)
    rng = np.random.default_rng(0)
    write_moments(tmp_path / "m.bin", rng.standard_normal((3000, 517)).astype(np.float16))
    args = argparse.Namespace(data=[tmp_path / "m.bin"], teacher=tmp_path / "teacher.pt", start="fresh", graph="",
                              graph_root=None, hops=0, steps=150, batch=64, lr=3e-3, temp=1.0, average=0.99,
                              holdout=0.1, eval_every=150, out=tmp_path / "student.pt", seed=0)
    r = train(args)
    assert r["kl"] < r["kl0"], r
    ck, s = load_actor(tmp_path / "student.pt", native=False, device="cuda")
    assert ck["taught_steps"] == 150
