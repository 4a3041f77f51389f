"""Writes the golden fixtures of the hop path from the REFERENCE's own code (run in the build container, where the
reference project adventure-gpt/flyguy is mounted; its Python imports here, nothing of it is copied).

  python tests/golden/make_golden.py [--ref REFERENCE_CHECKOUT]

Each committed fixture tests/golden/<case>.npz holds one network and what the reference computes on it:
  net          the network as NET.bin bytes, written by the reference's flyguy/native/export.py:write_net
               (so the FLY1 reader of this package is pinned too)
  P0..P6       the seven weight arrays (export.py:params_from_torch order: W in play, gain, theta, in_w, in_b, out_w,
               out_b)
  obs, teacher a seeded batch and teacher logits; inv_temp the teacher's 1/temperature
  logits       FlyActor.forward with gradients on (the gather path, flyguy/fly.py:290-305)
  logits_sparse  the same through the sparse-product path (_Hop, flyguy/fly.py:51-72), gather_limit = 0
  loss, dlogits  KL(softmax(teacher*inv_temp) || softmax(logits)) averaged over the batch, and its gradient
  G0..G6       the weights' gradients of that loss by torch autograd through the reference's FlyActor
  A0..A6       the weights after one torch.optim.Adam step (lr 1e-3 for W and the plugs, 3e-4 for gain / theta:
               teach.py's groups, flyguy/teach.py:138-141) from those gradients

Cases:
  toy_h2 / toy_h3 / toy_h4   a made-up 80-neuron connectome (this script's own generator) as FlyActor builds it for
                             2, 3 and 4 hops: sensory re-drive, shared weights across hops, rows without edges
  toy_wide_h3                a made-up 700-neuron connectome, 3 hops, batch 96
  syn_small                  a small seeded synthetic graph (flyguy_b200.synth) loaded into the reference's FlyActor
                             by filling its buffers (duplicate edges, Zipf hubs, no re-drive)

With the reference's bot/model.pt present, it also writes tests/golden/_model/ (git-ignored, too large to commit):
model.net.bin, model.params.bin and model_ref.npz (obs, teacher, logits, dlogits, G0..G6 at batch 64).
"""
from __future__ import annotations

import argparse
import os
import io
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def toy_connectome(path: Path, n: int, n_sens: int, n_dn: int, edges: int, seed: int) -> None:
    """A random directed graph without self-loops or repeated pairs, in the reference's graph-file layout."""
    rng = np.random.default_rng(seed)
    key = rng.choice(n * n, size=edges * 2, replace=False)
    pre, post = key // n, key % n
    keep = pre != post
    pre, post = pre[keep][:edges], post[keep][:edges]
    o = np.lexsort((post, pre))
    pre, post = pre[o].astype(np.int32), post[o].astype(np.int32)
    ids = rng.permutation(n)
    np.savez(path, body=np.arange(n) + 5000, cls=np.array(["x"] * n), pre=pre, post=post,
             nt=rng.choice(["acetylcholine", "gaba", "glutamate", "histamine"], n),
             syn=rng.integers(1, 50, len(pre)).astype(np.int32),
             sensory=np.sort(ids[:n_sens]).astype(np.int32), descending=np.sort(ids[n_sens:n_sens + n_dn]).astype(np.int32))


def synthetic_actor(FlyActor, s, P):
    """The reference's FlyActor with its buffers filled from a synthetic structure (its __init__ builds from a
    connectome file; the forward and autograd only read these buffers, flyguy/fly.py:105-154)."""
    import torch.nn as nn
    f = FlyActor.__new__(FlyActor)
    nn.Module.__init__(f)
    K = s["hops"]
    f.n_neurons, f.n_conn, f.hops, f.obs_dim, f.fan = s["n_neurons"], s["n_w"], K, s["obs_dim"], s["fan"]
    f.whole_graph, f.gather_limit, f.kernel, f.sizes = False, 60_000_000, "torch", list(s["sizes"])

    def buf(name, a):
        f.register_buffer(name, torch.as_tensor(np.ascontiguousarray(a)), persistent=False)
    f.used = 0
    for k in range(1, K + 1):
        h = s["hop"][k - 1]
        rows = np.repeat(np.arange(s["sizes"][k]), np.diff(h["crow"]))
        c = np.asarray(h["col"], np.int64)
        t = np.lexsort((rows, c))
        buf(f"e{k}", np.asarray(h["widx"], np.int64)); buf(f"r{k}", rows); buf(f"c{k}", c)
        buf(f"crow{k}", np.asarray(h["crow"], np.int64)); buf(f"tcrow{k}", np.asarray(h["tcrow"], np.int64))
        buf(f"tcol{k}", rows[t]); buf(f"tperm{k}", t)
        buf(f"ci{k}", c.astype(np.int32)); buf(f"tci{k}", rows[t].astype(np.int32))
        buf(f"n{k}", np.asarray(h["nid"], np.int64))
        buf(f"s{k}", np.zeros(0, np.int64)); buf(f"d{k}", np.zeros(0, np.int64))
        f.used += len(c)
    f.in_play = s["n_w"]
    buf("n0", np.asarray(s["n0"], np.int64)); buf("dn_rows", np.asarray(s["dn_rows"], np.int64))
    n_s, fan = s["n_s"], s["fan"]
    rows = np.repeat(np.arange(n_s), fan)
    cols = np.asarray(s["in_col"], np.int64)
    t = np.lexsort((rows, cols))
    buf("in_r", rows); buf("in_c", cols); buf("in_crow", np.asarray(s["in_crow"], np.int64))
    buf("in_tcrow", np.asarray(s["in_tcrow"], np.int64)); buf("in_tcol", rows[t]); buf("in_tperm", t)
    buf("in_ci", cols.astype(np.int32)); buf("in_tci", rows[t].astype(np.int32))
    W, gain, theta, in_w, in_b, ow, ob = [torch.as_tensor(np.asarray(p, np.float32)) for p in P]
    f.w, f.gain, f.theta = nn.Parameter(W.clone()), nn.Parameter(gain.clone()), nn.Parameter(theta.clone())
    f.in_w, f.in_b = nn.Parameter(in_w.clone()), nn.Parameter(in_b.clone())
    f.out = nn.Linear(s["n_dn"], s["n_act"])
    with torch.no_grad():
        f.out.weight.copy_(ow.view(s["n_act"], s["n_dn"]))
        f.out.bias.copy_(ob)
    return f


def run_case(f, write_net, params_from_torch, structure, B: int, seed: int, inv_temp: float) -> dict:
    g = torch.Generator().manual_seed(seed)
    obs = torch.randn(B, f.obs_dim, generator=g)
    teacher = 2.0 * torch.randn(B, f.out.out_features, generator=g)
    with tempfile.TemporaryDirectory() as tmp:
        s = write_net(f, Path(tmp) / "net.bin")
        net = np.frombuffer((Path(tmp) / "net.bin").read_bytes(), np.uint8).copy()
    P = [np.array(p, np.float32, copy=True) for p in params_from_torch(f, s)]   # (copies: some are views of the live weights)
    f.zero_grad()
    f.gather_limit = 10 ** 18
    logits = f(obs)
    lp = torch.log_softmax(logits, -1)
    pt = torch.softmax(teacher * inv_temp, -1)
    loss = (pt * (torch.log_softmax(teacher * inv_temp, -1) - lp)).sum(-1).mean()
    dl = torch.autograd.grad(loss, logits, retain_graph=True)[0]
    loss.backward()
    G = [f.w.grad.numpy()[s["wmap"]], f.gain.grad.numpy(), f.theta.grad.numpy(), f.in_w.grad.numpy(),
         f.in_b.grad.numpy(), f.out.weight.grad.numpy().reshape(-1), f.out.bias.grad.numpy()]
    out = {"net": net, "obs": obs.numpy(), "teacher": teacher.numpy(), "inv_temp": np.float32(inv_temp),
           "logits": logits.detach().numpy(), "loss": np.float64(loss.item()), "dlogits": dl.numpy()}
    f.gather_limit = 0
    try:
        out["logits_sparse"] = f(obs).detach().numpy()
    except RuntimeError:
        out["logits_sparse"] = out["logits"]
    for i in range(7):
        out[f"P{i}"], out[f"G{i}"] = np.asarray(P[i], np.float32), np.asarray(G[i], np.float32)
    # one Adam step with teach.py's groups (W and plugs at lr, gain/theta at 0.3 lr)
    plugs = [p for k, p in f.named_parameters() if k not in ("w", "gain", "theta")]
    opt = torch.optim.Adam([{"params": [f.w], "lr": 1e-3}, {"params": [f.gain, f.theta], "lr": 3e-4},
                            {"params": plugs, "lr": 1e-3}])
    opt.step()
    A = params_from_torch(f, s)
    for i in range(7):
        out[f"A{i}"] = np.asarray(A[i], np.float32)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("FLYGUY_REF"), required="FLYGUY_REF" not in os.environ,
                    help="checkout of the reference project (default: the FLYGUY_REF environment variable)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    sys.path.insert(0, str(REPO))
    from flyguy.fly import FlyActor                              # the reference's
    from flyguy.native.export import params_from_torch, structure, write_net
    from flyguy_b200.synth import make_synthetic
    torch.set_num_threads(8)
    cases = {}
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        toy_connectome(tmp / "toy.npz", 80, 14, 7, 420, seed=0)
        toy_connectome(tmp / "wide.npz", 700, 90, 40, 6000, seed=1)
        for hops in (2, 3, 4):
            torch.manual_seed(hops)
            f = FlyActor(tmp / "toy.npz", 517, 90, hops=hops, fan=5)
            with torch.no_grad():                                 # lively, so that the comparison means something
                sign = torch.where(torch.rand_like(f.w) < 0.2, -1.0, 1.0)
                f.w.abs_().mul_(4.0 * sign); f.out.weight.normal_(0, 0.3); f.theta.fill_(-2.0)
                f.gain.mul_(1 + 0.2 * torch.randn_like(f.gain)); f.in_b.normal_(0, 0.2)
            cases[f"toy_h{hops}"] = run_case(f, write_net, params_from_torch, structure, 40, 10 + hops, 1.0)
        torch.manual_seed(7)
        f = FlyActor(tmp / "wide.npz", 517, 90, hops=3, fan=8)
        with torch.no_grad():
            sign = torch.where(torch.rand_like(f.w) < 0.2, -1.0, 1.0)
            f.w.abs_().mul_(2.0 * sign); f.out.weight.normal_(0, 0.2); f.theta.fill_(-2.5)
        cases["toy_wide_h3"] = run_case(f, write_net, params_from_torch, structure, 96, 21, 2.0)
        s, P = make_synthetic(sizes=(300, 700, 500, 60), total_edges=30_000, fan=8, seed=3)
        f = synthetic_actor(FlyActor, s, P)
        cases["syn_small"] = run_case(f, write_net, params_from_torch, structure, 64, 31, 1.0)
    for name, d in cases.items():
        buf = io.BytesIO()
        np.savez_compressed(buf, **d)
        (HERE / f"{name}.npz").write_bytes(buf.getvalue())
        print(f"{name}: {len(buf.getvalue()) / 1024:.0f} KiB, logits max {np.abs(d['logits']).max():.3f}, "
              f"firing descending share {np.mean(d['logits'] != d['P6']):.2f}, "
              f"sparse vs gather {np.abs(d['logits'] - d['logits_sparse']).max():.2e}")
    model = Path(args.ref) / "bot" / "model.pt"
    if model.exists():
        from flyguy.model import build_model
        ck = torch.load(model, map_location="cpu", weights_only=False)
        ac = build_model({**ck["config"]["model"], "fly_kernel": "torch"})
        ac.load_state_dict(ck["model"], strict=False)
        f = ac.actor
        d = run_case(f, write_net, params_from_torch, structure, 64, 41, 1.0)
        out = HERE / "_model"
        out.mkdir(exist_ok=True)
        d["net"].tofile(out / "model.net.bin")
        from flyguy_b200.netfile import write_params
        write_params([d[f"P{i}"] for i in range(7)], out / "model.params.bin")
        np.savez(out / "model_ref.npz", **{k: v for k, v in d.items() if k != "net" and not k.startswith(("P", "A"))})
        print(f"model.pt: written to {out} (logits max {np.abs(d['logits']).max():.1f})")


if __name__ == "__main__":
    main()
