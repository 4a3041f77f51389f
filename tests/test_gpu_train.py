"""The standalone teaching trainer (fg_train; the reference's flyguy_train program, flyguy/native/flyguy_train.cu:
631-788) on a small synthetic network: it learns, writes FLYP / FLYO in the reference's formats, is deterministic,
matches the same steps driven from Python through the library bit for bit, restarts from its own save with the
optimiser state, stops on a STOP file, holds a chunk out and scores it every --eval-every steps, answers --check like
the reference's export.py batch (against the oracle), and revives silent neurons exactly as the CPU restatement of
the reference's revive() does (oracle/revival.py)."""
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import REPO
from flyguy_b200 import native, netfile, synth

pytestmark = pytest.mark.gpu
TRAIN = REPO / "flyguy_b200" / "fg_train"
M64 = (1 << 64) - 1


def _setup(tmp_path):
    s, P = synth.make_synthetic(sizes=(300, 600, 500, 120), total_edges=20000, seed=3)
    netfile.write_net(s, tmp_path / "NET.bin")
    netfile.write_params(P, tmp_path / "P0.bin", step=0)
    data = tmp_path / "data"
    data.mkdir()
    for i, (n, seed) in enumerate(((700, 31), (500, 32))):
        obs, teacher = synth.make_batch(n, seed=seed)
        netfile.write_chunk(obs, teacher, data / f"chunk_{i:03d}.bin")
        os.utime(data / f"chunk_{i:03d}.bin", (1_000_000 + i, 1_000_000 + i))     # chunk_000 is the older one
    return s, P, data


def _run(tmp_path, params, out, *opts):
    cmd = [str(TRAIN), str(tmp_path / "NET.bin"), str(params), str(tmp_path / "data"), str(out), "--batch", "64",
           "--log", "10", "--eval-batches", "2", "--save-sec", "1e9", "--lr", "1e-3", *map(str, opts)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def _splitmix64(x):
    x = (x + 0x9E3779B97F4A7C15) & M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M64
    return x ^ (x >> 31)


def test_trainer_learns_and_writes_the_reference_formats(tmp_path, cuda):
    s, P, data = _setup(tmp_path)
    log = _run(tmp_path, tmp_path / "P0.bin", tmp_path / "out", "--steps", 40)
    kls = [float(m) for m in re.findall(r"^step \d+ \| kl ([0-9.]+) agree [0-9.]+ \| lr", log, re.M)]
    assert len(kls) == 4 and kls[-1] < kls[0], log
    assert "eval @0 chunk_001.bin (at the start)" in log
    step, W = netfile.read_params(tmp_path / "out.bin", s)
    assert step == 40 and all(np.isfinite(a).all() for a in W)
    assert netfile.read_params(tmp_path / "out.ema.bin", s)[0] == 40
    st, adam_t, M, V = netfile.read_opt(tmp_path / "out.opt.bin", s)
    assert (st, adam_t) == (40, 40) and any(np.abs(m).max() > 0 for m in M)
    # deterministic: the same run again writes the same bytes
    _run(tmp_path, tmp_path / "P0.bin", tmp_path / "again", "--steps", 40)
    assert (tmp_path / "out.bin").read_bytes() == (tmp_path / "again.bin").read_bytes()
    # a restart from its own save goes on with the running average and the optimiser state
    log2 = _run(tmp_path, tmp_path / "out.bin", tmp_path / "out", "--steps", 10)
    assert "from step 40 with its optimiser state" in log2
    assert netfile.read_params(tmp_path / "out.bin", s)[0] == 50
    assert netfile.read_opt(tmp_path / "out.opt.bin", s)[1] == 50


def test_trainer_steps_equal_the_library_driven_from_python(tmp_path, cuda):
    """Three trainer steps = the same draws (counter-based), the same fused step and the same schedule through
    flyguy_b200.native from Python: identical weights."""
    import torch
    s, P, data = _setup(tmp_path)
    _run(tmp_path, tmp_path / "P0.bin", tmp_path / "t3", "--steps", 3, "--eval-batches", 0)
    chunks = [netfile.read_chunk(data / f"chunk_{i:03d}.bin") for i in range(2)]
    obs_all = np.concatenate([c[0] for c in chunks]).astype(np.float32)
    tl_all = np.concatenate([c[1] for c in chunks]).astype(np.float32)
    total, B, seed = len(obs_all), 64, 12345
    h = native.Handle(s, B)
    h.set_params(P, 0)
    h.set_params(P, 1)
    f32 = np.float32
    lr, lr_n, lr_p, lr_min = f32(1e-3), f32(1e-4), f32(3e-4), f32(3e-5)
    for step in range(3):
        sel = [_splitmix64(seed ^ ((step << 32) | b)) % total for b in range(B)]
        h.zero_grad()
        h.teach(torch.as_tensor(obs_all[sel]).cuda(), torch.as_tensor(tl_all[sel]).cuda(), 1.0, loss_norm=B)
        sched = f32(0.5 ** ((step + 1) / 20000.0))
        rate = lambda base: float(max(lr_min * base / lr, base * sched))
        h.step(rate(lr), rate(lr_n), rate(lr_p), 0.0, 0.999)
    want = [a.cpu().numpy() for a in h.get(0)]
    got = netfile.read_params(tmp_path / "t3.bin", s)[1]
    for i in range(7):
        assert np.array_equal(got[i], want[i]), i


def test_trainer_stops_on_request(tmp_path, cuda):
    s, P, data = _setup(tmp_path)
    (tmp_path / "st.STOP").write_text("")
    log = _run(tmp_path, tmp_path / "P0.bin", tmp_path / "st", "--eval-batches", 0)
    assert "stopped on request @1" in log
    assert (tmp_path / "st.STOP.done").exists() and netfile.read_params(tmp_path / "st.bin", s)[0] == 1


def test_survey_counts_and_squared_inputs(tmp_path, cuda):
    """fg_survey: per row, the samples whose state is positive (= the layers the forward leaves) and the summed squared
    pre-activations (= float64 recomputation from the layer below), and the loss at temperature 1 (= the oracle)."""
    import torch
    from conftest import rel
    from oracle.oracle import Oracle, loss
    s, P, data = _setup(tmp_path)
    B = 256
    obs, teacher = synth.make_batch(B, seed=44)
    h = native.Handle(s, B)
    h.set_params(P, 0)
    h.set_params(P, 1)
    fired, sq, st = h.survey(torch.as_tensor(obs).cuda(), torch.as_tensor(teacher).cuda())
    fired, sq = fired.cpu().numpy(), sq.cpu().numpy()
    layers = [h.layer(k, B).cpu().numpy().astype(np.float64) for k in range(len(s["sizes"]))]
    off = 0
    W = P[0].astype(np.float64)
    for k, L in enumerate(layers):
        rows = L.shape[0]
        assert np.array_equal(fired[off:off + rows], (L > 0).sum(1)), k
        if k:
            hop = s["hop"][k - 1]
            z = np.zeros_like(L)
            r = np.repeat(np.arange(rows), np.diff(hop["crow"]))
            np.add.at(z, r, W[hop["widx"]][:, None] * layers[k - 1][hop["col"]])
            assert rel(sq[off:off + rows], (z * z).sum(1)) < 1e-4, k
        off += rows
    kl_sum, agreements, _ = loss(Oracle(s).forward(P, obs), teacher, 1.0)
    assert abs(st[0] - kl_sum) < 1e-4 * abs(kl_sum)
    assert abs(st[1] - agreements) <= 1


def test_revive_brings_silent_neurons_back_with_the_output_unchanged(tmp_path, cuda):
    """Revival with every rate at zero (so the one step after it changes no weight): the saved weights equal the CPU
    restatement's (oracle/revival.py: the reference's revive() steps on the oracle's forward, the same census draws),
    the loss before and after is the same, and the planted silent neurons are among those revived."""
    from conftest import rel
    from oracle import revival
    s, P, data = _setup(tmp_path)
    n_s = s["sizes"][0]
    P = [a.copy() for a in P]
    planted = np.asarray(s["hop"][0]["nid"])[:60]
    P[2][planted] = 20.0                          # 60 layer-1 neurons whose threshold no input reaches: silent
    netfile.write_params(P, tmp_path / "Ps.bin", step=0)
    log = _run(tmp_path, tmp_path / "Ps.bin", tmp_path / "rv", "--steps", 1, "--revive-every", 1, "--revive-first", 1,
               "--revive-batches", 2, "--eval-batches", 1, "--lr", 0, "--lr-neuron", 0, "--lr-plug", 0, "--lr-min", 0)
    m = re.search(r"revival @0: (\d+) silent of \d+ .* still silent (\d+); kl ([0-9.]+) -> ([0-9.]+)", log)
    assert m, log
    n_dead, still, kl0, kl1 = int(m.group(1)), int(m.group(2)), m.group(3), m.group(4)
    assert n_dead >= 60 and still < n_dead and kl0 == kl1, log
    assert re.search(r"^eval @0 chunk_001.bin \(at the start\) \| average: kl [0-9.]+ agree [0-9.]+ \| weights: kl "
                     r"[0-9.]+ agree [0-9.]+ \| firing [0-9.]+(/[0-9.]+){3} \| silent \d+/\d+$", log, re.M), log
    chunks = [netfile.read_chunk(data / f"chunk_{i:03d}.bin") for i in range(2)]
    obs_all = np.concatenate([c[0] for c in chunks]).astype(np.float32)
    tl_all = np.concatenate([c[1] for c in chunks]).astype(np.float32)
    want, silent = revival.revive(s, P, obs_all, tl_all, seed=12345 + 3, batches=2, B=64, target=0.4)
    assert len(silent) == n_dead and set(planted) <= set(silent.tolist())
    got = netfile.read_params(tmp_path / "rv.bin", s)[1]
    for i in range(7):
        assert rel(got[i], want[i]) < 1e-4, i
    assert np.array_equal(np.sign(got[0]), np.sign(want[0]))


def test_check_mode_answers_like_the_reference_batch_check(tmp_path, cuda):
    """fg_train --check NET PARAMS BATCH (a FLYB batch of 40 samples, not a multiple of 32): loss, agreement, the
    first sample's first logits and every array's gradient norm and sum - against the oracle."""
    from oracle.oracle import Oracle, loss
    s, P, data = _setup(tmp_path)
    obs, teacher = synth.make_batch(40, seed=77)
    netfile.write_batch(obs, teacher, tmp_path / "batch.bin")
    r = subprocess.run([str(TRAIN), "--check", str(tmp_path / "NET.bin"), str(tmp_path / "P0.bin"),
                        str(tmp_path / "batch.bin")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = r.stdout
    o = Oracle(s)
    lg = o.forward(P, obs)
    kl, agree, dl = loss(lg, teacher, 1.0)
    G = o.backward(P, obs, dl)
    m = re.search(r"40 samples \| loss ([0-9.]+) agree ([0-9.]+)", out)
    assert m, out
    assert abs(float(m.group(1)) - kl / 40) < 1e-5 * max(1.0, kl / 40) and float(m.group(2)) == round(agree / 40, 4)
    got_lg = [float(v) for v in re.search(r"logits\[0\]\[:5\]((?: -?[0-9.]+)+)", out).group(1).split()]
    assert np.allclose(got_lg, lg[0, :5], rtol=1e-5, atol=2e-6)
    for i, name in enumerate(("W", "gain", "theta", "in_w", "in_b", "out_w", "out_b")):
        m = re.search(rf"grad {name}\s+norm ([0-9.e+-]+) sum ([0-9.e+-]+)", out)
        norm = float(np.linalg.norm(G[i].astype(np.float64)))
        assert abs(float(m.group(1)) - norm) <= 1e-4 * norm + 1e-12, (name, m.group(1), norm)


def test_holdout_is_scored_every_eval_every_steps_and_never_learned_from(tmp_path, cuda):
    """--holdout 1: the newest chunk at the start (chunk_001) stays out of the ring - the steps equal the library
    driven from Python on chunk_000's samples alone - and --eval-every 5 scores it at steps 0, 5 and 10."""
    import torch
    s, P, data = _setup(tmp_path)
    log = _run(tmp_path, tmp_path / "P0.bin", tmp_path / "ho", "--steps", 10, "--holdout", 1, "--eval-every", 5,
               "--eval-batches", 1)
    assert [int(v) for v in re.findall(r"^eval @(\d+) chunk_001.bin \(held out\)", log, re.M)] == [0, 5, 10], log
    assert "ring 1, newest chunk_000.bin" in log
    obs0, tl0 = netfile.read_chunk(data / "chunk_000.bin")
    obs0, tl0 = obs0.astype(np.float32), tl0.astype(np.float32)
    B, seed = 64, 12345
    h = native.Handle(s, B)
    h.set_params(P, 0)
    h.set_params(P, 1)
    f32 = np.float32
    lr, lr_n, lr_p, lr_min = f32(1e-3), f32(1e-4), f32(3e-4), f32(3e-5)
    for step in range(10):
        sel = [_splitmix64(seed ^ ((step << 32) | b)) % len(obs0) for b in range(B)]
        h.zero_grad()
        h.teach(torch.as_tensor(obs0[sel]).cuda(), torch.as_tensor(tl0[sel]).cuda(), 1.0, loss_norm=B)
        sched = f32(0.5 ** ((step + 1) / 20000.0))
        rate = lambda base: float(max(lr_min * base / lr, base * sched))  # noqa: E731
        h.step(rate(lr), rate(lr_n), rate(lr_p), 0.0, 0.999)
    want = [a.cpu().numpy() for a in h.get(0)]
    got = netfile.read_params(tmp_path / "ho.bin", s)[1]
    for i in range(7):
        assert np.array_equal(got[i], want[i]), i
