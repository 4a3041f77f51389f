"""Parity of the CUDA path (through the C-ABI of libflyguy_b200.so) with the reference's outputs (golden fixtures)
and with the CPU oracle, on the golden networks and on the benchmark's synthetic graph.

Tolerances (max|diff| / max|ref|, the reference's own measure): fp32 states - logits 1e-5 with identical argmax,
gradients 1e-4 (core_check.py accepts 2e-3); 16-bit states - logits 1e-2, and >= 99.9% argmax agreement with the
oracle's emulation of the same 16-bit format (the kernel's own error; the format's is reported beside it)."""
import numpy as np
import pytest

from conftest import CASES, REPO, load_case, rel
from flyguy_b200 import native, synth
from oracle.oracle import Oracle, adam

pytestmark = pytest.mark.gpu
TOL_FP32, TOL_GRAD, TOL_BF16 = 1e-5, 1e-4, 1e-2


def _pad(a, n):
    """Rows up to a multiple of n by repeating the last row (what NativeFlyActor._piece does)."""
    pad = (-len(a)) % n
    return np.concatenate([a, np.repeat(a[-1:], pad, 0)]) if pad else a


def _handle(s, P, max_batch, flags=0):
    h = native.Handle(s, max_batch, flags)
    h.set_params(P, 0)
    h.set_params(P, 1)
    return h


def _t(a):
    import torch
    return torch.as_tensor(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.mark.parametrize("case", CASES)
def test_forward_fp32_matches_reference(case, cuda):
    s, P, d = load_case(case)
    B = len(d["obs"])
    obs = _pad(d["obs"], 32)
    h = _handle(s, P, len(obs))
    got = h.forward(_t(obs)).cpu().numpy()[:B]
    assert rel(got, d["logits"]) < TOL_FP32
    assert (got.argmax(1) == d["logits"].argmax(1)).all()
    again = h.forward(_t(obs), ema=1).cpu().numpy()[:B]          # the running average starts as the weights
    assert np.array_equal(got, again)


@pytest.mark.parametrize("case", CASES)
def test_layers_match_oracle(case, cuda):
    s, P, d = load_case(case)
    obs = _pad(d["obs"], 32)
    h = _handle(s, P, len(obs))
    h.forward(_t(obs))
    _, lay = Oracle(s, threads=4).forward(P, obs, layers=True)
    off = 0
    for k, n in enumerate(s["sizes"]):
        got = h.layer(k, len(obs)).cpu().numpy().T
        want = lay[:, off:off + n]
        assert np.abs(got - want).max() <= TOL_FP32 * max(np.abs(want).max(), 1e-6), k
        off += n


@pytest.mark.parametrize("case", CASES)
def test_backward_matches_reference(case, cuda):
    s, P, d = load_case(case)
    B = len(d["obs"])
    obs = _pad(d["obs"], 32)
    dl = np.zeros((len(obs), s["n_act"]), np.float32)
    dl[:B] = d["dlogits"]                                           # padded samples carry no gradient
    h = _handle(s, P, len(obs))
    h.zero_grad()
    h.forward(_t(obs))
    h.backward(_t(dl))
    G = [g.cpu().numpy() for g in h.get(4)]
    for i in range(7):
        assert rel(G[i], d[f"G{i}"]) < TOL_GRAD, i
    h.backward(_t(dl))                                              # a second call ADDS (fc_backward semantics)
    G2 = [g.cpu().numpy() for g in h.get(4)]
    for i in range(7):
        assert rel(G2[i], 2 * d[f"G{i}"]) < TOL_GRAD, i


@pytest.mark.parametrize("case", ["toy_wide_h3", "syn_small"])
def test_teach_step_matches_reference(case, cuda):
    """fg_teach (forward + KL loss + backward fused) gives the reference's loss and gradients."""
    s, P, d = load_case(case)
    B = len(d["obs"])
    assert B % 32 == 0
    h = _handle(s, P, B)
    h.zero_grad()
    logits = _t(np.zeros((B, s["n_act"])))
    kl, agree = h.teach(_t(d["obs"]), _t(d["teacher"]), float(d["inv_temp"]), logits=logits)
    assert abs(kl / B - float(d["loss"])) <= 1e-5 * max(1.0, abs(float(d["loss"])))
    assert agree == float((d["logits"].argmax(1) == (d["teacher"] * d["inv_temp"]).argmax(1)).sum())
    assert rel(logits.cpu().numpy(), d["logits"]) < TOL_FP32
    G = [g.cpu().numpy() for g in h.get(4)]
    for i in range(7):
        assert rel(G[i], d[f"G{i}"]) < TOL_GRAD, i


@pytest.mark.parametrize("case", ["toy_h3", "syn_small"])
def test_adam_step_matches_oracle(case, cuda):
    s, P, d = load_case(case)
    obs = _pad(d["obs"], 32)
    h = _handle(s, P, len(obs))
    h.zero_grad()
    h.forward(_t(obs))
    dl = np.zeros((len(obs), s["n_act"]), np.float32)
    dl[:len(d["obs"])] = d["dlogits"]
    h.backward(_t(dl))
    G = [g.cpu().numpy() for g in h.get(4)]
    for max_norm in (0.0, 0.05):
        h2 = _handle(s, P, len(obs))
        h2.copy(4, 1, [_t(g) for g in G])
        norm = h2.step(1e-3, 3e-4, 1e-3, max_norm, 0.999)
        P2, M, V, E = [p.copy() for p in P], [np.zeros_like(p) for p in P], [np.zeros_like(p) for p in P], \
            [p.copy() for p in P]
        want_norm = adam(P2, [g.copy() for g in G], M, V, E, 1, 1e-3, 3e-4, 1e-3, max_norm, 0.999)
        assert abs(norm - want_norm) <= 1e-5 * max(want_norm, 1e-12)
        for which, want in ((0, P2), (1, E), (2, M), (3, V)):
            got = [g.cpu().numpy() for g in h2.get(which)]
            for i in range(7):
                tol = 1e-6 * max(np.abs(want[i]).max(), 1e-30)
                assert np.abs(got[i] - want[i]).max() <= tol, (which, i)
        assert h2.adam_t() == 1


@pytest.mark.parametrize("case", CASES)
def test_forward_bf16_close_to_reference(case, cuda):
    s, P, d = load_case(case)
    B = len(d["obs"])
    obs = _pad(d["obs"], 32)
    h = _handle(s, P, len(obs), native.FG_ACT_BF16)
    got = h.forward(_t(obs)).cpu().numpy()[:B]
    assert rel(got, d["logits"]) < TOL_BF16
    # against the oracle's emulation of bf16 states the only differences left are fp32 sum orders
    emu = Oracle(s).forward(P, d["obs"], states="bf16+obs")
    assert rel(got, emu) < 2e-3


def test_model_pt_matches_reference(cuda):
    """The shipped bot/model.pt network (trimmed male-CNS graph, 3,688,058 edge-steps, sensory re-drive, weights
    shared across hops): logits and all seven gradients against the reference's FlyActor."""
    base = REPO / "tests" / "golden" / "_model"
    if not (base / "model.net.bin").exists():
        pytest.skip("tests/golden/_model not generated (needs the reference's bot/model.pt)")
    from flyguy_b200.netfile import read_params
    d = dict(np.load(base / "model_ref.npz"))
    h = native.Handle(base / "model.net.bin", 64)
    _, P = read_params(base / "model.params.bin", h.s)
    h.set_params(P)
    h.zero_grad()
    got = h.forward(_t(d["obs"])).cpu().numpy()
    assert rel(got, d["logits"]) < TOL_FP32
    assert (got.argmax(1) == d["logits"].argmax(1)).all()
    h.backward(_t(d["dlogits"]))
    G = [g.cpu().numpy() for g in h.get(4)]
    for i in range(7):
        assert rel(G[i], d[f"G{i}"]) < TOL_GRAD, i
    for flag in (native.FG_ACT_BF16, native.FG_ACT_F16):
        hb = native.Handle(base / "model.net.bin", 64, flag)
        hb.set_params(P)
        got16 = hb.forward(_t(d["obs"])).cpu().numpy()
        assert rel(got16, d["logits"]) < TOL_BF16
        assert (got16.argmax(1) == d["logits"].argmax(1)).all()        # model.pt's logits have wide margins


# ------------------------------------------------------------------ the benchmark graph (2,992,734 edges)
@pytest.fixture(scope="module")
def flygraph():
    return synth.make_synthetic()


def _spread(n, k):
    return np.unique(np.linspace(0, n - 1, k).astype(np.int64))


def test_synthetic_fp32_batch4096_matches_oracle(flygraph, cuda):
    """Config 1: fp32, batch 4,096 - samples spread over the batch against the oracle, identical argmax."""
    s, P = flygraph
    obs, _ = synth.make_batch(4096, seed=11)
    h = _handle(s, P, 4096, native.FG_INFER_ONLY)
    got = h.forward(_t(obs)).cpu().numpy()
    idx = _spread(4096, 96)
    want = Oracle(s).forward(P, obs[idx])
    assert rel(got[idx], want) < TOL_FP32
    assert (got[idx].argmax(1) == want.argmax(1)).all()
    assert np.isfinite(got).all()


def test_synthetic_16bit_batch65536(flygraph, cuda):
    """Config 2 at batch 65,536, 16-bit states.

    The kernel's error: its logits against the oracle's EMULATION of the same format (every layer but the last rounded
    to nearest even where the kernel stores it, the plug's observation values rounded likewise, sums in double) - over
    the whole batch for bf16 (config 2 as written), over a quarter of it for fp16: within 1e-2 (measured ~1e-4) and
    >= 99.9% argmax agreement (hop_check.py's measure and the bar for the bf16-activation path).
    The format's own error: the emulation against the fp32 forward (the GPU fp32 path, itself checked against the
    oracle's fp32 forward on spread samples here). Rounding every stored state to bf16's 8-bit mantissa moves ~0.6% of
    this random network's argmaxes (1% of its samples have a top-2 logit gap below 0.002 logit standard deviations);
    fp16's 11 bits move ~0.05%. That limit is printed and bounded below, not claimed as 99.9%."""
    import torch
    s, P = flygraph
    B = 65536
    obs, _ = synth.make_batch(B, seed=12)
    x = _t(obs)
    h32 = _handle(s, P, 16384, native.FG_INFER_ONLY)
    got32 = torch.cat([h32.forward(x[i:i + 16384]) for i in range(0, B, 16384)]).cpu().numpy()
    h32.close()
    o = Oracle(s)
    idx = _spread(B, 64)
    want = o.forward(P, obs[idx])
    assert rel(got32[idx], want) < TOL_FP32
    assert (got32[idx].argmax(1) == want.argmax(1)).all()
    kernel, fmt = {}, {}
    for name, flag, n in (("bf16", native.FG_ACT_BF16, B), ("f16", native.FG_ACT_F16, B // 4)):
        h = _handle(s, P, B, flag)
        got = h.forward(x).cpu().numpy()
        h.close()
        emu = o.forward(P, obs[:n], states=name + "+obs")
        kernel[name] = (rel(got[:n], emu), float(np.mean(got[:n].argmax(1) == emu.argmax(1))))
        fmt[name] = float(np.mean(emu.argmax(1) == got32[:n].argmax(1)))
        assert rel(got, got32) < TOL_BF16, name
        assert kernel[name][0] < TOL_BF16, (name, kernel[name])
        assert kernel[name][1] >= 0.999, (name, kernel[name])
    print(f"kernel vs emulation (rel, argmax agreement): {kernel}; format limit (emulation vs fp32 argmax "
          f"agreement): {fmt}")
    assert fmt["bf16"] >= 0.99 and fmt["f16"] >= 0.999, fmt


@pytest.mark.parametrize("case", CASES)
def test_forward_f16_matches_reference(case, cuda):
    s, P, d = load_case(case)
    B = len(d["obs"])
    obs = _pad(d["obs"], 32)
    h = _handle(s, P, len(obs), native.FG_ACT_F16)
    got = h.forward(_t(obs)).cpu().numpy()[:B]
    assert rel(got, d["logits"]) < 2e-3
    assert np.mean(got.argmax(1) == d["logits"].argmax(1)) >= 0.97


def test_synthetic_4hop_forward_and_gradients(cuda):
    """The 4-hop network (145,113 neurons, 8.4M connections): fp32 logits and a 32-sample batch's gradients against
    the oracle, bf16 logits within the 16-bit tolerance - the same kernels, one more hop."""
    import torch
    from oracle.oracle import loss
    s, P = synth.make_synthetic4()
    obs, teacher = synth.make_batch(1024, seed=16)
    h = _handle(s, P, 1024)
    got = h.forward(_t(obs)).cpu().numpy()
    idx = _spread(1024, 32)
    want = Oracle(s).forward(P, obs[idx])
    assert rel(got[idx], want) < TOL_FP32
    assert (got[idx].argmax(1) == want.argmax(1)).all()
    small = 32
    h.zero_grad()
    lg = torch.empty(small, s["n_act"], device="cuda")
    h.teach(_t(obs[:small]), _t(teacher[:small]), 1.0, logits=lg)
    G = [g.cpu().numpy() for g in h.get(4)]
    want_lg = Oracle(s).forward(P, obs[:small])
    _, _, dl = loss(want_lg, teacher[:small], 1.0)
    want_g = Oracle(s).backward(P, obs[:small], dl)
    for i in range(7):
        assert rel(G[i], want_g[i]) < TOL_GRAD, i
    hb = _handle(s, P, 1024, native.FG_ACT_BF16)
    assert rel(hb.forward(_t(obs)).cpu().numpy()[idx], want) < TOL_BF16


def test_synthetic_training_gradients(flygraph, cuda):
    """Config 3's step on the benchmark graph: gradients of a 64-sample batch against the oracle; at batch 16,384 the
    gradient is the sum of its halves' (linearity over samples)."""
    import torch
    s, P = flygraph
    obs, teacher = synth.make_batch(16384, seed=13)
    h = _handle(s, P, 16384)
    h.zero_grad()
    small = 64
    lg = torch.empty(small, s["n_act"], device="cuda")
    h.teach(_t(obs[:small]), _t(teacher[:small]), 1.0, logits=lg)
    G = [g.cpu().numpy() for g in h.get(4)]
    from oracle.oracle import loss
    want_lg = Oracle(s).forward(P, obs[:small])
    _, _, dl = loss(want_lg, teacher[:small], 1.0)
    want = Oracle(s).backward(P, obs[:small], dl)
    assert rel(lg.cpu().numpy(), want_lg) < TOL_FP32
    for i in range(7):
        assert rel(G[i], want[i]) < TOL_GRAD, i
    # linearity: teach on all 16,384 == backward of the two halves with the same dl
    h.zero_grad()
    lg_all = torch.empty(16384, s["n_act"], device="cuda")
    h.teach(_t(obs), _t(teacher), 1.0, logits=lg_all)
    G_all = [g.cpu().numpy() for g in h.get(4)]
    _, _, dl_all = loss(lg_all.cpu().numpy(), teacher, 1.0)
    h.zero_grad()
    for lo in (0, 8192):
        h.forward(_t(obs[lo:lo + 8192]))
        h.backward(_t(dl_all[lo:lo + 8192]))
    G_halves = [g.cpu().numpy() for g in h.get(4)]
    for i in range(7):
        assert rel(G_halves[i], G_all[i]) < TOL_GRAD, i


def test_errors_leave_the_handle_usable(cuda):
    s, P, d = load_case("syn_small")
    h = _handle(s, P, 64)
    with pytest.raises(native.FlyguyError, match="multiple of 32"):
        h.forward(_t(d["obs"][:33]))
    with pytest.raises(native.FlyguyError, match="max_batch"):
        h.forward(_t(np.zeros((96, s["obs_dim"]))))
    got = h.forward(_t(d["obs"])).cpu().numpy()
    assert rel(got, d["logits"]) < TOL_FP32
    hi = _handle(s, P, 64, native.FG_INFER_ONLY)
    hi.forward(_t(d["obs"]))
    with pytest.raises(native.FlyguyError, match="inference only"):
        hi.backward(_t(d["dlogits"]))


@pytest.mark.parametrize("B", [8192, 33024])
def test_host_buffer_forward_matches_device_forward(flygraph, B, cuda):
    """fg_forward_host (pinned host buffers, copies overlapped with compute; 8,192 runs as pieces of 1,024 / 3,072 /
    4,096 samples, 33,024 as 2,048 / 6,144 / 18,432 / 6,400 - the last not a whole 1,024-sample hop chunk) gives the
    device forward's logits bit for bit."""
    import torch
    s, P = flygraph
    obs, _ = synth.make_batch(B, seed=14)
    h = _handle(s, P, B, native.FG_ACT_BF16)
    dev = h.forward(_t(obs)).cpu()
    host_obs = torch.from_numpy(obs).pin_memory()
    host_out = torch.empty(B, s["n_act"]).pin_memory()
    h.forward_host(host_obs, host_out)
    assert torch.equal(dev, host_out)


def test_stream_binding_and_zero_copy_gradient(cuda):
    """Work goes to torch's current stream; the flat gradient is the library's memory (zero copy)."""
    import torch
    s, P, d = load_case("syn_small")
    h = _handle(s, P, 64)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        h.zero_grad()
        h.forward(_t(d["obs"]))
        h.backward(_t(d["dlogits"]))
        flat = h.flat(4)
        flat.mul_(2.0)                                              # in place, as an all-reduce would
    st.synchronize()
    G = [g.cpu().numpy() for g in h.get(4)]
    for i in range(7):
        assert rel(G[i], 2 * d[f"G{i}"]) < TOL_GRAD, i


def test_untrimmed_graph_config4_matches_oracle(cuda):
    """Config 4's graph (166,700 neurons, 15,283,167 edges, hops 2-3 over all edges with shared weights, sensory
    drive re-added at every hop): logits and all gradients of a 64-sample teaching step against the oracle, and a batch
    in two pieces (fg_teach_ex with the loss over both) equal to one piece."""
    import torch
    from oracle.oracle import loss
    s, P = synth.make_full_graph()
    obs, teacher = synth.make_batch(64, seed=21)
    h = _handle(s, P, 64)
    lg = torch.empty(64, s["n_act"], device="cuda")
    h.zero_grad()
    h.teach(_t(obs), _t(teacher), 1.0, logits=lg)
    G = [g.cpu().numpy() for g in h.get(4)]
    o = Oracle(s)
    want_lg = o.forward(P, obs)
    _, _, dl = loss(want_lg, teacher, 1.0)
    want = o.backward(P, obs, dl)
    assert rel(lg.cpu().numpy(), want_lg) < TOL_FP32
    for i in range(7):
        assert rel(G[i], want[i]) < TOL_GRAD, i
    h.zero_grad()
    for lo in (0, 32):
        h.teach(_t(obs[lo:lo + 32]), _t(teacher[lo:lo + 32]), 1.0, loss_norm=64)
    G2 = [g.cpu().numpy() for g in h.get(4)]
    for i in range(7):
        assert rel(G2[i], G[i]) < TOL_GRAD, i
