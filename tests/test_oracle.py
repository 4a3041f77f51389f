"""The CPU oracle pinned against the reference's own outputs (tests/golden, written from the reference's FlyActor by
tests/golden/make_golden.py), the wire formats, and the synthetic graph generator. CPU only."""
import numpy as np
import pytest

from conftest import CASES, GOLDEN, load_case, rel
from flyguy_b200 import netfile, synth
from oracle.oracle import Oracle, adam, loss


@pytest.mark.parametrize("case", CASES)
def test_oracle_forward_matches_reference(case):
    s, P, d = load_case(case)
    got = Oracle(s, threads=4).forward(P, d["obs"])
    assert rel(got, d["logits"]) < 1e-6
    assert rel(got, d["logits_sparse"]) < 1e-5          # the reference's two paths agree with each other too
    assert (got.argmax(1) == d["logits"].argmax(1)).all()


@pytest.mark.parametrize("case", CASES)
def test_oracle_loss_and_backward_match_reference(case):
    s, P, d = load_case(case)
    o = Oracle(s, threads=4)
    kl, agree, dl = loss(d["logits"], d["teacher"], float(d["inv_temp"]))
    B = len(d["obs"])
    assert abs(kl / B - float(d["loss"])) < 1e-5 * max(1.0, abs(float(d["loss"])))
    assert rel(dl, d["dlogits"]) < 1e-5
    assert agree == float((d["logits"].argmax(1) == (d["teacher"] * d["inv_temp"]).argmax(1)).sum())
    G = o.backward(P, d["obs"], d["dlogits"])
    for i in range(7):
        assert rel(G[i], d[f"G{i}"]) < 2e-6, netfile.PARAM_NAMES[i]


@pytest.mark.parametrize("case", CASES)
def test_oracle_adam_matches_torch_adam(case):
    """One step of the library's Adam (flyguy/native/flyguy_train.cu:194-203) equals torch.optim.Adam with teach.py's
    groups on the reference's gradient, relative to the largest step."""
    s, P, d = load_case(case)
    P2 = [p.copy() for p in P]
    M = [np.zeros_like(p) for p in P]
    V = [np.zeros_like(p) for p in P]
    E = [p.copy() for p in P]
    G = [d[f"G{i}"].copy() for i in range(7)]
    adam(P2, G, M, V, E, 1, 1e-3, 3e-4, 1e-3, 0.0, 0.999)
    for i in range(7):
        want = d[f"A{i}"] - P[i]
        assert np.abs((P2[i] - P[i]) - want).max() <= 2e-3 * max(np.abs(want).max(), 1e-12), netfile.PARAM_NAMES[i]
        assert np.allclose(E[i], 0.999 * P[i] + 0.001 * P2[i], rtol=1e-6, atol=1e-7)


def test_adam_clipping_and_bias_correction_cap():
    rng = np.random.default_rng(0)
    P = [rng.standard_normal(n).astype(np.float32) for n in (50, 7, 7, 9, 3, 12, 2)]
    G = [10 * rng.standard_normal(len(p)).astype(np.float32) for p in P]
    norm = float(np.sqrt(sum((g.astype(np.float64) ** 2).sum() for g in G)))
    zeros = lambda: [np.zeros_like(p) for p in P]  # noqa: E731
    P2, M, V, E = [p.copy() for p in P], zeros(), zeros(), [p.copy() for p in P]
    g = adam(P2, G, M, V, E, 1, 1e-2, 1e-2, 1e-2, max_norm=1.0)
    assert abs(g - norm) < 1e-4 * norm
    assert np.allclose(M[0], 0.1 * G[0] / norm, rtol=1e-5)            # clipped to norm 1 before the moments
    P3, M3, V3, E3 = [p.copy() for p in P], zeros(), zeros(), [p.copy() for p in P]
    adam(P3, G, M3, V3, E3, 10**9, 1e-2, 1e-2, 1e-2)                   # t capped at 100000: c1 = c2 = 1 - tiny
    assert np.isfinite(P3[0]).all()


@pytest.mark.parametrize("case", CASES)
def test_netfile_roundtrip_is_byte_identical(case, tmp_path):
    """The reference's NET.bin (written by its export.py) reads and writes back byte for byte."""
    d = dict(np.load(GOLDEN / f"{case}.npz"))
    s, _, _ = load_case(case)
    netfile.write_net(s, tmp_path / "n.bin")
    assert (tmp_path / "n.bin").read_bytes() == d["net"].tobytes()


def test_params_roundtrip(tmp_path):
    s, P, _ = load_case("toy_h3")
    netfile.write_params(P, tmp_path / "p.bin", step=17)
    step, Q = netfile.read_params(tmp_path / "p.bin", s)
    assert step == 17 and all(np.array_equal(a, b) for a, b in zip(P, Q))


def test_bad_netfile_rejected(tmp_path):
    (tmp_path / "bad.bin").write_bytes(b"FLY2" + bytes(64))
    with pytest.raises(ValueError):
        netfile.read_net(tmp_path / "bad.bin")


def test_synthetic_graph_statistics():
    """Exact edge total, layer sizes, CSR order with sources ascending, Zipf hubs, duplicates kept, determinism."""
    s, P = synth.make_synthetic()
    assert s["sizes"] == list(synth.FLYGUY_SIZES) and s.edges() == synth.FLYGUY_EDGES
    assert s["n_w"] == synth.FLYGUY_EDGES and s["n_neurons"] == sum(synth.FLYGUY_SIZES)
    assert [len(p) for p in P] == s.param_sizes()
    h = s["hop"][0]
    rows = np.repeat(np.arange(s["sizes"][1]), np.diff(h["crow"]))
    key = rows.astype(np.int64) * s["sizes"][0] + h["col"]
    assert (np.diff(key) >= 0).all()                                     # CSR by destination, sources ascending
    assert np.diff(h["crow"]).min() >= 1
    share_top = np.bincount(h["col"]).max() / len(h["col"])
    assert 0.3 < share_top < 0.45                                        # Zipf(1.5): ~38% on the top source
    assert len(np.unique(key)) < 0.5 * len(key)                          # duplicate pairs kept
    deg = np.diff(h["crow"])
    assert 30 < deg.mean() < 40
    s2, P2 = synth.make_synthetic()
    assert all(np.array_equal(a, b) for a, b in zip(P, P2))
    assert np.array_equal(s2["hop"][1]["col"], s["hop"][1]["col"])


def test_oracle_on_synthetic_is_sample_independent():
    """The logits of a sample do not depend on the rest of the batch (what the sharded bench relies on)."""
    s, P = synth.make_synthetic(sizes=(200, 400, 300, 40), total_edges=12_000, seed=5)
    obs, _ = synth.make_batch(16, seed=2)
    o = Oracle(s, threads=2)
    full = o.forward(P, obs)
    assert np.array_equal(full[5:9], o.forward(P, obs[5:9]))


def test_reference_cpu_forward_matches_oracle():
    """The reference's own CPU forward (flyguy/native/fly_infer.cpp, built from source into oracle/_ref) against
    the oracle on the golden networks: the CPU baseline computes the same thing."""
    from oracle.oracle import REF_LIB, RefInfer
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libfly_infer.so not built (reference sources absent)")
    for case in ("toy_h3", "syn_small"):
        s, P, d = load_case(case)
        r = RefInfer(s, P, threads=3)
        got = r.forward(d["obs"])
        r.close()
        assert rel(got, d["logits"]) < 1e-5


def test_16bit_rounding_is_round_to_nearest_even():
    """The emulation's rounding (fo_round16) against torch's own fp32 -> bf16 / fp16 conversions (round to nearest
    even), on random values, exact halfway cases, tiny and huge values and fp16 subnormals."""
    import torch
    from oracle.oracle import round16
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100_000).astype(np.float32) * 10.0 ** rng.integers(-8, 8, 100_000),
                        np.float32([0.0, -0.0, 1.0, 65504.0, 70000.0, 6e-8, 3e-5, 1e-40, 3e38])])
    bits = rng.integers(0, 2 ** 16, 10_000).astype(np.uint32) << 16 | np.uint32(0x8000)    # bf16 halfway points
    x = np.concatenate([x, bits.view(np.float32)[np.isfinite(bits.view(np.float32))]])
    for fmt, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        want = torch.from_numpy(x).to(dt).float().numpy()
        assert np.array_equal(round16(x, fmt), want, equal_nan=True), fmt


def test_16bit_state_emulation_rounds_where_the_kernels_store():
    """states="bf16"/"f16": every layer but the last holds 16-bit values, the last layer and the logits are computed in
    double from them; "+obs" also rounds the plug's inputs. fp32 mode is the reference's forward."""
    from oracle.oracle import round16
    s, P, d = load_case("toy_h3")
    o = Oracle(s, threads=2)
    sizes = np.cumsum([0] + list(s["sizes"]))
    for fmt in ("bf16", "f16"):
        lg, lay = o.forward(P, d["obs"], layers=True, states=fmt)
        for k in range(len(s["sizes"])):
            part = lay[:, sizes[k]:sizes[k + 1]]
            same = np.array_equal(round16(part, fmt), part)
            assert same if k + 1 < len(s["sizes"]) else not same, (fmt, k)
        assert rel(lg, d["logits"]) < 2e-2
        assert not np.array_equal(o.forward(P, d["obs"], states=fmt + "+obs"), lg)
    assert np.array_equal(o.forward(P, d["obs"], states="fp32"), o.forward(P, d["obs"]))
