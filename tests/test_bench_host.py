"""Host-side arithmetic of bench.py (no GPU): the roofline's DRAM traffic taken from the committed ncu summary and
scaled to a run's per-GPU batch, and the algorithmic bytes the roofline divides by."""
import importlib.util
import json

from conftest import REPO


def _bench():
    spec = importlib.util.spec_from_file_location("bench", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_traffic_scales_with_the_per_gpu_batch():
    b = _bench()
    t = json.loads((REPO / "profiles" / "traffic.json").read_text())
    W = b.WORKLOADS["infer"]
    full = b.traffic_of("hop_fwd", W, t["bf16"]["batch"])
    assert full == round(t["bf16"]["hop_fwd"])
    assert b.traffic_of("hop_fwd", W, t["bf16"]["batch"] // 8) == round(t["bf16"]["hop_fwd"] / 8)
    assert b.traffic_of("hop_fwd", b.WORKLOADS["train"], t["train"]["batch"]) == round(t["train"]["hop_fwd"])


def test_no_traffic_for_other_graphs_or_sources():
    b = _bench()
    assert b.traffic_of("hop_fwd", b.WORKLOADS["infer"], 65536, "uniform") is None
    assert b.traffic_of("hop_fwd", b.WORKLOADS["infer4"], 65536) is None
    assert b.traffic_of("hop_fwd", b.WORKLOADS["full"], 16384) is None


def test_hop_forward_algorithmic_bytes_match_the_stated_figure():
    """24.47 GB per step at bf16, batch 65,536 on the config-2 graph: every layer written once and read once, edge
    arrays once."""
    b = _bench()
    from flyguy_b200 import synth
    s, _ = synth.make_synthetic()
    assert abs(b.algo_bytes("hop_fwd", s, 65536, 2) - 24.47e9) < 0.01e9


def test_training_bytes_count_only_what_the_plan_visits():
    """The training step's algorithmic bytes follow the plan: forward classes count every row, backward classes only
    the live rows and their pairs, so a plan with fewer live rows moves fewer backward bytes and the same forward
    bytes."""
    b = _bench()
    from flyguy_b200 import synth
    s, _ = synth.make_synthetic(sizes=(300, 700, 500, 60), total_edges=30_000, seed=3)

    def plan(frac):
        hops = []
        for k, hh in enumerate(s["hop"]):
            rows, n_src, E = s["sizes"][k + 1], s["sizes"][k], len(hh["col"])
            hops.append({"rows": rows, "n_src": n_src, "edges": E, "pairs": E, "tpairs": int(E * frac),
                         "live_dst": int(rows * frac), "live_src": int(n_src * frac), "live_edges": int(E * frac)})
        return b.with_live_pairs({"hops": hops, "plug_live": int(300 * frac), "n_s": 300, "fan": 8, "n_dn": 60})
    full = b.train_bytes(plan(1.0), s, 1024, 100_000, False)
    half = b.train_bytes(plan(0.5), s, 1024, 100_000, False)
    for k in ("plug_fwd", "hop_fwd", "out_fwd", "loss", "out_bwd", "adam"):
        assert full[k] == half[k], k
    for k in ("act_bwd", "wgrad", "hop_bwd_t", "plug_bwd"):
        assert half[k] < full[k], k
    assert full["hop_fwd"] == b.algo_bytes("hop_fwd", s, 1024, 4)
    assert full["adam"] == 36 * 100_000
