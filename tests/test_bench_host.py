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
