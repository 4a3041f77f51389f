#!/usr/bin/env python
"""Benchmark of the connectome hop path on B200: one JSON line (rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload infer|infer16|infer32|train|full] [--sources zipf|uniform] [--impl ours|reference]
  (N > 1: python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N)

Workloads (the reference's BASELINE configs, synthetic inputs: the seeded 2,992,734-edge 3-hop graph of
flyguy_b200.synth, obs ~ N(0,1), teacher logits ~ N(0,2^2)):
  infer    (default) config 2 - rollout inference, bf16 states / fp32 accumulation / fp32 weights, global batch 65,536
           sharded over the N GPUs with no collective; metric decisions/sec
  infer32  config 1 - fp32 forward, batch 4,096 per GPU; metric decisions/sec
  train    config 3 - distillation step (forward, fused KL loss, backward, Adam lr 3e-4), global batch 16,384 data-parallel
           with one NCCL all-reduce (average) of the flat fp32 gradient per step; metric train samples/sec

A step is one pass of the hop path over the rank's batch with its inputs resident in HBM; the L2 is flushed (a 256 MiB
write) between timed steps, outside the timed events. `value` = all ranks' units / the max over ranks of the summed
per-step device time. `e2e` = the same metric through the library's host-buffer entry points (fg_forward_host; for
train: pinned H2D of obs + teacher, the next step's copied on a side stream while this step computes, fg_teach,
all-reduce, fc_step, D2H of the loss), host copies inside the timed region. `roofline` = the dominant kernel class's algorithmic bytes / its CUDA-event time over the timed region.
`--impl reference` times the reference's own CPU implementation (flyguy/native/fly_infer.cpp built from source into
oracle/_ref; for training, which the reference does in torch on the CPU, the oracle's C port) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

WORKLOADS = {
    "infer": dict(cfg=2, batch=65536, per_gpu=False, flags="bf16", metric="decisions/sec", unit="decisions/s",
                  dtype="bf16", desc="config 2: bf16-state forward (fp32 accumulation, fp32 weights), global batch "
                                     "65,536 batch-sharded, no collective"),
    "infer16": dict(cfg=2, batch=65536, per_gpu=False, flags="f16", metric="decisions/sec", unit="decisions/s",
                    dtype="f16", desc="config 2 with fp16 states (the reference's 16-bit state format; fp32 "
                                      "accumulation, fp32 weights), global batch 65,536 batch-sharded, no collective"),
    "infer32": dict(cfg=1, batch=4096, per_gpu=True, flags="fp32", metric="decisions/sec", unit="decisions/s",
                    dtype="f32", desc="config 1: fp32 forward, batch 4,096 per GPU"),
    "train": dict(cfg=3, batch=16384, per_gpu=False, flags="train", metric="train samples/sec", unit="samples/s",
                  dtype="f32", desc="config 3: distillation step (forward, KL loss, backward, Adam) fp32, global "
                                    "batch 16,384 data-parallel, one NCCL all-reduce of the flat gradient per step"),
    "infer4": dict(cfg="4-hop", batch=65536, per_gpu=False, flags="bf16", graph="h4", metric="decisions/sec",
                   unit="decisions/s", dtype="bf16",
                   desc="4-hop network (145,113 neurons, 8.4M connections; docs/HOW_IT_WORKS.md:57-59): bf16-state "
                        "forward, global batch 65,536 batch-sharded, no collective"),
    "train4": dict(cfg="4-hop", batch=16384, per_gpu=False, flags="train", graph="h4", metric="train samples/sec",
                   unit="samples/s", dtype="f32",
                   desc="4-hop network: distillation step (forward, KL loss, backward, Adam) fp32, global batch "
                        "16,384 data-parallel, one NCCL all-reduce of the flat gradient per step"),
    "play": dict(cfg="play", batch=8, per_gpu=False, flags="play", metric="decisions/sec", unit="decisions/s",
                 dtype="f32", desc="playing: one decision for 8 cars per call through the reference's fly_* "
                                   "interface (fly_forward: host observations in, host logits and the first car's "
                                   "firing bytes out), fp32, the config-2 graph; latency-bound"),
    "model_infer": dict(cfg="model.pt", batch=65536, per_gpu=False, flags="bf16", graph="model",
                        metric="decisions/sec", unit="decisions/s", dtype="bf16",
                        desc="the shipped bot/model.pt network (trimmed 3-hop graph, 3,688,058 edge-steps over "
                             "2,992,734 shared weights, sensory re-drive, plug fan 16): bf16-state forward, global batch "
                             "65,536 batch-sharded, no collective"),
    "model_infer32": dict(cfg="model.pt", batch=4096, per_gpu=True, flags="fp32", graph="model",
                          metric="decisions/sec", unit="decisions/s", dtype="f32",
                          desc="bot/model.pt network: fp32 forward, batch 4,096 per GPU"),
    "model_train": dict(cfg="model.pt", batch=16384, per_gpu=False, flags="train", graph="model",
                        metric="train samples/sec", unit="samples/s", dtype="f32",
                        desc="bot/model.pt network: distillation step (forward, KL loss, backward over every row - "
                             "nothing is pruned on this graph - and Adam) fp32, global batch 16,384 data-parallel"),
    "model_play": dict(cfg=0, batch=1, per_gpu=False, flags="play", graph="model", metric="decisions/sec",
                       unit="decisions/s", dtype="f32",
                       desc="config 0 on the GPU: one decision per fly_forward call (batch 1) on the bot/model.pt "
                            "network, host observations in, host logits and firing bytes out; latency-bound"),
    "full": dict(cfg=4, batch=32768, per_gpu=False, flags="train", graph="full", metric="train samples/sec",
                 unit="samples/s", dtype="f32",
                 desc="config 4: the untrimmed graph (166,700 neurons, 15,283,167 edges, every hop past the first over "
                      "all edges with shared weights, sensory drive at every hop): forward + backward + Adam fp32, "
                      "global batch 32,768 data-parallel (pieces of at most 16,384 per GPU, one all-reduce per step)"),
}
PIECE = 16384          # largest batch one handle runs at once (config 4: memory for the 166,700-row layers)
ROOF_CLASS = "hop_fwd"      # the dominant kernel class of every workload: timed live in the timed region
LR = 3e-4
FALLBACK_HBM_GBS = 6650.0


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="infer")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="wall time budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-train", action="store_true", help="default workload: leave out the config-3 training block")
    ap.add_argument("--no-check", action="store_true", help="leave out the 16-bit argmax-agreement check")
    ap.add_argument("--no-overlap", action="store_true",
                    help="training at N > 1: one all-reduce of the whole gradient after the backward instead of the "
                         "packed gradient or buckets overlapping the backward")
    ap.add_argument("--batch", type=int, default=0, help="override the global batch (profiling of a small case only)")
    ap.add_argument("--sources", choices=["zipf", "uniform"], default="zipf",
                    help="source distribution of the 3-hop synthetic graph (configs 1-3): Zipf(1.5) ranks, or uniform "
                         "(no L2 locality from hub sources, and every row of every layer feeds the output)")
    a = ap.parse_args()
    a.warmup = max(3, a.warmup)
    return a


# ------------------------------------------------------------------ helpers
def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


class Clocks:
    """nvidia-smi sampled every 50 ms (with timestamps) from before the warm-up; mark_start / mark_end bracket the
    timed region and the summary keeps the samples taken inside it (within 0.1 s). A region shorter than the sampling
    interval falls back to the sample nearest its middle (and says so)."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.path = index, None, None
        self.t0 = self.t1 = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-f", self.path], stdout=subprocess.DEVNULL,
                                         stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        import datetime
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10 or not f[1].isdigit() or int(f[1]) != self.index:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(f[2]), float(f[3]), float(f[4]), f[6:10]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        t0 = self.t0 if self.t0 is not None else rows[0][0]
        t1 = self.t1 if self.t1 is not None else rows[-1][0]
        inside = [r for r in rows if t0 - 0.1 <= r[0] <= t1 + 0.1]
        nearest = not inside
        if nearest:
            mid = 0.5 * (t0 + t1)
            inside = [min(rows, key=lambda r: abs(r[0] - mid))]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[4]) if v.lower().startswith("active")})
        load = [r for r in inside if r[3] > 300.0] or inside
        out = {"sm_mhz": statistics.median(r[1] for r in load), "sm_max_mhz": max(r[2] for r in rows),
               "reasons": reasons, "samples": len(inside), "samples_under_load": len([r for r in inside if r[3] > 300.0]),
               "power_w_max": max(r[3] for r in inside), "gpu_index": self.index,
               "timed_region_s": round(t1 - t0, 4), "sampling_ms": 50}
        if nearest:
            out["nearest_sample"] = True
        return out


def algo_bytes(cls: str, s, B: int, act: int) -> float:
    """Algorithmic HBM bytes of one step's launches of a kernel class: every layer read / written once, edge arrays
    (int32 source + fp32 weight) and row pointers once."""
    n, K = s["sizes"], s["hops"]
    E = s.edges()
    rows = sum(n[1:])
    if cls == "hop_fwd":
        return act * B * sum(n[k] + n[k + 1] for k in range(K)) + 8 * E + 4 * rows
    if cls == "plug_fwd":
        return (s["obs_dim"] * 4 + n[0] * act) * B
    if cls == "out_fwd":
        return (n[K] * act + s["n_act"] * 4) * B
    return 0.0


def train_bytes(plan, s, B: int, flat_len: int, redrive: bool) -> dict:
    """Algorithmic HBM bytes of one fp32 training step per kernel class, counting only what the step's plan visits:
    the forward touches every row (each layer written once and read once, every edge record once); the backward only
    the rows whose gradient can be non-zero (live rows), their merged pairs and the edge weights of those pairs; Adam
    reads P, G, M, V, EMA and writes P, M, V, EMA over the flat parameter buffer."""
    n, K = s["sizes"], s["hops"]
    hops = plan["hops"]
    E = sum(h["edges"] for h in hops)
    chunks = (B + 255) // 256                           # the backward's 256-sample chunks
    out = {
        "plug_fwd": (s["obs_dim"] + n[0] * (2 if redrive else 1)) * 4 * B,
        "hop_fwd": 4 * B * sum(n[k] + n[k + 1] for k in range(K)) + 8 * E + 4 * sum(n[1:]),
        "out_fwd": (plan["n_dn"] + 2 * s["n_act"]) * 4 * B,
        "loss": 3 * s["n_act"] * 4 * B,
        "out_bwd": (s["n_act"] + 2 * plan["n_dn"]) * 4 * B,
        "act_bwd": 3 * 4 * B * hops[-1]["live_dst"],
        # the weight gradient's last step (k_sd_reduce): each live pair's per-chunk partials, its forward pair and edge
        # range, and each of its edges' weight-gradient word read and written
        "wgrad": sum(4 * h["live_pairs_"] * chunks + 12 * h["live_pairs_"] + 12 * h["live_edges"] for h in hops),
        # transposed product with the weight-gradient products fused in: read gz of the live rows and the live source
        # rows' states (the products and the fused neuron backward), write the layer below's live rows (gz, or gh0
        # below the first hop), read the pair records, write the per-chunk weight-gradient partials
        "hop_bwd_t": sum(4 * B * (h["live_dst"] + 2 * h["live_src"]) + 8 * h["tpairs"] + 4 * h["tpairs"] * chunks
                         for h in hops),
        "plug_bwd": 4 * B * (3 * plan["plug_live"] + s["obs_dim"]),
        "adam": 36 * flat_len,
    }
    return {k: float(v) for k, v in out.items()}


def with_live_pairs(plan):
    """plan['hops'][k]['live_pairs_']: merged pairs of the live rows (the transposed pairs kept are exactly those)."""
    for h in plan["hops"]:
        h["live_pairs_"] = h["tpairs"]
    return plan


# ------------------------------------------------------------------ our arm
MODEL_DIR = Path(os.environ.get("FLYGUY_MODEL_DIR", REPO / "tests" / "golden" / "_model"))


def make_graph(W, sources="zipf"):
    from flyguy_b200 import netfile, synth
    if W.get("graph") == "model":
        net, params = MODEL_DIR / "model.net.bin", MODEL_DIR / "model.params.bin"
        if not (net.exists() and params.exists()):
            raise SystemExit(f"{net} / {params} are missing: tests/golden/make_golden.py writes them from the "
                             "reference's bot/model.pt")
        s = netfile.read_net(net)
        return s, netfile.read_params(params, s)[1]
    if W.get("graph") == "full":
        return synth.make_full_graph()
    if W.get("graph") == "h4":
        return synth.make_synthetic4(uniform=sources == "uniform")
    return synth.make_synthetic(uniform=sources == "uniform")


def run_ours(a, W, rank, world, dev, torch, dist, graph=None):
    from flyguy_b200 import native, synth
    s, P = graph or make_graph(W, a.sources)
    Bg = (a.batch or W["batch"]) * (world if W["per_gpu"] else 1)
    B = Bg // world
    assert B % 32 == 0 and B * world == Bg, "the batch must split into multiples of 32"
    flags = {"bf16": native.FG_ACT_BF16, "f16": native.FG_ACT_F16, "fp32": native.FG_INFER_ONLY,
             "train": 0}[W["flags"]]
    piece = min(B, PIECE) if W.get("graph") == "full" else B
    h = native.Handle(s, piece, flags, device=dev)
    h.set_params(P, 0)
    h.set_params(P, 1)
    obs_np, teacher_np = synth.make_batch(B, seed=1000 + rank)
    obs = torch.from_numpy(obs_np).to(dev)
    teacher = torch.from_numpy(teacher_np).to(dev)
    logits = torch.empty(B, s["n_act"], device=dev)
    flush = torch.empty(64 * 2 ** 20, dtype=torch.float32, device=dev)      # 256 MiB > 126 MB L2
    train = W["flags"] == "train"
    grad = h.flat(4) if train else None
    # data-parallel mean: where the gradient's structural zeros are at least half of it (a graph whose backward
    # reaches few rows), one all-reduce of the packed gradient after the backward; otherwise the library's gradient
    # buckets, each started as soon as the backward finishes it (one piece a step); --no-overlap: one all-reduce of
    # the whole flat gradient after the backward
    from flyguy_b200.dist import BucketedMean, PackedMean
    packed = bucketed = None
    if train and world > 1 and not a.no_overlap:
        packed = PackedMean(h)
        if not packed.worth_it():
            packed = None
            bucketed = BucketedMean(h) if piece == B else None

    def mean_grad():
        if world == 1:
            return
        if packed:
            packed()
        elif bucketed:
            bucketed.finish()
        else:
            dist.all_reduce(grad, op=dist.ReduceOp.AVG)

    def step():
        if train:
            h.zero_grad()
            for lo in range(0, B, piece):
                h.teach(obs[lo:lo + piece], teacher[lo:lo + piece], 1.0, logits=None, stats=False, loss_norm=B)
            if bucketed:
                bucketed.start()
            mean_grad()
            h.step(LR, 0.3 * LR, LR, 0.0, 0.999)
        else:
            h.forward(obs, 0, out=logits)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with Clocks(int(os.environ.get("LOCAL_RANK", dev.index or 0))) as clk:
        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize(dev)
        # ---- timed region (device time, per-step CUDA events; L2 flushed between steps outside the events)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        h.timing(True, classes=[ROOF_CLASS])        # events around the roofline kernel's launches only
        launches0 = h.launches()
        barrier()
        torch.cuda.synchronize(dev)
        clk.mark_start()
        for e0, e1 in evs:
            flush.zero_()
            e0.record()
            step()
            e1.record()
        torch.cuda.synchronize(dev)
        clk.mark_end()
        barrier()
    launches = h.launches() - launches0
    kern = h.timing_read()
    h.timing(False)
    # per-class breakdown: a separate pass of a few steps with every class timed (not part of the timed region)
    h.timing(True)
    n_bd = min(a.steps, 5)
    for _ in range(n_bd):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    bd = h.timing_read()
    h.timing(False)
    t_dev = sum(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3
    t_max = max_over_ranks(t_dev)
    value = Bg * a.steps / t_max
    clocks = clk.summary()
    # ---- roofline of the dominant kernel class
    kern_step = {k: (ms / a.steps, n // a.steps) for k, (ms, n) in kern.items() if n}
    bd_step = {k: (ms / n_bd, n // n_bd) for k, (ms, n) in bd.items() if n}
    dom = ROOF_CLASS
    act = 2 if W["flags"] in ("bf16", "f16") else 4
    byts = algo_bytes(dom, s, B, act)
    peak, peak_src = peaks()
    achieved = byts / (kern_step[dom][0] / 1e3) / 1e9 if byts else None
    roof = {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1) if achieved else None, "peak": peak,
            "unit": "GB/s", "frac": round(achieved / peak, 4) if achieved else None, "traffic": traffic_of(dom, W, B, a.sources),
            "algorithmic_bytes_per_step": byts, "launches_per_step": kern_step[dom][1],
            "ms_per_step": round(kern_step[dom][0], 4), "peak_source": peak_src,
            "largest_class_in_breakdown": max(bd_step, key=lambda k: bd_step[k][0])}
    # whole-step view. Inference: the path's algorithmic bytes per decision (each layer written and read once, edge
    # arrays once per launch) x rate. Training: the bytes the step's plan really moves (train_bytes: the backward over
    # live rows only), per kernel class against that class's measured time, and summed against the step time.
    N_rows, E = sum(s["sizes"]), s.edges()
    if train:
        plan = with_live_pairs(h.plan())
        redrive = any((np.asarray(hh["drow"]) >= 0).any() for hh in s["hop"])
        tb = train_bytes(plan, s, B, int(grad.numel()), bool(redrive))
        ms_step = t_max / a.steps * 1e3
        step_roof = {"bytes_per_step": round(sum(tb.values())), "bytes_per_unit": round(sum(tb.values()) / B, 1),
                     "achieved_gbs_per_gpu": round(sum(tb.values()) / (ms_step / 1e3) / 1e9, 1),
                     "frac": round(sum(tb.values()) / (ms_step / 1e3) / 1e9 / peak, 4),
                     "kernels": {k: {"ms": round(bd_step[k][0], 4), "bytes": round(v),
                                     "frac": round(v / (bd_step[k][0] / 1e3) / 1e9 / peak, 4)}
                                 for k, v in tb.items() if k in bd_step and bd_step[k][0] > 0},
                     "live_rows": [hh["live_dst"] for hh in plan["hops"]],
                     "rows": [hh["rows"] for hh in plan["hops"]],
                     "live_pairs": [hh["tpairs"] for hh in plan["hops"]],
                     "pairs": [hh["pairs"] for hh in plan["hops"]],
                     "how": "algorithmic bytes of what the plan visits (forward: all rows; backward: live rows, their "
                            "pairs and edge weights; Adam over the flat buffer) / measured time; per-kernel times "
                            "from the breakdown pass"}
    else:
        per_unit = 2 * act * N_rows + s["obs_dim"] * 4 + s["n_act"] * 4 + (8 * E + 4 * sum(s["sizes"][1:])) / B
        step_roof = {"bytes_per_unit": round(per_unit, 1),
                     "achieved_gbs_per_gpu": round(per_unit * value / world / 1e9, 1),
                     "frac": round(per_unit * value / world / 1e9 / peak, 4)}
    # ---- argmax agreement of the 16-bit path (rank 0): the last step's logits on samples spread over the batch,
    # against the oracle's emulation of the same 16-bit format (the kernel's error) and its fp32 forward (the
    # format's error)
    agreement = None
    if rank == 0 and W["flags"] in ("bf16", "f16") and not a.no_check:
        agreement = argmax_agreement(s, P, obs_np, logits.cpu().numpy(), W["flags"])
    # ---- e2e through the host-buffer entry points
    e2e = None if a.no_e2e else run_e2e(a, W, h, s, obs_np, teacher_np, B, Bg, world, dev, torch, dist, barrier,
                                          max_over_ranks, grad, piece, bucketed, packed)
    # ---- CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(W, s, P, a.cpu_seconds)
    out = {"metric": W["metric"], "value": round(value, 1), "unit": W["unit"], "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": round(t_max / a.steps * 1e3, 4), "higher_is_better": True,
           "scaling": "weak" if W["per_gpu"] else "strong", "vs_baseline": None, "dtype": W["dtype"],
           "data": (f"the reference's bot/model.pt network and weights ({'/'.join(f'{v:,}' for v in s['sizes'])} "
                    f"neurons, {s['n_w']:,} weights, {E:,} edge-steps, sensory re-drive); synthetic obs ~ N(0,1), "
                    "teacher ~ N(0,4)" if W.get("graph") == "model" else
                    "synthetic: seeded untrimmed graph (166,700 neurons, 15,283,167 edges, lognormal in-degree mean 92, "
                    "Zipf(1.5) sources), obs ~ N(0,1), teacher ~ N(0,4)" if W.get("graph") == "full" else
                    f"synthetic: seeded {len(s['sizes']) - 1}-hop graph "
                    f"({'/'.join(f'{v:,}' for v in s['sizes'])} neurons, {s['n_w']:,} edges, lognormal "
                    f"in-degree mean 35, {'Zipf(1.5)' if a.sources == 'zipf' else 'uniform'} sources), obs ~ N(0,1), "
                    "teacher ~ N(0,4)"),
           "config": {"workload": W["desc"], "baseline_config": W["cfg"], "global_batch": Bg, "per_gpu_batch": B,
                      "parallelism": ((f"dp{world}, one all-reduce of the packed gradient ({packed.n:,} of "
                                       f"{packed.flat_len:,} floats: its structural zeros left out)" if packed else
                                       f"dp{world}, gradient all-reduce in {len(bucketed.early)} early + "
                                       f"{len(bucketed.late)} late buckets overlapping the backward" if bucketed else
                                       "dp1 (one GPU: no all-reduce)" if world == 1 else
                                       f"dp{world}, one gradient all-reduce per step") if train
                                      else f"batch-sharded x{world}, no collective"),
                      "l2": "flushed between timed steps (256 MiB write, outside the step events)",
                      "graph": ("bot/model.pt (trimmed male-CNS 3-hop graph)" if W.get("graph") == "model"
                                else "synthetic untrimmed 166,700-neuron graph" if W.get("graph") == "full"
                                else f"synthetic flyguy-sized {len(s['sizes']) - 1}-hop, {a.sources} sources"),
                      "edges": s["n_w"],
                      "edge_steps": E,
                      "pieces_per_step": (B + piece - 1) // piece,
                      "hop_kernel": "CUDA cores"},
           "roofline": roof, "step_roofline": step_roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
           **({"argmax_agreement": agreement} if agreement else {}),
           "gpu_launches": int(launches),
           "kernels_ms_per_step": {k: round(v[0], 4) for k, v in bd_step.items()},
           "kernels_breakdown": f"separate pass of {n_bd} steps after the timed region, every class timed"}
    return out


def argmax_agreement(s, P, obs_np, got, fmt: str, n: int = 2048) -> dict:
    """Argmax agreement of the GPU's 16-bit-state logits on n samples spread over the batch with the oracle's
    emulation of that format and with its fp32 forward (the reference's arithmetic)."""
    from oracle.oracle import Oracle
    idx = np.unique(np.linspace(0, len(obs_np) - 1, n).astype(np.int64))
    o = Oracle(s, threads=os.cpu_count() or 1)
    emu = o.forward(P, obs_np[idx], states=fmt + "+obs")
    ref = o.forward(P, obs_np[idx])
    g = got[idx]
    rel = lambda x, y: float(np.abs(x - y).max() / max(np.abs(y).max(), 1e-30))  # noqa: E731
    return {"samples": int(len(idx)), "vs_emulation": float(np.mean(g.argmax(1) == emu.argmax(1))),
            "vs_fp32_reference": float(np.mean(g.argmax(1) == ref.argmax(1))),
            "emulation_vs_fp32_reference": float(np.mean(emu.argmax(1) == ref.argmax(1))),
            "rel_vs_emulation": rel(g, emu), "rel_vs_fp32_reference": rel(g, ref),
            "how": f"oracle/fly_oracle.c: {fmt} emulation (states rounded where the kernels store them) and fp32 "
                   "forward, on samples spread over the last timed step's batch"}


def traffic_of(cls: str, W, B: int, sources: str = "zipf") -> float | None:
    """Per-step DRAM bytes of the kernel class from the committed ncu summary (profiles/traffic.json), if any, scaled
    from the capture's per-GPU batch to B in proportion to the samples."""
    p = REPO / "profiles" / "traffic.json"
    if not p.exists() or W.get("graph"):
        return None
    d = json.loads(p.read_text()).get(W["flags"] + ("" if sources == "zipf" else "/" + sources), {})
    v = d.get(cls)
    return round(float(v) * B / d["batch"]) if v is not None else None


def run_e2e(a, W, h, s, obs_np, teacher_np, B, Bg, world, dev, torch, dist, barrier, max_over_ranks, grad, piece,
            bucketed=None, packed=None):
    train = W["flags"] == "train"
    obs_h = torch.from_numpy(obs_np).pin_memory()
    out_h = torch.empty(B, s["n_act"]).pin_memory()
    if train:
        # a training loop's input pipeline: step i's obs and teacher cross PCIe on a copy stream while step i - 1
        # computes (two device buffers); the first step's copy is not hidden, and every copy is inside the timed loop
        teach_h = torch.from_numpy(teacher_np).pin_memory()
        obs_d = [torch.empty_like(obs_h, device=dev) for _ in range(2)]
        teach_d = [torch.empty_like(teach_h, device=dev) for _ in range(2)]
        cs = torch.cuda.Stream(device=dev)
        ready = [torch.cuda.Event() for _ in range(2)]
        main = torch.cuda.current_stream(dev)

        def upload(i):
            # (the buffer's last reader, step i - 2, has finished: every step ends with the host waiting for it)
            with torch.cuda.stream(cs):
                obs_d[i % 2].copy_(obs_h, non_blocking=True)
                teach_d[i % 2].copy_(teach_h, non_blocking=True)
                ready[i % 2].record(cs)

        def step(i, last):
            if not last:
                upload(i + 1)
            main.wait_event(ready[i % 2])
            od, td = obs_d[i % 2], teach_d[i % 2]
            h.zero_grad()
            st = None
            for lo in range(0, B, piece):
                st = h.teach(od[lo:lo + piece], td[lo:lo + piece], 1.0, logits=None, stats=world == 1,
                             loss_norm=B)
            if world > 1:
                if packed:
                    packed()
                elif bucketed:
                    bucketed.start()
                    bucketed.finish()
                else:
                    dist.all_reduce(grad, op=dist.ReduceOp.AVG)
                h.step(LR, 0.3 * LR, LR, 0.0, 0.999)
                h.sync()                             # the loss sums come back after the step
            else:
                h.step(LR, 0.3 * LR, LR, 0.0, 0.999)
                h.sync()
            return st
        h2d, d2h = (obs_np.nbytes + teacher_np.nbytes), 16
    else:
        def upload(i):
            pass

        def step(i, last):
            h.forward_host(obs_h, out_h)
        h2d, d2h = obs_np.nbytes, out_h.numel() * 4
    upload(0)
    for i in range(2):
        step(i, i == 1)
    torch.cuda.synchronize(dev)
    barrier()
    t0 = time.perf_counter()
    upload(0)
    for i in range(a.steps):
        step(i, i + 1 == a.steps)
    t = time.perf_counter() - t0
    barrier()
    t = max_over_ranks(t)
    return {"value": round(Bg * a.steps / t, 1), "unit": W["unit"], "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h),
            "path": ("obs/teacher H2D (pinned; the next step's on a copy stream during this step) + fg_teach + "
                     "fc_step + D2H loss" if train
                     else "fg_forward_host (pinned host obs -> host logits; pieces growing from 1/32 of the batch, each upload hidden behind the previous piece's forward)")}


# ------------------------------------------------------------------ CPU baseline / reference arm
def _ref_forward(s, P, threads):
    from oracle.oracle import REF_LIB, Oracle, RefInfer
    if REF_LIB.exists():
        return RefInfer(s, P, threads=threads), "reference", "flyguy/native/fly_infer.cpp (oracle/_ref, g++ -O3 " \
            "-march=x86-64-v3 -ffast-math), one handle per thread"
    o = Oracle(s, threads=threads)
    return type("O", (), {"forward": lambda self, x: o.forward(P, x), "close": lambda self: None})(), "port", \
        "oracle/fly_oracle.c forward (OpenMP)"


def cpu_baseline(W, s, P, budget: float):
    """The reference's CPU path timed on this host's cores on a bounded sample sized to ~`budget` seconds."""
    return _cpu_baseline(W, s, P, budget)


def _cpu_baseline(W, s, P, budget: float):
    """The reference's CPU path timed on this host's cores on a bounded sample sized to ~`budget` seconds."""
    from flyguy_b200 import synth
    threads = os.cpu_count() or 1
    if W["flags"] == "train":
        return _cpu_train(s, P, threads, budget, steps=1)
    r, kind, what = _ref_forward(s, P, threads)
    obs, _ = synth.make_batch(threads * 8, seed=7)
    t0 = time.perf_counter()
    r.forward(obs)
    dt = time.perf_counter() - t0
    n = int(max(threads, min(200_000, budget / max(dt, 1e-6) * len(obs))))
    obs, _ = synth.make_batch(n, seed=8)
    t0 = time.perf_counter()
    r.forward(obs)
    dt = time.perf_counter() - t0
    r.close()
    return {"value": round(n / dt, 1), "unit": W["unit"], "cores": threads, "kind": kind,
            "sample": f"{n} decisions of the same workload (synthetic graph, obs ~ N(0,1)) in {dt:.1f} s; {what}",
            "cpu": _cpu_model()}


def _cpu_train(s, P, threads, budget, steps):
    """The oracle's C port of the training step: forward + KL loss + backward on a sample, then Adam over every
    weight (the reference trains on the CPU through torch, which is not available on the GPU box)."""
    from flyguy_b200 import synth
    from oracle.oracle import Oracle, adam, loss
    o = Oracle(s, threads=threads)
    M = [np.zeros_like(p) for p in P]
    V = [np.zeros_like(p) for p in P]
    E = [p.copy() for p in P]
    Q = [p.copy() for p in P]

    def one(n, seed):
        obs, teacher = synth.make_batch(n, seed=seed)
        lg = o.forward(Q, obs)
        _, _, dl = loss(lg, teacher, 1.0)
        G = o.backward(Q, obs, dl)
        adam(Q, G, M, V, E, 1, LR, 0.3 * LR, LR)
    n = threads * 2
    t0 = time.perf_counter()
    one(n, 7)
    dt = time.perf_counter() - t0
    n = int(max(threads, min(16384, budget / max(dt, 1e-6) * n / steps)))
    n = max(32, n // 32 * 32)
    t0 = time.perf_counter()
    for i in range(steps):
        one(n, 9 + i)
    dt = time.perf_counter() - t0
    return {"value": round(n * steps / dt, 1), "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{steps} training step(s) of {n} samples (forward, KL loss, backward, Adam over all "
                      f"{sum(len(p) for p in P):,} weights) in {dt:.1f} s; oracle/fly_oracle.c (OpenMP, double sums)",
            "cpu": _cpu_model()}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(a, W):
    """The reference's CPU implementation of the path, W warm-up + K timed steps of a bounded sample each."""
    from flyguy_b200 import synth
    s, P = make_graph(W, a.sources)
    threads = os.cpu_count() or 1
    Bg = W["batch"]
    if W["flags"] == "train":
        cb = _cpu_train(s, P, threads, budget=max(2.0, 90.0 / (a.steps + a.warmup)), steps=1)
        n = int(cb["sample"].split(" samples")[0].split()[-1])
        from oracle.oracle import Oracle, adam, loss
        o = Oracle(s, threads=threads)
        M, V, E, Q = [np.zeros_like(p) for p in P], [np.zeros_like(p) for p in P], [p.copy() for p in P], \
            [p.copy() for p in P]

        def step(i):
            obs, teacher = synth.make_batch(n, seed=100 + i)
            lg = o.forward(Q, obs)
            _, _, dl = loss(lg, teacher, 1.0)
            adam(Q, o.backward(Q, obs, dl), M, V, E, i + 1, LR, 0.3 * LR, LR)
        kind, what = "port", "oracle/fly_oracle.c training step (OpenMP)"
        r = None
    else:
        r, kind, what = _ref_forward(s, P, threads)
        obs0, _ = synth.make_batch(threads * 8, seed=5)
        t0 = time.perf_counter()
        r.forward(obs0)
        per = (time.perf_counter() - t0) / len(obs0)
        n = int(max(threads, min(Bg, max(2.0, 90.0 / (a.steps + a.warmup)) / per)))
        obs, _ = synth.make_batch(n, seed=6)

        def step(i):
            r.forward(obs)
    for i in range(a.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(a.steps):
        step(a.warmup + i)
    dt = time.perf_counter() - t0
    if r is not None:
        r.close()
    value = n * a.steps / dt
    return {"impl": "reference", "metric": W["metric"], "value": round(value, 1), "unit": W["unit"],
            "n_gpus": 0, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt / a.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak" if W["per_gpu"] else "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (same graph and obs distribution as our arm)",
            "config": {"workload": W["desc"], "baseline_config": W["cfg"], "global_batch": Bg,
                       "sample_per_step": n, "parallelism": f"{threads} host threads"},
            "cpu_baseline": {"value": round(value, 1), "unit": W["unit"], "cores": threads, "kind": kind,
                             "sample": f"{n} units per step; {what}", "cpu": _cpu_model()},
            "e2e": {"value": round(value, 1), "unit": W["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def _play_calls(fwd, obs_pool, n):
    """n calls of fwd on the pool's observation batches in turn; seconds per call (host wall clock)."""
    t0 = time.perf_counter()
    for i in range(n):
        fwd(obs_pool[i % len(obs_pool)])
    return (time.perf_counter() - t0) / n


def run_play(a, W, reference: bool):
    """The playing path: fly_forward for 8 cars per call, host buffers in and out, timed per call on the host clock
    (a decision is latency); K steps of CALLS calls after W warm-up steps. Ours: the GPU library; the reference: its
    CPU library (oracle/_ref/libfly_infer.so, one thread, as the bot calls it)."""
    import ctypes
    from flyguy_b200 import synth
    from flyguy_b200.play import Player
    s, P = make_graph(W, a.sources)
    ref = REPO / "oracle" / "_ref" / "libfly_infer.so"
    pool = [synth.make_batch(W["batch"], seed=700 + i)[0] for i in range(16)]
    CALLS = 50 if reference else 200                   # (the CPU library takes milliseconds a call)
    players = {}
    if not reference:
        players["gpu"] = Player(s, P)
    if ref.exists() and (reference or not a.no_cpu_baseline):
        players["cpu"] = Player(s, P, lib=ctypes.CDLL(str(ref)))
    key = "cpu" if reference else "gpu"
    if key not in players:
        return {"impl": "reference" if reference else "ours", "unavailable": f"{ref} is not built"}
    fwd = lambda o, p=players[key]: p.forward(o, tap=True)
    _play_calls(fwd, pool, CALLS * a.warmup)
    clk = None
    if reference:
        per = [_play_calls(fwd, pool, CALLS) for _ in range(a.steps)]
    else:
        import torch
        with Clocks(torch.cuda.current_device()) as clk:
            clk.mark_start()
            per = [_play_calls(fwd, pool, CALLS) for _ in range(a.steps)]
            clk.mark_end()
    dt = sum(per) / len(per)
    value = W["batch"] / dt
    out = {"metric": W["metric"], "value": round(value, 1), "unit": W["unit"], "n_gpus": 0 if reference else 1,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt * CALLS * 1e3, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": ("the reference's bot/model.pt network and weights, obs ~ N(0,1)" if W.get("graph") == "model"
                    else "synthetic: the config-2 graph, obs ~ N(0,1)"),
           "config": {"workload": W["desc"], "baseline_config": W["cfg"], "cars_per_call": W["batch"],
                      "calls_per_step": CALLS, "timing": "host wall clock per fly_forward call",
                      "latency_ms_per_call": round(dt * 1e3, 4)},
           "roofline": None,
           "e2e": {"value": round(value, 1), "unit": W["unit"], "h2d_bytes_per_step": CALLS * W["batch"] * s["obs_dim"] * 4,
                   "d2h_bytes_per_step": CALLS * (W["batch"] * s["n_act"] * 4 + int(sum(s["sizes"])))}}
    if reference:
        out.update(impl="reference", cpu_baseline={"value": round(value, 1), "unit": W["unit"], "cores": 1,
                                                   "kind": "reference", "sample": f"{CALLS} calls per step; "
                                                   "flyguy/native/fly_infer.cpp fly_forward", "cpu": _cpu_model()})
    else:
        cpu = None
        if "cpu" in players:
            dc = _play_calls(lambda o, p=players["cpu"]: p.forward(o, tap=True), pool, 50)
            cpu = {"value": round(W["batch"] / dc, 1), "unit": W["unit"], "cores": 1, "kind": "reference",
                   "sample": f"50 calls of 8 cars, {dc * 1e3:.3f} ms per call; flyguy/native/fly_infer.cpp "
                             "fly_forward (oracle/_ref), one thread", "cpu": _cpu_model()}
        out.update(cpu_baseline=cpu, clocks=clk.summary(), gpu_launches=int((len(s["hop"]) + 2) * CALLS * a.steps))
    return out


def main():
    a = args_()
    W = WORKLOADS[a.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if W["flags"] == "play":                    # one process plays; under torchrun the other ranks have nothing to do
        if rank == 0:
            print(json.dumps(run_play(a, W, a.impl == "reference")), flush=True)
        return
    if a.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(a, W)), flush=True)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", torch.cuda.current_device())
    try:
        graph = make_graph(W, a.sources)
        out = run_ours(a, W, rank, world, dev, torch, dist, graph)
        if a.workload == "infer" and not a.no_train and not a.batch:
            # config 3 at the same N on the same graph: the training half of BASELINE's metric
            torch.cuda.empty_cache()
            tr = run_ours(a, WORKLOADS["train"], rank, world, dev, torch, dist, graph)
            out["train"] = {k: tr[k] for k in ("metric", "value", "unit", "ms_per_step", "scaling", "dtype", "config",
                                               "roofline", "step_roofline", "e2e", "cpu_baseline", "clocks",
                                               "gpu_launches", "kernels_ms_per_step") if k in tr}
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
