"""Teach a fly network to choose what another network chooses - flyguy/teach.py with its hop path on B200.

  python -m flyguy_b200.teach --data MOMENTS.bin [MORE.bin ...] --teacher TEACHER.pt [--start fresh | CKPT.pt]
        [--graph GRAPH.npz] [--hops 3] [--steps 3000] [--batch 128] [--lr 4e-4] [--temp 0.5] [--average 0.999]
        [--holdout 0.05] [--eval-every 250] [--out runs/teach/student.pt] [--seed 0] [--graph-root DIR]

Same recipe as the reference (flyguy/teach.py:69-170): the loss is KL(softmax(teacher / temp) || softmax(student)),
Adam with the strengths and the plugs at lr and gain / threshold at 0.3 lr, the rate falling to a tenth by the last
step, a running average of the weights (young averages follow closely: keep = min(average, step / (step + 9))) that is
scored on the held-out end of every data file and saved. The difference is where it runs: the student's forward, the
loss, the backward pass, Adam and the running average are one fused library step on the GPU per batch (fg_teach +
fc_step), and the teacher is a fly network run by the same library (fp32 states).

DATA: "FLYD" files (observations as 16-bit floats) or "FLYR" recordings of the bot (flyguy/teach.py:53-66).
With several GPUs (torchrun), each rank takes its own batches and the gradient is averaged before every step.
"""
from __future__ import annotations

import argparse
import struct
import time
from pathlib import Path

import numpy as np
import torch

from . import dist
from .model import build_actor, load_actor, save_actor


def moments(path: Path) -> np.ndarray:
    """[n, obs size] float16 observations of a FLYD file or a FLYR recording."""
    with open(path, "rb") as fh:
        kind = fh.read(4)
        if kind == b"FLYD":
            n, od, _ = struct.unpack("<qii", fh.read(16))
            return np.memmap(path, np.float16, "r", 20, (n, od))
        if kind == b"FLYR":
            od, extra = struct.unpack("<ii", fh.read(8))
            rec = 8 + extra + 2 * od
            n = (path.stat().st_size - 12) // rec
            raw = np.memmap(path, np.uint8, "r", 12, (n, rec))
            return np.ascontiguousarray(raw[:, 8 + extra:]).view(np.float16)
    raise SystemExit(f"{path}: neither a FLYD file nor a recording of the bot")


def write_moments(path: Path, obs: np.ndarray) -> None:
    """A FLYD file of observations (no teacher answers: answer size 0)."""
    obs = np.ascontiguousarray(obs, np.float16)
    with open(path, "wb") as fh:
        fh.write(b"FLYD" + struct.pack("<qii", obs.shape[0], obs.shape[1], 0))
        fh.write(obs.tobytes())


class Teacher:
    """A fly network's logits for a batch (fp32 states, no gradients)."""

    def __init__(self, path: Path, device, graph_root=None):
        _, self.actor = load_actor(path, native=False, device=device, graph_root=graph_root)
        self.actor.requires_grad_(False)

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.actor(x).float()


def train(args) -> dict:
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(args.seed)
    rank = torch.distributed.get_rank() if dist.on() else 0
    rng = np.random.default_rng(args.seed + 1000 * rank)
    teacher = Teacher(args.teacher, dev, args.graph_root)
    tck = torch.load(args.teacher, map_location="cpu", weights_only=False)
    if args.start == "fresh":
        cfg = dict(tck["config"]["model"])
        cfg.update(fly_graph=args.graph or cfg.get("fly_graph"), fly_hops=args.hops or cfg.get("fly_hops", 3),
                   fly_batch=max(args.batch, 32))
        student, step0 = build_actor(cfg, graph_root=args.graph_root), 0
    else:
        sck, student = load_actor(args.start, native=True, device="cpu", graph_root=args.graph_root)
        cfg, step0 = dict(sck["config"]["model"], fly_batch=max(args.batch, 32)), int(sck.get("taught_steps", 0))
        student.max_batch = max(args.batch, 32)
    student = student.to(dev)
    opt = student.native_adam(args.lr)
    h = student.engine().training_handle()
    seen, unseen = [], []
    for p in args.data:
        m = moments(p)
        cut = len(m) - max(1, int(len(m) * args.holdout))
        seen.append(m[:cut])
        unseen.append(m[cut:])
    seen = torch.from_numpy(np.concatenate(seen).astype(np.float32))
    un = np.concatenate(unseen)
    unseen = torch.from_numpy(un[:: max(1, len(un) // 4096)].astype(np.float32))
    inv_t = 1.0 / args.temp
    B = (args.batch + 31) // 32 * 32

    @torch.no_grad()
    def score() -> tuple[float, float]:
        same = kl = 0.0
        for i in range(0, len(unseen), 512):
            x = unseen[i:i + 512].to(dev)
            t = teacher(x)
            s = student.engine().run_average(x)
            same += float((t.argmax(-1) == s.argmax(-1)).sum())
            target = torch.softmax(t * inv_t, -1)
            kl += float((target * (torch.log(target.clamp_min(1e-12)) - torch.log_softmax(s, -1))).sum())
        return same / len(unseen), kl / len(unseen)

    a0, k0 = score()
    if rank == 0:
        print(student.describe(), flush=True)
        print(f"start | unseen: same first choice {a0:.3f}, distance {k0:.3f} | {len(seen):,} moments to learn from",
              flush=True)
    t0, run, a, k = time.time(), 0.0, a0, k0
    for step in range(1, args.steps + 1):
        lr = args.lr * 0.1 ** (step / args.steps)
        idx = np.sort(rng.integers(0, len(seen), B))
        x = seen[torch.as_tensor(idx)].to(dev, non_blocking=True)
        t = teacher(x)
        h.zero_grad()
        kl_sum, _ = h.teach(x.contiguous(), t.contiguous(), inv_t)
        if dist.on():
            dist.mean_([h.flat(4)])
        keep = min(args.average, step / (step + 9.0))
        h.step(lr, 0.3 * lr, lr, 0.0, keep)
        run = kl_sum / B if step == 1 else 0.98 * run + 0.02 * kl_sum / B
        if step % args.eval_every == 0 or step == args.steps:
            a, k = score()
            if rank == 0:
                print(f"step {step:,} | distance {run:.3f} | unseen: same first choice {a:.3f}, distance {k:.3f} | "
                      f"{step * B * (torch.distributed.get_world_size() if dist.on() else 1) / (time.time() - t0):,.0f}"
                      f" moments a second", flush=True)
                student.pull()
                avg = student.engine().average_state()
                save_actor(args.out, avg, dict(cfg, fly_kernel="torch"), step0 + step,
                           taught_by=Path(args.teacher).name, unseen_same_first_choice=a)
    return {"agree0": a0, "kl0": k0, "agree": a, "kl": k, "distance": run}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--data", nargs="+", type=Path, required=True)
    ap.add_argument("--teacher", type=Path, required=True)
    ap.add_argument("--start", default="fresh")
    ap.add_argument("--graph", default="")
    ap.add_argument("--graph-root", default=None)
    ap.add_argument("--hops", type=int, default=0)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--lr", type=float, default=4e-4)
    ap.add_argument("--temp", type=float, default=0.5)
    ap.add_argument("--average", type=float, default=0.999)
    ap.add_argument("--holdout", type=float, default=0.05)
    ap.add_argument("--eval-every", type=int, default=250)
    ap.add_argument("--out", type=Path, default=Path("runs/teach/student.pt"))
    ap.add_argument("--seed", type=int, default=0)
    train(ap.parse_args())


if __name__ == "__main__":
    main()
