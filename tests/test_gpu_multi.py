"""Data-parallel training on two GPUs over NCCL (skipped with fewer than two GPUs): each rank runs the fused teaching
step on its half of the batch, the library's flat gradient is averaged in place by flyguy_b200.dist, and the
result equals one process's gradient of the whole batch (the reference's DP hook, flyguy/fly_native.py:78-81)."""
import os
import socket
from pathlib import Path

import numpy as np
import pytest

from conftest import load_case, rel

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out, mode="one"):
    import torch
    import torch.distributed as td
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                          device_id=torch.device("cuda", rank))
    try:
        from flyguy_b200 import dist, native
        s, P, d = load_case("syn_small")
        B = len(d["obs"]) // world
        h = native.Handle(s, B, device=torch.device("cuda", rank))
        h.set_params(P)
        obs = torch.as_tensor(d["obs"][rank * B:(rank + 1) * B]).cuda()
        teacher = torch.as_tensor(d["teacher"][rank * B:(rank + 1) * B]).cuda()
        mean = dist.BucketedMean(h) if mode == "bucketed" else dist.PackedMean(h) if mode == "packed" else None
        h.zero_grad()
        h.teach(obs, teacher, float(d["inv_temp"]))
        assert dist.on()
        if mode == "bucketed":                         # buckets started as the backward finishes them
            mean.start()
            mean.finish()
        elif mode == "packed":                         # one all-reduce of the gradient without its structural zeros
            mean()
        else:
            dist.mean_([h.flat(4)])
        G = [g.cpu().numpy() for g in h.get(4)]
        np.savez(Path(out) / f"r{rank}.npz", *G)
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("mode", ["one", "bucketed", "packed"])
def test_two_gpu_gradient_mean_equals_full_batch(tmp_path, cuda, mode):
    """One all-reduce after the backward, the library's buckets each started on a side stream when the backward
    reaches its stage, or one all-reduce of the packed gradient: each way the averaged gradient is the whole batch's."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), mode), nprocs=2, start_method="spawn")
    # one process, the whole batch: the mean over ranks of per-half gradients (each scaled by 1/half) equals the
    # gradient of the whole batch (scaled by 1/B)
    from flyguy_b200 import native
    s, P, d = load_case("syn_small")
    h = native.Handle(s, len(d["obs"]))
    h.set_params(P)
    h.zero_grad()
    h.teach(torch.as_tensor(d["obs"]).cuda(), torch.as_tensor(d["teacher"]).cuda(), float(d["inv_temp"]))
    want = [g.cpu().numpy() for g in h.get(4)]
    for r in range(2):
        got = np.load(tmp_path / f"r{r}.npz")
        for i in range(7):
            assert rel(got[f"arr_{i}"], want[i]) < 1e-4, (r, i)


def test_gradient_buckets_cover_the_flat_gradient_and_their_events_fire(cuda):
    """fg_grad_buckets: the ranges cover [0, flat length) once; on the synthetic graph (hops on disjoint strength
    ranges) the output plug and every hop's strengths are early buckets, on a graph whose hops share strengths only the
    output plug is; every stage event of a step has completed once the step has."""
    import torch
    from flyguy_b200 import native, synth
    for s, want_early in ((synth.make_synthetic(sizes=(300, 700, 500, 60), total_edges=30_000, seed=3)[0], 4),
                          (load_case("toy_h3")[0], None)):
        P = [np.zeros(n, np.float32) for n in s.param_sizes()]
        h = native.Handle(s, 64)
        h.set_params(P)
        buckets = sorted(h.grad_buckets())
        n = h.flat(4).numel()
        at = 0
        for lo, hi, st in buckets:
            assert lo == at and hi > lo, buckets
            at = hi
        assert at == n
        early = [b for b in buckets if b[2] >= 0]
        if want_early is not None:
            assert len(early) == want_early and {b[2] for b in early} == {0, 1, 2, 3}
        else:
            assert 0 in {b[2] for b in early}
        evs = {st: torch.cuda.Event() for st in {b[2] for b in early}}
        for st, ev in evs.items():
            h.set_stage_event(st, ev)
        obs = torch.randn(64, s["obs_dim"], device="cuda")
        h.zero_grad()
        h.teach(obs, torch.randn(64, s["n_act"], device="cuda"), 1.0)
        torch.cuda.synchronize()
        assert all(ev.query() for ev in evs.values())
        with pytest.raises(native.FlyguyError):
            h.set_stage_event(99, evs[0])


def test_packed_gradient_leaves_out_only_zeros(cuda):
    """fg_grad_pack: after a teaching step, packing the gradient, zeroing it and unpacking gives the same gradient bit
    for bit - the strengths left out of the packed set had an exactly zero gradient; on a Zipf-source graph (most rows
    unread, so the backward reaches few) the packed gradient is a fraction of the flat one."""
    import torch
    from flyguy_b200 import native, synth
    for s, smaller in ((synth.make_synthetic(sizes=(300, 700, 500, 60), total_edges=30_000, seed=3)[0], True),
                       (load_case("toy_h3")[0], False)):
        P = [np.random.default_rng(1).normal(size=n).astype(np.float32) * 0.1 for n in s.param_sizes()]
        h = native.Handle(s, 64)
        h.set_params(P)
        obs = torch.randn(64, s["obs_dim"], device="cuda")
        h.zero_grad()
        h.teach(obs, torch.randn(64, s["n_act"], device="cuda"), 1.0)
        flat = h.flat(4)
        want = flat.clone()
        n = h.grad_pack()
        if smaller:                                    # (about 54% here: 10,928 of 30,000 strengths + the rest)
            assert n < 0.6 * flat.numel(), (n, flat.numel())
        buf = torch.full((n,), float("nan"), device="cuda")
        assert h.grad_pack(buf) == n
        h.zero_grad()
        h.grad_pack(buf, unpack=True)
        torch.cuda.synchronize()
        assert torch.equal(flat, want)
        with pytest.raises(native.FlyguyError):
            h.grad_pack(torch.empty(max(n - 1, 1), device="cuda"))

