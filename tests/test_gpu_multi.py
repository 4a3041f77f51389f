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


def _rank(rank, world, port, out):
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
        h.zero_grad()
        h.teach(obs, teacher, float(d["inv_temp"]))
        assert dist.on()
        dist.mean_([h.flat(4)])
        G = [g.cpu().numpy() for g in h.get(4)]
        np.savez(Path(out) / f"r{rank}.npz", *G)
    finally:
        td.destroy_process_group()


def test_two_gpu_gradient_mean_equals_full_batch(tmp_path, cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
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
