"""Several GPUs: one process per GPU, every optimiser step on the mean gradient of all of them.

The reference leaves this as a stub (flyguy/dist.py:8-13: on() is False, mean_ has no body). Here it is
torch.distributed: on() is true in an initialised process group of more than one rank, and mean_ averages tensors in
place across the ranks with one all-reduce per tensor (NCCL over NVLink on GPUs, gloo on CPU). NativeAdam passes the
library's flat gradient buffer itself (one contiguous ~3.5M-float array), so a step costs exactly one all-reduce.
"""
from __future__ import annotations

import torch
import torch.distributed as td


def on() -> bool:
    return td.is_available() and td.is_initialized() and td.get_world_size() > 1


def mean_(tensors) -> None:
    """In place: every tensor becomes the mean of that tensor over all ranks."""
    if not on():
        return
    world = td.get_world_size()
    avg = td.get_backend() == "nccl"
    for t in tensors:
        if avg:
            td.all_reduce(t, op=td.ReduceOp.AVG)
        else:                                             # gloo has no AVG
            td.all_reduce(t, op=td.ReduceOp.SUM)
            t.div_(world)
