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


class BucketedMean:
    """The mean of a handle's flat gradient over all ranks, taken in the library's buckets (fg_grad_buckets) so that
    most of it crosses NVLink while the backward is still running: a bucket whose values are final early (the output
    plug's arrays, each hop's strengths when no later hop shares them) is all-reduced on a side stream as soon as the
    backward records its stage event; the rest after the backward returns. The result is the same in-place average as
    mean_([flat]) (the same reduction on the same values, per range).

        mean = BucketedMean(handle)          # once: buckets, events, the side stream
        handle.teach(...)                    # enqueues the step; its backward records the stage events
        mean.start()                         # early buckets wait on their events on the side stream
        mean.finish()                        # the remaining buckets; the current stream waits for all of them
    """

    def __init__(self, handle):
        self.h = handle
        self.grad = handle.flat(4)
        self.stream = torch.cuda.Stream(device=handle.device)
        hops = len(handle.layout()[1])
        self.events = {}
        for _, _, st in handle.grad_buckets():
            if st >= 0 and st not in self.events:
                ev = torch.cuda.Event()
                handle.set_stage_event(st, ev)
                self.events[st] = ev
        buckets = handle.grad_buckets()
        # the backward reaches stage 0 (output plug) first, then hops+..., 1 (the hops top down)
        self.early = sorted([b for b in buckets if b[2] >= 0], key=lambda b: 0 if b[2] == 0 else hops + 1 - b[2])
        self.late = [b for b in buckets if b[2] < 0]
        self.works = []

    def _reduce(self, lo, hi):
        t = self.grad[lo:hi]
        if td.get_backend() == "nccl":
            return td.all_reduce(t, op=td.ReduceOp.AVG, async_op=True)
        w = td.all_reduce(t, op=td.ReduceOp.SUM, async_op=True)
        w.wait()
        t.div_(td.get_world_size())
        return None

    def start(self) -> None:
        self.works = []
        if not on():
            return
        with torch.cuda.stream(self.stream):
            for lo, hi, st in self.early:
                self.stream.wait_event(self.events[st])
                self.works.append(self._reduce(lo, hi))

    def finish(self) -> None:
        if not on():
            return
        main = torch.cuda.current_stream(self.grad.device)
        with torch.cuda.stream(self.stream):
            self.stream.wait_stream(main)
            for lo, hi, _ in self.late:
                self.works.append(self._reduce(lo, hi))
        for w in self.works:
            if w is not None:
                w.wait()                                 # the current (main) stream waits for the NCCL work
        main.wait_stream(self.stream)
        self.works = []


class PackedMean:
    """The mean of a handle's gradient over all ranks, all-reduced without its structural zeros (fg_grad_pack): on a
    graph whose backward reaches few rows (the benchmark's Zipf graph: 170,679 of 2,992,734 strengths can get a
    gradient) the packed gradient is a fraction of the flat one, so one small all-reduce after the backward replaces
    the full 14 MB one. The strengths left out are exactly zero on every rank, so the result is the same average.

        mean = PackedMean(handle)            # once: the packed buffer
        handle.teach(...)
        mean()                               # pack, all-reduce (average), unpack - on the current stream
    """

    def __init__(self, handle):
        self.h = handle
        self.n = handle.grad_pack()
        self.flat_len = handle.flat(4).numel()
        self.buf = torch.empty(max(self.n, 1), dtype=torch.float32, device=handle.device)

    def worth_it(self) -> bool:
        """The packed gradient is at most half the flat one."""
        return 2 * self.n <= self.flat_len

    def __call__(self) -> None:
        if not on():
            return
        self.h.grad_pack(self.buf, unpack=False)
        b = self.buf[:self.n]
        if td.get_backend() == "nccl":
            td.all_reduce(b, op=td.ReduceOp.AVG)
        else:
            td.all_reduce(b, op=td.ReduceOp.SUM)
            b.div_(td.get_world_size())
        self.h.grad_pack(self.buf, unpack=True)

