"""Binds a FlyActor's torch parameters to library handles on the actor's CUDA device.

The weights live in torch (the checkpoint's tensors); before a forward they are pushed into the library when any of
them changed (torch's per-tensor version counters, as flyguy/fly.py:192-196 does for its compiled path). Batches are
split into pieces of at most `max_batch` and padded to a multiple of 32 by repeating the last observation
(flyguy/fly_native.py:198-213); with gradients, a backward over several pieces runs each piece's forward again
(flyguy/fly_native.py:46-58).
"""
from __future__ import annotations

import torch

from . import native
from .netfile import structure_of_actor

MAX_INFER_BATCH = 65536


def _pad32(x: torch.Tensor) -> torch.Tensor:
    pad = (-x.shape[0]) % 32
    return x if not pad else torch.cat([x, x[-1:].expand(pad, -1)])


class Engine:
    def __init__(self, actor):
        self.actor = actor
        self.device = actor.gain.device
        self.s = structure_of_actor(actor)
        self.wmap = torch.as_tensor(self.s["wmap"], device=self.device)
        self.max_batch = int(getattr(actor, "max_batch", 2048))
        self.train = None                      # fp32 handle with gradient and optimiser state
        self.infer_h = {}                      # (half,) -> forward-only handle
        self._ver = {}
        self.gen = 0                           # bumped by every training-handle forward (states overwritten)
        self.hook = torch.zeros(1, device=self.device, requires_grad=True)   # makes autograd call _Logits.backward

    # ---- weights
    def tensors(self):
        a = self.actor
        return [a.w.detach()[self.wmap].contiguous(), a.gain.detach(), a.theta.detach(), a.in_w.detach(),
                a.in_b.detach(), a.out.weight.detach().reshape(-1), a.out.bias.detach()]

    def _version(self):
        a = self.actor
        return tuple(p._version for p in (a.w, a.gain, a.theta, a.in_w, a.in_b, a.out.weight, a.out.bias)) + \
            tuple(p.data_ptr() for p in (a.w, a.gain))

    def push(self, h, also_average: bool = False) -> None:
        ts = [t.float().contiguous() for t in self.tensors()]
        h.copy(0, 1, ts)
        if also_average:
            h.copy(1, 1, ts)
        self._ver[id(h)] = self._version()

    def _fresh(self, h, also_average=False) -> None:
        if self._ver.get(id(h)) != self._version():
            self.push(h, also_average)

    def training_handle(self):
        if self.train is None:
            with torch.cuda.device(self.device):
                self.train = native.Handle(self.s, self.max_batch, 0, device=self.device)
            self.push(self.train, also_average=True)
        self._fresh(self.train)
        return self.train

    # ---- forward without gradients
    def infer(self, obs: torch.Tensor, states: str = "f32") -> torch.Tensor:
        """Forward without gradients; states "f32", "f16" (the reference's 16-bit "cuda16" states) or "bf16"."""
        B = obs.shape[0]
        if states == "f32" and self.train is not None and B <= self.max_batch:
            return self._piece(self.training_handle(), obs)
        cap = min(MAX_INFER_BATCH, max(32, (B + 31) // 32 * 32))
        h = self.infer_h.get(states)
        if h is None or h.max_batch < cap:
            if h is not None:
                h.close()
            flags = {"f32": native.FG_INFER_ONLY, "f16": native.FG_ACT_F16, "bf16": native.FG_ACT_BF16}[states]
            with torch.cuda.device(self.device):
                h = native.Handle(self.s, cap, flags, device=self.device)
            self.infer_h[states] = h
            self._ver.pop(id(h), None)
        self._fresh(h)
        return torch.cat([self._piece(h, obs[i:i + h.max_batch]) for i in range(0, B, h.max_batch)]) \
            if B > h.max_batch else self._piece(h, obs)

    def _piece(self, h, obs: torch.Tensor) -> torch.Tensor:
        b = obs.shape[0]
        x = _pad32(obs.float()).contiguous()
        out = h.forward(x, 0)
        if h is self.train:
            self.gen += 1
        return out[:b]

    # ---- forward / backward with gradients
    def run(self, obs: torch.Tensor) -> torch.Tensor:
        h = self.training_handle()
        mb = h.max_batch
        if obs.shape[0] <= mb:
            return self._piece(h, obs)
        return torch.cat([self._piece(h, obs[i:i + mb]) for i in range(0, obs.shape[0], mb)])

    def backward_into_library(self, obs: torch.Tensor, g: torch.Tensor, gen: int) -> None:
        """dlogits g of the batch obs: the weights' gradients are ADDED to the library's gradient."""
        h = self.training_handle()
        n, mb = obs.shape[0], h.max_batch
        for i in range(0, n, mb):
            if not (n <= mb and self.gen == gen):           # several pieces, or something ran in between
                self._piece(h, obs[i:i + mb])
            gi = g[i:i + mb].float()
            pad = (-gi.shape[0]) % 32
            if pad:
                gi = torch.cat([gi, gi.new_zeros(pad, gi.shape[1])])
            h.backward(gi.contiguous())

    def logits_autograd(self, obs: torch.Tensor, to_torch: bool = True) -> torch.Tensor:
        """Logits with a backward through the library: to_torch - gradients into the parameters' .grad (FlyActor);
        else they accumulate in the library's gradient (NativeFlyActor + NativeAdam)."""
        return _Logits.apply(obs, self.hook, self, to_torch)

    def run_average(self, obs: torch.Tensor) -> torch.Tensor:
        """Forward with the library's running average of the weights (fc_forward with ema 1), no gradients."""
        h = self.training_handle()
        outs = []
        for i in range(0, obs.shape[0], h.max_batch):
            x = obs[i:i + h.max_batch]
            b = x.shape[0]
            outs.append(h.forward(_pad32(x.float()).contiguous(), 1)[:b])
            self.gen += 1
        return torch.cat(outs) if len(outs) > 1 else outs[0]

    def average_state(self):
        """A copy of the actor (no library handle) holding the library's running average of the weights."""
        import copy
        a = copy.deepcopy(self.actor)
        E = self.train.get(1)
        with torch.no_grad():
            a.w[self.wmap.to(a.w.device)] = E[0].to(a.w.device)
            for p, v in ((a.gain, E[1]), (a.theta, E[2]), (a.in_w, E[3]), (a.in_b, E[4]), (a.out.weight, E[5]),
                         (a.out.bias, E[6])):
                p.copy_(v.view_as(p))
        return a

    def pull(self) -> None:
        """The library's weights -> the torch parameters (after a library optimiser step)."""
        a = self.actor
        P = self.train.get(0)
        with torch.no_grad():
            a.w[self.wmap] = P[0]
            for p, v in ((a.gain, P[1]), (a.theta, P[2]), (a.in_w, P[3]), (a.in_b, P[4]), (a.out.weight, P[5]),
                         (a.out.bias, P[6])):
                p.copy_(v.view_as(p))
        self._ver[id(self.train)] = self._version()

    def grads_to_torch(self) -> None:
        """The library's gradient ADDED into the parameters' .grad (W scattered through the in-play map)."""
        a = self.actor
        G = self.train.get(4)
        gw = torch.zeros_like(a.w)
        gw[self.wmap] = G[0]
        for p, g in ((a.w, gw), (a.gain, G[1]), (a.theta, G[2]), (a.in_w, G[3]), (a.in_b, G[4]),
                     (a.out.weight, G[5].view_as(a.out.weight)), (a.out.bias, G[6])):
            if p.requires_grad:
                p.grad = g.clone() if p.grad is None else p.grad + g


class _Logits(torch.autograd.Function):
    """Logits of the library's forward; backward through the library, gradients into the torch parameters."""

    @staticmethod
    def forward(ctx, obs, hook, eng, to_torch):
        ctx.eng, ctx.obs, ctx.to_torch = eng, obs, to_torch
        out = eng.run(obs)
        ctx.gen = eng.gen
        return out

    @staticmethod
    def backward(ctx, g):
        eng = ctx.eng
        h = eng.training_handle()
        if ctx.to_torch:
            h.zero_grad()
        eng.backward_into_library(ctx.obs, g, ctx.gen)
        if ctx.to_torch:
            eng.grads_to_torch()
            h.zero_grad()
        return None, None, None, None

