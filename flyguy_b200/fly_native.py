"""NativeFlyActor and NativeAdam: the reference's library-backed actor and optimiser (flyguy/fly_native.py), on the
B200 library.

NativeFlyActor IS a FlyActor (same weights and checkpoint keys). Forward with gradients hands the backward pass to the
library, which ADDS the weights' gradients to its own gradient buffer (flyguy/fly_native.py:37-58); `native_adam()`
returns the optimiser that zeroes that buffer, averages it over the data-parallel ranks (dist.mean_ on the library's
flat gradient, in place - no copies), takes the Adam step in the library (strengths at lr, gain / theta at
lr * lr_neuron, plugs at lr * lr_plug, optional clipping, running average of the weights) and copies the new weights
back into the torch parameters (flyguy/fly_native.py:61-103).
"""
from __future__ import annotations

import numpy as np
import torch

from . import dist
from .fly import FlyActor


class NativeAdam:
    """The actor's optimiser as a trainer sees it; the work is done by the library."""

    def __init__(self, actor: "NativeFlyActor", lr: float, max_norm: float = 0.0, ema: float = 0.999):
        self.actor, self.max_norm, self.ema = actor, max_norm, ema
        self.param_groups = [{"lr": lr}]
        self.grad_norm = 0.0

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.actor.engine().training_handle().zero_grad()

    def step(self) -> None:
        a = self.actor
        h = a.engine().training_handle()
        if dist.on():                                      # several GPUs: the mean of every rank's gradient
            dist.mean_([h.flat(4)])
        lr = float(self.param_groups[0]["lr"])
        self.grad_norm = h.step(lr, lr * a.lr_neuron, lr * a.lr_plug, float(self.max_norm), float(self.ema))
        a.pull()

    def state_dict(self) -> dict:
        h = self.actor.engine().training_handle()
        out = {"native": True, "adam_t": h.adam_t()}
        for name, which in (("ema", 1), ("m", 2), ("v", 3)):
            out[name] = [t.cpu() for t in h.get(which)]
        return out

    def load_state_dict(self, d: dict) -> None:
        if not d.get("native") or "m" not in d:           # (a torch Adam's state: the library starts its own)
            return
        h = self.actor.engine().training_handle()
        dev = self.actor.gain.device
        for name, which in (("ema", 1), ("m", 2), ("v", 3)):
            h.copy(which, 1, [t.to(dev).float().contiguous() for t in d[name]])
        h.adam_t(int(d.get("adam_t", 0)))


class NativeFlyActor(FlyActor):
    lr_neuron, lr_plug = 0.3, 1.0       # rates of gain / threshold and of the plugs, as shares of the strengths'

    def __init__(self, *args, max_batch: int = 2048, **kw):
        super().__init__(*args, **kw)
        self.max_batch = int(max_batch)

    def native_adam(self, lr: float, max_norm: float = 0.0) -> NativeAdam | None:
        if not self.gain.is_cuda:
            return None
        self.engine().training_handle()
        return NativeAdam(self, lr, max_norm)

    # ---- weights between torch and the library (flyguy/fly_native.py:169-188)
    def push(self, also_average: bool = False) -> None:
        eng = self.engine()
        eng.push(eng.training_handle(), also_average)

    def pull(self) -> None:
        self.engine().pull()

    def _fetch(self, which: int) -> list[torch.Tensor]:
        return self.engine().training_handle().get(which)

    def _store(self, which: int, tensors: list[torch.Tensor]) -> None:
        self.engine().training_handle().copy(which, 1, [t.contiguous().float() for t in tensors])

    def forward(self, obs: torch.Tensor, extra: torch.Tensor | None = None) -> torch.Tensor:
        if not obs.is_cuda:
            return super().forward(obs, extra)            # raises: no CPU path
        obs = obs.float()
        eng = self.engine()
        if torch.is_grad_enabled():
            return eng.logits_autograd(obs, to_torch=False)
        return eng.run(obs)


def grad_arrays(actor: NativeFlyActor) -> list[np.ndarray]:
    """The gradient the library gathered since zero_grad (flyguy/fly_native.py:224-226)."""
    return [t.cpu().numpy() for t in actor._fetch(4)]
