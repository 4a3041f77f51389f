"""FlyActor: flyguy's fly-wired actor, with its hop path on the B200 library.

Same constructor, buffers, parameters and state-dict keys as the reference's FlyActor (flyguy/fly.py:75-154), so a
reference checkpoint (bot/model.pt, keys actor.w / gain / theta / in_w / in_b / out.weight / out.bias) loads
unchanged. The forward pass runs in libflyguy_b200.so for CUDA tensors - with autograd: the backward pass also runs
in the library and lands in the parameters' .grad like the reference's torch path (flyguy/fly.py:286-305). There is
no CPU compute path here: CPU tensors raise (the reference's CPU play path, fly_infer.cpp, stays the reference's).

The structure comes from flyguy_b200.wiring (the layers, each hop's connections in CSR order by destination and by
source); this class lays it out under the reference's buffer names (e{k}, r{k}, c{k}, crow{k}, tcrow{k}, tcol{k},
tperm{k}, ci{k}, tci{k}, n{k}, s{k}, d{k}, n0, dn_rows, in_*), which the NET.bin writer reads.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

from .wiring import by_key, row_starts, wire

ROOT = Path(__file__).resolve().parents[1]
INHIBITORY = ("gaba", "glutamate", "histamine")     # transmitters whose connections start with a negative strength


def plug_columns(n_s: int, obs_dim: int, fan: int, seed: int) -> np.ndarray:
    """The observation indices each sensory row listens to: per row, in row order, one draw of `fan` distinct indices
    from numpy default_rng(seed), sorted - the reference's draws (flyguy/fly.py:141-143), so a checkpoint's in_w meets
    the same observation values."""
    rng = np.random.default_rng(seed)
    return np.concatenate([np.sort(rng.choice(obs_dim, size=fan, replace=False)) for _ in range(n_s)]
                          or [np.zeros(0, np.int64)]).astype(np.int64)


def starting_strengths(g, total: np.ndarray) -> np.ndarray:
    """1.5 x synapse count / the target's incoming synapse count, negative for inhibitory transmitters (the
    reference's starting point, flyguy/fly.py:134-137)."""
    pre, post = g["pre"].astype(np.int64), g["post"].astype(np.int64)
    neg = np.isin(g["nt"], INHIBITORY)[pre]
    return (np.where(neg, -1.5, 1.5).astype(np.float32) * g["syn"].astype(np.float32)
            / np.maximum(total[post], 1.0)).astype(np.float32)


class FlyActor(nn.Module):
    memory = 0

    def __init__(self, graph: str | Path, obs_dim: int, n_actions: int, hops: int = 3, fan: int = 16,
                 out_gain: float = 0.01, seed: int = 0):
        super().__init__()
        p = Path(graph)
        g = np.load(p if p.is_absolute() or p.exists() else ROOT / p)
        n = len(g["body"])
        pre, post = g["pre"].astype(np.int64), g["post"].astype(np.int64)
        self.n_neurons, self.n_conn, self.hops, self.obs_dim, self.fan = n, len(pre), hops, obs_dim, fan
        self.whole_graph = "in_total" not in g.files
        self.gather_limit = 60_000_000           # kept for API compatibility (the reference's torch-path switch)
        self.kernel = "b200"                     # every kernel name of the reference maps to the B200 library; for
        #                                          forward without gradients "cuda16" selects fp16 states (as the
        #                                          reference's cuda16 kernels) and "bf16" bf16 states
        wiring = wire(pre, post, g["sensory"], g["descending"], n, hops)
        if not len(wiring.dn_rows):
            raise ValueError(f"{p.name}: none of the descending neurons is {hops} synapses or fewer from a sensory "
                             "neuron along the wiring")
        self.sizes = wiring.sizes
        for k, hw in enumerate(wiring.hop, start=1):
            tcol = hw.rows[hw.tperm]
            for name, a in (("e", hw.edges), ("r", hw.rows), ("c", hw.cols), ("crow", hw.row_ptr),
                            ("tcrow", hw.tcol_ptr), ("tcol", tcol), ("tperm", hw.tperm),
                            ("ci", hw.cols.astype(np.int32)), ("tci", tcol.astype(np.int32)), ("n", hw.neurons),
                            ("s", hw.sensory_rows), ("d", hw.drive_rows)):
                self._buf(f"{name}{k}", a)
        self.used = int(sum(len(hw.edges) for hw in wiring.hop))
        self.in_play = int(wiring.kept(self.n_conn).sum())
        self._buf("n0", wiring.layers[0])
        self._buf("dn_rows", wiring.dn_rows)
        # weights: a strength per connection (normalised by the target's incoming synapses in the WHOLE graph, which
        # a trimmed file carries as in_total), a gain and a threshold parameter per neuron
        if self.whole_graph:
            total = np.bincount(post, weights=g["syn"].astype(np.float64), minlength=n).astype(np.float32)
        else:
            if hops > int(g["hops"]):
                raise ValueError(f"{p.name} keeps only the connections of a {int(g['hops'])}-hop network")
            total = g["in_total"].astype(np.float32)
        self.w = nn.Parameter(torch.as_tensor(starting_strengths(g, total)))
        self.gain = nn.Parameter(torch.ones(n))
        self.theta = nn.Parameter(torch.full((n,), -4.0))
        # input plug: sensory row i hears `fan` observation values; output plug: descending rows -> action logits
        n_s = self.sizes[0]
        cols = plug_columns(n_s, obs_dim, fan, seed)
        rows = np.repeat(np.arange(n_s, dtype=np.int64), fan)
        t = by_key(cols, rows, n_s)
        for name, a in (("in_r", rows), ("in_c", cols), ("in_crow", row_starts(rows, n_s)),
                        ("in_tcrow", row_starts(cols[t], obs_dim)), ("in_tcol", rows[t]), ("in_tperm", t),
                        ("in_ci", cols.astype(np.int32)), ("in_tci", rows[t].astype(np.int32))):
            self._buf(name, a)
        # (the order of the random draws below is the reference's, so a seeded run starts from the same numbers)
        self.in_w = nn.Parameter(torch.randn(n_s * fan) / fan ** 0.5)
        self.in_b = nn.Parameter(torch.zeros(n_s))
        self.out = nn.Linear(len(wiring.dn_rows), n_actions)
        nn.init.orthogonal_(self.out.weight, out_gain)
        nn.init.zeros_(self.out.bias)
        self._engine = None

    def _buf(self, name: str, a: np.ndarray) -> None:
        self.register_buffer(name, torch.as_tensor(np.ascontiguousarray(a)), persistent=False)

    def describe(self) -> str:
        plug = self.in_w.numel() + self.in_b.numel() + sum(q.numel() for q in self.out.parameters())
        return (f"{self.hops}-hop fly network over a {self.n_neurons:,}-neuron, {self.n_conn:,}-connection graph: "
                f"layers {self.sizes}, {self.in_play:,} connections used ({self.used:,} connection steps per "
                f"decision); plugs: {self.fan} observation values per sensory neuron in, {len(self.dn_rows):,} "
                f"descending neurons out ({plug:,} weights)")

    def __deepcopy__(self, memo):
        """Copies share no library handle (two Python objects must not drive one network in the library)."""
        import copy
        cls = self.__class__
        new = cls.__new__(cls)
        memo[id(self)] = new
        for k, v in self.__dict__.items():
            new.__dict__[k] = None if k == "_engine" else copy.deepcopy(v, memo)
        return new

    # ---- the library
    def engine(self):
        from .engine import Engine
        if self._engine is None or self._engine.device != self.gain.device:
            self._engine = Engine(self)
        return self._engine

    def forward(self, obs: torch.Tensor, extra: torch.Tensor | None = None) -> torch.Tensor:
        if not obs.is_cuda:
            raise RuntimeError("flyguy_b200 runs the hop path on the GPU: move the actor and the observations to "
                               "CUDA (the CPU play path is the reference's fly_infer)")
        obs = obs.float()
        eng = self.engine()
        if torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()):
            return eng.logits_autograd(obs)
        return eng.infer(obs, states={"cuda16": "f16", "bf16": "bf16"}.get(self.kernel, "f32"))
