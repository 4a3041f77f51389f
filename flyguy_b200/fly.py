"""FlyActor: flyguy's fly-wired actor, with its hop path on the B200 library.

Same constructor, buffers, parameters and state-dict keys as the reference's FlyActor (flyguy/fly.py:75-154), so a
reference checkpoint (bot/model.pt, keys actor.w / gain / theta / in_w / in_b / out.weight / out.bias) loads
unchanged. The forward pass runs in libflyguy_b200.so for CUDA tensors - with autograd: the backward pass also runs
in the library and lands in the parameters' .grad like the reference's torch path (flyguy/fly.py:286-305). There is
no CPU compute path here: CPU tensors raise (the reference's CPU play path, fly_infer.cpp, stays the reference's).

Structure (flyguy/fly.py:91-126): the neurons that matter after hop k are those within k synapses downstream of a
sensory neuron AND within hops-k synapses upstream of a descending neuron; hop k keeps the connections from the
layer-(k-1) set into the layer-k set, in CSR order by destination (sources ascending) and by source. The input plug
draws, per sensory neuron in play, `fan` distinct observation indices from numpy default_rng(seed) - the same draws
in the same order as the reference, so that a checkpoint's in_w meets the same observation values.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

ROOT = Path(__file__).resolve().parents[1]
INHIBITORY = ("gaba", "glutamate", "histamine")


def reachable(start: np.ndarray, src: np.ndarray, dst: np.ndarray, n: int, steps: int) -> list[np.ndarray]:
    """masks[k][i]: neuron i is in `start` or reachable from it in at most k steps along src -> dst."""
    mask = np.zeros(n, bool)
    mask[start] = True
    masks = [mask]
    for _ in range(steps):
        nxt = masks[-1].copy()
        nxt[dst[masks[-1][src]]] = True
        masks.append(nxt)
    return masks


def row_pointer(rows: np.ndarray, n_rows: int) -> np.ndarray:
    counts = np.bincount(rows, minlength=n_rows)
    out = np.zeros(n_rows + 1, np.int64)
    np.cumsum(counts, out=out[1:])
    return out


def plug_columns(n_s: int, obs_dim: int, fan: int, seed: int) -> np.ndarray:
    """fan distinct observation indices per sensory row, sorted within the row (flyguy/fly.py:141-143: one
    rng.choice(obs_dim, fan, replace=False) per row from default_rng(seed), in row order)."""
    rng = np.random.default_rng(seed)
    out = np.empty((n_s, fan), np.int64)
    for i in range(n_s):
        out[i] = np.sort(rng.choice(obs_dim, size=fan, replace=False))
    return out.reshape(-1)


class FlyActor(nn.Module):
    memory = 0

    def __init__(self, graph: str | Path, obs_dim: int, n_actions: int, hops: int = 3, fan: int = 16,
                 out_gain: float = 0.01, seed: int = 0):
        super().__init__()
        p = Path(graph)
        g = np.load(p if p.is_absolute() or p.exists() else ROOT / p)
        n = len(g["body"])
        pre, post = g["pre"].astype(np.int64), g["post"].astype(np.int64)
        syn = g["syn"].astype(np.float32)
        sens, dn = g["sensory"].astype(np.int64), g["descending"].astype(np.int64)
        self.n_neurons, self.n_conn, self.hops, self.obs_dim, self.fan = n, len(pre), hops, obs_dim, fan
        self.whole_graph = "in_total" not in g.files
        self.gather_limit = 60_000_000           # kept for API compatibility (the reference's torch-path switch)
        self.kernel = "b200"                     # every kernel name of the reference maps to the B200 library; for
        #                                          forward without gradients "cuda16" selects fp16 states (as the
        #                                          reference's cuda16 kernels) and "bf16" bf16 states
        down = reachable(sens, pre, post, n, hops)
        up = reachable(dn, post, pre, n, hops)
        layers = [np.flatnonzero(down[k] & up[hops - k]) for k in range(hops + 1)]
        self.sizes = [len(s) for s in layers]
        where = []
        for s in layers:
            w = np.full(n, -1, np.int64)
            w[s] = np.arange(len(s))
            where.append(w)
        sensory = np.zeros(n, bool)
        sensory[sens] = True
        self.used = 0
        in_play = np.zeros(len(pre), bool)
        for k in range(1, hops + 1):
            m = np.flatnonzero((where[k - 1][pre] >= 0) & (where[k][post] >= 0))
            r, c = where[k][post[m]], where[k - 1][pre[m]]
            by_dst = np.lexsort((c, r))
            m, r, c = m[by_dst], r[by_dst], c[by_dst]
            by_src = np.lexsort((r, c))
            ids = layers[k]
            self._buf(f"e{k}", m); self._buf(f"r{k}", r); self._buf(f"c{k}", c)
            self._buf(f"crow{k}", row_pointer(r, len(ids))); self._buf(f"tcrow{k}", row_pointer(c[by_src], len(layers[k - 1])))
            self._buf(f"tcol{k}", r[by_src]); self._buf(f"tperm{k}", by_src)
            self._buf(f"ci{k}", c.astype(np.int32)); self._buf(f"tci{k}", r[by_src].astype(np.int32))
            self._buf(f"n{k}", ids)
            self._buf(f"s{k}", np.flatnonzero(sensory[ids]))
            self._buf(f"d{k}", where[0][ids[sensory[ids]]])
            self.used += len(m)
            in_play[m] = True
        self.in_play = int(in_play.sum())
        self._buf("n0", layers[0])
        reach_dn = where[hops][dn] >= 0
        assert reach_dn.any(), "no descending neuron can be reached in this many hops"
        self._buf("dn_rows", where[hops][dn[reach_dn]])
        if "in_total" in g.files:
            assert hops <= int(g["hops"]), f"this graph file holds the connections of a {int(g['hops'])}-hop network only"
            total = g["in_total"].astype(np.float32)
        else:
            total = np.zeros(n, np.float32)
            np.add.at(total, post, syn)
        sign = np.where(np.isin(g["nt"][pre], INHIBITORY), -1.0, 1.0).astype(np.float32)
        self.w = nn.Parameter(torch.as_tensor(1.5 * sign * syn / np.maximum(total[post], 1.0)))
        self.gain = nn.Parameter(torch.ones(n))
        self.theta = nn.Parameter(torch.full((n,), -4.0))
        n_s = self.sizes[0]
        cols = plug_columns(n_s, obs_dim, fan, seed)
        rows = np.repeat(np.arange(n_s), fan)
        t = np.lexsort((rows, cols))
        self._buf("in_r", rows); self._buf("in_c", cols); self._buf("in_crow", row_pointer(rows, n_s))
        self._buf("in_tcrow", row_pointer(cols[t], obs_dim)); self._buf("in_tcol", rows[t]); self._buf("in_tperm", t)
        self._buf("in_ci", cols.astype(np.int32)); self._buf("in_tci", rows[t].astype(np.int32))
        self.in_w = nn.Parameter(torch.randn(n_s * fan) / fan ** 0.5)
        self.in_b = nn.Parameter(torch.zeros(n_s))
        self.out = nn.Linear(len(self.dn_rows), n_actions)
        nn.init.orthogonal_(self.out.weight, out_gain)
        nn.init.zeros_(self.out.bias)
        self._engine = None

    def _buf(self, name: str, a: np.ndarray) -> None:
        self.register_buffer(name, torch.as_tensor(np.ascontiguousarray(a)), persistent=False)

    def describe(self) -> str:
        plug = self.in_w.numel() + self.in_b.numel() + sum(p.numel() for p in self.out.parameters())
        return (f"fly actor: {self.n_neurons:,} neurons and {self.n_conn:,} connections in the graph; {self.hops} hops: "
                f"{self.in_play:,} connections and {sum(self.sizes):,} neuron states in play (per hop {self.sizes}), "
                f"{self.used:,} connection steps a decision; learned outside the fly: {plug:,} numbers (each sensory "
                f"neuron hears {self.fan} observation values; {len(self.dn_rows):,} descending neurons -> actions)")

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
