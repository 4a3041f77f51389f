"""The fly actor of a flyguy model config / checkpoint (the fly branch of flyguy/model.py:225-232 and build_model
285-292): `fly_graph`, `fly_hops`, `fly_fan`, `fly_kernel`, `fly_batch`. Checkpoints are flyguy's torch dicts
{"model": {"actor.w", "actor.gain", "actor.theta", "actor.in_w", "actor.in_b", "actor.out.weight",
"actor.out.bias", ... critic ...}, "steps", "config": {"model": cfg}}; only the actor's keys are read (the critic and
the dense/attention actors are not part of the hop path).
"""
from __future__ import annotations

from pathlib import Path

import torch

from .fly import FlyActor
from .fly_native import NativeFlyActor

OBS_DIM = 517        # flyguy's observation with ball prediction and opponents' inputs (flyguy/obs.py:34-40)
N_ACTIONS = 90       # flyguy's action table (flyguy/actions.py)


def build_actor(cfg: dict, obs_dim: int = OBS_DIM, n_actions: int = N_ACTIONS, native: bool = True,
                graph_root: str | Path | None = None):
    """The actor of a model config: NativeFlyActor (library optimiser) or FlyActor (torch optimisers)."""
    if not cfg.get("fly_graph"):
        raise ValueError("not a fly model config (no fly_graph)")
    graph = Path(cfg["fly_graph"])
    if graph_root is not None and not graph.is_absolute():
        graph = Path(graph_root) / graph
    kw = dict(hops=int(cfg.get("fly_hops", 3)), fan=int(cfg.get("fly_fan", 16)))
    if native:
        a = NativeFlyActor(graph, obs_dim, n_actions, max_batch=int(cfg.get("fly_batch", 2048)), **kw)
    else:
        a = FlyActor(graph, obs_dim, n_actions, **kw)
    kern = cfg.get("fly_kernel", "torch")
    a.kernel = kern if kern in ("cuda16", "bf16") else "b200"
    return a


def actor_state(model_state: dict) -> dict:
    return {k[len("actor."):]: v for k, v in model_state.items() if k.startswith("actor.")}


def load_actor(path: str | Path, native: bool = True, device: str | torch.device = "cuda",
               graph_root: str | Path | None = None, obs_dim: int = OBS_DIM):
    ck = torch.load(path, map_location="cpu", weights_only=False)
    a = build_actor(ck["config"]["model"], obs_dim=obs_dim, native=native, graph_root=graph_root)
    a.load_state_dict(actor_state(ck["model"]))
    return ck, a.to(device)


def save_actor(path: str | Path, actor, cfg: dict, steps: int, **extra) -> None:
    """A checkpoint in flyguy's layout with this actor's weights (flyguy/teach.py:167-169)."""
    sd = {"actor." + k: v.detach().cpu() for k, v in actor.state_dict().items()}
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    torch.save({"model": sd, "steps": steps, "taught_steps": steps, "config": {"model": dict(cfg)}, **extra}, path)
