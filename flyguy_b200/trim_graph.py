"""The part of a connectome graph file that a network of N hops uses, as a graph file of its own.

  python -m flyguy_b200.trim_graph GRAPH.npz OUT.npz [--hops 3] [--weights IN.pt OUT.pt]

Restates flyguy/trim_graph.py on this package's FlyActor (same structure rules, flyguy/fly.py:91-126): a connection
matters only if some hop of an N-hop network computes it - its source can carry the signal at that hop and its target
can still reach a descending neuron in the hops left. OUT holds every array of GRAPH unchanged (neurons are not
renumbered) except
  pre, post, syn       the kept connections, in their old order (flyguy/trim_graph.py:49-51)
  in_total             every neuron's incoming synapse count in the WHOLE graph (the starting strengths are normalised
                       by it, so a network built from OUT starts exactly like one built from GRAPH; 45-46)
  hops                 the hop count it was cut for (a network of that many hops or fewer can be built from it; 52)
  whole_connections    the connection count of GRAPH (53)
and a network built from OUT is the same network: the same neurons at every hop, the connections in the same order
(checked before OUT is written, as the reference does at 56-63).

--weights IN.pt OUT.pt cuts a checkpoint trained on GRAPH down to the kept connections and points its config at OUT
(flyguy/trim_graph.py:69-96). The connections that are cut never took part in a decision, so the cut network computes
the same function: this is checked on the structures (every hop's connections map one to one, with the same
strengths), and, when a GPU is present, on the actors' answers for 64 random game states through the B200 library
(the reference compares them on its CPU torch path, which this package does not have).
"""
from __future__ import annotations

import argparse
from pathlib import Path

import numpy as np
import torch

from .fly import ROOT, FlyActor


def in_play(graph: str | Path, hops: int) -> np.ndarray:
    """keep[i]: connection i of the graph is computed by some hop of a `hops`-hop network (flyguy/trim_graph.py:33-40)."""
    f = FlyActor(graph, 16, 2, hops=hops, fan=16)
    keep = np.zeros(f.n_conn, bool)
    for k in range(1, hops + 1):
        keep[getattr(f, f"e{k}").numpy()] = True
    assert int(keep.sum()) == f.in_play
    return keep


def same_network(a: FlyActor, b: FlyActor, keep: np.ndarray) -> None:
    """b (built from the trimmed file) is a (built from the whole one) with connection i renumbered to
    cumsum(keep)[i] - 1: the same layers, the same connections per hop in the same order, the same strengths."""
    new_index = np.cumsum(keep) - 1
    assert a.sizes == b.sizes, (a.sizes, b.sizes)
    assert torch.equal(a.w.detach()[torch.as_tensor(keep)], b.w.detach())
    for k in range(a.hops + 1):
        assert torch.equal(getattr(a, f"n{k}"), getattr(b, f"n{k}"))
        if k:
            assert np.array_equal(new_index[getattr(a, f"e{k}").numpy()], getattr(b, f"e{k}").numpy())
            assert torch.equal(getattr(a, f"c{k}"), getattr(b, f"c{k}"))
            assert torch.equal(getattr(a, f"r{k}"), getattr(b, f"r{k}"))
    assert torch.equal(a.dn_rows, b.dn_rows)


def trim(graph: str | Path, out: str | Path, hops: int, verbose: bool = True) -> np.ndarray:
    """Writes the trimmed graph file OUT and returns the kept-connection mask (flyguy/trim_graph.py:43-66)."""
    graph, out = Path(graph), Path(out)
    keep = in_play(graph, hops)
    g = np.load(graph)
    if "in_total" in g.files:
        raise ValueError(f"{graph} is trimmed already")
    total = np.zeros(len(g["body"]), np.int64)
    np.add.at(total, g["post"].astype(np.int64), g["syn"].astype(np.int64))
    arrays = {k: g[k] for k in g.files}
    for k in ("pre", "post", "syn"):
        arrays[k] = g[k][keep]
    arrays["in_total"] = total
    arrays["hops"] = np.int64(hops)
    arrays["whole_connections"] = np.int64(len(keep))
    out.parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out, **arrays)
    a, b = FlyActor(graph, 16, 2, hops=hops), FlyActor(out, 16, 2, hops=hops)
    same_network(a, b, keep)
    if verbose:
        print(f"{out}: {int(keep.sum()):,} of {len(keep):,} connections ({hops} hops), "
              f"{out.stat().st_size / 2 ** 20:.1f} MB (was {graph.stat().st_size / 2 ** 20:.1f}); "
              f"neurons per hop {b.sizes}")
    return keep


def trim_weights(src: str | Path, dst: str | Path, keep: np.ndarray, graph_name: str,
                 graph_root: str | Path | None = None, verbose: bool = True) -> float | None:
    """A checkpoint trained on the whole graph with its strengths cut to the kept connections and its config's
    fly_graph set to graph_name (flyguy/trim_graph.py:69-96). Returns the largest difference of the two actors' action
    scores on 64 random game states when a GPU is present (else None: the structural check has run in trim)."""
    from .model import actor_state, build_actor
    src, dst = Path(src), Path(dst)
    ck = torch.load(src, map_location="cpu", weights_only=False)
    if ck["model"]["actor.w"].numel() != len(keep):
        raise ValueError("this checkpoint was not trained on that graph")
    cfg = dict(ck["config"]["model"])
    new = dict(ck)
    new["model"] = dict(ck["model"])
    new["model"]["actor.w"] = ck["model"]["actor.w"][torch.as_tensor(keep)].clone()
    new["config"] = dict(ck["config"])
    new["config"]["model"] = dict(cfg, fly_graph=graph_name)
    worst = None
    if torch.cuda.is_available():
        whole = build_actor(cfg, native=False, graph_root=graph_root)
        cut = build_actor(new["config"]["model"], native=False, graph_root=graph_root)
        whole.load_state_dict(actor_state(ck["model"]))
        cut.load_state_dict(actor_state(new["model"]))
        whole, cut = whole.cuda().eval(), cut.cuda().eval()
        torch.manual_seed(0)
        obs = torch.randn(64, whole.obs_dim, device="cuda")
        with torch.no_grad():
            x, y = whole(obs), cut(obs)
        worst = float((x - y).abs().max())
        if not (torch.equal(x.argmax(-1), y.argmax(-1)) and worst <= 1e-4 * float(x.abs().max())):
            raise AssertionError(f"the cut checkpoint answers differently (largest difference {worst:.3g})")
    dst.parent.mkdir(parents=True, exist_ok=True)
    torch.save(new, dst)
    if verbose:
        check = f"largest difference in 64 x 90 action scores {worst:.2g}" if worst is not None else "no GPU: structure checked"
        print(f"{dst}: {new['model']['actor.w'].numel():,} strengths, {dst.stat().st_size / 2 ** 20:.1f} MB "
              f"(was {src.stat().st_size / 2 ** 20:.1f}); {check}")
    return worst


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("graph", type=Path)
    ap.add_argument("out", type=Path)
    ap.add_argument("--hops", type=int, default=3)
    ap.add_argument("--weights", nargs=2, type=Path, metavar=("IN.pt", "OUT.pt"))
    args = ap.parse_args(argv)
    keep = trim(args.graph, args.out, args.hops)
    if args.weights:
        try:
            name = args.out.resolve().relative_to(ROOT).as_posix()
        except ValueError:
            name = str(args.out.resolve())
        trim_weights(args.weights[0], args.weights[1], keep, name)


if __name__ == "__main__":
    main()
