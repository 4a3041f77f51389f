"""Cut a connectome graph file down to the connections an N-hop fly network computes.

  python -m flyguy_b200.trim_graph GRAPH.npz OUT.npz [--hops 3] [--weights IN.pt OUT.pt]

The kept connections are exactly the ones flyguy_b200.wiring assigns to some hop (a connection whose source can carry
the signal at that hop and whose target can still reach a descending neuron in the hops left; the reference's rule,
flyguy/trim_graph.py:33-40 and flyguy/fly.py:91-126). The output file is the graph file with
  pre, post, syn         only the kept connections, still in graph order (neurons are never renumbered)
  in_total               each neuron's incoming synapse count in the WHOLE graph - the starting strengths are normalised
                         by it, so a network built from OUT starts exactly like one built from GRAPH
  hops                   the hop count it was cut for (a network of at most that many hops can be built from it)
  whole_connections      the connection count of GRAPH
and every other array as it was - the reference's trimmed-file layout (flyguy/trim_graph.py:43-56), which its
FlyActor reads. Before anything is written the wiring of OUT is checked to be the wiring of GRAPH with connection i
renumbered to its rank among the kept ones.

--weights IN.pt OUT.pt: a checkpoint trained on GRAPH with its strengths cut to the kept connections and its config's
fly_graph pointed at OUT (flyguy/trim_graph.py:69-96). The cut connections never took part in a decision, so both
checkpoints compute the same function; with a GPU present that is checked on 64 random game states through the B200
library before the file is written.
"""
from __future__ import annotations

import argparse
import tempfile
from pathlib import Path

import numpy as np
import torch

from .fly import ROOT
from .wiring import Wiring, wire


def wiring_of(graph_file, hops: int) -> Wiring:
    g = np.load(graph_file)
    return wire(g["pre"], g["post"], g["sensory"], g["descending"], len(g["body"]), hops)


def in_play(graph: str | Path, hops: int) -> np.ndarray:
    """Mask over the graph's connections: computed by some hop of a `hops`-hop network."""
    g = np.load(graph)
    return wiring_of(graph, hops).kept(len(g["pre"]))


def check_same_wiring(whole: Wiring, cut: Wiring, keep: np.ndarray) -> None:
    """cut (from the trimmed file) is whole (from the full graph) with connection i renumbered to rank(i) among the
    kept ones: the same layers and descending rows, and per hop the same connections in the same order."""
    rank = np.cumsum(keep) - 1
    problems = []
    if whole.sizes != cut.sizes:
        problems.append(f"layer sizes {whole.sizes} != {cut.sizes}")
    else:
        for k in range(whole.hops + 1):
            if not np.array_equal(whole.layers[k], cut.layers[k]):
                problems.append(f"layer {k} neurons differ")
        for k, (a, b) in enumerate(zip(whole.hop, cut.hop), start=1):
            if not (np.array_equal(rank[a.edges], b.edges) and np.array_equal(a.rows, b.rows)
                    and np.array_equal(a.cols, b.cols)):
                problems.append(f"hop {k} connections differ")
        if not np.array_equal(whole.dn_rows, cut.dn_rows):
            problems.append("descending rows differ")
    if problems:
        raise AssertionError("the trimmed file does not wire the same network: " + "; ".join(problems))


def trim(graph: str | Path, out: str | Path, hops: int, verbose: bool = True) -> np.ndarray:
    """Writes the trimmed graph file `out`; returns the kept-connection mask."""
    graph, out = Path(graph), Path(out)
    g = np.load(graph)
    if "in_total" in g.files:
        raise ValueError(f"{graph} is trimmed already (it holds the connections of a {int(g['hops'])}-hop network)")
    whole = wiring_of(graph, hops)
    keep = whole.kept(len(g["pre"]))
    arrays = {k: g[k] for k in g.files}
    arrays.update({k: g[k][keep] for k in ("pre", "post", "syn")})
    arrays["in_total"] = np.bincount(g["post"].astype(np.int64), weights=g["syn"].astype(np.int64),
                                     minlength=len(g["body"])).astype(np.int64)
    arrays["hops"] = np.int64(hops)
    arrays["whole_connections"] = np.int64(len(keep))
    out.parent.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory(dir=out.parent) as tmp:      # checked before it takes the output's name
        staged = Path(tmp) / out.name
        np.savez_compressed(staged, **arrays)
        check_same_wiring(whole, wiring_of(staged, hops), keep)
        staged.replace(out)
    if verbose:
        print(f"{out}: kept {int(keep.sum()):,} of {len(keep):,} connections for {hops} hops "
              f"(layers {whole.sizes}); {out.stat().st_size / 2 ** 20:.1f} MB, the whole graph "
              f"{graph.stat().st_size / 2 ** 20:.1f} MB")
    return keep


def cut_checkpoint(ck: dict, keep: np.ndarray, graph_name: str) -> dict:
    """A copy of checkpoint `ck` with actor.w cut to the kept connections and its config's fly_graph = graph_name;
    every other entry is carried over unchanged."""
    w = ck["model"]["actor.w"]
    if w.numel() != len(keep):
        raise ValueError(f"this checkpoint was not trained on that graph ({w.numel():,} strengths, the graph has "
                         f"{len(keep):,} connections)")
    model = dict(ck["model"], **{"actor.w": w[torch.as_tensor(keep)].clone()})
    config = dict(ck["config"], model=dict(ck["config"]["model"], fly_graph=graph_name))
    return dict(ck, model=model, config=config)


def answers_differ(ck_a: dict, ck_b: dict, graph_root=None) -> float:
    """Largest difference of the two checkpoints' action scores on 64 seeded random game states, through the B200
    library; raises if an argmax differs or the difference exceeds 1e-4 of the scores' size."""
    from .model import actor_state, build_actor
    actors = []
    for ck in (ck_a, ck_b):
        a = build_actor(ck["config"]["model"], native=False, graph_root=graph_root)
        a.load_state_dict(actor_state(ck["model"]))
        actors.append(a.cuda().eval())
    obs = torch.randn(64, actors[0].obs_dim, generator=torch.Generator().manual_seed(0)).cuda()
    with torch.no_grad():
        x, y = actors[0](obs), actors[1](obs)
    worst = float((x - y).abs().max())
    if not torch.equal(x.argmax(-1), y.argmax(-1)) or worst > 1e-4 * float(x.abs().max()):
        raise AssertionError(f"the cut checkpoint answers differently (largest difference {worst:.3g})")
    return worst


def trim_weights(src: str | Path, dst: str | Path, keep: np.ndarray, graph_name: str,
                 graph_root: str | Path | None = None, verbose: bool = True) -> float | None:
    """Writes the cut checkpoint; returns the largest answer difference (None without a GPU: the wiring check in
    trim() is then the check)."""
    src, dst = Path(src), Path(dst)
    ck = torch.load(src, map_location="cpu", weights_only=False)
    new = cut_checkpoint(ck, keep, graph_name)
    worst = answers_differ(ck, new, graph_root) if torch.cuda.is_available() else None
    dst.parent.mkdir(parents=True, exist_ok=True)
    torch.save(new, dst)
    if verbose:
        how = f"action scores agree to {worst:.2g} on 64 states" if worst is not None else "no GPU: wiring checked"
        print(f"{dst}: {new['model']['actor.w'].numel():,} strengths (was {len(keep):,}); {how}")
    return worst


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("graph", type=Path)
    ap.add_argument("out", type=Path)
    ap.add_argument("--hops", type=int, default=3)
    ap.add_argument("--weights", nargs=2, type=Path, metavar=("IN.pt", "OUT.pt"))
    a = ap.parse_args(argv)
    keep = trim(a.graph, a.out, a.hops)
    if a.weights:
        out = a.out.resolve()
        name = out.relative_to(ROOT).as_posix() if out.is_relative_to(ROOT) else str(out)
        trim_weights(a.weights[0], a.weights[1], keep, name)


if __name__ == "__main__":
    main()
