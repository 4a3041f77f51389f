"""Seeded synthetic connectomes in the hop-path wire format (the `structure` dict of `netfile`).

The benchmark graphs of the hop path are synthetic: the same layer sizes as flyguy's trimmed 3-hop male-CNS graph
(16,894 sensory -> 46,393 -> 37,748 -> 1,332 descending neurons, 2,992,734 edges) with made-up wiring whose
statistics are fixed here. One numpy `default_rng(seed)` stream draws everything, in this order:

1. per hop k=1..K, in-degree of every destination row: round(lognormal(ln(mean_deg) - sigma^2/2, sigma)), at least 1;
   then all hops together are rescaled (largest remainder) to exactly `total_edges`;
2. per hop: a permutation of the source layer, then the sources of every edge: Zipf(`zipf`) ranks, ranks beyond the
   source layer rejected, rank r -> perm[r-1] (duplicate (dst, src) pairs are kept: they are a sum);
   `uniform=True` draws sources uniformly instead (no L2 locality from hubs);
3. the input plug: `fan` distinct observation indices per sensory neuron (sorted);
4. weights: edge w ~ N(0, 1/sqrt(in-degree of its row)), plug in ~ N(0, 0.35), plug out ~ N(0, 1/sqrt(n_dn)).
Neurons start at gain 1 and theta -4 (threshold softplus(-4) = 0.018), biases 0 - the reference's own start values
(flyguy/fly.py:138-139, 150, 154).

Layers are distinct neuron sets (neuron ids: layer 0 first, then layer 1, ...), no sensory re-drive, every neuron of
the last layer is a descending neuron, and every edge has its own weight (widx = identity) - so `n_w` equals the
edge count, like a trimmed graph whose hops use disjoint connections.

`make_full_graph` builds the untrimmed-graph workload: one square graph over all neurons, every hop past the first
using all of its edges (shared weights across hops) with the sensory drive re-injected at every hop, the recurrence
of the reference's blind check (tests/test_fly.py:29-41).
"""
from __future__ import annotations

import numpy as np

from .netfile import Structure, csr_ptr, transpose_order

FLYGUY_SIZES = (16894, 46393, 37748, 1332)
FLYGUY_EDGES = 2_992_734
OBS_DIM = 517
N_ACT = 90


def _largest_remainder(raw: np.ndarray, total: int) -> np.ndarray:
    """Scale positive integer counts to sum exactly to `total` (Hamilton's method), each count at least 1."""
    scaled = raw.astype(np.float64) * (total / raw.sum())
    base = np.floor(scaled).astype(np.int64)
    extra = int(total - base.sum())
    if extra > 0:
        order = np.argsort(-(scaled - base), kind="stable")
        base[order[:extra]] += 1
    zero = base < 1
    if zero.any():                                   # keep every row alive, take the surplus from the largest rows
        surplus = int(zero.sum())
        base[zero] = 1
        for i in np.argsort(-base, kind="stable")[:surplus]:
            base[i] -= 1
    assert base.sum() == total and base.min() >= 1
    return base


def _zipf_sources(rng: np.random.Generator, n: int, n_src: int, a: float) -> np.ndarray:
    out, need = [], n
    while need > 0:
        r = rng.zipf(a, int(need * 1.25) + 64)
        r = r[r <= n_src][:need]
        out.append(r)
        need -= len(r)
    return np.concatenate(out) - 1 if out else np.zeros(0, np.int64)


def _plug_cols(rng: np.random.Generator, n_s: int, obs_dim: int, fan: int) -> np.ndarray:
    """`fan` distinct observation indices per sensory row, sorted within the row (the reference draws its plug the
    same way, flyguy/fly.py:141-148, though from its own stream)."""
    cols = np.empty((n_s, fan), np.int64)
    step = 4096
    for i in range(0, n_s, step):
        keys = rng.random((min(step, n_s - i), obs_dim))
        cols[i:i + step] = np.sort(np.argpartition(keys, fan - 1, axis=1)[:, :fan], axis=1)
    return cols.reshape(-1)


def _plug(s: Structure, rng: np.random.Generator, n_s: int, obs_dim: int, fan: int) -> None:
    cols = _plug_cols(rng, n_s, obs_dim, fan)
    rows = np.repeat(np.arange(n_s), fan)
    t = transpose_order(rows, cols)
    s.update(in_crow=csr_ptr(rows, n_s), in_col=cols, in_tcrow=csr_ptr(cols[t], obs_dim), in_tcol=rows[t], in_tperm=t)


def make_synthetic(sizes=FLYGUY_SIZES, total_edges: int = FLYGUY_EDGES, fan: int = 8, obs_dim: int = OBS_DIM,
                   n_act: int = N_ACT, mean_deg: float = 35.0, sigma: float = 1.0, zipf: float = 1.5,
                   uniform: bool = False, seed: int = 0) -> tuple[Structure, list[np.ndarray]]:
    """The seeded synthetic K-hop graph. Returns (structure, params) where params are the seven weight arrays in
    the library's order: W, gain, theta, in_w, in_b, out_w (row = action), out_b."""
    rng = np.random.default_rng(seed)
    sizes = [int(v) for v in sizes]
    K = len(sizes) - 1
    raw = [np.maximum(1, np.round(rng.lognormal(np.log(mean_deg) - 0.5 * sigma * sigma, sigma, sizes[k + 1])))
           .astype(np.int64) for k in range(K)]
    cut = np.cumsum([0] + [len(r) for r in raw])
    deg_all = _largest_remainder(np.concatenate(raw), total_edges)
    deg = [deg_all[cut[k]:cut[k + 1]] for k in range(K)]
    offs = np.cumsum([0] + sizes)                    # neuron ids: the layers one after another
    s = Structure(obs_dim=obs_dim, n_act=n_act, hops=K, n_neurons=int(offs[-1]), n_s=sizes[0], fan=fan,
                  n_dn=sizes[K], sizes=sizes, hop=[])
    w_off = 0
    row_deg = []
    for k in range(K):
        n_src, n_dst = sizes[k], sizes[k + 1]
        E = int(deg[k].sum())
        perm = rng.permutation(n_src)
        src = rng.integers(0, n_src, E) if uniform else perm[_zipf_sources(rng, E, n_src, zipf)]
        rows = np.repeat(np.arange(n_dst), deg[k])
        o = np.lexsort((src, rows))                  # CSR by destination, sources ascending inside a row
        rows, src = rows[o], src[o]
        t = transpose_order(rows, src)
        widx = np.arange(w_off, w_off + E)
        s["hop"].append({"nid": offs[k + 1] + np.arange(n_dst), "crow": csr_ptr(rows, n_dst), "col": src,
                         "widx": widx, "tcrow": csr_ptr(src[t], n_src), "tcol": rows[t], "twidx": widx[t],
                         "drow": np.full(n_dst, -1, np.int64)})
        row_deg.append(deg[k][rows])
        w_off += E
    s.update(n_w=w_off, wmap=np.arange(w_off), n0=np.arange(sizes[0]), dn_rows=np.arange(sizes[K]))
    _plug(s, rng, sizes[0], obs_dim, fan)
    W = (rng.standard_normal(w_off) / np.sqrt(np.concatenate(row_deg))).astype(np.float32)
    in_w = (0.35 * rng.standard_normal(sizes[0] * fan)).astype(np.float32)
    out_w = (rng.standard_normal((n_act, sizes[K])) / np.sqrt(sizes[K])).astype(np.float32)
    params = [W, np.ones(s["n_neurons"], np.float32), np.full(s["n_neurons"], -4.0, np.float32), in_w,
              np.zeros(sizes[0], np.float32), out_w.reshape(-1), np.zeros(n_act, np.float32)]
    s.check()
    return s, params


# the 4-hop variant (docs/HOW_IT_WORKS.md:57-59: 145,113 neurons, 8.4 million connections): the 3-hop layers with a
# second 46,393-neuron layer and a 34,101-neuron fourth, as distinct neuron sets
FLYGUY4_SIZES = (16894, 46393, 46393, 34101, 1332)
FLYGUY4_EDGES = 8_400_000


def make_synthetic4(uniform: bool = False, seed: int = 0) -> tuple[Structure, list[np.ndarray]]:
    """The seeded synthetic 4-hop graph (same generator as make_synthetic)."""
    return make_synthetic(sizes=FLYGUY4_SIZES, total_edges=FLYGUY4_EDGES, uniform=uniform, seed=seed)


def make_full_graph(n_neurons: int = 166_700, n_edges: int = 15_283_167, n_sens: int = 16_894, n_dn: int = 1_332,
                    hops: int = 3, fan: int = 8, obs_dim: int = OBS_DIM, n_act: int = N_ACT, mean_deg: float = 92.0,
                    sigma: float = 1.2, zipf: float = 1.5, seed: int = 0) -> tuple[Structure, list[np.ndarray]]:
    """The untrimmed-graph workload: sensory -> all neurons (edges from sensory sources) -> all -> all, each hop past
    the first using every edge of the square graph with one shared weight per edge, the sensory drive added at every
    hop; the logits read the descending neurons of the last hop."""
    rng = np.random.default_rng(seed)
    raw = np.maximum(1, np.round(rng.lognormal(np.log(mean_deg) - 0.5 * sigma * sigma, sigma, n_neurons))).astype(np.int64)
    deg = _largest_remainder(raw, n_edges)
    perm = rng.permutation(n_neurons)
    src = perm[_zipf_sources(rng, n_edges, n_neurons, zipf)]
    rows = np.repeat(np.arange(n_neurons), deg)
    o = np.lexsort((src, rows))
    rows, src = rows[o], src[o]
    sens = np.sort(rng.choice(n_neurons, n_sens, replace=False))
    dn = np.sort(rng.choice(np.setdiff1d(np.arange(n_neurons), sens), n_dn, replace=False))
    spos = np.full(n_neurons, -1, np.int64)
    spos[sens] = np.arange(n_sens)
    s = Structure(obs_dim=obs_dim, n_act=n_act, hops=hops, n_neurons=n_neurons, n_s=n_sens, fan=fan, n_dn=n_dn,
                  sizes=[n_sens] + [n_neurons] * hops, hop=[])
    eid = np.arange(n_edges)
    for k in range(hops):
        if k == 0:                                   # from the sensory layer: only edges whose source is sensory
            m = spos[src] >= 0
            r, c, w = rows[m], spos[src[m]], eid[m]
            n_src = n_sens
        else:
            r, c, w, n_src = rows, src, eid, n_neurons
        t = transpose_order(r, c)
        s["hop"].append({"nid": np.arange(n_neurons), "crow": csr_ptr(r, n_neurons), "col": c, "widx": w,
                         "tcrow": csr_ptr(c[t], n_src), "tcol": r[t], "twidx": w[t], "drow": spos.copy()})
    s.update(n_w=n_edges, wmap=eid.copy(), n0=sens, dn_rows=dn)
    _plug(s, rng, n_sens, obs_dim, fan)
    W = (rng.standard_normal(n_edges) / np.sqrt(deg[rows])).astype(np.float32)
    in_w = (0.35 * rng.standard_normal(n_sens * fan)).astype(np.float32)
    out_w = (rng.standard_normal((n_act, n_dn)) / np.sqrt(n_dn)).astype(np.float32)
    params = [W, np.ones(n_neurons, np.float32), np.full(n_neurons, -4.0, np.float32), in_w,
              np.zeros(n_sens, np.float32), out_w.reshape(-1), np.zeros(n_act, np.float32)]
    s.check()
    return s, params


def make_batch(n: int, obs_dim: int = OBS_DIM, n_act: int = N_ACT, seed: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """Seeded observations ~ N(0, 1) [n, obs_dim] and teacher logits ~ N(0, 2^2) [n, n_act], fp32."""
    rng = np.random.default_rng(seed)
    obs = rng.standard_normal((n, obs_dim), dtype=np.float32)
    teacher = (2.0 * rng.standard_normal((n, n_act), dtype=np.float32)).astype(np.float32)
    return obs, teacher
