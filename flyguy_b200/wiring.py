"""Which neurons and connections of a connectome a K-hop fly network computes, and in what order.

A decision enters at the sensory neurons and leaves K synapses later at the descending neurons (flyguy/fly.py:91-126
states the rule this module implements). Instead of carrying reachability masks hop by hop, every neuron gets two
hop distances, found by breadth-first sweeps over the edge list:

  depth[i]  the fewest synapses from any sensory neuron to i      (0 for a sensory neuron)
  height[i] the fewest synapses from i to any descending neuron   (0 for a descending neuron)

Neuron i takes part after hop k exactly when depth[i] <= k and height[i] <= K - k: it can already carry the signal and
can still deliver it in the hops that are left. Layer k lists those neurons in ascending id; hop k uses the
connections from a layer-(k-1) neuron into a layer-k neuron. A hop's connections are ordered by (destination row,
source row), ties in graph order - the CSR the kernels walk - and its transpose by (source row, destination row), ties
in CSR position. Both orders are produced with one stable sort of a combined integer key.

The result is plain numpy (a `Wiring`), shared by FlyActor (which keeps the reference's buffer names), the graph
trimmer and the NET.bin exporter.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

UNREACHED = np.iinfo(np.int64).max


def hop_distance(start: np.ndarray, src: np.ndarray, dst: np.ndarray, n: int, limit: int) -> np.ndarray:
    """Fewest edges src -> dst from any neuron in `start` to each neuron, counted up to `limit` (UNREACHED beyond)."""
    dist = np.full(n, UNREACHED, np.int64)
    dist[start] = 0
    frontier = np.zeros(n, bool)
    frontier[start] = True
    for d in range(1, limit + 1):
        hit = np.zeros(n, bool)
        hit[dst[frontier[src]]] = True
        new = hit & (dist == UNREACHED)
        if not new.any():
            break
        dist[new] = d
        frontier = new
    return dist


def row_starts(sorted_rows: np.ndarray, n_rows: int) -> np.ndarray:
    """CSR row pointer of entries already sorted by row: position of the first entry of every row, and the end."""
    return np.searchsorted(sorted_rows, np.arange(n_rows + 1), side="left").astype(np.int64)


def by_key(major: np.ndarray, minor: np.ndarray, minor_count: int) -> np.ndarray:
    """Stable order by (major, minor): one argsort of major * minor_count + minor."""
    return np.argsort(major.astype(np.int64) * max(minor_count, 1) + minor, kind="stable")


@dataclass
class HopWiring:
    """Hop k: its connections (graph indices), by destination row then source row, and their transpose."""
    edges: np.ndarray            # graph index of each connection, CSR order
    rows: np.ndarray             # destination row (in layer k) of each
    cols: np.ndarray             # source row (in layer k - 1) of each
    row_ptr: np.ndarray          # CSR pointer over layer k
    tperm: np.ndarray            # CSR position of each connection in by-source order
    tcol_ptr: np.ndarray         # pointer over layer k - 1 into the by-source order
    neurons: np.ndarray          # neuron ids of layer k
    sensory_rows: np.ndarray     # rows of layer k that are sensory neurons (their plug drive is added again)
    drive_rows: np.ndarray       # ... and their rows in layer 0


@dataclass
class Wiring:
    n_neurons: int
    hops: int
    layers: list[np.ndarray]                 # neuron ids per layer 0..K, ascending
    hop: list[HopWiring] = field(default_factory=list)
    dn_rows: np.ndarray = None               # rows of layer K that are descending neurons (the output plug's inputs)

    @property
    def sizes(self) -> list[int]:
        return [len(s) for s in self.layers]

    def kept(self, n_conn: int) -> np.ndarray:
        """Mask of the graph's connections that some hop computes."""
        m = np.zeros(n_conn, bool)
        for h in self.hop:
            m[h.edges] = True
        return m


def wire(pre: np.ndarray, post: np.ndarray, sensory: np.ndarray, descending: np.ndarray, n: int,
         hops: int) -> Wiring:
    pre, post = np.asarray(pre, np.int64), np.asarray(post, np.int64)
    depth = hop_distance(np.asarray(sensory, np.int64), pre, post, n, hops)
    height = hop_distance(np.asarray(descending, np.int64), post, pre, n, hops)
    layers = [np.flatnonzero((depth <= k) & (height <= hops - k)) for k in range(hops + 1)]
    slot = []                                        # row of each neuron in each layer, -1 outside it
    for ids in layers:
        s = np.full(n, -1, np.int64)
        s[ids] = np.arange(len(ids))
        slot.append(s)
    is_sensory = np.zeros(n, bool)
    is_sensory[np.asarray(sensory, np.int64)] = True
    w = Wiring(n, hops, layers)
    for k in range(1, hops + 1):
        r_all, c_all = slot[k][post], slot[k - 1][pre]
        sel = np.flatnonzero((r_all >= 0) & (c_all >= 0))
        n_rows, n_cols = len(layers[k]), len(layers[k - 1])
        o = by_key(r_all[sel], c_all[sel], n_cols)
        edges, rows, cols = sel[o], r_all[sel][o], c_all[sel][o]
        t = by_key(cols, rows, n_rows)
        sens_rows = np.flatnonzero(is_sensory[layers[k]])
        w.hop.append(HopWiring(edges=edges, rows=rows, cols=cols, row_ptr=row_starts(rows, n_rows), tperm=t,
                               tcol_ptr=row_starts(cols[t], n_cols), neurons=layers[k], sensory_rows=sens_rows,
                               drive_rows=slot[0][layers[k][sens_rows]]))
    top = slot[hops][np.asarray(descending, np.int64)]
    w.dn_rows = top[top >= 0]
    return w
