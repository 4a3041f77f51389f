"""CPU restatement of the trainer's revival of silent neurons - TEST INFRASTRUCTURE ONLY.

The steps are the reference's revive() (flyguy/native/flyguy_train.cu:479-551) as fg_train carries them out, with the
samples and surveys restated on the CPU: the census batches are redrawn with the trainer's counter-based draw
(splitmix64) from the same chunks, every forward is the oracle's (oracle/fly_oracle.c, pinned to the reference), so the
weights it returns are what a correct revival writes:
  1. silent = neurons in a layer past the sensory one, not sensory, whose state is positive for none of the surveyed
     samples in any of their rows;
  2. per weight (each once): into a silent neuron -> its size (at least 1e-4) with the sign bit 0 of
     splitmix64(seed ^ weight index) gives (1: +, 0: -); else from a silent neuron -> 0; silent neurons' gain 1 and
     theta -4; the action weights of silent descending rows 0;
  3. three passes: survey, rms of each neuron's pre-activation (largest over its rows), incoming weights of each
     silent neuron (each weight once, in hop / row / edge order) times clamp(target / rms, 0.02, 200).
Used by tests/test_gpu_train.py only; the product never imports it.
"""
from __future__ import annotations

import numpy as np

from .oracle import Oracle

M64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M64
    return x ^ (x >> 31)


def draw(obs_all: np.ndarray, teacher_all: np.ndarray, seed: int, counter: int, B: int):
    """The trainer's batch `counter` for `seed` from the concatenated chunks (oldest first)."""
    n = len(obs_all)
    sel = [splitmix64(seed ^ ((counter << 32) | b)) % n for b in range(B)]
    return obs_all[sel], teacher_all[sel]


def survey(o: Oracle, P, obs_all, teacher_all, seed: int, batches: int, B: int):
    """Per row of every layer: samples with a positive state, and the summed squared pre-activation."""
    fired = sq = None
    for i in range(batches):
        x, _ = draw(obs_all, teacher_all, seed, i, B)
        _, h = o.forward(P, x, layers=True)
        _, z = o.forward(P, x, layers=True, pre=True)
        f, q = (h > 0).sum(0), (z.astype(np.float64) ** 2).sum(0)
        fired, sq = (f, q) if fired is None else (fired + f, sq + q)
    return fired, sq, batches * B


def revive(s, P, obs_all, teacher_all, seed: int, batches: int, B: int, target: float):
    """(new weights [7 arrays], silent neuron ids) after one revival of network `s` with weights P."""
    o = Oracle(s, threads=4)
    P = [np.array(a, np.float32, copy=True) for a in P]
    fired, _, _ = survey(o, P, obs_all, teacher_all, seed, batches, B)
    n_s = s["n_s"]
    hidden = np.zeros(s["n_neurons"], bool)
    count = np.zeros(s["n_neurons"], np.int64)
    row = n_s
    for h in s["hop"]:
        nid = np.asarray(h["nid"])
        hidden[nid] = True
        np.add.at(count, nid, fired[row:row + len(nid)])
        row += len(nid)
    hidden[np.asarray(s["n0"])] = False
    silent = hidden & (count == 0)
    touched = np.zeros(s["n_w"], bool)
    for k, h in enumerate(s["hop"]):
        nid = np.asarray(h["nid"])
        below = np.asarray(s["hop"][k - 1]["nid"]) if k else np.asarray(s["n0"])
        crow, col, widx = (np.asarray(h[x]) for x in ("crow", "col", "widx"))
        for t in range(len(nid)):
            for e in range(crow[t], crow[t + 1]):
                w = int(widx[e])
                if touched[w]:
                    continue
                if silent[nid[t]]:
                    mag = max(abs(float(P[0][w])), 1e-4)
                    P[0][w] = np.float32(mag if splitmix64(seed ^ w) & 1 else -mag)
                    touched[w] = True
                elif silent[below[col[e]]]:
                    P[0][w] = 0.0
                    touched[w] = True
    P[1][silent] = 1.0
    P[2][silent] = -4.0
    top = np.asarray(s["hop"][-1]["nid"])
    dead_cols = silent[top[np.asarray(s["dn_rows"])]]
    ow = P[5].reshape(s["n_act"], s["n_dn"])
    ow[:, dead_cols] = 0.0
    for _ in range(3):
        _, sq, samples = survey(o, P, obs_all, teacher_all, seed, batches, B)
        rms = np.zeros(s["n_neurons"], np.float32)
        row = n_s
        for h in s["hop"]:
            nid = np.asarray(h["nid"])
            r = np.sqrt(sq[row:row + len(nid)] / samples).astype(np.float32)
            np.maximum.at(rms, nid, r)
            row += len(nid)
        scaled = np.zeros(s["n_w"], bool)
        for h in s["hop"]:
            nid = np.asarray(h["nid"])
            crow, widx = np.asarray(h["crow"]), np.asarray(h["widx"])
            for t in range(len(nid)):
                g = nid[t]
                if not silent[g] or rms[g] <= 0:
                    continue
                f = np.float32(min(200.0, max(0.02, target / float(rms[g]))))
                for e in range(crow[t], crow[t + 1]):
                    w = int(widx[e])
                    if not scaled[w]:
                        P[0][w] = np.float32(P[0][w] * f)
                        scaled[w] = True
    return P, np.flatnonzero(silent)
