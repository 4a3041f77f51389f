"""The network's wire formats: NET.bin (structure), PARAMS.bin (weights), and the in-memory `Structure` dict.

These are the formats the reference's native library reads (flyguy/native/export.py:9-16 documents them; the
reader is flyguy/native/flyguy_train.cu:230-256), kept byte-for-byte so that a NET.bin written by the reference's
`export.py net` loads into this library and the other way round:

NET.bin, little endian, int32 unless noted: b"FLY1", obs_dim, n_act, hops, n_neurons, n_w, n_s, fan, n_dn,
sizes[hops+1], E[hops]; plug: in_crow[n_s+1], in_col[E_in], in_tcrow[obs_dim+1], in_tcol[E_in], in_tperm[E_in];
n0[n_s]; per hop k: nid[N_k], crow[N_k+1], col[E_k], widx[E_k], tcrow[N_{k-1}+1], tcol[E_k], twidx[E_k], drow[N_k];
dn_rows[n_dn]; wmap[n_w].  (E_in = n_s * fan.)

PARAMS.bin: b"FLYP", step (int64), float32 W[n_w], gain[n_neurons], theta[n_neurons], in_w[E_in], in_b[n_s],
out_w[n_act * n_dn] (row = action), out_b[n_act]   (flyguy/native/export.py:14-15, 73-88).

Meaning of a hop's arrays (flyguy/fly.py:107-121 builds them): rows of hop k are the neurons in play after k hops;
crow/col is the CSR by destination row with sources (rows of layer k-1) ascending inside a row; widx maps an edge to
its weight in W; tcrow/tcol/twidx are the same edges by source (stable order by (source, destination)); nid is the
neuron id of a row (index of its gain/theta); drow is the sensory-plug row whose drive is re-added to the row, or -1.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

HEADER = ("obs_dim", "n_act", "hops", "n_neurons", "n_w", "n_s", "fan", "n_dn")
HOP_KEYS = ("nid", "crow", "col", "widx", "tcrow", "tcol", "twidx", "drow")
PARAM_NAMES = ("W", "gain", "theta", "in_w", "in_b", "out_w", "out_b")


def csr_ptr(rows: np.ndarray, n_rows: int) -> np.ndarray:
    """Row pointer of CSR entries sorted by row (flyguy/fly.py:46-48)."""
    return np.concatenate([[0], np.cumsum(np.bincount(rows, minlength=n_rows))]).astype(np.int64)


def transpose_order(rows: np.ndarray, cols: np.ndarray) -> np.ndarray:
    """Permutation of CSR-by-row entries into by-column order, ties by row (flyguy/fly.py:112)."""
    return np.lexsort((rows, cols))


class Structure(dict):
    """The index arrays of one network (the dict flyguy/native/export.py:32-49 builds), plus checks."""

    def param_sizes(self) -> list[int]:
        return [self["n_w"], self["n_neurons"], self["n_neurons"], self["n_s"] * self["fan"], self["n_s"],
                self["n_act"] * self["n_dn"], self["n_act"]]

    def edges(self) -> int:
        return int(sum(len(h["col"]) for h in self["hop"]))

    def check(self) -> None:
        K, sz = self["hops"], self["sizes"]
        assert len(sz) == K + 1 and len(self["hop"]) == K and sz[0] == self["n_s"]
        assert len(self["in_crow"]) == self["n_s"] + 1 and len(self["in_col"]) == self["n_s"] * self["fan"]
        assert int(self["in_crow"][-1]) == self["n_s"] * self["fan"]
        assert len(self["n0"]) == self["n_s"] and len(self["dn_rows"]) == self["n_dn"]
        for k, h in enumerate(self["hop"]):
            n_dst, n_src, E = sz[k + 1], sz[k], len(h["col"])
            assert len(h["nid"]) == n_dst and len(h["crow"]) == n_dst + 1 and int(h["crow"][-1]) == E
            assert len(h["tcrow"]) == n_src + 1 and int(h["tcrow"][-1]) == E and len(h["drow"]) == n_dst
            assert len(h["widx"]) == E and len(h["tcol"]) == E and len(h["twidx"]) == E
            if E:
                assert 0 <= int(h["col"].min()) and int(h["col"].max()) < n_src
                assert 0 <= int(h["widx"].min()) and int(h["widx"].max()) < self["n_w"]
            assert int(np.max(h["nid"], initial=-1)) < self["n_neurons"]
            assert int(np.max(h["drow"], initial=-1)) < self["n_s"]
        assert int(np.max(self["dn_rows"], initial=-1)) < sz[K]


def write_net(s: Structure, path: str | Path) -> None:
    """NET.bin in the reference's "FLY1" layout (flyguy/native/export.py:52-65)."""
    i32 = lambda a: np.ascontiguousarray(a, dtype=np.int32).tobytes()  # noqa: E731
    with open(path, "wb") as fh:
        fh.write(b"FLY1")
        fh.write(struct.pack("<8i", *[int(s[k]) for k in HEADER]))
        fh.write(i32(s["sizes"]))
        fh.write(i32([len(h["col"]) for h in s["hop"]]))
        for k in ("in_crow", "in_col", "in_tcrow", "in_tcol", "in_tperm", "n0"):
            fh.write(i32(s[k]))
        for h in s["hop"]:
            for k in HOP_KEYS:
                fh.write(i32(h[k]))
        fh.write(i32(s["dn_rows"]))
        fh.write(i32(s["wmap"]))


def read_net(path: str | Path) -> Structure:
    raw = Path(path).read_bytes()
    if raw[:4] != b"FLY1":
        raise ValueError(f"{path}: not a FLY1 network file")
    at = [4]

    def take(n: int) -> np.ndarray:
        a = np.frombuffer(raw, np.int32, n, at[0]).astype(np.int64)
        at[0] += 4 * n
        return a
    hd = take(8)
    s = Structure({k: int(v) for k, v in zip(HEADER, hd)})
    K = s["hops"]
    s["sizes"] = [int(v) for v in take(K + 1)]
    E = take(K)
    e_in = s["n_s"] * s["fan"]
    for k, n in (("in_crow", s["n_s"] + 1), ("in_col", e_in), ("in_tcrow", s["obs_dim"] + 1), ("in_tcol", e_in),
                 ("in_tperm", e_in), ("n0", s["n_s"])):
        s[k] = take(n)
    s["hop"] = []
    for k in range(K):
        n_dst, n_src = s["sizes"][k + 1], s["sizes"][k]
        lens = {"nid": n_dst, "crow": n_dst + 1, "col": E[k], "widx": E[k], "tcrow": n_src + 1, "tcol": E[k],
                "twidx": E[k], "drow": n_dst}
        s["hop"].append({key: take(lens[key]) for key in HOP_KEYS})
    s["dn_rows"] = take(s["n_dn"])
    s["wmap"] = take(s["n_w"])
    if at[0] != len(raw):
        raise ValueError(f"{path}: {len(raw) - at[0]} bytes after the network")
    s.check()
    return s


def write_params(arrs: list[np.ndarray], path: str | Path, step: int = 0) -> None:
    with open(path, "wb") as fh:
        fh.write(b"FLYP")
        fh.write(struct.pack("<q", step))
        for a in arrs:
            fh.write(np.ascontiguousarray(a, dtype=np.float32).tobytes())


def read_params(path: str | Path, s: Structure) -> tuple[int, list[np.ndarray]]:
    raw = Path(path).read_bytes()
    if raw[:4] != b"FLYP":
        raise ValueError(f"{path}: not a FLYP weights file")
    step = struct.unpack("<q", raw[4:12])[0]
    out, off = [], 12
    for n in s.param_sizes():
        out.append(np.frombuffer(raw, np.float32, n, off).copy())
        off += 4 * n
    return step, out


def write_chunk(obs: np.ndarray, teacher: np.ndarray, path: str | Path) -> None:
    """A FLYD chunk of recorded teacher data (flyguy/native/flyguy_train.cu:13-14, 374-386): "FLYD", n (int64),
    obs_dim, n_act (int32), then the n observations and the n teacher-logit rows as IEEE fp16."""
    obs = np.ascontiguousarray(obs, dtype=np.float16)
    teacher = np.ascontiguousarray(teacher, dtype=np.float16)
    if obs.ndim != 2 or teacher.ndim != 2 or len(obs) != len(teacher) or not len(obs):
        raise ValueError("write_chunk: obs [n, obs_dim] and teacher [n, n_act] with n > 0")
    with open(path, "wb") as fh:
        fh.write(b"FLYD")
        fh.write(struct.pack("<qii", len(obs), obs.shape[1], teacher.shape[1]))
        fh.write(obs.tobytes())
        fh.write(teacher.tobytes())


def read_chunk(path: str | Path) -> tuple[np.ndarray, np.ndarray]:
    raw = Path(path).read_bytes()
    if raw[:4] != b"FLYD":
        raise ValueError(f"{path}: not a FLYD chunk")
    n, od, na = struct.unpack("<qii", raw[4:20])
    obs = np.frombuffer(raw, np.float16, n * od, 20).reshape(n, od)
    teacher = np.frombuffer(raw, np.float16, n * na, 20 + 2 * n * od).reshape(n, na)
    return obs, teacher


def write_batch(obs: np.ndarray, teacher: np.ndarray, path: str | Path) -> None:
    """A fixed batch for `fg_train --check`: "FLYB", n (int32), obs [n, obs_dim] then teacher [n, n_act] float32 (the
    layout export.py batch writes, flyguy/native/export.py:142-143)."""
    obs, teacher = np.ascontiguousarray(obs, np.float32), np.ascontiguousarray(teacher, np.float32)
    assert obs.shape[0] == teacher.shape[0]
    with open(path, "wb") as fh:
        fh.write(b"FLYB" + struct.pack("<i", obs.shape[0]) + obs.tobytes() + teacher.tobytes())


def read_opt(path: str | Path, s: Structure) -> tuple[int, int, list[np.ndarray], list[np.ndarray]]:
    """A FLYO optimiser state (flyguy/native/flyguy_train.cu:288-293): "FLYO", step, adam_t (int64), then M and V of
    each of the seven arrays in turn. Returns (step, adam_t, M, V)."""
    raw = Path(path).read_bytes()
    if raw[:4] != b"FLYO":
        raise ValueError(f"{path}: not a FLYO optimiser file")
    step, adam_t = struct.unpack("<qq", raw[4:20])
    M, V, off = [], [], 20
    for n in s.param_sizes():
        M.append(np.frombuffer(raw, np.float32, n, off).copy())
        V.append(np.frombuffer(raw, np.float32, n, off + 4 * n).copy())
        off += 8 * n
    return step, adam_t, M, V


def structure_of_actor(f) -> Structure:
    """The structure of a FlyActor (this package's or the reference's: the same buffer names), with only the
    connections in play as weights (flyguy/native/export.py:32-49)."""
    import torch
    K = f.hops
    used = torch.unique(torch.cat([getattr(f, f"e{k}") for k in range(1, K + 1)])).cpu().numpy()
    comp = np.full(f.n_conn, -1, np.int64)
    comp[used] = np.arange(len(used))
    s = Structure(obs_dim=f.obs_dim, n_act=f.out.out_features, hops=K, n_neurons=f.n_neurons, n_w=len(used),
                  n_s=f.sizes[0], fan=f.fan, n_dn=len(f.dn_rows), sizes=list(f.sizes), wmap=used,
                  in_crow=f.in_crow.cpu().numpy(), in_col=f.in_ci.cpu().numpy().astype(np.int64),
                  in_tcrow=f.in_tcrow.cpu().numpy(), in_tcol=f.in_tci.cpu().numpy().astype(np.int64),
                  in_tperm=f.in_tperm.cpu().numpy(), n0=f.n0.cpu().numpy(), dn_rows=f.dn_rows.cpu().numpy(), hop=[])
    for k in range(1, K + 1):
        g = lambda name: getattr(f, f"{name}{k}").cpu().numpy()  # noqa: E731
        widx = comp[g("e")]
        drow = np.full(f.sizes[k], -1, np.int64)
        drow[g("s")] = g("d")
        s["hop"].append({"nid": g("n"), "crow": g("crow"), "col": g("ci").astype(np.int64), "widx": widx,
                         "tcrow": g("tcrow"), "tcol": g("tci").astype(np.int64), "twidx": widx[g("tperm")],
                         "drow": drow})
    s.check()
    return s


def params_of_actor(f, s: Structure) -> list[np.ndarray]:
    """The seven weight arrays of a FlyActor in the library's order (flyguy/native/export.py:68-70)."""
    d = lambda t: t.detach().cpu().numpy().astype(np.float32)  # noqa: E731
    return [d(f.w)[s["wmap"]], d(f.gain), d(f.theta), d(f.in_w), d(f.in_b), d(f.out.weight).reshape(-1), d(f.out.bias)]
