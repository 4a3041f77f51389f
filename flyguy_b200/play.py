"""The playing network on the GPU through the reference's fly_* interface (flyguy/native/fly_infer.cpp; the library's
fly_create / fly_set_* / fly_forward, csrc/fg_fly.cu): a decision for a few cars from host observations, with the
visualizer's firing bytes of the first car. `fly_arrays` builds the arguments the way FlyActor._native does
(flyguy/fly.py:216-233), from a structure and its seven weight arrays; any library with the fly_* interface (this one,
or the reference's CPU library) takes them.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import native
from .netfile import Structure


def _softplus(x: np.ndarray) -> np.ndarray:
    import torch
    return torch.nn.functional.softplus(torch.as_tensor(np.asarray(x, np.float32))).numpy()


def fly_arrays(s: Structure, params) -> dict:
    """The fly_set_plug / fly_set_hop / fly_set_out arguments: connections by source neuron with their strengths in
    that order, gain and threshold (softplus(theta)) per row, re-drive rows, the output plug."""
    W, gain, theta, in_w, in_b, out_w, out_b = [np.asarray(p, np.float32).reshape(-1) for p in params]
    thr = _softplus(theta)
    i32 = lambda a: np.ascontiguousarray(a, np.int32)
    f32 = lambda a: np.ascontiguousarray(a, np.float32)
    n0 = np.asarray(s["n0"], np.int64)
    plug = [i32(s["in_crow"]), i32(s["in_col"]), f32(in_w), f32(in_b), f32(gain[n0]), f32(thr[n0])]
    hops = []
    for k, h in enumerate(s["hop"]):
        nid = np.asarray(h["nid"], np.int64)
        hops.append((len(nid), s["sizes"][k], [i32(h["tcrow"]), i32(h["tcol"]), f32(W[np.asarray(h["twidx"], np.int64)]),
                                               f32(gain[nid]), f32(thr[nid]), i32(h["drow"])]))
    out = [i32(s["dn_rows"]), f32(out_w), f32(out_b)]
    return dict(obs_dim=s["obs_dim"], n_act=s["n_act"], plug=plug, hops=hops, out=out)


def bind_fly(L: ctypes.CDLL) -> ctypes.CDLL:
    """The argument types FlyActor._native sets (flyguy/fly.py:209-215)."""
    vp, ci = ctypes.c_void_p, ctypes.c_int
    L.fly_create.restype, L.fly_create.argtypes = vp, [ci, ci, ci]
    L.fly_set_plug.restype, L.fly_set_plug.argtypes = None, [vp, ci, ci] + [vp] * 6
    L.fly_set_hop.restype, L.fly_set_hop.argtypes = None, [vp, ci, ci, ci, ci] + [vp] * 6
    L.fly_set_out.restype, L.fly_set_out.argtypes = None, [vp, ci, vp, vp, vp]
    L.fly_forward.restype, L.fly_forward.argtypes = None, [vp, vp, ci, vp, vp]
    L.fly_free.restype, L.fly_free.argtypes = None, [vp]
    return L


class Player:
    """A fly_* handle of `lib` (default: this library, the GPU) set up from a structure and weights."""

    def __init__(self, s: Structure, params, lib: ctypes.CDLL | None = None):
        self.L = bind_fly(lib or native.lib())
        a = fly_arrays(s, params)
        self._keep = a                                   # (the arrays stay alive while the handle may read them)
        ptr = lambda x: x.ctypes.data_as(ctypes.c_void_p)
        self.h = self.L.fly_create(a["obs_dim"], a["n_act"], len(a["hops"]))
        if not self.h:
            raise native.FlyguyError(self._err())
        self.L.fly_set_plug(self.h, s["n_s"], len(a["plug"][1]), *map(ptr, a["plug"]))
        for k, (rows, src, arrs) in enumerate(a["hops"]):
            self.L.fly_set_hop(self.h, k, rows, src, len(arrs[1]), *map(ptr, arrs))
        self.L.fly_set_out(self.h, len(a["out"][0]), *map(ptr, a["out"]))
        self._check()
        self.n_act, self.total = a["n_act"], int(sum(s["sizes"]))

    def _err(self) -> str:
        return self.L.fg_fly_last_error().decode() if hasattr(self.L, "fg_fly_last_error") else ""

    def _check(self) -> None:
        msg = self._err()
        if msg:
            raise native.FlyguyError(msg)

    def forward(self, obs: np.ndarray, tap: bool = False):
        x = np.ascontiguousarray(obs, np.float32)
        out = np.empty((x.shape[0], self.n_act), np.float32)
        shade = np.zeros(self.total, np.uint8) if tap else None
        ptr = lambda v: None if v is None else v.ctypes.data_as(ctypes.c_void_p)
        self.L.fly_forward(self.h, ptr(x), x.shape[0], ptr(out), ptr(shade))
        self._check()
        return (out, shade) if tap else out

    def close(self) -> None:
        if getattr(self, "h", None):
            self.L.fly_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
