"""CPU ORACLE for the flyguy hop path - TEST INFRASTRUCTURE ONLY.

Python face of oracle/fly_oracle.c (the C restatement of the reference's forward, loss, backward and Adam; see the
citations there) and of oracle/_ref/libfly_infer.so (the reference's own CPU forward, flyguy/native/fly_infer.cpp,
compiled from its source by oracle/Makefile). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs
use this module, as the checker and the CPU baseline; the product path (flyguy_b200) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libfly_oracle.so"
REF_LIB = HERE / "_ref" / "libfly_infer.so"
_lib = None
_lock = threading.Lock()


class _Net(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int) for k in ("obs_dim", "n_act", "hops", "n_neurons", "n_w", "n_s", "fan", "n_dn")] + \
               [(k, ctypes.c_void_p) for k in ("sizes", "in_crow", "in_col", "n0", "dn_rows", "nid", "crow", "col",
                                                "widx", "drow")]


def _build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE), str(LIB)], check=True)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not LIB.exists() or LIB.stat().st_mtime < (HERE / "fly_oracle.c").stat().st_mtime:
                _build()
            L = ctypes.CDLL(str(LIB))
            vp, ci, cf = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
            L.fo_forward.restype, L.fo_forward.argtypes = ci, [vp, vp, vp, ci, vp, vp, ci]
            L.fo_forward_q.restype, L.fo_forward_q.argtypes = ci, [vp, vp, vp, ci, vp, vp, ci, ci]
            L.fo_round16.restype, L.fo_round16.argtypes = None, [vp, vp, ctypes.c_longlong, ci]
            L.fo_backward.restype, L.fo_backward.argtypes = ci, [vp, vp, vp, vp, ci, vp, ci]
            L.fo_loss.restype = None
            L.fo_loss.argtypes = [vp, vp, ci, ci, cf, vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
            L.fo_grad_norm.restype, L.fo_grad_norm.argtypes = ctypes.c_double, [vp, vp]
            L.fo_adam.restype = ctypes.c_double
            L.fo_adam.argtypes = [vp] * 6 + [ctypes.c_longlong, cf, cf, cf, cf, cf]
            _lib = L
    return _lib


# fo_forward_q's qmode per state format (fly_oracle.c: q16)
QMODES = {"fp32": 0, "bf16": 1, "f16": 2, "bf16+obs": 1 | 16, "f16+obs": 2 | 16}


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Oracle:
    """The oracle bound to one network structure (a netfile.Structure)."""

    def __init__(self, s, threads: int = 0):
        self.s, self.threads = s, int(threads or min(os.cpu_count() or 1, 16))
        self._keep = []
        K = s["hops"]

        def arr(a):
            a = _i32(a)
            self._keep.append(a)
            return a

        def table(key):
            ptrs = (ctypes.c_void_p * K)(*[_ptr(arr(h[key])) for h in s["hop"]])
            self._keep.append(ptrs)
            return ctypes.cast(ptrs, ctypes.c_void_p).value
        n = _Net(*[int(s[k]) for k in ("obs_dim", "n_act", "hops", "n_neurons", "n_w", "n_s", "fan", "n_dn")])
        n.sizes, n.in_crow, n.in_col = _ptr(arr(s["sizes"])), _ptr(arr(s["in_crow"])), _ptr(arr(s["in_col"]))
        n.n0, n.dn_rows = _ptr(arr(s["n0"])), _ptr(arr(s["dn_rows"]))
        for key in ("nid", "crow", "col", "widx", "drow"):
            setattr(n, key, table(key))
        self.net = n
        self.sizes = s.param_sizes()

    def _params(self, P):
        P = [_f32(p).reshape(-1) for p in P]
        assert [len(p) for p in P] == self.sizes, "weights do not fit this network"
        return P, (ctypes.c_void_p * 7)(*[_ptr(p) for p in P])

    def forward(self, P, obs: np.ndarray, layers: bool = False, states: str = "fp32", pre: bool = False):
        """obs [B, obs_dim] -> logits [B, n_act] (and, with layers=True, every layer's firing [B, sum of sizes]).

        states: "fp32" - the reference's forward; "bf16" / "f16" - 16-bit state emulation: every layer but the last
        rounded (to nearest even) to that type where a 16-bit-state kernel stores it, the sums still in double;
        "bf16+obs" / "f16+obs" - the plug's observation values rounded to that type as well. pre=True: the layers
        returned are the pre-activations (the plug's drive for layer 0, z for the hop layers) instead of the states."""
        obs = _f32(obs)
        B = obs.shape[0]
        P, pp = self._params(P)
        out = np.empty((B, self.s["n_act"]), np.float32)
        lay = np.empty((B, int(sum(self.s["sizes"]))), np.float32) if layers else None
        rc = lib().fo_forward_q(ctypes.byref(self.net), pp, _ptr(obs), B, _ptr(out), _ptr(lay) if layers else None,
                                self.threads, QMODES[states] | (32 if pre else 0))
        assert rc == 0, "oracle forward ran out of memory"
        return (out, lay) if layers else out

    def backward(self, P, obs: np.ndarray, dlogits: np.ndarray, G=None):
        """Gradients of sum <dlogits, logits> over the batch, ADDED to G (seven float32 arrays; zeros if None)."""
        obs, dl = _f32(obs), _f32(dlogits)
        P, pp = self._params(P)
        G = [np.zeros(n, np.float32) for n in self.sizes] if G is None else G
        gp = (ctypes.c_void_p * 7)(*[_ptr(g) for g in G])
        rc = lib().fo_backward(ctypes.byref(self.net), pp, _ptr(obs), _ptr(dl), obs.shape[0], gp, self.threads)
        assert rc == 0, "oracle backward ran out of memory"
        return G


def round16(x: np.ndarray, fmt: str) -> np.ndarray:
    """x rounded to the 16-bit state format fmt ("bf16" / "f16"), as fp32: the emulation's rounding (fly_oracle.c q16)."""
    x = _f32(x)
    out = np.empty_like(x)
    lib().fo_round16(_ptr(x), _ptr(out), x.size, QMODES[fmt])
    return out


def loss(logits: np.ndarray, teacher: np.ndarray, inv_temp: float = 1.0):
    """(kl summed over the batch, argmax agreements, dl [B, n_act])."""
    logits, teacher = _f32(logits), _f32(teacher)
    B, A = logits.shape
    dl = np.empty_like(logits)
    kl, ag = ctypes.c_double(), ctypes.c_double()
    lib().fo_loss(_ptr(logits), _ptr(teacher), B, A, float(inv_temp), _ptr(dl), ctypes.byref(kl), ctypes.byref(ag))
    return kl.value, ag.value, dl


def adam(P, G, M, V, EMA, t: int, lr: float, lr_neuron: float, lr_plug: float, max_norm: float = 0.0,
         ema: float = 0.999) -> float:
    """One in-place Adam step over the seven arrays of each of P, M, V, EMA (fc_step); t = the step count after the
    increment. Returns the pre-clip gradient norm (0 when max_norm is 0)."""
    sizes = (ctypes.c_longlong * 7)(*[len(p) for p in P])
    tab = lambda L: (ctypes.c_void_p * 7)(*[_ptr(a) for a in L])  # noqa: E731
    for L in (P, G, M, V, EMA):
        assert all(a.dtype == np.float32 and a.flags.c_contiguous for a in L)
    return lib().fo_adam(tab(P), tab(G), tab(M), tab(V), tab(EMA), sizes, int(t), lr, lr_neuron, lr_plug, max_norm, ema)


# ------------------------------------------------------------------ the reference's own CPU forward (fly_infer.cpp)
class RefInfer:
    """flyguy/native/fly_infer.cpp compiled from source (oracle/_ref/libfly_infer.so), fed the way
    flyguy/fly.py:187-241 feeds it: per hop the edges by SOURCE with their weights in that order, the threshold
    softplus(theta) precomputed. One handle per thread, the batch split between the threads."""

    def __init__(self, s, P, threads: int = 1):
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} is not built (make -C oracle with the reference mounted)")
        L = ctypes.CDLL(str(REF_LIB))
        vp, ci = ctypes.c_void_p, ctypes.c_int
        L.fly_create.restype, L.fly_create.argtypes = vp, [ci, ci, ci]
        L.fly_set_plug.restype, L.fly_set_plug.argtypes = None, [vp, ci, ci] + [vp] * 6
        L.fly_set_hop.restype, L.fly_set_hop.argtypes = None, [vp, ci, ci, ci, ci] + [vp] * 6
        L.fly_set_out.restype, L.fly_set_out.argtypes = None, [vp, ci, vp, vp, vp]
        L.fly_forward.restype, L.fly_forward.argtypes = None, [vp, vp, ci, vp, vp]
        L.fly_free.restype, L.fly_free.argtypes = None, [vp]
        self.L, self.s, self.threads = L, s, max(1, int(threads))
        W, gain, theta, in_w, in_b, ow, ob = [_f32(p).reshape(-1) for p in P]
        thr = np.where(theta > 20, theta, np.log1p(np.exp(np.minimum(theta, 20)))).astype(np.float32)
        self._keep = []

        def k(a):
            self._keep.append(a)
            return _ptr(a)
        n0 = np.asarray(s["n0"])
        plug = [_i32(s["in_crow"]), _i32(s["in_col"]), in_w, _f32(in_b), _f32(gain[n0]), _f32(thr[n0])]
        hops = []
        for h in s["hop"]:
            nid = np.asarray(h["nid"])
            hops.append([_i32(h["tcrow"]), _i32(h["tcol"]), _f32(W[np.asarray(h["twidx"])]), _f32(gain[nid]),
                         _f32(thr[nid]), _i32(h["drow"])])
        out = [_i32(s["dn_rows"]), _f32(ow), _f32(ob)]
        self.handles = []
        for _ in range(self.threads):
            hd = L.fly_create(s["obs_dim"], s["n_act"], s["hops"])
            L.fly_set_plug(hd, s["n_s"], len(plug[1]), *[k(a) for a in plug])
            for i, a in enumerate(hops):
                L.fly_set_hop(hd, i, s["sizes"][i + 1], s["sizes"][i], len(a[1]), *[k(x) for x in a])
            L.fly_set_out(hd, len(out[0]), *[k(a) for a in out])
            self.handles.append(hd)

    def forward(self, obs: np.ndarray) -> np.ndarray:
        obs = _f32(obs)
        B = obs.shape[0]
        out = np.empty((B, self.s["n_act"]), np.float32)
        parts = np.array_split(np.arange(B), len(self.handles))

        def run(i):
            p = parts[i]
            if len(p):
                self.L.fly_forward(self.handles[i], _ptr(obs) + int(p[0]) * obs.strides[0], len(p),
                                   _ptr(out) + int(p[0]) * out.strides[0], None)
        ts = [threading.Thread(target=run, args=(i,)) for i in range(len(self.handles))]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        return out

    def close(self) -> None:
        for hd in self.handles:
            self.L.fly_free(hd)
        self.handles = []
