"""Records the reference's OWN ctypes binding of the fc_* library driving a training step, for replay against
libflyguy_b200.so on a GPU (tests/test_gpu_binding.py). Run in the build container, where the reference project
adventure-gpt/flyguy is importable; nothing of it is copied.

  python tests/golden/make_binding_golden.py [--ref REFERENCE_CHECKOUT]

The reference's flyguy/fly_native.py (NativeFlyActor, NativeAdam, grad_arrays: fly_native.py:34-215) is imported and
run unchanged on the CPU, with three stand-ins so that it runs without a GPU: torch tensors report is_cuda, CUDA
synchronisation is a no-op, and ctypes.CDLL returns a recording library. The recording library keeps whatever
argtypes / restype the reference declares on each entry point (fly_native.py:135-145) and executes every call on the
CPU oracle (oracle/fly_oracle.c: forward, backward, Adam - itself pinned to the reference's outputs), so the
reference's own code paths - pieces beyond max_batch with padding, the second forward of each piece inside backward,
push / pull / fetch through fc_copy, the Adam step with its three rates, the optimiser state - produce the call
sequence and the values a correct library returns. The recording's gradient is also checked here against torch
autograd through the reference's plain FlyActor.

tests/golden/binding_toy_h3.npz holds:
  meta     JSON: the network's NET.bin name, the declarations (restype / argtypes per entry point, as the reference set
           them) and the calls in order: entry point, scalar arguments, named input / output arrays, return value
  net      the NET.bin bytes the reference's fc_create was given (written by its export.write_net)
  a<i>     the arrays the calls read or write (inputs as the reference passed them, outputs as the oracle computed)
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import io
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _arr(ptr: int, n: int, dtype=np.float32) -> np.ndarray:
    """n values at a host address (the CPU tensors the reference hands the library)."""
    ct = {np.float32: ctypes.c_float, np.int64: ctypes.c_longlong}[dtype]
    return np.ctypeslib.as_array((ct * n).from_address(int(ptr)))


class Recorder:
    """The fc_* library as the reference's ctypes binding sees it, executed on the CPU oracle."""

    def __init__(self):
        self.decl, self.calls, self.arrays, self._hash = {}, [], [], {}
        self.net_bytes = None
        outer = self

        class Fn:
            def __init__(self, name):
                self.name, self.argtypes, self.restype = name, None, None

            def __call__(self, *args):
                outer.decl[self.name] = {"restype": _tname(self.restype), "argtypes": [_tname(t) for t in
                                                                                        (self.argtypes or [])]}
                return getattr(outer, "_do_" + self.name)(*args)

        self._Fn = Fn

    def __getattr__(self, name):
        if name.startswith("fc_"):
            f = self._Fn(name)
            self.__dict__[name] = f
            return f
        raise AttributeError(name)

    # ---- recording helpers
    def _keep(self, a: np.ndarray) -> int:
        a = np.ascontiguousarray(a)
        key = hashlib.sha1(a.tobytes() + str(a.dtype).encode() + str(a.shape).encode()).hexdigest()
        if key not in self._hash:
            self._hash[key] = len(self.arrays)
            self.arrays.append(a.copy())
        return self._hash[key]

    def _log(self, fn, scalars, inputs=None, outputs=None, ret=None):
        self.calls.append({"fn": fn, "scalars": scalars,
                           "in": {k: self._keep(v) for k, v in (inputs or {}).items()},
                           "out": {k: self._keep(v) for k, v in (outputs or {}).items()},
                           "ret": ret})

    # ---- the entry points (flyguy_train.cu:569-629 semantics), reached through the declared Fn objects
    def _do_fc_create(self, path: bytes, max_batch: int):
        from flyguy_b200.netfile import read_net
        from oracle.oracle import Oracle
        self.net_bytes = Path(path.decode()).read_bytes()
        self.s = read_net(path.decode())
        self.o = Oracle(self.s, threads=2)
        self.maxB = int(max_batch)
        self.sizes = self.s.param_sizes()
        self.state = {w: [np.zeros(n, np.float32) for n in self.sizes] for w in range(5)}
        self.t = 0
        self.last_obs = None
        self._log("fc_create", [int(max_batch)])
        return 1

    def _do_fc_sizes(self, core, out):
        v = self.sizes + [self.s["obs_dim"], self.s["n_act"], self.maxB]
        for i, x in enumerate(v):
            out[i] = x
        self._log("fc_sizes", [], outputs={"sizes": np.asarray(v, np.int64)})

    def _do_fc_copy(self, core, which, to_core, ptrs):
        arrs = [_arr(ptrs[i], n) for i, n in enumerate(self.sizes)]
        if to_core:
            for i in range(7):
                self.state[which][i][:] = arrs[i]
            self._log("fc_copy", [int(which), int(to_core)], inputs={f"p{i}": arrs[i] for i in range(7)})
        else:
            for i in range(7):
                arrs[i][:] = self.state[which][i]
            self._log("fc_copy", [int(which), int(to_core)], outputs={f"p{i}": self.state[which][i] for i in range(7)})

    def _do_fc_forward(self, core, obs_ptr, B, out_ptr, ema):
        obs = _arr(obs_ptr, B * self.s["obs_dim"]).reshape(B, -1).copy()
        lg = self.o.forward(self.state[1 if ema else 0], obs)
        _arr(out_ptr, B * self.s["n_act"])[:] = lg.reshape(-1)
        self.last_obs = obs
        self._log("fc_forward", [int(B), int(ema)], inputs={"obs": obs}, outputs={"logits": lg})

    def _do_fc_zero_grad(self, core):
        for g in self.state[4]:
            g[:] = 0
        self._log("fc_zero_grad", [])

    def _do_fc_backward(self, core, dl_ptr, B):
        dl = _arr(dl_ptr, B * self.s["n_act"]).reshape(B, -1).copy()
        self.o.backward(self.state[0], self.last_obs, dl, self.state[4])
        self._log("fc_backward", [int(B)], inputs={"dlogits": dl})

    def _do_fc_grad_norm(self, core):
        n = float(np.sqrt(sum(float((g.astype(np.float64) ** 2).sum()) for g in self.state[4])))
        self._log("fc_grad_norm", [], ret=n)
        return n

    def _do_fc_step(self, core, lr, lr_neuron, lr_plug, max_norm, ema):
        from oracle.oracle import adam
        self.t += 1
        P, M, V, E = (self.state[w] for w in (0, 2, 3, 1))
        n = adam(P, self.state[4], M, V, E, self.t, float(lr), float(lr_neuron), float(lr_plug), float(max_norm),
                 float(ema))
        self._log("fc_step", [float(lr), float(lr_neuron), float(lr_plug), float(max_norm), float(ema)], ret=float(n))
        return float(n)

    def _do_fc_adam_t(self, core, set_):
        if set_ >= 0:
            self.t = int(set_)
        self._log("fc_adam_t", [int(set_)], ret=int(self.t))
        return self.t


def _tname(t) -> str | None:
    if t is None:
        return None
    return t.__name__


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("FLYGUY_REF"), required="FLYGUY_REF" not in os.environ,
                    help="checkout of the reference project (default: the FLYGUY_REF environment variable)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(HERE))
    from make_golden import toy_connectome
    from oracle.oracle import lib as oracle_lib
    oracle_lib()                                            # (loaded before ctypes.CDLL is replaced)
    import flyguy.fly_native as fn                          # the reference's
    torch.set_num_threads(4)
    rec = Recorder()
    real_cdll, real_sync, real_is_cuda = ctypes.CDLL, torch.cuda.synchronize, torch.Tensor.is_cuda
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        toy_connectome(tmp / "toy.npz", 80, 14, 7, 420, seed=0)
        torch.manual_seed(3)
        actor = fn.NativeFlyActor(tmp / "toy.npz", 517, 90, hops=3, fan=5, max_batch=32)
        with torch.no_grad():                               # lively weights (as the golden toy_h3 case)
            sign = torch.where(torch.rand_like(actor.w) < 0.2, -1.0, 1.0)
            actor.w.abs_().mul_(4.0 * sign); actor.out.weight.normal_(0, 0.3); actor.theta.fill_(-2.0)
            actor.gain.mul_(1 + 0.2 * torch.randn_like(actor.gain)); actor.in_b.normal_(0, 0.2)
        import copy
        plain = copy.deepcopy(actor)                        # (NativeFlyActor.__deepcopy__ gives a plain FlyActor)
        g = torch.Generator().manual_seed(5)
        obs = torch.randn(40, 517, generator=g)             # 40 > max_batch: two pieces, the second padded to 32
        teacher = 2.0 * torch.randn(40, 90, generator=g)
        fn.DLL = Path(__file__)                              # (exists: _ready() goes on to load "the library")
        ctypes.CDLL = lambda *a, **k: rec                    # noqa: E731
        torch.cuda.synchronize = lambda *a, **k: None
        torch.Tensor.is_cuda = property(lambda self: True)
        try:
            opt = actor.native_adam(1e-3, max_norm=1.0)     # _ready: declarations, fc_create, fc_sizes, push
            assert opt is not None
            with torch.no_grad():
                acting = actor(obs)                          # acting: forward in pieces, no gradient
            opt.zero_grad()
            logits = actor(obs)                              # learning: _NativeLogits
            pt = torch.softmax(teacher, -1)
            loss = (pt * (torch.log_softmax(teacher, -1) - torch.log_softmax(logits, -1))).sum(-1).mean()
            loss.backward()                                  # each piece's forward again, then fc_backward
            grads = fn.grad_arrays(actor)                    # fc_copy(4, to host)
            opt.step()                                       # fc_step(lr, 0.3 lr, lr, 1.0, 0.999), then pull
            state = opt.state_dict()                         # fc_adam_t, fc_copy(1/2/3, to host)
            stepped = [t.detach().clone() for t in actor._tensors()]
        finally:
            ctypes.CDLL, torch.cuda.synchronize = real_cdll, real_sync
            torch.Tensor.is_cuda = real_is_cuda
        # the recording's gradient against torch autograd through the reference's plain FlyActor
        plain.zero_grad()
        lg = plain(obs)
        (pt * (torch.log_softmax(teacher, -1) - torch.log_softmax(lg, -1))).sum(-1).mean().backward()
        wmap = actor._wmap.cpu().numpy()
        want = [plain.w.grad.numpy()[wmap], plain.gain.grad.numpy(), plain.theta.grad.numpy(),
                plain.in_w.grad.numpy(), plain.in_b.grad.numpy(), plain.out.weight.grad.numpy().reshape(-1),
                plain.out.bias.grad.numpy()]
        for i in range(7):
            d = np.abs(grads[i].reshape(-1) - want[i]).max() / max(np.abs(want[i]).max(), 1e-30)
            assert d < 1e-5, (i, d)
        d = np.abs(acting.numpy() - lg.detach().numpy()).max() / np.abs(lg.detach().numpy()).max()
        assert d < 1e-5, d
        assert state["adam_t"] == 1 and len(stepped) == 7
    meta = {"network": "toy_h3 connectome (80 neurons, 3 hops, fan 5) as the reference's NativeFlyActor builds it",
            "max_batch": 32, "batch": 40, "declarations": rec.decl, "calls": rec.calls}
    buf = io.BytesIO()
    np.savez_compressed(buf, meta=np.frombuffer(json.dumps(meta).encode(), np.uint8),
                        net=np.frombuffer(rec.net_bytes, np.uint8), **{f"a{i}": a for i, a in enumerate(rec.arrays)})
    (HERE / "binding_toy_h3.npz").write_bytes(buf.getvalue())
    print(f"{len(rec.calls)} calls ({', '.join(sorted(set(c['fn'] for c in rec.calls)))}), {len(rec.arrays)} arrays, "
          f"{len(buf.getvalue()) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
