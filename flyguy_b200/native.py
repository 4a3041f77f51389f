"""ctypes binding of libflyguy_b200.so (the C-ABI of include/flyguy_b200.h) and a torch-facing handle.

The library is loaded from the package directory (built in-tree by flyguy_b200/csrc/build.py). There is no CPU or
eager fallback: if the library is missing or fails to load, `lib()` raises.
"""
from __future__ import annotations

import ctypes
import os
import tempfile
from pathlib import Path

import numpy as np

from .netfile import Structure, read_net, write_net

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("FLYGUY_B200_LIB", PKG / "libflyguy_b200.so"))   # (override: a variant build)
FG_ACT_BF16, FG_INFER_ONLY, FG_ACT_F16 = 1, 2, 4
_lib = None

# the exported symbols and their ctypes signatures: (restype, argtypes)
_vp, _ci, _cf, _cll = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_longlong
SIGNATURES = {
    "fc_create": (_vp, [ctypes.c_char_p, _ci]),
    "fc_sizes": (None, [_vp, ctypes.POINTER(_cll)]),
    "fc_copy": (None, [_vp, _ci, _ci, ctypes.POINTER(_vp)]),
    "fc_forward": (None, [_vp, _vp, _ci, _vp, _ci]),
    "fc_zero_grad": (None, [_vp]),
    "fc_backward": (None, [_vp, _vp, _ci]),
    "fc_grad_norm": (_cf, [_vp]),
    "fc_step": (_cf, [_vp, _cf, _cf, _cf, _cf, _cf]),
    "fc_adam_t": (_cll, [_vp, _cll]),
    "fc_sync": (None, [_vp]),
    "fg_create": (_vp, [ctypes.c_char_p, _ci, _ci]),
    "fg_destroy": (None, [_vp]),
    "fg_status": (_ci, [_vp]),
    "fg_last_error": (ctypes.c_char_p, [_vp]),
    "fg_clear_error": (None, [_vp]),
    "fc_set_stream": (None, [_vp, _vp]),
    "fg_flat": (_ci, [_vp, _ci, ctypes.POINTER(_vp), ctypes.POINTER(_cll)]),
    "fg_offsets": (None, [_vp, ctypes.POINTER(_cll)]),
    "fg_layout": (_ci, [_vp, ctypes.POINTER(_ci), ctypes.POINTER(_cll)]),
    "fg_plan": (_ci, [_vp, ctypes.POINTER(_cll), _ci]),
    "fg_grad_buckets": (_ci, [_vp, ctypes.POINTER(_cll), _ci]),
    "fg_set_stage_event": (_ci, [_vp, _ci, _vp]),
    "fg_grad_pack": (_cll, [_vp, _vp, _cll, _ci]),
    "fg_teach": (_ci, [_vp, _vp, _vp, _ci, _cf, _vp, ctypes.POINTER(ctypes.c_double)]),
    "fg_teach_ex": (_ci, [_vp, _vp, _vp, _ci, _cf, _cf, _vp, ctypes.POINTER(ctypes.c_double)]),
    "fg_forward_host": (_ci, [_vp, _vp, _ci, _vp, _ci]),
    "fg_layer": (_ci, [_vp, _ci, _vp, _ci]),
    "fg_launches": (_cll, [_vp]),
    "fg_timing": (_ci, [_vp, _ci]),
    "fg_timing_classes": (_ci, [_vp, ctypes.c_uint]),
    "fg_timing_read": (_ci, [_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_cll), _ci]),
    "fg_kl_loss_noalloc": (_ci, [_vp, _vp, _ci, _ci, _cf, _vp, _vp, _vp]),
    "fg_noalloc_last_error": (ctypes.c_char_p, []),
    "fg_hop_fwd": (_ci, [_vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _vp, _vp]),
    "fg_hop_bwd": (_ci, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _vp, _vp, _vp]),
    "fg_hop_last_error": (ctypes.c_char_p, []),
    "fg_train_main": (_ci, [_ci, ctypes.POINTER(ctypes.c_char_p)]),
    "fg_survey": (_ci, [_vp, _vp, _vp, _ci, _ci, _vp, _vp, ctypes.POINTER(ctypes.c_double)]),
    "fly_create": (_vp, [_ci, _ci, _ci]),
    "fly_set_plug": (None, [_vp, _ci, _ci] + [_vp] * 6),
    "fly_set_hop": (None, [_vp, _ci, _ci, _ci, _ci] + [_vp] * 6),
    "fly_set_out": (None, [_vp, _ci, _vp, _vp, _vp]),
    "fly_forward": (None, [_vp, _vp, _ci, _vp, _vp]),
    "fly_free": (None, [_vp]),
    "fg_fly_last_error": (ctypes.c_char_p, []),
}
KERNEL_CLASSES = ("layout", "fold", "plug_fwd", "hop_fwd", "out_fwd", "loss", "out_bwd", "act_bwd", "wgrad",
                  "hop_bwd_t", "plug_bwd", "adam", "norm")


class FlyguyError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it is not built or does not load."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FlyguyError(f"{LIB_PATH} is not built: run `python -m flyguy_b200.csrc.build` (or "
                              "__graft_entry__.build()); flyguy_b200 has no fallback path")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


class Handle:
    """One network in the library, bound to torch tensors on one CUDA device.

    Arrays are exchanged as torch CUDA tensors (fp32, contiguous). `flags` 0: fp32 states, training buffers;
    FG_ACT_BF16: bf16 states, forward only; FG_INFER_ONLY: fp32 states, forward only."""

    def __init__(self, s: Structure | str | Path, max_batch: int, flags: int = 0, device=None):
        """s: a Structure, or the path of a NET.bin file."""
        import torch
        self.torch = torch
        self.L = lib()
        self.max_batch, self.flags = int(max_batch), int(flags)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        with torch.cuda.device(self.device), tempfile.TemporaryDirectory() as tmp:
            if isinstance(s, (str, Path)):
                path = Path(s)
                s = read_net(path)
            else:
                path = Path(tmp) / "net.bin"
                write_net(s, path)
            self.s = s
            torch.cuda.synchronize()
            self.h = self.L.fg_create(str(path).encode(), self.max_batch, self.flags)
        if not self.h:
            raise FlyguyError(f"fg_create: {self.L.fg_last_error(None).decode()}")
        sizes = (ctypes.c_longlong * 10)()
        self.L.fc_sizes(self.h, sizes)
        self.sizes = [int(v) for v in sizes[:7]]
        off = (ctypes.c_longlong * 8)()
        self.L.fg_offsets(self.h, off)
        self.offsets = [int(v) for v in off]
        self.check()

    # ---- plumbing
    def check(self) -> None:
        if self.L.fg_status(self.h):
            msg = self.L.fg_last_error(self.h).decode()
            self.L.fg_clear_error(self.h)
            raise FlyguyError(msg)

    def bind_stream(self) -> None:
        self.L.fc_set_stream(self.h, self.torch.cuda.current_stream(self.device).cuda_stream)

    def close(self) -> None:
        if getattr(self, "h", None):
            self.L.fg_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def flat(self, which: int):
        """The library's flat array (0 weights, 1 average, 2 m, 3 v, 4 gradient) as a zero-copy torch tensor."""
        p, n = ctypes.c_void_p(), ctypes.c_longlong()
        if self.L.fg_flat(self.h, which, ctypes.byref(p), ctypes.byref(n)):
            self.check()
        return _wrap(p.value, int(n.value), self.device)

    def layout(self):
        sizes = (ctypes.c_int * 64)()
        pairs = (ctypes.c_longlong * 64)()
        K = self.L.fg_layout(self.h, sizes, pairs)
        self.check()
        return [int(v) for v in sizes[:K + 1]], [int(v) for v in pairs[:K]]

    def plan(self) -> dict:
        """The work plan's counts (fg_plan): per hop {rows, n_src, edges, pairs, tpairs, live_dst, live_src,
        live_edges}, and the plug backward's live sensory rows."""
        buf = (ctypes.c_longlong * 512)()
        n = self.L.fg_plan(self.h, buf, 512)
        self.check()
        keys = ("rows", "n_src", "edges", "pairs", "tpairs", "live_dst", "live_src", "live_edges")
        hops = [{k: int(buf[8 * i + j]) for j, k in enumerate(keys)} for i in range((n - 4) // 8)]
        t = n - 4
        return {"hops": hops, "plug_live": int(buf[t]), "n_s": int(buf[t + 1]), "fan": int(buf[t + 2]),
                "n_dn": int(buf[t + 3])}

    def grad_pack(self, buf=None, unpack: bool = False) -> int:
        """fg_grad_pack: the gradient without its structural zeros into `buf` (a float32 device tensor; unpack: back
        from it). Without buf, the packed length."""
        self.bind_stream()
        if buf is None:
            n = self.L.fg_grad_pack(self.h, None, 0, 0)
        else:
            if buf.dtype != self.torch.float32 or not buf.is_contiguous() or buf.device != self.device:
                raise FlyguyError("grad_pack: buf must be a contiguous float32 tensor on the handle's device")
            n = self.L.fg_grad_pack(self.h, buf.data_ptr(), buf.numel(), 1 if unpack else 0)
        if n < 0:
            self.check()
        return int(n)

    def grad_buckets(self) -> list[tuple[int, int, int]]:
        """(first, end, stage) ranges of the flat gradient (fg_grad_buckets): stage s >= 0 final once the backward
        reaches stage s, -1 at its end."""
        buf = (ctypes.c_longlong * 96)()
        n = self.L.fg_grad_buckets(self.h, buf, 32)
        self.check()
        return [(int(buf[3 * i]), int(buf[3 * i + 1]), int(buf[3 * i + 2])) for i in range(n)]

    def set_stage_event(self, stage: int, event) -> None:
        """Record `event` (a torch.cuda.Event, or None) when the backward reaches `stage` (fg_set_stage_event)."""
        handle = None
        if event is not None:
            event.record()                                    # (creates the underlying CUDA event)
            handle = event.cuda_event
        if self.L.fg_set_stage_event(self.h, int(stage), handle):
            self.check()

    # ---- weights
    def set_params(self, params, which: int = 0) -> None:
        torch = self.torch
        ts = [torch.as_tensor(np.asarray(p, np.float32).reshape(-1)).to(self.device) for p in params]
        assert [t.numel() for t in ts] == self.sizes, "weights do not fit this network"
        self.copy(which, 1, ts)

    def copy(self, which: int, to_core: int, tensors) -> None:
        for t in tensors:
            if t is not None:
                assert t.is_cuda and t.is_contiguous() and t.dtype == self.torch.float32
        arr = (ctypes.c_void_p * 7)(*[_ptr(t) for t in tensors])
        self.bind_stream()
        self.L.fc_copy(self.h, which, to_core, arr)
        self.check()

    def get(self, which: int):
        out = [self.torch.empty(n, device=self.device) for n in self.sizes]
        self.copy(which, 0, out)
        return out

    # ---- compute
    def forward(self, obs, ema: int = 0, out=None):
        torch = self.torch
        B = obs.shape[0]
        out = torch.empty(B, self.s["n_act"], device=self.device) if out is None else out
        self.bind_stream()
        self.L.fc_forward(self.h, _ptr(obs), B, _ptr(out), ema)
        self.check()
        return out

    def backward(self, dlogits) -> None:
        self.bind_stream()
        self.L.fc_backward(self.h, _ptr(dlogits), dlogits.shape[0])
        self.check()

    def zero_grad(self) -> None:
        self.bind_stream()
        self.L.fc_zero_grad(self.h)
        self.check()

    def step(self, lr, lr_neuron, lr_plug, max_norm=0.0, ema=0.999) -> float:
        self.bind_stream()
        g = self.L.fc_step(self.h, lr, lr_neuron, lr_plug, max_norm, ema)
        self.check()
        return float(g)

    def grad_norm(self) -> float:
        self.bind_stream()
        g = self.L.fc_grad_norm(self.h)
        self.check()
        return float(g)

    def adam_t(self, set_to: int = -1) -> int:
        v = self.L.fc_adam_t(self.h, int(set_to))
        self.check()
        return int(v)

    def teach(self, obs, teacher, inv_temp: float = 1.0, logits=None, stats: bool = True, loss_norm: float = 0.0):
        """Fused forward + KL loss + backward (gradient ADDED); loss_norm: samples the loss averages over (0: B)."""
        self.bind_stream()
        st = (ctypes.c_double * 2)() if stats else None
        rc = self.L.fg_teach_ex(self.h, _ptr(obs), _ptr(teacher), obs.shape[0], float(inv_temp),
                                float(loss_norm or obs.shape[0]), _ptr(logits), st)
        if rc:
            self.check()
        return (float(st[0]), float(st[1])) if stats else None

    def forward_host(self, obs_host, logits_host, ema: int = 0) -> None:
        """obs_host / logits_host: contiguous CPU tensors (pinned for overlap)."""
        self.bind_stream()
        rc = self.L.fg_forward_host(self.h, obs_host.data_ptr(), obs_host.shape[0], logits_host.data_ptr(), ema)
        if rc:
            self.check()

    def survey(self, obs, teacher=None, ema: int = 0, fired=None, sq=None):
        """The firing survey of one batch (fg_survey): per row of every layer the samples whose state is positive and
        the sum of the squared pre-activations, ADDED to fired / sq (int32 / float32 [sum of layer sizes], made when
        None); with teacher, (KL sum, agreements) at temperature 1 as the third result."""
        R = int(sum(self.s["sizes"]))
        if fired is None:
            fired = self.torch.zeros(R, dtype=self.torch.int32, device=self.device)
        if sq is None:
            sq = self.torch.zeros(R, dtype=self.torch.float32, device=self.device)
        st = (ctypes.c_double * 2)() if teacher is not None else None
        self.bind_stream()
        if self.L.fg_survey(self.h, _ptr(obs), _ptr(teacher), obs.shape[0], ema, _ptr(fired), _ptr(sq), st):
            self.check()
        return fired, sq, ((float(st[0]), float(st[1])) if st is not None else None)

    def layer(self, k: int, B: int):
        rows = self.s["sizes"][k]
        out = self.torch.empty(rows, B, device=self.device)
        self.bind_stream()
        if self.L.fg_layer(self.h, k, _ptr(out), B):
            self.check()
        return out

    def launches(self) -> int:
        return int(self.L.fg_launches(self.h))

    def timing(self, on: bool, classes=None) -> None:
        """Per-launch CUDA-event timing: of every kernel class, or of the named ones (KERNEL_CLASSES) only."""
        if on and classes is not None:
            mask = 0
            for k in classes:
                mask |= 1 << KERNEL_CLASSES.index(k)
            rc = self.L.fg_timing_classes(self.h, mask)
        else:
            rc = self.L.fg_timing(self.h, int(on))
        if rc:
            self.check()

    def timing_read(self) -> dict:
        """{kernel class: (milliseconds, launches)} since the last read."""
        n = len(KERNEL_CLASSES)
        ms, cnt = (ctypes.c_double * n)(), (ctypes.c_longlong * n)()
        if self.L.fg_timing_read(self.h, ms, cnt, n) < 0:
            self.check()
        return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(KERNEL_CLASSES)}

    def sync(self) -> None:
        self.L.fc_sync(self.h)
        self.check()


class _CudaArray:
    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _wrap(ptr: int, n: int, device):
    import torch
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaArray(ptr, n), device=device)


def kl_loss_noalloc(logits, teacher, inv_temp: float, dlogits, stats, stream=None) -> None:
    """KL loss and its gradient without any device allocation (fg_kl_loss_noalloc): logits, teacher, dlogits [B, n_act]
    and stats [2] are caller-owned CUDA fp32 tensors; the work is queued on `stream` (default: torch's current)."""
    import torch
    named = {"logits": logits, "teacher": teacher, "dlogits": dlogits, "stats": stats}
    for k, t in named.items():
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise FlyguyError(f"{k} must be a contiguous float32 CUDA tensor")
        if t.device != logits.device:
            raise FlyguyError(f"{k} is on {t.device}, logits on {logits.device}")
    if logits.dim() != 2 or teacher.shape != logits.shape or dlogits.shape != logits.shape:
        raise FlyguyError(f"logits, teacher and dlogits must share one [B, n_act] shape "
                          f"(got {tuple(logits.shape)}, {tuple(teacher.shape)}, {tuple(dlogits.shape)})")
    if stats.numel() < 2:
        raise FlyguyError("stats needs room for 2 floats")
    L = lib()
    with torch.cuda.device(logits.device):                     # the entry point works on the current device
        st = (stream or torch.cuda.current_stream(logits.device)).cuda_stream
        rc = L.fg_kl_loss_noalloc(logits.data_ptr(), teacher.data_ptr(), logits.shape[0], logits.shape[1],
                                  float(inv_temp), dlogits.data_ptr(), stats.data_ptr(), st)
    if rc:
        raise FlyguyError(L.fg_noalloc_last_error().decode())


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def header_symbols(path: Path | None = None) -> list[str]:
    """The entry points include/flyguy_b200.h declares."""
    import re
    path = path or PKG.parent / "include" / "flyguy_b200.h"
    text = Path(path).read_text()
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b((?:fc|fg|fly)_\w+)\s*\(", text, re.M)))


def default_threads() -> int:
    return os.cpu_count() or 1
