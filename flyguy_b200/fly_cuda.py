"""The per-hop autograd operator of the reference's CUDA path (flyguy/fly_cuda.py HopCuda, lines 78-115), on the
library's fg_hop_fwd / fg_hop_bwd instead of kernels compiled at run time by CuPy: the same arguments, the same
[neurons, batch] states, the same 16-bit mode (states read as fp16, sums in fp32, the gradient scaled by its largest
magnitude first). A maintainer points the reference's `from .fly_cuda import HopCuda` (flyguy/fly.py:172) here and
`FlyActor(kernel="cuda" | "cuda16")` runs without CuPy.
"""
from __future__ import annotations

import torch

from . import native


def available() -> bool:
    """Mirrors the reference's fly_cuda.available(): the library loads and a GPU is present."""
    try:
        native.lib()
    except native.FlyguyError:
        return False
    return torch.cuda.is_available()


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check(rc: int) -> None:
    if rc:
        raise native.FlyguyError(native.lib().fg_hop_last_error().decode())


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


class HopCuda(torch.autograd.Function):
    """z[target, b] = sum over connections (source -> target) of strength * h[source, b]; states are [neurons, batch].
    crow / col: the connections by target (CSR, int64 / int32); tcrow / tcol / tperm: the same by source."""

    @staticmethod
    def forward(ctx, w, h, crow, col, tcrow, tcol, tperm, half: bool):
        n_rows, batch = crow.numel() - 1, h.shape[1]
        if not (h.is_cuda and w.is_cuda):
            raise native.FlyguyError("HopCuda runs on CUDA tensors only (flyguy_b200 has no CPU path)")
        if batch % 32 or not h.is_contiguous():
            raise native.FlyguyError("HopCuda: h must be contiguous [neurons, batch] with batch a multiple of 32")
        w = w.detach().float().contiguous()
        h32 = h.detach().float().contiguous()
        out = torch.empty(n_rows, batch, device=h.device)
        _check(native.lib().fg_hop_fwd(_p(w), _p(h32), _p(crow), _p(col), n_rows, h.shape[0], batch, int(half),
                                       _p(out), _stream(h.device)))
        ctx.save_for_backward(w, h32, crow, col, tcrow, tcol, tperm)
        ctx.half = half
        return out

    @staticmethod
    def backward(ctx, gz):
        w, h, crow, col, tcrow, tcol, tperm = ctx.saved_tensors
        n_rows, batch = gz.shape
        gz = gz.detach().float().contiguous()
        gw = torch.empty_like(w) if ctx.needs_input_grad[0] else None
        gh = torch.empty(h.shape[0], batch, device=gz.device) if ctx.needs_input_grad[1] else None
        if gw is not None or gh is not None:
            _check(native.lib().fg_hop_bwd(_p(w), _p(h), _p(gz), _p(crow), _p(col), _p(tcrow), _p(tcol), _p(tperm),
                                           n_rows, h.shape[0], batch, int(ctx.half), _p(gw), _p(gh),
                                           _stream(gz.device)))
        return gw, gh, None, None, None, None, None, None
