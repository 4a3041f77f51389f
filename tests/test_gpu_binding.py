"""The drop-in boundary driven by the reference's OWN binding: the fc_* calls that the reference's NativeFlyActor /
NativeAdam / grad_arrays (flyguy/fly_native.py:34-215) made in a recorded training step - with the argtypes and
restypes it declares (fly_native.py:135-145), in its order, with its buffers - are replayed against
libflyguy_b200.so on the GPU, and every value the library hands back is compared with what a correct library returns
(the CPU oracle's values in the recording, whose gradient was checked against the reference's torch autograd when the
recording was made: tests/golden/make_binding_golden.py).

What the recorded step covers: fc_create on the reference's own NET.bin (export.write_net) and fc_sizes (the size
check of fly_native.py:155), push of the weights and of the running average (fc_copy to the library), forward
without gradients in two pieces of max_batch = 32 (40 samples, the second piece padded by repeating the last row),
zero_grad, the learning forward, backward (each piece forwarded again, then fc_backward), grad_arrays (fc_copy of
the gradient out), NativeAdam.step (fc_step with the rates lr, 0.3 lr, lr, clipping at 1.0, average 0.999, then pull)
and NativeAdam.state_dict (fc_adam_t, and the running average, m and v fetched)."""
import ctypes
import json
import tempfile
from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN, rel
from flyguy_b200 import native

pytestmark = pytest.mark.gpu

CTYPES = {"c_void_p": ctypes.c_void_p, "c_char_p": ctypes.c_char_p, "c_int": ctypes.c_int,
          "c_float": ctypes.c_float, "c_long": ctypes.c_long, "c_longlong": ctypes.c_longlong,
          "LP_c_long": ctypes.POINTER(ctypes.c_long), "LP_c_longlong": ctypes.POINTER(ctypes.c_longlong),
          "LP_c_void_p": ctypes.POINTER(ctypes.c_void_p), None: None}


def _declared(meta):
    """libflyguy_b200.so loaded the way the reference loads its library: ctypes.CDLL by path, with the reference's
    declarations (a CDLL object of its own, so nothing else's declarations interfere)."""
    lib = ctypes.CDLL(str(native.LIB_PATH))
    for name, d in meta["declarations"].items():
        f = getattr(lib, name)
        f.restype = CTYPES[d["restype"]]
        f.argtypes = [CTYPES[t] for t in d["argtypes"]]
    return lib


def test_reference_binding_replays_against_this_library(cuda):
    import torch
    d = np.load(GOLDEN / "binding_toy_h3.npz")
    meta = json.loads(d["meta"].tobytes())
    A = [d[f"a{i}"] for i in range(sum(k.startswith("a") for k in d.files))]
    lib = _declared(meta)
    with tempfile.TemporaryDirectory() as tmp:
        net = Path(tmp) / "net.bin"
        net.write_bytes(d["net"].tobytes())
        core = None
        sizes = None
        checked = {}
        pushed = next(c for c in meta["calls"] if c["fn"] == "fc_copy" and c["scalars"] == [0, 1])["in"]
        for i, c in enumerate(meta["calls"]):
            fn, sc = c["fn"], c["scalars"]
            ins = {k: torch.as_tensor(A[v]).to(cuda).contiguous() for k, v in c["in"].items()}
            want = {k: A[v] for k, v in c["out"].items()}
            where = f"call {i} {fn}{tuple(sc)}"
            if fn == "fc_create":
                torch.cuda.synchronize()
                core = lib.fc_create(str(net).encode(), sc[0])
                assert core, f"{where}: {native.lib().fg_last_error(None).decode()}"
                continue
            if fn == "fc_sizes":
                buf = (ctypes.c_long * 10)()
                lib.fc_sizes(core, buf)
                assert list(buf) == list(want["sizes"]), where
                sizes = [int(v) for v in buf[:7]]
                continue
            if fn == "fc_copy":
                which, to_core = sc
                ts = [ins[f"p{j}"] for j in range(7)] if to_core else \
                    [torch.full((n,), float("nan"), device=cuda) for n in sizes]
                lib.fc_copy(core, which, to_core, (ctypes.c_void_p * 7)(*[t.data_ptr() for t in ts]))
                torch.cuda.synchronize()
                if not to_core:
                    tol = {0: 1e-5, 1: 1e-5, 2: 1e-4, 3: 1e-3, 4: 1e-4}[which]
                    for j in range(7):
                        got = ts[j].cpu().numpy()
                        if which == 0:                   # stepped weights: compare the Adam update itself
                            before = A[pushed[f"p{j}"]]
                            assert rel(got - before, want[f"p{j}"] - before) < 1e-3, (where, j)
                        else:
                            assert rel(got, want[f"p{j}"]) < tol, (where, j)
                    checked[f"fc_copy{which}"] = True
            elif fn == "fc_forward":
                out = torch.full((sc[0], want["logits"].shape[1]), float("nan"), device=cuda)
                lib.fc_forward(core, ins["obs"].data_ptr(), sc[0], out.data_ptr(), sc[1])
                torch.cuda.synchronize()
                got = out.cpu().numpy()
                assert rel(got, want["logits"]) < 1e-5, where
                assert (got.argmax(1) == want["logits"].argmax(1)).all(), where
                checked["fc_forward"] = checked.get("fc_forward", 0) + 1
            elif fn == "fc_zero_grad":
                lib.fc_zero_grad(core)
            elif fn == "fc_backward":
                lib.fc_backward(core, ins["dlogits"].data_ptr(), sc[0])
            elif fn == "fc_step":
                n = lib.fc_step(core, *sc)
                torch.cuda.synchronize()
                assert abs(n - c["ret"]) <= 1e-4 * abs(c["ret"]), (where, n, c["ret"])
            elif fn == "fc_adam_t":
                assert lib.fc_adam_t(core, sc[0]) == c["ret"], where
            else:
                raise AssertionError(f"unexpected call {fn}")
            assert native.lib().fg_status(core) == 0, native.lib().fg_last_error(core).decode()
        native.lib().fg_destroy(core)
    assert checked.get("fc_forward", 0) == 6 and all(checked.get(f"fc_copy{w}") for w in (0, 1, 2, 3, 4)), checked
