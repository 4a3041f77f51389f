"""The C-ABI library without a GPU: it loads, exports every entry point include/flyguy_b200.h declares, and turns bad
input into an error status instead of ending the process. No compute calls here."""
import ctypes
import subprocess

import numpy as np
import pytest

from conftest import REPO
from flyguy_b200 import native, netfile, synth


def test_library_loads_and_exports_the_header():
    L = native.lib()
    declared = native.header_symbols()
    assert set(declared) == set(native.exported_symbols())
    for name in declared:
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(native.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(declared) <= exported


def test_reference_binding_names_are_all_there():
    """Every symbol the reference's ctypes binding sets up (flyguy/fly_native.py:137-145) exists with that name."""
    for name in ("fc_create", "fc_sizes", "fc_copy", "fc_forward", "fc_zero_grad", "fc_backward", "fc_grad_norm",
                 "fc_step", "fc_adam_t"):
        assert name in native.exported_symbols()


def _create(path, max_batch=64, flags=0):
    L = native.lib()
    h = L.fg_create(str(path).encode(), max_batch, flags)
    return h, L.fg_last_error(None).decode()


def test_corrupt_network_file_is_an_error_not_an_exit(tmp_path):
    s, _ = synth.make_synthetic(sizes=(40, 60, 50, 10), total_edges=900, seed=1)
    good = tmp_path / "good.bin"
    netfile.write_net(s, good)
    raw = bytearray(good.read_bytes())
    cases = {
        "magic": b"FLY9" + raw[4:],
        "short": raw[: len(raw) // 2],
        "trailing": raw + b"\0\0\0\0",
        "index": None,
    }
    bad_col = netfile.Structure(s)
    bad_col["hop"] = [dict(h) for h in s["hop"]]
    bad_col["hop"][1]["col"] = bad_col["hop"][1]["col"].copy()
    bad_col["hop"][1]["col"][3] = 10_000                     # a source beyond the layer
    for name, data in cases.items():
        p = tmp_path / f"{name}.bin"
        if data is None:
            netfile.write_net(bad_col, p)
        else:
            p.write_bytes(bytes(data))
        h, msg = _create(p)
        assert not h and "NET.bin" in msg, (name, msg)
    h, msg = _create(tmp_path / "missing.bin")
    assert not h and "cannot open" in msg


def test_bad_max_batch_is_an_error(tmp_path):
    s, _ = synth.make_synthetic(sizes=(40, 60, 50, 10), total_edges=900, seed=1)
    netfile.write_net(s, tmp_path / "n.bin")
    h, msg = _create(tmp_path / "n.bin", max_batch=33)
    assert not h and "multiple of 32" in msg


def test_null_handle_calls_do_not_crash():
    L = native.lib()
    L.fc_zero_grad(None)
    assert L.fg_teach(None, None, None, 32, 1.0, None, None) == -1


def test_hop_operator_argument_errors_are_statuses():
    """fg_hop_fwd / fg_hop_bwd check their arguments before any GPU work: a bad batch or a missing buffer is -1 and a
    message, never a crash."""
    L = native.lib()
    assert L.fg_hop_fwd(None, None, None, None, 10, 10, 33, 0, None, None) == -1
    assert "multiple of 32" in L.fg_hop_last_error().decode()
    assert L.fg_hop_fwd(None, None, None, None, 10, 10, 64, 0, None, None) == -1
    assert "null pointer" in L.fg_hop_last_error().decode()
    assert L.fg_hop_bwd(None, None, None, None, None, None, None, None, -1, 10, 64, 0, None, None, None) == -1
    assert "negative" in L.fg_hop_last_error().decode()


def test_noalloc_wrapper_checks_its_tensors():
    """kl_loss_noalloc refuses, before any device call, tensors the entry point would write out of bounds of or read
    on the wrong device: non-CUDA, non-fp32, non-contiguous, mismatched shapes, a too-small stats buffer."""
    import torch
    from flyguy_b200 import native
    x = torch.zeros(32, 90)
    with pytest.raises(native.FlyguyError, match="CUDA tensor"):
        native.kl_loss_noalloc(x, x, 1.0, x, torch.zeros(2))


def test_reference_binding_fixture_names_exported_entry_points():
    """The recorded binding (tests/golden/binding_toy_h3.npz, made from the reference's fly_native.py) declares only
    entry points this library exports and include/flyguy_b200.h declares."""
    import json
    from conftest import GOLDEN
    d = np.load(GOLDEN / "binding_toy_h3.npz")
    meta = json.loads(d["meta"].tobytes())
    lib = ctypes.CDLL(str(native.LIB_PATH))
    declared = set(native.header_symbols())
    for name in meta["declarations"]:
        assert hasattr(lib, name) and name in declared, name
    assert {c["fn"] for c in meta["calls"]} >= {"fc_create", "fc_sizes", "fc_copy", "fc_forward", "fc_backward",
                                                  "fc_zero_grad", "fc_step", "fc_adam_t"}
