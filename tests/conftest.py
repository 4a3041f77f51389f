"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on a CPU-only machine."""
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(REPO))

CASES = ["toy_h2", "toy_h3", "toy_h4", "toy_wide_h3", "syn_small"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libflyguy_b200.so")


def load_case(name: str):
    """(structure, params, fixture dict) of a golden case written by tests/golden/make_golden.py."""
    from flyguy_b200.netfile import read_net
    d = dict(np.load(GOLDEN / f"{name}.npz"))
    with tempfile.NamedTemporaryFile(suffix=".bin", delete=False) as fh:
        fh.write(d["net"].tobytes())
    s = read_net(fh.name)
    Path(fh.name).unlink()
    return s, [d[f"P{i}"] for i in range(7)], d


def rel(a, b) -> float:
    """max|a - b| / max|b| (the reference's parity measure, flyguy/hop_check.py:34-48)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)) if b.size else 0.0


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
