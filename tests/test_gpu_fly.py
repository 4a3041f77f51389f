"""The fly_* interface on the GPU (csrc/fg_fly.cu) against the reference's own CPU library (flyguy/native/
fly_infer.cpp, compiled from its source into oracle/_ref): the same arrays - built as FlyActor._native builds them -
give the same logits and the same visualizer bytes for batches of 1, 7 and 64 cars, on graphs with duplicate
connections, shared weights and sensory re-drive."""
import ctypes

import numpy as np
import pytest

from conftest import REPO, load_case, rel
from flyguy_b200 import synth
from flyguy_b200.play import Player

pytestmark = pytest.mark.gpu
REF = REPO / "oracle" / "_ref" / "libfly_infer.so"


@pytest.mark.parametrize("graph", ["syn", "toy_h3", "toy_h4"])
def test_fly_interface_matches_reference_cpu_library(graph, cuda):
    if not REF.exists():
        pytest.skip("oracle/_ref/libfly_infer.so is not built (make -C oracle)")
    if graph == "syn":
        s, P = synth.make_synthetic(sizes=(300, 600, 500, 120), total_edges=20000, seed=3)
    else:
        s, P, _ = load_case(graph)
    gpu = Player(s, P)
    cpu = Player(s, P, lib=ctypes.CDLL(str(REF)))
    for B in (1, 7, 64):
        obs, _ = synth.make_batch(B, seed=100 + B)
        lg, tap = gpu.forward(obs, tap=True)
        want, want_tap = cpu.forward(obs, tap=True)
        assert rel(lg, want) < 1e-6, (graph, B)
        assert (lg.argmax(1) == want.argmax(1)).all()
        d = np.abs(tap.astype(np.int32) - want_tap.astype(np.int32))
        assert d.max() <= 1 and (d == 0).mean() > 0.999, (graph, B)
