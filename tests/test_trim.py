"""Graph trimming (flyguy_b200.trim_graph) against the reference's own trim (fixture tests/golden/trim_wide.npz, made
by tests/golden/make_trim_golden.py with flyguy/trim_graph.py), on the CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from flyguy_b200 import trim_graph
from flyguy_b200.fly import FlyActor

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
from make_golden import toy_connectome  # noqa: E402


@pytest.fixture(scope="module")
def wide(tmp_path_factory):
    p = tmp_path_factory.mktemp("trim") / "wide.npz"
    toy_connectome(p, 700, 90, 40, 6000, seed=1)
    return p


@pytest.mark.parametrize("hops", [2, 3])
def test_trim_matches_reference(wide, tmp_path, hops):
    ref = np.load(GOLDEN / "trim_wide.npz")
    keep = trim_graph.trim(wide, tmp_path / "out.npz", hops, verbose=False)
    assert np.array_equal(keep, ref[f"keep_h{hops}"])
    g, whole = np.load(tmp_path / "out.npz"), np.load(wide)
    for k in ("pre", "post", "syn", "in_total", "hops", "whole_connections"):
        assert g[k].dtype == ref[f"{k}_h{hops}"].dtype and np.array_equal(g[k], ref[f"{k}_h{hops}"]), k
    for k in whole.files:                                    # everything else unchanged, neurons not renumbered
        if k not in ("pre", "post", "syn"):
            assert np.array_equal(g[k], whole[k]), k


def test_trimmed_graph_limits(wide, tmp_path):
    trim_graph.trim(wide, tmp_path / "h3.npz", 3, verbose=False)
    with pytest.raises(ValueError, match="trimmed already"):
        trim_graph.trim(tmp_path / "h3.npz", tmp_path / "again.npz", 3, verbose=False)
    a, b = FlyActor(wide, 16, 2, hops=2), FlyActor(tmp_path / "h3.npz", 16, 2, hops=2)   # fewer hops: the same network
    assert a.sizes == b.sizes
    for k in range(3):
        assert torch.equal(getattr(a, f"n{k}"), getattr(b, f"n{k}"))
    assert torch.allclose(a.w.detach()[getattr(a, "e1")], b.w.detach()[getattr(b, "e1")])
    with pytest.raises(ValueError, match="only the connections of a 3-hop network"):
        FlyActor(tmp_path / "h3.npz", 16, 2, hops=4)


def test_trim_weights_cuts_checkpoint(wide, tmp_path):
    torch.manual_seed(0)
    n_conn = len(np.load(wide)["pre"])
    cfg = {"fly_graph": str(wide), "fly_hops": 3, "fly_fan": 16}
    f = FlyActor(wide, 517, 90, hops=3, fan=16)
    sd = {"actor." + k: v.detach().clone() for k, v in f.state_dict().items()}
    sd["actor.w"] = torch.randn(n_conn)
    sd["critic.x"] = torch.ones(3)                         # other keys ride along unchanged
    torch.save({"model": sd, "steps": 7, "config": {"model": cfg, "other": 1}}, tmp_path / "in.pt")
    keep = trim_graph.trim(wide, tmp_path / "h3.npz", 3, verbose=False)
    worst = trim_graph.trim_weights(tmp_path / "in.pt", tmp_path / "out.pt", keep, str(tmp_path / "h3.npz"),
                                    verbose=False)
    new = torch.load(tmp_path / "out.pt", weights_only=False)
    assert torch.equal(new["model"]["actor.w"], sd["actor.w"][torch.as_tensor(keep)])
    assert torch.equal(new["model"]["critic.x"], sd["critic.x"]) and new["steps"] == 7
    assert new["config"]["model"] == dict(cfg, fly_graph=str(tmp_path / "h3.npz")) and new["config"]["other"] == 1
    if not torch.cuda.is_available():
        assert worst is None
    with pytest.raises(ValueError, match="not trained on that graph"):
        trim_graph.trim_weights(tmp_path / "out.pt", tmp_path / "bad.pt", keep, "x", verbose=False)


def test_trim_cli(wide, tmp_path, capsys):
    trim_graph.main([str(wide), str(tmp_path / "cli.npz"), "--hops", "2"])
    assert "of 6,000 connections for 2 hops" in capsys.readouterr().out
    assert int(np.load(tmp_path / "cli.npz")["hops"]) == 2
