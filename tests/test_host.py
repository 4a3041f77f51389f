"""The reference-facing host code on the CPU: FlyActor's structure (byte-identical NET.bin to the reference's), its
checkpoint layout, dist.mean_ over two gloo ranks, and a missing rank detected on the host."""
import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import GOLDEN, REPO

sys.path.insert(0, str(GOLDEN))
from make_golden import toy_connectome  # noqa: E402  (the fixture script's own made-up connectome)

from flyguy_b200 import netfile, synth  # noqa: E402
from flyguy_b200.fly import FlyActor  # noqa: E402


@pytest.fixture(scope="module")
def toys(tmp_path_factory):
    d = tmp_path_factory.mktemp("toys")
    toy_connectome(d / "toy.npz", 80, 14, 7, 420, seed=0)
    toy_connectome(d / "wide.npz", 700, 90, 40, 6000, seed=1)
    return d


@pytest.mark.parametrize("case,graph,hops,fan", [("toy_h2", "toy.npz", 2, 5), ("toy_h3", "toy.npz", 3, 5),
                                                 ("toy_h4", "toy.npz", 4, 5), ("toy_wide_h3", "wide.npz", 3, 8)])
def test_structure_is_byte_identical_to_the_references(toys, tmp_path, case, graph, hops, fan):
    """The structure this FlyActor builds from a connectome writes the same NET.bin as the reference's FlyActor
    (the golden file was written by the reference's export.write_net) - same layers, CSR orders, plug wiring."""
    f = FlyActor(toys / graph, 517, 90, hops=hops, fan=fan)
    s = netfile.structure_of_actor(f)
    netfile.write_net(s, tmp_path / "n.bin")
    want = np.load(GOLDEN / f"{case}.npz")["net"].tobytes()
    assert (tmp_path / "n.bin").read_bytes() == want


def test_checkpoint_layout(toys):
    f = FlyActor(toys / "toy.npz", 517, 90, hops=3, fan=5)
    sd = f.state_dict()
    assert set(sd) == {"w", "gain", "theta", "in_w", "in_b", "out.weight", "out.bias"}
    assert sd["w"].shape == (f.n_conn,) and sd["gain"].shape == (f.n_neurons,)
    assert sd["in_w"].shape == (f.sizes[0] * 5,) and sd["out.weight"].shape == (90, len(f.dn_rows))
    g = FlyActor(toys / "toy.npz", 517, 90, hops=3, fan=5)
    g.load_state_dict(sd)
    assert "fly network" in f.describe() and str(f.used) not in ("", "0")


def test_cpu_forward_is_refused(toys):
    f = FlyActor(toys / "toy.npz", 517, 90, hops=3, fan=5)
    with pytest.raises(RuntimeError, match="GPU"):
        f(torch.zeros(2, 517))


def test_trimmed_hops_refused(toys, tmp_path):
    """A trimmed graph file holds one hop count's connections; more hops are refused (flyguy/fly.py:131)."""
    g = dict(np.load(toys / "toy.npz"))
    g["in_total"], g["hops"] = np.ones(80, np.float32), np.array(2)
    np.savez(tmp_path / "trim.npz", **g)
    with pytest.raises(ValueError, match="2-hop network"):
        FlyActor(tmp_path / "trim.npz", 517, 90, hops=3, fan=5)


# ------------------------------------------------------------------ several ranks (gloo on the CPU)
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mean_worker(rank, world, port, out):
    import torch.distributed as td
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    td.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    from flyguy_b200 import dist
    assert dist.on()
    a = torch.full((1000,), float(rank + 1))
    b = torch.arange(7, dtype=torch.float32) * (rank + 1)
    dist.mean_([a, b])
    torch.save({"a": a, "b": b}, Path(out) / f"r{rank}.pt")
    td.destroy_process_group()


def test_dist_mean_over_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_mean_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        d = torch.load(tmp_path / f"r{r}.pt")
        assert torch.allclose(d["a"], torch.full((1000,), 1.5))
        assert torch.allclose(d["b"], torch.arange(7, dtype=torch.float32) * 1.5)


class _FakePackHandle:
    """The host side of fg_grad_pack on the CPU: a flat gradient whose entries 0..63 outside `idx` are structural
    zeros, packed as flat[idx] then flat[64:] (the library's layout: the strengths that can change, then the rest)."""

    def __init__(self, rank):
        self.device = torch.device("cpu")
        self.idx = torch.tensor([3, 5, 17, 40, 41, 63])
        self.g = torch.zeros(100)
        self.g[self.idx] = torch.arange(6, dtype=torch.float32) * (rank + 1)
        self.g[64:] = torch.linspace(-1, 1, 36) * (rank + 1)

    def flat(self, which):
        return self.g

    def grad_pack(self, buf=None, unpack=False):
        n = len(self.idx) + 36
        if buf is None:
            return n
        if unpack:
            self.g[self.idx] = buf[:len(self.idx)]
            self.g[64:] = buf[len(self.idx):n]
        else:
            buf[:len(self.idx)] = self.g[self.idx]
            buf[len(self.idx):n] = self.g[64:]
        return n


def _packed_worker(rank, world, port, out):
    import torch.distributed as td
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    td.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    from flyguy_b200 import dist
    h = _FakePackHandle(rank)
    mean = dist.PackedMean(h)
    assert mean.n == 42 and mean.worth_it()
    mean()
    torch.save(h.g, Path(out) / f"r{rank}.pt")
    td.destroy_process_group()


def test_dist_packed_mean_over_two_gloo_ranks(tmp_path):
    """dist.PackedMean: pack, all-reduce (average), unpack - the same mean as all-reducing the whole flat gradient, and
    the structural zeros left out stay zero."""
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_packed_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    want = (_FakePackHandle(0).g + _FakePackHandle(1).g) / 2
    for r in range(world):
        got = torch.load(tmp_path / f"r{r}.pt")
        assert torch.allclose(got, want)
        assert torch.count_nonzero(got[:64]) == 5          # idx entries (the first is 0 * 1.5) and nothing else


def test_dist_off_without_a_group():
    from flyguy_b200 import dist
    t = torch.ones(3)
    assert not dist.on()
    dist.mean_([t])
    assert torch.equal(t, torch.ones(3))


def _lonely_worker(rank, world, port, out):
    """Rank 0 of a world of 2 whose peer never joins: the rendezvous times out with an error, on the host."""
    import torch.distributed as td
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        td.init_process_group("gloo", rank=0, world_size=2, timeout=timedelta(seconds=3))
        Path(out, "joined").write_text("unexpected")
    except Exception as e:                                   # noqa: BLE001
        Path(out, "error").write_text(type(e).__name__ + ": " + str(e)[:200])


def test_missing_rank_is_detected_on_the_host(tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_lonely_worker, args=(1, _free_port(), str(tmp_path)), nprocs=1, start_method="spawn")
    assert (tmp_path / "error").exists() and not (tmp_path / "joined").exists()


def test_flyd_chunk_round_trip(tmp_path):
    obs, teacher = synth.make_batch(50, seed=8)
    netfile.write_chunk(obs, teacher, tmp_path / "chunk_000.bin")
    o2, t2 = netfile.read_chunk(tmp_path / "chunk_000.bin")
    assert np.array_equal(o2, obs.astype(np.float16)) and np.array_equal(t2, teacher.astype(np.float16))
    raw = (tmp_path / "chunk_000.bin").read_bytes()
    assert raw[:4] == b"FLYD" and len(raw) == 20 + 2 * 50 * (517 + 90)


def test_trainer_argument_errors_exit_without_a_gpu():
    """fg_train_main reads its command line before touching the GPU: usage and bad options are exit status 1."""
    from flyguy_b200 import train
    assert train.main([]) == 1
    assert train.main(["a", "b", "c", "d", "--batch", "33"]) == 1
    assert train.main(["a", "b", "c", "d", "--bogus", "1"]) == 1
