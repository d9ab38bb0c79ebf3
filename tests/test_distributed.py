"""Multi-process host logic on CPU (gloo, world size 2): token-sharded
calibration accumulators are merged with one all-reduce."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mxwave_b200.calibration import ActivationCollector
from mxwave_b200.calibration_stream import _shard_bounds


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        col = ActivationCollector({"a.weight": 64, "b.weight": 32}, ("mean-abs", "rms", "block-hessian"))
        # Rank r observed 10*(r+1) tokens of a.weight; only rank 0 observed b.weight.
        col._counts["a.weight"] = 10 * (rank + 1)
        col._absolute_sums["a.weight"] = torch.full((64,), float(rank + 1))
        col._square_sums["a.weight"] = torch.full((64,), float(rank + 2))
        col._gram_sums["a.weight"] = torch.full((2, 32, 32), float(rank + 3))
        if rank == 0:
            col._counts["b.weight"] = 5
            col._absolute_sums["b.weight"] = torch.arange(32, dtype=torch.float32)
            col._square_sums["b.weight"] = torch.ones(32)
            col._gram_sums["b.weight"] = torch.eye(32).unsqueeze(0)
        col.all_reduce(device=torch.device("cpu"))
        torch.save({"counts": col.observation_counts, "abs_a": col._absolute_sums["a.weight"],
                    "sq_a": col._square_sums["a.weight"], "gram_a": col._gram_sums["a.weight"],
                    "abs_b": col._absolute_sums["b.weight"], "gram_b": col._gram_sums["b.weight"]},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_collector_all_reduce_over_two_gloo_ranks(tmp_path) -> None:
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for rank in range(2):
        r = torch.load(tmp_path / f"rank{rank}.pt")
        assert r["counts"] == {"a.weight": 30, "b.weight": 5}
        assert torch.equal(r["abs_a"], torch.full((64,), 3.0))
        assert torch.equal(r["sq_a"], torch.full((64,), 5.0))
        assert torch.equal(r["gram_a"], torch.full((2, 32, 32), 7.0))
        assert torch.equal(r["abs_b"], torch.arange(32, dtype=torch.float32))
        assert torch.equal(r["gram_b"], torch.eye(32).unsqueeze(0))


def _unobserved_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        col = ActivationCollector({"a.weight": 32, "c.weight": 32}, ("rms",))
        col._counts["a.weight"] = 1
        col._square_sums["a.weight"] = torch.ones(32)
        col.all_reduce(device=torch.device("cpu"))
        try:
            col.finalize()
            msg = "no error"
        except ValueError as exc:
            msg = str(exc)
        with open(os.path.join(out_dir, f"msg{rank}.txt"), "w") as f:
            f.write(msg)
    finally:
        dist.destroy_process_group()


def test_target_unobserved_on_every_rank_still_fails(tmp_path) -> None:
    port = _free_port()
    mp.start_processes(_unobserved_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for rank in range(2):
        assert "did not observe 1 target(s): ['c.weight']" in (tmp_path / f"msg{rank}.txt").read_text()


@pytest.mark.parametrize("n,world", [(1, 2), (7, 2), (128, 8), (5, 3)])
def test_sequence_shards_cover_every_sequence_once(n, world) -> None:
    spans = [_shard_bounds(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
