"""Host logic of ActivationCollector that needs no GPU: when a shared input
(q/k/v, gate/up) may be reduced once for several targets."""

from __future__ import annotations

import torch

from mxwave_b200.calibration import ActivationCollector


def _counting_collector() -> tuple[ActivationCollector, list[int]]:
    col = ActivationCollector({"q.weight": 64, "k.weight": 64}, ("rms",))
    calls: list[int] = []

    def fake_reduce(activation: torch.Tensor, width: int):
        calls.append(1)
        x = activation.reshape(-1, width).float()
        return x.shape[0], None, (x * x).sum(0), None

    col._reduce = fake_reduce  # type: ignore[method-assign]
    return col, calls


def test_same_unchanged_tensor_is_reduced_once() -> None:
    col, calls = _counting_collector()
    x = torch.randn(3, 5, 64)
    col.update("q.weight", x)
    col.update("k.weight", x)
    assert len(calls) == 1 and col.reduced_reads == 1
    assert col.observation_counts == {"q.weight": 15, "k.weight": 15}


def test_in_place_change_forces_a_new_read() -> None:
    col, calls = _counting_collector()
    x = torch.randn(3, 5, 64)
    col.update("q.weight", x)
    x.mul_(2)
    col.update("k.weight", x)
    assert len(calls) == 2
    assert torch.allclose(col._square_sums["k.weight"], 4 * col._square_sums["q.weight"])


def test_inference_tensors_are_always_re_read() -> None:
    col, calls = _counting_collector()
    with torch.inference_mode():
        x = torch.randn(3, 5, 64)
        col.update("q.weight", x)
        col.update("k.weight", x)
    assert len(calls) == 2
