"""GPU: routed-expert moments and the GGUF MXFP4 repack against the
reference (run on CPU) and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mxwave_b200.gguf import repack_mxfp4_blocks
from mxwave_b200.routed_calibration import RoutedLayerMoments
from oracle import oracle
from tests.reference_pkg import import_reference

pytestmark = pytest.mark.gpu


def _routes(tokens: int, top_k: int, experts: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(experts, generator=g)[:top_k] for _ in range(tokens)])
    return ids, torch.rand(tokens, top_k, generator=g)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tokens,top_k,experts,hidden,inter", [(64, 2, 8, 256, 96), (1000, 8, 128, 2048, 768)])
def test_routed_moments_match_reference(tokens, top_k, experts, hidden, inter, dtype, cuda_device) -> None:
    ref = import_reference("mxwave.routed_calibration")
    ids, weights = _routes(tokens, top_k, experts, tokens + experts)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(tokens, hidden, generator=g).to(dtype)
    down = torch.randn(tokens * top_k, inter, generator=g).to(dtype)
    want = ref.RoutedLayerMoments.create(experts, hidden, inter, torch.device("cpu"))
    got = RoutedLayerMoments.create(experts, hidden, inter, cuda_device)
    for _ in range(2):  # two batches accumulate
        want.update_inputs(x, ids, weights)
        want.update_down(down, ids, weights)
        got.update_inputs(x.to(cuda_device), ids.to(cuda_device), weights.to(cuda_device))
        got.update_down(down.to(cuda_device), ids.to(cuda_device), weights.to(cuda_device))
    torch.testing.assert_close(got.input_squares.cpu(), want.input_squares, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(got.down_squares.cpu(), want.down_squares, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(got.route_mass.cpu(), want.route_mass, rtol=1e-5, atol=1e-6)
    assert torch.equal(got.observations.cpu(), want.observations)
    assert torch.equal(got.down_observations.cpu(), want.down_observations)
    stats_g, meta_g = got.finalize(3)
    stats_w, meta_w = want.finalize(3)
    assert stats_g.keys() == stats_w.keys()
    assert meta_g["retained_unweighted_targets"] == meta_w["retained_unweighted_targets"]
    for name in stats_w:
        torch.testing.assert_close(stats_g[name], stats_w[name], rtol=1e-5, atol=1e-6)


def test_routed_moments_are_deterministic_and_validate_like_the_reference(cuda_device) -> None:
    ref = import_reference("mxwave.routed_calibration")
    ids, weights = _routes(500, 4, 32, 7)
    x = torch.randn(500, 512).to(cuda_device)
    outs = []
    for _ in range(2):
        m = RoutedLayerMoments.create(32, 512, 64, cuda_device)
        m.update_inputs(x, ids.to(cuda_device), weights.to(cuda_device))
        outs.append(m.input_squares.clone())
    assert torch.equal(outs[0], outs[1])
    m = RoutedLayerMoments.create(4, 64, 32, cuda_device)
    r = ref.RoutedLayerMoments.create(4, 64, 32, torch.device("cpu"))
    bad = torch.tensor([[0, 4]])
    with pytest.raises(ValueError) as e_ref:
        r.update_inputs(torch.zeros(1, 64), bad, torch.ones(1, 2))
    with pytest.raises(ValueError, match=str(e_ref.value)):
        m.update_inputs(torch.zeros(1, 64, device=cuda_device), bad.to(cuda_device), torch.ones(1, 2, device=cuda_device))


@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 64), (300, 5120), (2048, 768)])
def test_gguf_repack_is_byte_identical_to_reference(rows, cols, cuda_device) -> None:
    ref = import_reference("mxwave.gguf")
    g = torch.Generator().manual_seed(rows * cols)
    packed = torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.uint8)
    scales = torch.randint(0, 255, (rows, cols // 32), generator=g, dtype=torch.uint8)
    got = repack_mxfp4_blocks(packed.to(cuda_device), scales.to(cuda_device))
    assert np.array_equal(got, ref.repack_mxfp4_blocks(packed, scales))
    assert np.array_equal(got, oracle.gguf_repack(packed.numpy(), scales.numpy()))


def test_routed_finalize_is_bit_identical_on_the_same_accumulators(cuda_device) -> None:
    """finalize's device pass rounds exactly like the reference's per-expert CPU loop."""
    ref = import_reference("mxwave.routed_calibration")
    experts, hidden, inter = 16, 384, 96
    ids, weights = _routes(300, 2, experts - 3, 11)  # the last three experts never receive a route
    g = torch.Generator().manual_seed(4)
    want = ref.RoutedLayerMoments.create(experts, hidden, inter, torch.device("cpu"))
    want.update_inputs(torch.randn(300, hidden, generator=g), ids, weights)
    want.update_down(torch.randn(600, inter, generator=g), ids, weights)
    want.input_squares[2].zero_()  # a routed expert with no energy stays uncalibrated
    got = RoutedLayerMoments.create(experts, hidden, inter, cuda_device)
    for field in ("input_squares", "down_squares", "route_mass", "observations", "down_observations"):
        getattr(got, field).copy_(getattr(want, field))
    stats_g, meta_g = got.finalize(5)
    stats_w, meta_w = want.finalize(5)
    assert meta_g == meta_w
    assert list(stats_g) == list(stats_w)
    for name in stats_w:
        assert stats_g[name].device.type == "cpu" and stats_g[name].is_contiguous()
        assert torch.equal(stats_g[name], stats_w[name]), name
