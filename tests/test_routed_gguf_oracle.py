"""CPU: oracle restatements of routed-expert moments and the GGUF MXFP4
repack, pinned against the reference's own implementations."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.reference_pkg import import_reference


def _routes(tokens: int, top_k: int, experts: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(experts, generator=g)[:top_k] for _ in range(tokens)])
    weights = torch.rand(tokens, top_k, generator=g)
    return ids, weights


@pytest.mark.parametrize("tokens,top_k,experts,hidden,inter", [(50, 2, 8, 64, 32), (200, 4, 16, 96, 48)])
def test_routed_oracle_matches_reference(tokens, top_k, experts, hidden, inter) -> None:
    ref = import_reference("mxwave.routed_calibration")
    ids, weights = _routes(tokens, top_k, experts, tokens)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(tokens, hidden, generator=g)
    down = torch.randn(tokens * top_k, inter, generator=g)
    m = ref.RoutedLayerMoments.create(experts, hidden, inter, torch.device("cpu"))
    m.update_inputs(x, ids, weights)
    m.update_down(down, ids, weights)
    sq, mass, counts = oracle.routed_squares(x.numpy(), ids.numpy(), weights.numpy(), experts, False)
    np.testing.assert_allclose(m.input_squares.numpy(), sq, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(m.route_mass.numpy(), mass, rtol=1e-5)
    assert np.array_equal(m.observations.numpy(), counts)
    dsq, _, _ = oracle.routed_squares(down.numpy(), ids.numpy(), weights.numpy(), experts, True)
    np.testing.assert_allclose(m.down_squares.numpy(), dsq, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rows,cols", [(1, 32), (5, 64), (33, 2048)])
def test_gguf_oracle_matches_reference(rows, cols) -> None:
    ref = import_reference("mxwave.gguf")
    g = torch.Generator().manual_seed(rows + cols)
    packed = torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.uint8)
    scales = torch.randint(0, 255, (rows, cols // 32), generator=g, dtype=torch.uint8)
    assert np.array_equal(oracle.gguf_repack(packed.numpy(), scales.numpy()), ref.repack_mxfp4_blocks(packed, scales))
