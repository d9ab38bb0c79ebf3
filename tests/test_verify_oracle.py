"""CPU: the float64 error-sum oracle reproduces the reference's SQNR family."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.reference_pkg import import_reference


def _case(rows: int, cols: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    o = (torch.randn(rows, cols, generator=g) * 0.02).to(torch.bfloat16)
    r = (o.float() + torch.randn(rows, cols, generator=g) * 1e-3).float()
    gamma = torch.rand(cols, generator=g) + 0.1
    x = torch.randn(64, cols, generator=g)
    h = torch.einsum("nbi,nbj->bij", x.view(64, -1, 32), x.view(64, -1, 32)) / 64 + 1e-3 * torch.eye(32)
    return o, r, gamma, h


@pytest.mark.parametrize("rows,cols", [(16, 64), (3, 5120), (40, 320)])
def test_oracle_matches_reference_sqnr_family(rows, cols) -> None:
    ver = import_reference("mxwave.verify")
    o, r, gamma, h = _case(rows, cols, rows + cols)
    on, rn = o.float().numpy(), r.numpy()
    s = oracle.error_sums(on, rn)
    assert abs(oracle.sqnr_db(s[0], s[1]) - ver.sqnr(o, r)) < 1e-4
    s = oracle.error_sums(on, rn, gamma=gamma.numpy())
    assert abs(oracle.sqnr_db(s[2], s[3]) - ver.channel_weighted_sqnr(o, r, gamma)) < 1e-4
    s = oracle.error_sums(on, rn, hessian=h.numpy())
    assert abs(oracle.sqnr_db(s[2], s[3]) - ver.block_hessian_weighted_sqnr(o, r, h)) < 1e-4


def test_oracle_clamps_a_zero_noise_floor_like_the_reference() -> None:
    ver = import_reference("mxwave.verify")
    o = torch.ones(2, 32)
    s = oracle.error_sums(o.numpy(), o.numpy())
    assert np.isclose(oracle.sqnr_db(s[0], s[1]), ver.sqnr(o, o))
