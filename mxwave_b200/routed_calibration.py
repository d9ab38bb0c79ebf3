"""Drop-in for ``mxwave.routed_calibration.RoutedLayerMoments`` on B200.

Same fields, constructor, validation messages and results as the reference
(mxwave/routed_calibration.py:55-170).  The accumulations run in one sm_100a
kernel (``mxw_accumulate_routed_squares``): the routes are grouped by expert
with a stable sort (host-side index bookkeeping on the device), then each
expert's squared, routing-weighted activations are summed in route order in
fp64 and added once -- deterministic, unlike an atomic index_add_.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}


def _accumulate(squares: torch.Tensor, mass: torch.Tensor | None, inputs: torch.Tensor, route_rows: torch.Tensor,
                route_w2: torch.Tensor, experts: torch.Tensor) -> None:
    """Add fl(fl(x^2) * w2) of each route's input row into its expert's row of `squares`."""
    device = squares.device
    order = torch.sort(experts, stable=True).indices
    counts = torch.bincount(experts, minlength=squares.shape[0])
    offsets = torch.zeros(squares.shape[0] + 1, dtype=torch.int64, device=device)
    torch.cumsum(counts, 0, out=offsets[1:])
    rows_sorted = route_rows[order].contiguous()
    w2_sorted = route_w2[order].contiguous()
    x = inputs.detach()
    if x.dtype not in _DTYPES:
        x = x.float()
    if x.stride(-1) != 1:
        x = x.contiguous()
    lib = _lib.load()
    with torch.cuda.device(device):
        status = lib.mxw_accumulate_routed_squares(
            x.data_ptr(), _DTYPES[x.dtype], x.shape[0], x.shape[1], x.stride(0), rows_sorted.data_ptr(),
            w2_sorted.data_ptr(), rows_sorted.numel(), offsets.data_ptr(), squares.shape[0], squares.data_ptr(),
            None if mass is None else mass.data_ptr(), torch.cuda.current_stream(device).cuda_stream,
        )
    _lib.check(status, "mxw_accumulate_routed_squares")


@dataclass
class RoutedLayerMoments:
    """Bounded per-expert statistics, with no retained token activation history."""

    input_squares: torch.Tensor
    down_squares: torch.Tensor
    route_mass: torch.Tensor
    observations: torch.Tensor
    down_observations: torch.Tensor

    @classmethod
    def create(cls, experts: int, hidden: int, intermediate: int, device: torch.device) -> RoutedLayerMoments:
        """Allocate device-local accumulators for one complete unsharded MoE layer."""
        if min(experts, hidden, intermediate) <= 0:
            raise ValueError("Expert count and channel widths must be positive")
        if torch.device(device).type != "cuda":
            raise RuntimeError("mxwave_b200 accumulates routed moments on CUDA devices only (no CPU fallback)")
        return cls(
            torch.zeros((experts, hidden), dtype=torch.float32, device=device),
            torch.zeros((experts, intermediate), dtype=torch.float32, device=device),
            torch.zeros(experts, dtype=torch.float32, device=device),
            torch.zeros(experts, dtype=torch.int64, device=device),
            torch.zeros(experts, dtype=torch.int64, device=device),
        )

    def _routes(self, ids: torch.Tensor, weights: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        if (
            ids.ndim != 2
            or weights.shape != ids.shape
            or ids.dtype not in (torch.int32, torch.int64)
            or ids.device != self.input_squares.device
        ):
            raise ValueError("Expected matching device-local [tokens, top_k] route IDs/weights")
        if (
            ids.numel() == 0
            or bool((ids < 0).any())
            or bool((ids >= len(self.route_mass)).any())
            or not bool(torch.isfinite(weights).all())
            or bool((weights < 0).any())
        ):
            raise ValueError("Routing IDs or weights are empty, invalid, or non-finite")
        return ids.reshape(-1).long(), weights.detach().float().reshape(-1).square()

    @torch.no_grad()
    def update_inputs(self, inputs: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> None:
        """Accumulate gate/up inputs for exactly the expert routes selected at runtime."""
        routed_ids, mass = self._routes(ids, weights)
        if inputs.shape != (ids.shape[0], self.input_squares.shape[1]):
            raise ValueError("Gate/up activation shape does not match the actual token routes")
        # Route (t, k) reads token row t (the reference repeats each row top_k times).
        route_rows = torch.arange(routed_ids.numel(), device=routed_ids.device) // ids.shape[1]
        _accumulate(self.input_squares, self.route_mass, inputs, route_rows, mass, routed_ids)
        self.observations.add_(torch.bincount(routed_ids, minlength=len(self.route_mass)))

    @torch.no_grad()
    def update_down(self, inputs: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> None:
        """Accumulate token-major down-projection inputs, weighted by router weights squared."""
        routed_ids, mass = self._routes(ids, weights)
        if inputs.shape != (ids.numel(), self.down_squares.shape[1]):
            raise ValueError("Down inputs must have one row per token-major expert route")
        route_rows = torch.arange(routed_ids.numel(), device=routed_ids.device)
        _accumulate(self.down_squares, None, inputs, route_rows, mass, routed_ids)
        self.down_observations.add_(torch.bincount(routed_ids, minlength=len(self.route_mass)))

    def finalize(self, layer: int) -> tuple[dict[str, torch.Tensor], dict[str, Any]]:
        """Return observed, nonzero RMS targets; unseen targets remain explicitly uncalibrated."""
        if not torch.equal(self.observations, self.down_observations):
            raise ValueError("Gate/up and down captures do not cover the same routed observations")
        if not bool(torch.isfinite(self.input_squares).all()) or not bool(torch.isfinite(self.down_squares).all()):
            raise ValueError("Captured activation moments contain NaN or infinity")
        statistics: dict[str, torch.Tensor] = {}
        retained: list[str] = []
        masses = self.route_mass.cpu()
        counts = self.observations.cpu()
        gate = self.input_squares.cpu()
        down = self.down_squares.cpu()
        for expert in range(len(masses)):
            for projection, values in (("gate_proj", gate), ("up_proj", gate), ("down_proj", down)):
                name = f"model.layers.{layer}.mlp.experts.{expert}.{projection}.weight"
                mass = float(masses[expert])
                if mass <= 0 or not bool((values[expert] > 0).any()):
                    retained.append(name)
                    continue
                gamma = torch.sqrt(values[expert] / mass)
                gamma = (gamma / gamma.amax()).float().contiguous()
                statistics[name] = gamma
        return statistics, {
            "layer": layer,
            "routed_observations": counts.tolist(),
            "routing_weight_squared_mass": masses.tolist(),
            "calibrated_targets": len(statistics),
            "retained_unweighted_targets": retained,
        }


__all__ = ["RoutedLayerMoments"]
