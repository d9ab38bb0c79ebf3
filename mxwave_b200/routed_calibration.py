"""Drop-in for ``mxwave.routed_calibration.RoutedLayerMoments`` on B200.

The public surface is the reference's (mxwave/routed_calibration.py:55-170):
the five accumulator fields, ``create`` / ``update_inputs`` / ``update_down``
/ ``finalize``, their validation messages and the shape of ``finalize``'s
result.  The implementation is this package's own:

* the accumulators live in two device arenas (one fp32, one int64), so the
  whole layer state is two buffers that a token-sharded caller can
  all-reduce in two calls;
* route validation is one device reduction and one host read per update,
  instead of one host synchronisation per condition;
* accumulation is one sm_100a kernel (``mxw_accumulate_routed_squares``):
  routes are grouped by expert with a stable sort, and each expert's squared,
  routing-weighted activations are summed in route order in fp64 and added
  once -- deterministic, unlike an atomic ``index_add_``;
* ``finalize`` divides every expert's squares by its routing mass at once on
  the device (IEEE division, which is how the reference's CPU division
  rounds) and brings the quotients, masses and counts to the host in one
  transfer; the square root and the normalisation by the maximum then use
  torch's CPU kernels per expert row, as the reference does, because
  torch's vectorised CPU square root is not correctly rounded.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}
_PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def _accumulate(squares: torch.Tensor, mass: torch.Tensor | None, inputs: torch.Tensor, route_rows: torch.Tensor,
                route_w2: torch.Tensor, experts: torch.Tensor) -> None:
    """Add fl(fl(x^2) * w2) of each route's input row into its expert's row of `squares`."""
    device = squares.device
    order = torch.sort(experts, stable=True).indices
    offsets = torch.zeros(squares.shape[0] + 1, dtype=torch.int64, device=device)
    torch.cumsum(torch.bincount(experts, minlength=squares.shape[0]), 0, out=offsets[1:])
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


def _device_quotients(squares: torch.Tensor, mass: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per expert: squares / mass (IEEE division, as the reference's CPU division rounds) and
    whether the expert is calibrated (positive mass and some positive square)."""
    usable = (mass > 0) & (squares > 0).any(dim=1)
    safe_mass = torch.where(mass > 0, mass, torch.ones_like(mass))
    return squares / safe_mass[:, None], usable


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
        dev = torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("mxwave_b200 accumulates routed moments on CUDA devices only (no CPU fallback)")
        floats = torch.zeros(experts * (hidden + intermediate + 1), dtype=torch.float32, device=dev)
        counts = torch.zeros(2 * experts, dtype=torch.int64, device=dev)
        a, b = experts * hidden, experts * (hidden + intermediate)
        return cls(floats[:a].view(experts, hidden), floats[a:b].view(experts, intermediate), floats[b:],
                   counts[:experts], counts[experts:])

    def _routes(self, ids: torch.Tensor, weights: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Flattened expert ids and squared router weights, validated in one device reduction."""
        if (ids.ndim != 2 or weights.shape != ids.shape or ids.dtype not in (torch.int32, torch.int64)
                or ids.device != self.input_squares.device):
            raise ValueError("Expected matching device-local [tokens, top_k] route IDs/weights")
        experts = self.route_mass.numel()
        if ids.numel() == 0:
            raise ValueError("Routing IDs or weights are empty, invalid, or non-finite")
        w = weights.detach().float()
        invalid = ((ids < 0) | (ids >= experts)).any() | (~torch.isfinite(w)).any() | (w < 0).any()
        if bool(invalid):
            raise ValueError("Routing IDs or weights are empty, invalid, or non-finite")
        return ids.reshape(-1).long(), w.reshape(-1).square()

    @torch.no_grad()
    def update_inputs(self, inputs: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> None:
        """Accumulate gate/up inputs for exactly the expert routes selected at runtime."""
        routed_ids, w2 = self._routes(ids, weights)
        if inputs.shape != (ids.shape[0], self.input_squares.shape[1]):
            raise ValueError("Gate/up activation shape does not match the actual token routes")
        # Route (t, k) reads token row t: the kernel indexes rows, nothing is repeated.
        token_of_route = torch.arange(routed_ids.numel(), device=routed_ids.device) // ids.shape[1]
        _accumulate(self.input_squares, self.route_mass, inputs, token_of_route, w2, routed_ids)
        self.observations.add_(torch.bincount(routed_ids, minlength=self.route_mass.numel()))

    @torch.no_grad()
    def update_down(self, inputs: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> None:
        """Accumulate token-major down-projection inputs, weighted by router weights squared."""
        routed_ids, w2 = self._routes(ids, weights)
        if inputs.shape != (ids.numel(), self.down_squares.shape[1]):
            raise ValueError("Down inputs must have one row per token-major expert route")
        row_of_route = torch.arange(routed_ids.numel(), device=routed_ids.device)
        _accumulate(self.down_squares, None, inputs, row_of_route, w2, routed_ids)
        self.down_observations.add_(torch.bincount(routed_ids, minlength=self.route_mass.numel()))

    @torch.no_grad()
    def finalize(self, layer: int) -> tuple[dict[str, torch.Tensor], dict[str, Any]]:
        """Return observed, nonzero RMS targets; unseen targets remain explicitly uncalibrated."""
        same_routes = torch.equal(self.observations, self.down_observations)
        if not same_routes:
            raise ValueError("Gate/up and down captures do not cover the same routed observations")
        finite = torch.isfinite(self.input_squares).all() & torch.isfinite(self.down_squares).all()
        if not bool(finite):
            raise ValueError("Captured activation moments contain NaN or infinity")
        gate_q, gate_ok = _device_quotients(self.input_squares, self.route_mass)
        down_q, down_ok = _device_quotients(self.down_squares, self.route_mass)
        # One host transfer of everything the result needs.
        gate_q, down_q = gate_q.cpu(), down_q.cpu()
        flags = torch.stack([gate_ok, down_ok]).cpu().tolist()
        masses = self.route_mass.cpu().tolist()
        counts = self.observations.cpu().tolist()
        statistics: dict[str, torch.Tensor] = {}
        retained: list[str] = []
        for expert in range(len(masses)):
            for projection in _PROJECTIONS:
                name = f"model.layers.{layer}.mlp.experts.{expert}.{projection}.weight"
                down = projection == "down_proj"
                if not flags[1 if down else 0][expert]:
                    retained.append(name)
                    continue
                # The square root and the normalisation run on the host with torch's CPU
                # kernels, one expert row at a time as the reference applies them: torch's
                # vectorised CPU sqrt is not correctly rounded, so the device's IEEE sqrt would
                # differ from the reference's gammas in the last bit.
                root = torch.sqrt((down_q if down else gate_q)[expert])
                statistics[name] = (root / root.amax()).float().contiguous()
        return statistics, {
            "layer": layer,
            "routed_observations": counts,
            "routing_weight_squared_mass": masses,
            "calibrated_targets": len(statistics),
            "retained_unweighted_targets": retained,
        }


__all__ = ["RoutedLayerMoments"]
