"""Drop-in for ``mxwave.calibration``'s collector on B200.

``ActivationCollector`` and ``attach_activation_hooks`` keep the reference
signatures, validation and messages (mxwave/calibration.py:154-336).  Each
``update`` reads the activation once with the sm_100a statistics kernel
(sum |x|, sum x^2 and the diagonal 32x32 blocks of X^T X in one pass, fp32
partials folded in fp64) instead of casting the whole activation to fp32.

Inputs shared by several targets (q/k/v read one tensor, gate/up another) are
reduced once: when ``update`` sees the same live tensor object again,
unmodified (same version counter), the previous call's statistics are added
to the new target without re-reading the activation.
"""

from __future__ import annotations

import math
import weakref
from collections.abc import Iterable, Mapping
from typing import Any

import torch

from . import _lib
from .core import BLOCK_SIZE, HessianDampingMode

_OBJECTIVES: frozenset[str] = frozenset({"mean-abs", "rms", "block-hessian"})
_DTYPE_CODES = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}


def _expected_statistic_shape(objective: str, width: int) -> tuple[int, ...]:
    if width <= 0:
        raise ValueError(f"Calibration target width must be positive, got {width}")
    if objective == "block-hessian" and width % BLOCK_SIZE != 0:
        raise ValueError(
            f"Block-Hessian calibration target width {width} is not divisible by {BLOCK_SIZE}"
        )
    return (width // BLOCK_SIZE, BLOCK_SIZE, BLOCK_SIZE) if objective == "block-hessian" else (width,)


def validate_statistic(target_name: str, objective: str, tensor: torch.Tensor, width: int) -> None:
    """Numerical validation of one statistic (mxwave/calibration.py:395-424)."""
    expected_shape = _expected_statistic_shape(objective, width)
    if tensor.shape != expected_shape:
        raise ValueError(
            f"Calibration statistic {target_name!r}/{objective} has shape "
            f"{tuple(tensor.shape)}, expected {expected_shape}"
        )
    if tensor.dtype != torch.float32:
        raise ValueError(
            f"Calibration statistic {target_name!r}/{objective} must be float32, got {tensor.dtype}"
        )
    if not torch.isfinite(tensor).all():
        raise ValueError(f"Calibration statistic contains NaN or infinity: {target_name}/{objective}")
    if objective != "block-hessian":
        if (tensor < 0).any() or not (tensor > 0).any():
            raise ValueError(f"Calibration magnitudes must be non-negative and nonzero: {target_name}")
        return
    if (tensor.diagonal(dim1=-2, dim2=-1) < 0).any():
        raise ValueError(f"Calibration Hessian has a negative diagonal: {target_name}")
    if not torch.allclose(tensor, tensor.transpose(-1, -2), rtol=1e-4, atol=1e-5):
        raise ValueError(f"Calibration Hessian is not symmetric: {target_name}")


def accumulate_stats(
    x: torch.Tensor,
    sum_abs: torch.Tensor | None,
    sum_sq: torch.Tensor | None,
    gram_blocks: torch.Tensor | None,
) -> None:
    """Add the statistics of a 2-D activation slice [tokens, width] into fp32 buffers."""
    if x.device.type != "cuda":
        raise RuntimeError(f"mxwave_b200 runs on CUDA devices only; activation is on {x.device}")
    if x.dtype not in _DTYPE_CODES:
        x = x.to(torch.float32)
    if x.stride(-1) != 1 or (x.shape[0] > 1 and x.stride(0) < x.shape[1]):
        x = x.contiguous()
    if x.shape[0] == 0:
        return
    from . import ops  # noqa: F401  -- registers torch.ops.mxwave_b200

    torch.ops.mxwave_b200.accumulate_activation_stats_(x, sum_abs, sum_sq, gram_blocks)


class ActivationCollector:
    """Accumulate real module-input statistics without retaining activations.

    Same interface as mxwave.calibration.ActivationCollector
    (mxwave/calibration.py:154-279); sums live in fp32 on the activation's
    CUDA device and only finalized statistics are copied to the CPU.
    """

    def __init__(
        self,
        target_widths: Mapping[str, int],
        objectives: Iterable[str] = ("mean-abs",),
        *,
        hessian_damp: float = 1e-6,
        hessian_damp_mode: HessianDampingMode = "absolute",
        skip_first_tokens: int = 0,
    ) -> None:
        if not target_widths:
            raise ValueError("At least one calibration target is required")
        if not math.isfinite(hessian_damp) or hessian_damp < 0.0:
            raise ValueError("hessian_damp must be finite and non-negative")
        if hessian_damp_mode not in ("absolute", "relative"):
            raise ValueError(f"Unknown Hessian damping mode: {hessian_damp_mode}")
        if not isinstance(skip_first_tokens, int) or skip_first_tokens < 0:
            raise ValueError("skip_first_tokens must be a non-negative integer")
        normalized = frozenset(objectives)
        if not normalized:
            raise ValueError("At least one calibration objective is required")
        invalid = sorted(set(normalized).difference(_OBJECTIVES))
        if invalid:
            raise ValueError(f"Unsupported calibration objectives: {invalid}")
        for name, width in target_widths.items():
            if not name.endswith(".weight"):
                raise ValueError(f"Calibration target must be a weight name: {name!r}")
            if width <= 0:
                raise ValueError(f"Calibration target {name!r} has invalid width {width}")
            if "block-hessian" in normalized and width % BLOCK_SIZE != 0:
                raise ValueError(
                    f"Calibration target {name!r} width {width} is not divisible by {BLOCK_SIZE}"
                )
        self.target_widths = dict(target_widths)
        self.objectives = normalized
        self.hessian_damp = hessian_damp
        self.hessian_damp_mode = hessian_damp_mode
        self.skip_first_tokens = skip_first_tokens
        self._counts: dict[str, int] = {}
        self._absolute_sums: dict[str, torch.Tensor] = {}
        self._square_sums: dict[str, torch.Tensor] = {}
        self._gram_sums: dict[str, torch.Tensor] = {}
        # Statistics of the most recent activation, reused for a shared input.
        self._last_ref: weakref.ref | None = None
        self._last_version = -1
        self._last: tuple[int, torch.Tensor | None, torch.Tensor | None, torch.Tensor | None] | None = None
        self.reduced_reads = 0

    def update(self, target_name: str, activation: torch.Tensor) -> None:
        """Accumulate one invocation of a target module's input tensor."""
        width = self.target_widths.get(target_name)
        if width is None:
            raise KeyError(f"Unknown calibration target: {target_name}")
        if activation.ndim == 0 or activation.shape[-1] != width:
            raise ValueError(
                f"Input for {target_name!r} has shape {tuple(activation.shape)}, "
                f"expected final dimension {width}"
            )
        if self.skip_first_tokens:
            if activation.ndim != 3:
                raise ValueError("Token exclusion requires [batch, sequence, channels] inputs")
            if activation.shape[1] <= self.skip_first_tokens:
                raise ValueError("Token exclusion would remove every observation in a window")
        # Inference tensors carry no version counter, so an in-place change
        # between two hooks could not be seen: they are always re-read.
        version = None if activation.is_inference() else activation._version
        same = (version is not None and self._last is not None and self._last_ref is not None
                and self._last_ref() is activation and version == self._last_version)
        if same:
            count, d_abs, d_sq, d_gram = self._last
            self.reduced_reads += 1
        else:
            count, d_abs, d_sq, d_gram = self._reduce(activation.detach(), width)
            self._last = (count, d_abs, d_sq, d_gram)
            self._last_ref = weakref.ref(activation)
            self._last_version = version
        if count == 0:
            return
        self._counts[target_name] = self._counts.get(target_name, 0) + count
        for dest, delta in ((self._absolute_sums, d_abs), (self._square_sums, d_sq), (self._gram_sums, d_gram)):
            if delta is None:
                continue
            prev = dest.get(target_name)
            if prev is None:
                dest[target_name] = delta.clone()
            else:
                prev.add_(delta)

    def _reduce(self, activation: torch.Tensor, width: int):
        dev = activation.device
        if dev.type != "cuda":
            raise RuntimeError(f"mxwave_b200 runs on CUDA devices only; activation is on {dev}")
        want_abs = "mean-abs" in self.objectives
        want_sq = "rms" in self.objectives
        want_gram = "block-hessian" in self.objectives
        d_abs = torch.zeros(width, dtype=torch.float32, device=dev) if want_abs else None
        d_sq = torch.zeros(width, dtype=torch.float32, device=dev) if want_sq else None
        d_gram = (torch.zeros((width // BLOCK_SIZE, BLOCK_SIZE, BLOCK_SIZE), dtype=torch.float32, device=dev)
                  if want_gram else None)
        if self.skip_first_tokens:
            # [batch, seq, width] minus each sequence's first tokens: one
            # gather of the kept rows into a contiguous [tokens, width] slice,
            # then a single statistics pass (not one launch per sequence).
            kept = activation[:, self.skip_first_tokens:, :].reshape(-1, width)
            count = kept.shape[0]
            accumulate_stats(kept, d_abs, d_sq, d_gram)
        else:
            flat = activation.reshape(-1, width)
            count = flat.shape[0]
            accumulate_stats(flat, d_abs, d_sq, d_gram)
        return count, d_abs, d_sq, d_gram

    def _finalized(self, to_cpu: bool) -> dict[str, dict[str, torch.Tensor]]:
        missing = sorted(set(self.target_widths).difference(self._counts))
        if missing:
            raise ValueError(f"Calibration hooks did not observe {len(missing)} target(s): {missing[:5]}")
        result: dict[str, dict[str, torch.Tensor]] = {}
        from . import ops  # noqa: F401  -- registers torch.ops.mxwave_b200

        for objective in sorted(self.objectives):
            values: dict[str, torch.Tensor] = {}
            for name in sorted(self.target_widths):
                count = self._counts[name]
                width = self.target_widths[name]
                if objective == "mean-abs":
                    src = self._absolute_sums[name]
                    with torch.cuda.device(src.device):
                        value = torch.ops.mxwave_b200.finalize_moments(src, count, False)
                elif objective == "rms":
                    src = self._square_sums[name]
                    with torch.cuda.device(src.device):
                        value = torch.ops.mxwave_b200.finalize_moments(src, count, True)
                else:
                    src = self._gram_sums[name]
                    mode = _lib.MXW_DAMP_ABSOLUTE if self.hessian_damp_mode == "absolute" else _lib.MXW_DAMP_RELATIVE
                    with torch.cuda.device(src.device):
                        value = torch.ops.mxwave_b200.finalize_block_hessian(src, False, count,
                                                                             float(self.hessian_damp), mode)
                if to_cpu:
                    value = value.cpu().to(torch.float32).contiguous()
                validate_statistic(name, objective, value, width)
                values[name] = value
            result[objective] = values
        return result

    def finalize(self) -> dict[str, dict[str, torch.Tensor]]:
        """Return complete CPU float32 statistics, failing on every missed hook."""
        return self._finalized(to_cpu=True)

    def finalize_on_device(self) -> dict[str, dict[str, torch.Tensor]]:
        """Same statistics left on the activation device (no host round trip)."""
        return self._finalized(to_cpu=False)

    @property
    def observation_counts(self) -> dict[str, int]:
        return dict(self._counts)

    def all_reduce(self, group: Any = None, device: torch.device | None = None) -> None:
        """Sum this collector's accumulators and counts over a process group.

        For token-sharded calibration: every rank accumulates its own tokens,
        then one all-reduce (a single flat fp32 buffer, plus one int64 buffer
        of counts) gives every rank the totals.  A target this rank did not
        observe contributes zeros; a target no rank observed stays unobserved,
        so finalize() still reports it.
        """
        import torch.distributed as dist

        names = sorted(self.target_widths)
        if device is None:
            existing = next(iter(self._absolute_sums.values() or self._square_sums.values() or
                                 self._gram_sums.values()), None)
            device = existing.device if existing is not None else torch.device("cuda", torch.cuda.current_device())
        layout: list[tuple[dict[str, torch.Tensor], str, tuple[int, ...]]] = []
        for name in names:
            width = self.target_widths[name]
            if "mean-abs" in self.objectives:
                layout.append((self._absolute_sums, name, (width,)))
            if "rms" in self.objectives:
                layout.append((self._square_sums, name, (width,)))
            if "block-hessian" in self.objectives:
                layout.append((self._gram_sums, name, (width // BLOCK_SIZE, BLOCK_SIZE, BLOCK_SIZE)))
        sizes = [math.prod(shape) for _, _, shape in layout]
        flat = torch.zeros(sum(sizes), dtype=torch.float32, device=device)
        offset = 0
        for (dest, name, _shape), size in zip(layout, sizes):
            value = dest.get(name)
            if value is not None:
                flat[offset : offset + size].copy_(value.reshape(-1))
            offset += size
        counts = torch.tensor([self._counts.get(n, 0) for n in names], dtype=torch.int64, device=device)
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
        offset = 0
        for (dest, name, shape), size in zip(layout, sizes):
            dest[name] = flat[offset : offset + size].view(shape).clone()
            offset += size
        self._counts = {n: int(c) for n, c in zip(names, counts.tolist()) if int(c) > 0}
        self._last = None
        self._last_ref = None


def attach_activation_hooks(
    model: torch.nn.Module,
    collector: ActivationCollector,
    *,
    module_prefix: str = "",
) -> list[Any]:
    """Attach strict forward-pre-hooks to exact target modules (calibration.py:282-336)."""
    modules = dict(model.named_modules())
    handles: list[Any] = []
    missing: list[str] = []
    for target_name, width in sorted(collector.target_widths.items()):
        module_name = target_name.removesuffix(".weight")
        local_module_name = module_name
        if module_prefix:
            prefix = f"{module_prefix}."
            if not module_name.startswith(prefix):
                raise ValueError(
                    f"Calibration target {target_name!r} is outside module prefix {module_prefix!r}"
                )
            local_module_name = module_name.removeprefix(prefix)
        module = modules.get(local_module_name)
        if module is None:
            missing.append(local_module_name)
            continue
        weight = getattr(module, "weight", None)
        if not isinstance(weight, torch.Tensor) or weight.ndim != 2 or weight.shape[-1] != width:
            actual_shape = tuple(weight.shape) if isinstance(weight, torch.Tensor) else None
            raise ValueError(
                f"Calibration module {module_name!r} has weight shape {actual_shape}, "
                f"expected (*, {width})"
            )

        def capture(_module: torch.nn.Module, inputs: tuple[Any, ...], *, name: str = target_name) -> None:
            if not inputs or not isinstance(inputs[0], torch.Tensor):
                raise ValueError(f"Calibration module {name!r} received no tensor input")
            collector.update(name, inputs[0])

        handles.append(module.register_forward_pre_hook(capture))
    if missing:
        for handle in handles:
            handle.remove()
        raise ValueError(f"Model is missing {len(missing)} calibration module(s): {missing[:5]}")
    return handles


__all__ = ["ActivationCollector", "accumulate_stats", "attach_activation_hooks", "validate_statistic"]
