"""Drop-in for ``mxwave.core`` on B200: MXFP4 quantization through sm_100a kernels.

``quantize_mxfp4``, ``dequant_mxfp4`` and ``compute_block_hessian`` keep the
reference signatures, argument validation order, messages and exception
types (mxwave/core.py:30-58, 114-278).  Tensors must live on a CUDA device;
there is no CPU fallback.  Packed nibbles and E8M0 scales are bit-identical to
the reference's CPU fp32 implementation.
"""

from __future__ import annotations

import math
import weakref
from typing import Literal

import torch

from . import _lib

BLOCK_SIZE = 32
QUANTIZATION_REVISION = "mxfp4-rne-v2"
QuantizationMethod = Literal["rtn", "mse"]
HessianDampingMode = Literal["absolute", "relative"]

_DTYPE_CODES = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}


def _require_cuda(tensor: torch.Tensor, what: str) -> None:
    if tensor.device.type != "cuda":
        raise RuntimeError(
            f"mxwave_b200 runs on CUDA devices only; {what} is on {tensor.device} (no CPU fallback)"
        )


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _as_kernel_input(tensor: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Return (2-D tensor with unit column stride in a native dtype, dtype code)."""
    t = tensor
    if t.dtype not in _DTYPE_CODES:
        # The reference casts every input to fp32 first (core.py:167).
        t = t.to(torch.float32)
    if t.stride(-1) != 1 or t.stride(0) < t.shape[-1]:
        t = t.contiguous()
    return t, _DTYPE_CODES[t.dtype]


class _ValidatedCache:
    """Remembers statistic tensors already validated, keyed by identity + version.

    The reference re-validates gamma / hessian on every row chunk (one host
    synchronisation each).  A tensor that has not been modified since it was
    checked (same object, storage and version counter) is not re-checked.
    """

    def __init__(self) -> None:
        # id -> (weak reference, key): the weak reference proves the entry is
        # about this very object, not a later one that reuses its id.
        self._seen: dict[int, tuple[weakref.ref, tuple[int, int, tuple[int, ...]]]] = {}

    def key(self, t: torch.Tensor) -> tuple[int, int, tuple[int, ...]]:
        return (t.data_ptr(), t._version, tuple(t.shape))

    def ok(self, t: torch.Tensor) -> bool:
        if t.is_inference():  # no version counter: an in-place change would go unseen
            return False
        entry = self._seen.get(id(t))
        return entry is not None and entry[0]() is t and entry[1] == self.key(t)

    def add(self, t: torch.Tensor) -> None:
        if t.is_inference():
            return
        if len(self._seen) > 256:
            self._seen.clear()
        self._seen[id(t)] = (weakref.ref(t), self.key(t))


_gamma_ok = _ValidatedCache()
_hessian_ok = _ValidatedCache()


@torch.no_grad()
def quantize_mxfp4(
    tensor: torch.Tensor,
    scale_percentile: float = 99.5,
    gamma: torch.Tensor | None = None,
    hessian: torch.Tensor | None = None,
    method: QuantizationMethod = "mse",
    mse_clip_depth: int = 1,
    *,
    _flags: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize a float tensor to MXFP4 with MSE-optimal scale selection.

    Same contract as mxwave.core.quantize_mxfp4 (mxwave/core.py:114-251):
    returns packed [out, in//2] uint8 (element 2j in the low nibble) and
    scales [out, in//32] uint8 (E8M0 biased exponents), on the input's device.
    """
    if hessian is not None and gamma is not None:
        raise ValueError("hessian and gamma are mutually exclusive")
    if method not in ("rtn", "mse"):
        raise ValueError(f"Unsupported quantization method: {method}")
    if method == "rtn" and (gamma is not None or hessian is not None):
        raise ValueError("rtn does not use gamma or hessian weighting")
    if not 0.0 < scale_percentile <= 100.0:
        raise ValueError("scale_percentile must be in (0, 100]")
    if not isinstance(mse_clip_depth, int) or not 0 <= mse_clip_depth <= 8:
        raise ValueError("mse_clip_depth must be an integer in [0, 8]")
    if tensor.ndim != 2:
        raise ValueError(f"Expected a 2D weight tensor, got shape {tuple(tensor.shape)}")
    assert tensor.shape[-1] % BLOCK_SIZE == 0, (
        f"Last dim {tensor.shape[-1]} not divisible by BLOCK_SIZE={BLOCK_SIZE}"
    )
    _require_cuda(tensor, "the weight")
    rows, cols = tensor.shape
    num_blocks = cols // BLOCK_SIZE
    device = tensor.device

    hessian_f32: torch.Tensor | None = None
    if hessian is not None:
        if hessian.shape != (num_blocks, BLOCK_SIZE, BLOCK_SIZE):
            raise ValueError(
                "hessian must have shape "
                f"{(num_blocks, BLOCK_SIZE, BLOCK_SIZE)}, got {tuple(hessian.shape)}"
            )
        if not _hessian_ok.ok(hessian):
            if not torch.isfinite(hessian).all():
                raise ValueError("hessian contains NaN or infinity")
            _hessian_ok.add(hessian)
        hessian_f32 = hessian.to(device=device, dtype=torch.float32).contiguous()

    gamma_f32: torch.Tensor | None = None
    if gamma is not None and method == "mse":
        if gamma.shape != (cols,):
            raise ValueError(f"gamma must have shape {(cols,)}, got {tuple(gamma.shape)}")
        if not _gamma_ok.ok(gamma):
            if not torch.isfinite(gamma).all() or (gamma < 0).any():
                raise ValueError("gamma must contain finite, non-negative magnitudes")
            _gamma_ok.add(gamma)
        gamma_f32 = gamma.to(device=device, dtype=torch.float32).contiguous()

    w, _dtype_code = _as_kernel_input(tensor)
    if rows == 0:
        return (torch.empty((0, cols // 2), dtype=torch.uint8, device=device),
                torch.empty((0, num_blocks), dtype=torch.uint8, device=device))
    _ops()
    return torch.ops.mxwave_b200.quantize_mxfp4(
        w,
        float(scale_percentile),
        gamma_f32,
        hessian_f32,
        _lib.MXW_METHOD_RTN if method == "rtn" else _lib.MXW_METHOD_MSE,
        mse_clip_depth,
        _flags if _flags is not None else _device_flags(device),
    )


def _ops():
    """Register the torch operators (mxwave_b200.ops) on first use."""
    from . import ops

    return ops


_DEVICE_FLAGS: dict = {}


def _device_flags(device: torch.device) -> torch.Tensor:
    """A flag word for calls that pass none: one per (device, stream), cleared before each use.

    Its MXW_FLAG_RARE bit lets the rare-block pass return at once after a
    main pass that marked nothing, so it is zeroed on the current stream
    before every call; a bit left over from an earlier call would make every
    later call scan the scale bytes again.  Calls on one stream run in order,
    so the clear cannot race with an earlier call's rare-block pass; each
    stream has its own word for the same reason.  Nothing reads its
    MXW_FLAG_NONFINITE bit; callers that need it pass their own word.
    """
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    flags = _DEVICE_FLAGS.get(key)
    if flags is None:
        flags = torch.zeros(1, dtype=torch.int32, device=device)
        _DEVICE_FLAGS[key] = flags
    else:
        flags.zero_()
    return flags


@torch.no_grad()
def quantize_into(
    weight: torch.Tensor,
    packed: torch.Tensor,
    scales: torch.Tensor,
    *,
    scale_percentile: float = 99.5,
    gamma: torch.Tensor | None = None,
    hessian: torch.Tensor | None = None,
    method: QuantizationMethod = "mse",
    mse_clip_depth: int = 1,
    flags: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Quantize a 2-D CUDA weight into caller-owned outputs on `stream`.

    The pipeline building block behind the streamer: no validation beyond the
    C ABI's argument checks and no allocation.  `gamma` / `hessian` must be
    fp32 CUDA tensors already validated by the caller; `flags` (int32, one
    element) receives MXW_FLAG_NONFINITE for a NaN/inf input.
    """
    rows, cols = weight.shape
    w, dtype_code = _as_kernel_input(weight)
    handle = (stream or torch.cuda.current_stream(weight.device)).cuda_stream
    lib = _lib.load()
    with torch.cuda.device(weight.device):
        status = lib.mxw_quantize_mxfp4(
            w.data_ptr(), dtype_code, rows, cols, w.stride(0), float(scale_percentile),
            None if gamma is None else gamma.data_ptr(),
            None if hessian is None else hessian.data_ptr(),
            _lib.MXW_METHOD_RTN if method == "rtn" else _lib.MXW_METHOD_MSE, mse_clip_depth,
            packed.data_ptr(), scales.data_ptr(), None if flags is None else flags.data_ptr(), handle,
        )
    _lib.check(status, "mxw_quantize_mxfp4")


@torch.no_grad()
def dequant_mxfp4(
    packed: torch.Tensor,
    scales: torch.Tensor,
    shape: tuple[int, ...],
) -> torch.Tensor:
    """Dequantize MXFP4 packed weights back to float32 (mxwave/core.py:254-278)."""
    _require_cuda(packed, "packed")
    cols = shape[-1]
    rows = math.prod(shape) // cols
    _ops()
    return torch.ops.mxwave_b200.dequant_mxfp4(packed, scales, rows, cols).reshape(shape)


def _damp_block_hessian(hessian: torch.Tensor, damp: float, mode: HessianDampingMode) -> None:
    """Add absolute or per-block relative diagonal damping in place (core.py:61-69)."""
    if not math.isfinite(damp) or damp < 0:
        raise ValueError("Hessian damping must be finite and non-negative")
    if mode not in ("absolute", "relative"):
        raise ValueError(f"Unknown Hessian damping mode: {mode}")
    diagonal = hessian.diagonal(dim1=-2, dim2=-1)
    addition = damp if mode == "absolute" else diagonal.mean(dim=-1, keepdim=True) * damp
    diagonal.add_(addition)


@torch.no_grad()
def compute_block_hessian(
    X: torch.Tensor,
    block_size: int = BLOCK_SIZE,
    damp: float = 1e-6,
    damp_mode: HessianDampingMode = "absolute",
) -> torch.Tensor:
    """Block-diagonal Hessian H_b = X_b^T X_b / N with damping (mxwave/core.py:30-58)."""
    assert X.ndim == 2, f"Expected 2D activation matrix, got shape {X.shape}"
    N, K = X.shape
    assert K % block_size == 0, f"in_features {K} not divisible by block_size {block_size}"
    if block_size != BLOCK_SIZE:
        raise ValueError(f"mxwave_b200 computes {BLOCK_SIZE}-wide blocks only")
    if not math.isfinite(damp) or damp < 0:
        raise ValueError("Hessian damping must be finite and non-negative")
    if damp_mode not in ("absolute", "relative"):
        raise ValueError(f"Unknown Hessian damping mode: {damp_mode}")
    _require_cuda(X, "X")
    x, _dtype_code = _as_kernel_input(X)
    device = X.device
    gram = torch.zeros((K // BLOCK_SIZE, BLOCK_SIZE, BLOCK_SIZE), dtype=torch.float32, device=device)
    _ops()
    if N > 0:
        torch.ops.mxwave_b200.accumulate_activation_stats_(x, None, None, gram)
    return torch.ops.mxwave_b200.finalize_block_hessian(
        gram, False, max(N, 1), float(damp),
        _lib.MXW_DAMP_ABSOLUTE if damp_mode == "absolute" else _lib.MXW_DAMP_RELATIVE,
    )


__all__ = [
    "BLOCK_SIZE",
    "QUANTIZATION_REVISION",
    "HessianDampingMode",
    "QuantizationMethod",
    "compute_block_hessian",
    "dequant_mxfp4",
    "quantize_into",
    "quantize_mxfp4",
]
