"""Drop-in SQNR family of ``mxwave.verify`` on B200.

``sqnr``, ``channel_weighted_sqnr`` and ``block_hessian_weighted_sqnr`` keep
the reference's signatures, validation and messages (mxwave/verify.py:24-86);
their sums run in one sm_100a pass (``mxw_error_sums``) with fp64
accumulation instead of several fp32 torch reductions.  ``sqnr_packed``
goes further: it reads the packed MXFP4 bytes and scales directly, so the
engines' dequantized copy (mxwave/engine.py:439-458) is never materialised.

The returned values are ``10 * log10(signal / noise)`` with both sums clamped
below at 1e-12, as in the reference.  They agree with the reference's fp32
values to the precision of its own summation (about 1e-6 relative).
"""

from __future__ import annotations

import math
import threading

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}
_CLAMP = float(torch.tensor(1e-12, dtype=torch.float32))  # the reference clamps its fp32 sums


class _Workspaces:
    """One zeroed workspace per (device, stream); reused (the kernel leaves it zeroed)."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._ws: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        stream = torch.cuda.current_stream(device)
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
        with self._lock:
            ws = self._ws.get(key)
            if ws is None or ws.numel() < nbytes:
                ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
                self._ws[key] = ws
        return ws


_workspaces = _Workspaces()


def _as_matrix(t: torch.Tensor, cols: int) -> torch.Tensor:
    m = t.reshape(-1, cols)
    if t.dtype not in _DTYPES:
        m = m.float()
    if m.stride(-1) != 1:
        m = m.contiguous()
    return m


def _error_sums(
    original: torch.Tensor,
    *,
    reconstructed: torch.Tensor | None = None,
    packed: torch.Tensor | None = None,
    scales: torch.Tensor | None = None,
    gamma: torch.Tensor | None = None,
    hessian: torch.Tensor | None = None,
) -> list[float]:
    device = original.device
    if device.type != "cuda":
        raise RuntimeError(f"mxwave_b200 runs on CUDA devices only; the original tensor is on {device}")
    cols = original.shape[-1]
    o = _as_matrix(original, cols)
    rows = o.shape[0]
    r = None
    if reconstructed is not None:
        r = _as_matrix(reconstructed.to(device), cols)
    p = s = None
    if packed is not None:
        p = packed.to(device).reshape(rows, cols // 2).contiguous()
        s = scales.to(device).reshape(rows, cols // 32).contiguous()
    g = gamma.to(device=device, dtype=torch.float32).contiguous() if gamma is not None else None
    h = hessian.to(device=device, dtype=torch.float32).contiguous() if hessian is not None else None
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = int(lib.mxw_error_sums_workspace_size(rows, cols))
        ws = _workspaces.get(device, nbytes)
        sums = torch.empty(4, dtype=torch.float64, device=device)
        status = lib.mxw_error_sums(
            o.data_ptr(), _DTYPES[o.dtype], rows, cols, o.stride(0),
            None if r is None else r.data_ptr(), _DTYPES[r.dtype] if r is not None else 0,
            0 if r is None else r.stride(0),
            None if p is None else p.data_ptr(), None if s is None else s.data_ptr(),
            None if g is None else g.data_ptr(), None if h is None else h.data_ptr(),
            sums.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(device).cuda_stream,
        )
    _lib.check(status, "mxw_error_sums")
    return sums.tolist()


def _db(signal: float, noise: float) -> float:
    return float(10.0 * math.log10(max(signal, _CLAMP) / max(noise, _CLAMP)))


def block_hessian_weighted_sqnr(original: torch.Tensor, reconstructed: torch.Tensor, hessian: torch.Tensor) -> float:
    """Return SQNR in the block-quadratic activation reconstruction objective."""
    if original.shape != reconstructed.shape or original.ndim != 2:
        raise ValueError("original and reconstructed tensors must be same-shaped matrices")
    width = original.shape[1]
    if width % 32 != 0 or hessian.shape != (width // 32, 32, 32):
        raise ValueError(
            "hessian must have shape "
            f"{(width // 32, 32, 32)} for input width {width}, got {tuple(hessian.shape)}"
        )
    sums = _error_sums(original, reconstructed=reconstructed, hessian=hessian)
    return _db(sums[2], sums[3])


def channel_weighted_sqnr(
    original: torch.Tensor, reconstructed: torch.Tensor, channel_weights: torch.Tensor
) -> float:
    """Return SQNR after weighting each input channel by ``channel_weights**2``."""
    if original.shape != reconstructed.shape:
        raise ValueError("original and reconstructed tensors must have the same shape")
    if original.ndim < 1 or channel_weights.shape != (original.shape[-1],):
        raise ValueError(
            "channel_weights must match the last tensor dimension, got "
            f"{tuple(channel_weights.shape)} for {tuple(original.shape)}"
        )
    sums = _error_sums(original, reconstructed=reconstructed, gamma=channel_weights)
    return _db(sums[2], sums[3])


def sqnr(original: torch.Tensor, reconstructed: torch.Tensor) -> float:
    """Signal-to-quantization-noise ratio (dB): 10 log10(||x||^2 / ||x - x_hat||^2)."""
    if original.numel() != reconstructed.numel():
        raise ValueError("original and reconstructed tensors must have the same number of elements")
    if original.numel() == 0:
        return _db(0.0, 0.0)
    flat_o = original.reshape(1, -1)
    sums = _error_sums(flat_o, reconstructed=reconstructed.reshape(1, -1))
    return _db(sums[0], sums[1])


def sqnr_packed(
    original: torch.Tensor,
    packed: torch.Tensor,
    scales: torch.Tensor,
    *,
    gamma: torch.Tensor | None = None,
    hessian: torch.Tensor | None = None,
) -> tuple[float, float | None]:
    """SQNR of an MXFP4 quantization straight from its packed bytes and scales.

    Returns ``(sqnr, weighted)``: the plain SQNR, and the gamma- or
    Hessian-weighted SQNR when one is given (else None).  Equal to
    ``sqnr(original, dequant_mxfp4(packed, scales, original.shape))`` and its
    weighted companion, without the dequantized tensor.
    """
    if original.ndim != 2 or original.shape[1] % 32 != 0:
        raise ValueError("original must be a matrix whose width is a multiple of 32")
    rows, cols = original.shape
    if packed.shape != (rows, cols // 2) or scales.shape != (rows, cols // 32):
        raise ValueError("packed / scales do not match the original's shape")
    if gamma is not None and hessian is not None:
        raise ValueError("gamma and hessian are mutually exclusive")
    if gamma is not None and gamma.shape != (cols,):
        raise ValueError(f"gamma must have shape {(cols,)}, got {tuple(gamma.shape)}")
    if hessian is not None and hessian.shape != (cols // 32, 32, 32):
        raise ValueError(f"hessian must have shape {(cols // 32, 32, 32)}, got {tuple(hessian.shape)}")
    sums = _error_sums(original, packed=packed, scales=scales, gamma=gamma, hessian=hessian)
    weighted = _db(sums[2], sums[3]) if (gamma is not None or hessian is not None) else None
    return _db(sums[0], sums[1]), weighted


__all__ = ["block_hessian_weighted_sqnr", "channel_weighted_sqnr", "sqnr", "sqnr_packed"]
