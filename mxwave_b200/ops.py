"""torch custom operators over the C ABI (namespace ``mxwave_b200``).

Each operator wraps one entry point of include/mxwave_b200.h with a schema, a
CUDA implementation (allocation through torch's caching allocator on the
input's device, launch on torch's current stream) and a fake implementation,
so callers get shape propagation under FakeTensor / ``torch.compile`` and
``torch.library.opcheck`` coverage.  Argument validation with the
reference's messages stays in the host mirror (``mxwave_b200.core``,
``mxwave_b200.calibration``); these operators only enforce the C ABI's own
contract, and a non-OK status raises (ValueError for MXW_EINVAL).

Operators (reference function each one backs):

* ``quantize_mxfp4(weight, scale_percentile, gamma, hessian, method,
  mse_clip_depth, flags) -> (packed, scales)`` -- mxwave/core.py:114-251;
  ``flags`` is a caller-owned int32 word that receives MXW_FLAG_* bits.
* ``dequant_mxfp4(packed, scales, rows, cols) -> fp32`` -- core.py:254-278.
* ``accumulate_moments_(x, sum_abs, sum_sq)`` -- calibration.py:227-232.
* ``accumulate_activation_stats_(x, sum_abs?, sum_sq?, gram_blocks?)`` --
  calibration.py:226-236 in one read of ``x``.
* ``accumulate_xtx_(x, gram)`` -- the full X^T X on the tensor cores
  (the reference forms only its diagonal blocks, calibration.py:233-236).
* ``finalize_moments(sums, count, root) -> fp32`` -- calibration.py:262-266.
* ``finalize_block_hessian(gram, full, count, damp, mode) -> fp32`` --
  calibration.py:267-270 with core.py:61-69.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib

_DTYPE_CODES = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _cuda_2d(x: Tensor, what: str) -> tuple[Tensor, int]:
    """A 2-D view with unit column stride in a native dtype."""
    if x.device.type != "cuda":
        raise RuntimeError(f"mxwave_b200 runs on CUDA devices only; {what} is on {x.device} (no CPU fallback)")
    if x.ndim != 2:
        raise ValueError(f"{what} must be 2-D, got shape {tuple(x.shape)}")
    if x.dtype not in _DTYPE_CODES:
        x = x.to(torch.float32)
    if x.stride(-1) != 1 or (x.shape[0] > 1 and x.stride(0) < x.shape[1]):
        x = x.contiguous()
    return x, _DTYPE_CODES[x.dtype]


def _f32_buffer(t: Tensor, shape: tuple[int, ...], what: str) -> None:
    if t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous() or t.device.type != "cuda":
        raise ValueError(f"{what} must be a contiguous CUDA float32 tensor of shape {shape}")


# ------------------------------------------------------------------ quantize


@torch.library.custom_op("mxwave_b200::quantize_mxfp4", mutates_args=("flags",))
def quantize_mxfp4(
    weight: Tensor,
    scale_percentile: float,
    gamma: Tensor | None,
    hessian: Tensor | None,
    method: int,
    mse_clip_depth: int,
    flags: Tensor,
) -> tuple[Tensor, Tensor]:
    w, code = _cuda_2d(weight, "the weight")
    rows, cols = w.shape
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((rows, cols // 32), dtype=torch.uint8, device=w.device)
    if rows == 0:
        return packed, scales
    if flags.dtype != torch.int32 or flags.numel() < 1 or flags.device != w.device:
        raise ValueError("flags must be an int32 tensor on the weight's device")
    lib = _lib.load()
    with torch.cuda.device(w.device):
        status = lib.mxw_quantize_mxfp4(
            w.data_ptr(), code, rows, cols, w.stride(0), float(scale_percentile), _ptr(gamma), _ptr(hessian),
            method, mse_clip_depth, packed.data_ptr(), scales.data_ptr(), flags.data_ptr(), _stream(w.device),
        )
    _lib.check(status, "mxw_quantize_mxfp4")
    return packed, scales


@quantize_mxfp4.register_fake
def _(weight, scale_percentile, gamma, hessian, method, mse_clip_depth, flags):
    rows, cols = weight.shape
    return (weight.new_empty((rows, cols // 2), dtype=torch.uint8),
            weight.new_empty((rows, cols // 32), dtype=torch.uint8))


@torch.library.custom_op("mxwave_b200::dequant_mxfp4", mutates_args=())
def dequant_mxfp4(packed: Tensor, scales: Tensor, rows: int, cols: int) -> Tensor:
    if packed.device.type != "cuda":
        raise RuntimeError(f"mxwave_b200 runs on CUDA devices only; packed is on {packed.device} (no CPU fallback)")
    p = packed.reshape(rows, cols // 2).contiguous()
    s = scales.reshape(rows, cols // 32).to(device=packed.device).contiguous()
    out = torch.empty((rows, cols), dtype=torch.float32, device=packed.device)
    lib = _lib.load()
    with torch.cuda.device(packed.device):
        status = lib.mxw_dequant_mxfp4(p.data_ptr(), s.data_ptr(), rows, cols, out.data_ptr(), _stream(packed.device))
    _lib.check(status, "mxw_dequant_mxfp4")
    return out


@dequant_mxfp4.register_fake
def _(packed, scales, rows, cols):
    return packed.new_empty((rows, cols), dtype=torch.float32)


# ------------------------------------------------------------- calibration


@torch.library.custom_op("mxwave_b200::accumulate_moments_", mutates_args=("sum_abs", "sum_sq"))
def accumulate_moments_(x: Tensor, sum_abs: Tensor, sum_sq: Tensor) -> None:
    xx, code = _cuda_2d(x, "the activation")
    tokens, cols = xx.shape
    _f32_buffer(sum_abs, (cols,), "sum_abs")
    _f32_buffer(sum_sq, (cols,), "sum_sq")
    if tokens == 0:
        return
    lib = _lib.load()
    with torch.cuda.device(xx.device):
        status = lib.mxw_accumulate_moments(xx.data_ptr(), code, tokens, cols, max(xx.stride(0), cols),
                                            sum_abs.data_ptr(), sum_sq.data_ptr(), _stream(xx.device))
    _lib.check(status, "mxw_accumulate_moments")


@accumulate_moments_.register_fake
def _(x, sum_abs, sum_sq):
    return None


@torch.library.custom_op("mxwave_b200::accumulate_activation_stats_",
                         mutates_args=("sum_abs", "sum_sq", "gram_blocks"))
def accumulate_activation_stats_(x: Tensor, sum_abs: Tensor | None, sum_sq: Tensor | None,
                                 gram_blocks: Tensor | None) -> None:
    xx, code = _cuda_2d(x, "the activation")
    tokens, cols = xx.shape
    if sum_abs is not None:
        _f32_buffer(sum_abs, (cols,), "sum_abs")
    if sum_sq is not None:
        _f32_buffer(sum_sq, (cols,), "sum_sq")
    if gram_blocks is not None:
        _f32_buffer(gram_blocks, (cols // 32, 32, 32), "gram_blocks")
    if tokens == 0:
        return
    lib = _lib.load()
    with torch.cuda.device(xx.device):
        status = lib.mxw_accumulate_activation_stats(
            xx.data_ptr(), code, tokens, cols, max(xx.stride(0), cols), _ptr(sum_abs), _ptr(sum_sq),
            _ptr(gram_blocks), None, _stream(xx.device),
        )
    _lib.check(status, "mxw_accumulate_activation_stats")


@accumulate_activation_stats_.register_fake
def _(x, sum_abs, sum_sq, gram_blocks):
    return None


@torch.library.custom_op("mxwave_b200::accumulate_xtx_", mutates_args=("gram",))
def accumulate_xtx_(x: Tensor, gram: Tensor) -> None:
    if x.dtype != torch.bfloat16:
        raise ValueError("accumulate_xtx_ takes bf16 activations")
    xx, _code = _cuda_2d(x, "the activation")
    tokens, cols = xx.shape
    _f32_buffer(gram, (cols, cols), "gram")
    if tokens == 0:
        return
    lib = _lib.load()
    with torch.cuda.device(xx.device):
        status = lib.mxw_accumulate_xtx(xx.data_ptr(), tokens, cols, xx.stride(0), gram.data_ptr(), cols, None,
                                        _stream(xx.device))
    _lib.check(status, "mxw_accumulate_xtx")


@accumulate_xtx_.register_fake
def _(x, gram):
    return None


@torch.library.custom_op("mxwave_b200::finalize_moments", mutates_args=())
def finalize_moments(sums: Tensor, count: int, root: bool) -> Tensor:
    _f32_buffer(sums, (sums.shape[0],), "sums")
    out = torch.empty_like(sums)
    lib = _lib.load()
    cols = sums.shape[0]
    with torch.cuda.device(sums.device):
        if root:
            status = lib.mxw_finalize_moments(None, sums.data_ptr(), cols, count, None, out.data_ptr(),
                                              _stream(sums.device))
        else:
            status = lib.mxw_finalize_moments(sums.data_ptr(), None, cols, count, out.data_ptr(), None,
                                              _stream(sums.device))
    _lib.check(status, "mxw_finalize_moments")
    return out


@finalize_moments.register_fake
def _(sums, count, root):
    return torch.empty_like(sums)


@torch.library.custom_op("mxwave_b200::finalize_block_hessian", mutates_args=())
def finalize_block_hessian(gram: Tensor, full: bool, count: int, damp: float, mode: int) -> Tensor:
    if full:
        cols = gram.shape[-1]
        _f32_buffer(gram, (cols, cols), "gram")
    else:
        cols = gram.shape[0] * 32
        _f32_buffer(gram, (cols // 32, 32, 32), "gram")
    out = torch.empty((cols // 32, 32, 32), dtype=torch.float32, device=gram.device)
    lib = _lib.load()
    with torch.cuda.device(gram.device):
        status = lib.mxw_finalize_block_hessian(gram.data_ptr(), 1 if full else 0, cols, cols, count, float(damp),
                                                mode, out.data_ptr(), _stream(gram.device))
    _lib.check(status, "mxw_finalize_block_hessian")
    return out


@finalize_block_hessian.register_fake
def _(gram, full, count, damp, mode):
    cols = gram.shape[-1] if full else gram.shape[0] * 32
    return gram.new_empty((cols // 32, 32, 32), dtype=torch.float32)


OPS = (
    quantize_mxfp4,
    dequant_mxfp4,
    accumulate_moments_,
    accumulate_activation_stats_,
    accumulate_xtx_,
    finalize_moments,
    finalize_block_hessian,
)

__all__ = [
    "OPS",
    "accumulate_activation_stats_",
    "accumulate_moments_",
    "accumulate_xtx_",
    "dequant_mxfp4",
    "finalize_block_hessian",
    "finalize_moments",
    "quantize_mxfp4",
]
