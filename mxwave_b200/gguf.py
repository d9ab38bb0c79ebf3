"""Drop-in ``repack_mxfp4_blocks`` (mxwave/gguf.py:134-150) on B200.

The compressed-tensors MXFP4 pair (packed codes, E8M0 scales) is rewritten
as ggml ``block_mxfp4`` records by one sm_100a kernel (``mxw_repack_gguf_mxfp4``),
a pure byte shuffle; the result is returned as a host numpy array, as the
reference returns it.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib

BLOCK_SIZE = 32


def _validate_mxfp4_pair(name: str, packed: torch.Tensor, scale: torch.Tensor) -> tuple[int, int]:
    if packed.dtype is not torch.uint8 or scale.dtype is not torch.uint8:
        raise TypeError(f"MXFP4 tensor {name} must use uint8 packed weights and scales")
    if packed.ndim != 2 or scale.ndim != 2:
        raise ValueError(f"MXFP4 tensor {name} must have two-dimensional weights and scales")
    rows, packed_columns = (int(value) for value in packed.shape)
    logical_columns = packed_columns * 2
    if logical_columns % BLOCK_SIZE != 0:
        raise ValueError(f"MXFP4 tensor {name} has {logical_columns} columns; expected a multiple of {BLOCK_SIZE}")
    expected_scale_shape = (rows, logical_columns // BLOCK_SIZE)
    if tuple(int(value) for value in scale.shape) != expected_scale_shape:
        raise ValueError(
            f"MXFP4 scale for {name} has shape {tuple(scale.shape)}, expected {expected_scale_shape}"
        )
    return rows, logical_columns


def repack_mxfp4_blocks_device(packed: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """The ggml block_mxfp4 bytes [rows, blocks * 17] as a device uint8 tensor."""
    rows, cols = _validate_mxfp4_pair("weight", packed, scale)
    device = packed.device if packed.device.type == "cuda" else scale.device
    if device.type != "cuda":
        raise RuntimeError("mxwave_b200 repacks on CUDA devices only (no CPU fallback); move the tensors to a GPU")
    p = packed.to(device).contiguous()
    s = scale.to(device).contiguous()
    if p.data_ptr() % 16 != 0:
        p = p.clone()
    out = torch.empty((rows, (cols // BLOCK_SIZE) * 17), dtype=torch.uint8, device=device)
    lib = _lib.load()
    with torch.cuda.device(device):
        status = lib.mxw_repack_gguf_mxfp4(p.data_ptr(), s.data_ptr(), rows, cols, out.data_ptr(),
                                           torch.cuda.current_stream(device).cuda_stream)
    _lib.check(status, "mxw_repack_gguf_mxfp4")
    return out


def repack_mxfp4_blocks(packed: torch.Tensor, scale: torch.Tensor) -> np.ndarray:
    """Repack compressed-tensors MXFP4 into ggml ``block_mxfp4`` bytes (lossless)."""
    return repack_mxfp4_blocks_device(packed, scale).cpu().numpy()


__all__ = ["repack_mxfp4_blocks", "repack_mxfp4_blocks_device"]
