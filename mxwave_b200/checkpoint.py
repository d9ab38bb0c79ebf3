"""Drop-in for the chunked quantization loop of ``mxwave.checkpoint`` / ``mxwave.shard``.

* ``tensor_chunk_rows`` and ``iter_quantized_row_chunks`` keep the reference
  contract (mxwave/checkpoint.py:89-126): the same row-chunk bound, the same
  shape and finiteness errors (same messages), chunks yielded in order.  With
  this package's own row reader the loop reads the next chunks on a
  background thread while the current one is quantized (other readers are
  called on the caller's thread), and when ``quantize`` is this package's quantizer the NaN/inf
  check is folded into the kernel (a device flag word) instead of a separate
  ``isfinite`` reduction; the flag is read before the chunk is yielded, so a
  bad chunk still raises before anything of it is returned.
* ``read_tensor_row_range`` (mxwave/shard.py:220-237) reads the rows into
  pinned host memory and copies them to the device asynchronously on the
  current stream.
"""

from __future__ import annotations

import functools
import threading
from collections.abc import Callable, Iterator
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any, cast

import torch

from . import _lib
from . import core as _core

DEFAULT_TENSOR_CHUNK_MAX_ELEMENTS = 1_048_576


def tensor_chunk_rows(columns: int, max_rows: int, max_elements: int) -> int:
    """Bound rows by both the configured row limit and the matrix width (checkpoint.py:89-97)."""
    if columns <= 0 or max_rows <= 0 or max_elements <= 0:
        raise ValueError("Chunk dimensions and limits must be positive")
    if columns > max_elements:
        raise ValueError(
            f"One row has {columns} elements, above tensor_chunk_max_elements={max_elements}"
        )
    return min(max_rows, max_elements // columns)


class _FlagPool:
    """One reusable int32 flag word per CUDA device."""

    def __init__(self) -> None:
        self._flags: dict[int, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device) -> torch.Tensor:
        index = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            flag = self._flags.get(index)
            if flag is None:
                flag = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
                self._flags[index] = flag
        return flag


_flags = _FlagPool()


def _is_our_quantizer(quantize: Callable[..., Any]) -> bool:
    fn = quantize.func if isinstance(quantize, functools.partial) else quantize
    return fn is _core.quantize_mxfp4


def iter_quantized_row_chunks(
    read_rows: Callable[[int, int], torch.Tensor],
    quantize: Callable[[torch.Tensor], tuple[torch.Tensor, torch.Tensor]],
    *,
    rows: int,
    columns: int,
    max_rows: int,
    max_elements: int,
    name: str,
    prefetch: int | None = None,
) -> Iterator[tuple[int, int, torch.Tensor, torch.Tensor]]:
    """Read, validate, and quantize one element-bounded row slice at a time.

    ``prefetch`` chunks are read ahead on a background thread while the
    current one is quantized.  Peak memory is then (prefetch + 1) chunks
    instead of the reference's one, and ``read_rows`` is called from that
    thread, concurrently with the caller.  The default (None) prefetches 2
    chunks only when ``read_rows`` is this package's ``read_tensor_row_range``
    (which opens the file per call and is thread-safe) and reads on the
    caller's thread otherwise, as the reference does.
    """
    if prefetch is None:
        reader = read_rows.func if isinstance(read_rows, functools.partial) else read_rows
        prefetch = 2 if reader is read_tensor_row_range else 0
    chunk_rows = tensor_chunk_rows(columns, max_rows, max_elements)
    bounds = [(start, min(start + chunk_rows, rows)) for start in range(0, rows, chunk_rows)]
    if not bounds:
        return
    fused = _is_our_quantizer(quantize)
    pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="mxw-read") if prefetch > 0 else None
    # Reads issue their H2D copies on the caller's current stream, so they are
    # ordered before the kernels the caller launches on it.
    caller_stream = torch.cuda.current_stream() if torch.cuda.is_available() else None

    def read_on_caller_stream(a: int, b: int) -> torch.Tensor:
        if caller_stream is None:
            return read_rows(a, b)
        with torch.cuda.stream(caller_stream):
            return read_rows(a, b)
    pending: list[Future[torch.Tensor]] = []
    next_to_submit = 0

    def submit_reads() -> None:
        nonlocal next_to_submit
        while pool is not None and next_to_submit < len(bounds) and len(pending) < prefetch:
            a, b = bounds[next_to_submit]
            pending.append(pool.submit(read_on_caller_stream, a, b))
            next_to_submit += 1

    try:
        for index, (start, stop) in enumerate(bounds):
            if pool is None:
                weight = read_rows(start, stop)
            else:
                submit_reads()
                weight = pending.pop(0).result()
                submit_reads()
            if tuple(weight.shape) != (stop - start, columns):
                raise ValueError(f"Row slice has an unexpected shape for {name!r}")
            if fused and weight.device.type == "cuda":
                flag = _flags.get(weight.device)
                flag.zero_()
                packed, scales = quantize(weight, _flags=flag)
                if int(flag.item()) & _lib.MXW_FLAG_NONFINITE:
                    raise ValueError(f"Tensor contains NaN or infinity in rows [{start}, {stop}): {name}")
            else:
                if not torch.isfinite(weight).all():
                    raise ValueError(f"Tensor contains NaN or infinity in rows [{start}, {stop}): {name}")
                packed, scales = quantize(weight)
            del weight
            for tensor, width in ((packed, columns // 2), (scales, columns // 32)):
                if tuple(tensor.shape) != (stop - start, width) or tensor.dtype != torch.uint8:
                    raise ValueError(f"Quantized row slice has an unexpected shape or dtype: {name}")
            yield start, stop, packed, scales
            del packed, scales
            _ = index
    finally:
        if pool is not None:
            for fut in pending:
                fut.cancel()
            pool.shutdown(wait=True)


def read_tensor_row_range(
    shard: Any,
    key: str,
    start: int,
    stop: int,
    *,
    device: torch.device | str = "cpu",
) -> torch.Tensor:
    """Read the half-open row range ``[start, stop)`` of a matrix (shard.py:220-237).

    For a CUDA device the rows land in pinned host memory and are copied with
    a non-blocking H2D copy on the current stream (ordered before any kernel
    that later runs on that stream).
    """
    from safetensors import safe_open

    if start < 0 or stop <= start:
        raise ValueError("row range must satisfy 0 <= start < stop")
    with safe_open(str(shard.path), framework="pt", device="cpu") as sf:
        sliced = cast(torch.Tensor, sf.get_slice(key)[start:stop])
    if sliced.ndim != 2 or sliced.shape[0] != stop - start:
        raise ValueError(f"Tensor {key!r} cannot provide requested matrix rows [{start}, {stop})")
    target = torch.device(device)
    if target.type != "cuda":
        return sliced.to(target)
    pinned = sliced.pin_memory()
    out = pinned.to(target, non_blocking=True)
    # Keep the pinned staging buffer alive until the copy has run.
    event = torch.cuda.Event()
    event.record(torch.cuda.current_stream(target))
    _PinnedKeepAlive.hold(pinned, event)
    return out


class _PinnedKeepAlive:
    """Holds pinned staging buffers until their H2D copy has completed."""

    _lock = threading.Lock()
    _held: list[tuple[torch.Tensor, torch.cuda.Event]] = []

    @classmethod
    def hold(cls, tensor: torch.Tensor, event: torch.cuda.Event) -> None:
        with cls._lock:
            cls._held = [(t, e) for t, e in cls._held if not e.query()]
            cls._held.append((tensor, event))


__all__ = [
    "DEFAULT_TENSOR_CHUNK_MAX_ELEMENTS",
    "iter_quantized_row_chunks",
    "read_tensor_row_range",
    "tensor_chunk_rows",
]
