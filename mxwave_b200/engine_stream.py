"""Overlapped chunk stream for the reference engine's shard writer.

Replaces ``mxwave.engine._quantized_chunks`` (mxwave/engine.py:372-394), which
reads one 1,048,576-element row chunk at a time with ``safe_open`` into
pageable memory, copies it to the device, quantizes it, synchronises on the
chunk's finiteness check and hands device tensors to
``IncrementalSafeTensorsWriter.write_u8_chunk``, whose ``.cpu()`` copies them
back synchronously (mxwave/incremental_safetensors.py:138-150).

Here a whole tensor flows through a pipeline instead:

    reader thread   file -> pinned staging slab (``readinto`` at the tensor's
                    payload offset; one copy out of the page cache)
    h2d stream      staging slab -> device input ring slot
    compute stream  quantize (sm_100a kernel, fused NaN/inf flag word per slab)
    d2h stream      packed + scales + flag word -> pinned host buffers

Slabs are whole multiples of the reference's chunk rows, so every reference
chunk lies inside one slab.  The generator yields the reference's chunks in
order, as row views of pinned host tensors: the writer's ``.cpu()`` is then a
no-op.  The flag word of a slab is read (from pinned memory, no extra
synchronisation) before any chunk of it is yielded; a NaN or infinity yields
the slab's chunks before the offending one and raises the reference's
ValueError naming that chunk's rows, which is the order in which the reference
would have yielded and raised.  Output bytes do not depend on the slab size.

The streamed path is taken when the engine would call this package's
quantizer on a CUDA device for a BF16 / F16 / F32 tensor; otherwise (a test
that monkeypatches ``mxwave.engine.quantize_mxfp4``, a CPU device, another
dtype) the engine's original function runs unchanged.
"""

from __future__ import annotations

import functools
import queue
import threading
from collections.abc import Callable, Iterator
from typing import Any

import torch

from . import _lib
from . import core as _core
from .checkpoint import tensor_chunk_rows

_TORCH_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}
_DEFAULT_SLAB_BYTES = 64 << 20
_DEPTH = 3

_original: Callable[..., Any] | None = None


def _payload_start(path) -> int:
    with open(path, "rb") as f:
        head = f.read(8)
    if len(head) != 8:
        raise ValueError(f"Invalid safetensors header in {path}")
    return 8 + int.from_bytes(head, "little")


class _Rings:
    """Per-device pinned staging slabs, device rings, streams and flag words, reused across tensors."""

    def __init__(self, device: torch.device, slab_bytes: int) -> None:
        self.device = device
        self.slab_bytes = slab_bytes
        with torch.cuda.device(device):
            self.h2d = torch.cuda.Stream(device)
            self.compute = torch.cuda.Stream(device)
            self.d2h = torch.cuda.Stream(device)
        self.staging = [torch.empty(slab_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(_DEPTH)]
        self.staging_free = [None] * _DEPTH  # event: the H2D copy out of the slot has run
        self.inputs = [torch.empty(slab_bytes, dtype=torch.uint8, device=device) for _ in range(_DEPTH)]
        self.input_free = [None] * _DEPTH  # event: the quantize reading the slot has run
        self.flags = torch.zeros(_DEPTH, dtype=torch.int32, device=device)
        self.host_flags = torch.zeros(_DEPTH, dtype=torch.int32, pin_memory=True)


_RINGS: dict[tuple[int, int], _Rings] = {}


def _rings(device: torch.device, slab_bytes: int) -> _Rings:
    key = (device.index if device.index is not None else torch.cuda.current_device(), slab_bytes)
    r = _RINGS.get(key)
    if r is None:
        r = _RINGS[key] = _Rings(torch.device("cuda", key[0]), slab_bytes)
    return r


def _engine_quantizer() -> Any:
    import sys

    engine = sys.modules.get("mxwave.engine")
    return getattr(engine, "quantize_mxfp4", None) if engine is not None else None


def _validated_statistic(value: torch.Tensor | None, check: Callable[[torch.Tensor], None],
                         device: torch.device) -> torch.Tensor | None:
    if value is None:
        return None
    check(value)
    return value.to(device=device, dtype=torch.float32).contiguous()


def quantized_chunks(shard: Any, info: Any, cfg: Any, gamma: torch.Tensor | None,
                     hessian: torch.Tensor | None) -> Iterator[tuple[int, int, torch.Tensor, torch.Tensor]]:
    """Drop-in for mxwave.engine._quantized_chunks: (start, stop, packed, scales) host chunks in order."""
    device = torch.device(cfg.device)
    dtype = _TORCH_DTYPES.get(str(getattr(info, "dtype", "")))
    if (device.type != "cuda" or dtype is None or _engine_quantizer() is not _core.quantize_mxfp4
            or len(info.shape) != 2 or _original is None):
        if _original is None:
            raise RuntimeError("mxwave_b200.engine_stream is not installed")
        yield from _original(shard, info, cfg, gamma, hessian)
        return
    yield from _stream_tensor(shard, info, cfg, gamma, hessian, device, dtype)


def _stream_tensor(shard, info, cfg, gamma, hessian, device, dtype):
    rows, cols = (int(v) for v in info.shape)
    name = info.name
    chunk_rows = tensor_chunk_rows(cols, cfg.tensor_row_chunk_size, cfg.tensor_chunk_max_elements)
    if cols % 32 != 0:
        # The reference asserts on the first chunk (core.py:160); keep its path and message.
        yield from _original(shard, info, cfg, gamma, hessian)
        return
    elem = torch.empty((), dtype=dtype).element_size()
    row_bytes = cols * elem
    slab_rows = max(chunk_rows, (_DEFAULT_SLAB_BYTES // max(row_bytes, 1)) // chunk_rows * chunk_rows)
    slab_rows = min(slab_rows, -(-rows // chunk_rows) * chunk_rows)
    R = _rings(device, max(_DEFAULT_SLAB_BYTES, slab_rows * row_bytes))
    # quantize_mxfp4's own argument checks, in its order (mxwave/core.py:151-186).
    if hessian is not None and gamma is not None:
        raise ValueError("hessian and gamma are mutually exclusive")
    if cfg.method not in ("rtn", "mse"):
        raise ValueError(f"Unsupported quantization method: {cfg.method}")
    if cfg.method == "rtn" and (gamma is not None or hessian is not None):
        raise ValueError("rtn does not use gamma or hessian weighting")
    if not 0.0 < cfg.scale_percentile <= 100.0:
        raise ValueError("scale_percentile must be in (0, 100]")
    if not isinstance(cfg.mse_clip_depth, int) or not 0 <= cfg.mse_clip_depth <= 8:
        raise ValueError("mse_clip_depth must be an integer in [0, 8]")
    h = _validated_statistic(hessian, functools.partial(_check_hessian, cols), device)
    g = _validated_statistic(gamma if cfg.method == "mse" else None, functools.partial(_check_gamma, cols), device)
    base = _payload_start(shard.path) + int(info.data_offsets[0])
    slabs = [(a, min(a + slab_rows, rows)) for a in range(0, rows, slab_rows)]

    # Reader thread: file -> pinned staging slot, in slab order.
    ready: queue.Queue = queue.Queue()
    slots_free = threading.Semaphore(_DEPTH)
    stop = threading.Event()

    def reader() -> None:
        try:
            with open(shard.path, "rb", buffering=0) as f:
                for i, (a, b) in enumerate(slabs):
                    while not slots_free.acquire(timeout=0.1):
                        if stop.is_set():
                            return
                    slot = i % _DEPTH
                    ev = R.staging_free[slot]
                    if ev is not None:
                        ev.synchronize()
                    nbytes = (b - a) * row_bytes
                    view = memoryview(R.staging[slot].numpy())[:nbytes]
                    f.seek(base + a * row_bytes)
                    got = 0
                    while got < nbytes:
                        n = f.readinto(view[got:])
                        if not n:
                            raise ValueError(f"Tensor {name!r} payload is truncated in {shard.path}")
                        got += n
                    ready.put((i, None))
        except BaseException as exc:  # surfaced on the consumer thread
            ready.put((-1, exc))

    thread = threading.Thread(target=reader, name="mxw-engine-read", daemon=True)
    thread.start()
    pending: list[tuple[int, int, int, torch.Tensor, torch.Tensor, torch.cuda.Event]] = []
    try:
        with torch.cuda.device(device):
            R.compute.wait_stream(torch.cuda.current_stream(device))
            next_slab = 0

            def enqueue() -> None:
                nonlocal next_slab
                i = next_slab
                a, b = slabs[i]
                idx, exc = ready.get()
                if exc is not None:
                    raise exc
                slot = i % _DEPTH
                n = b - a
                nbytes = n * row_bytes
                if R.input_free[slot] is not None:
                    R.h2d.wait_event(R.input_free[slot])
                with torch.cuda.stream(R.h2d):
                    R.inputs[slot][:nbytes].copy_(R.staging[slot][:nbytes], non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(R.h2d)
                R.staging_free[slot] = copied
                slots_free.release()
                weight = R.inputs[slot][:nbytes].view(dtype).view(n, cols)
                packed = torch.empty((n, cols // 2), dtype=torch.uint8, pin_memory=True)
                scales = torch.empty((n, cols // 32), dtype=torch.uint8, pin_memory=True)
                R.compute.wait_event(copied)
                with torch.cuda.stream(R.compute):
                    flag = R.flags[slot : slot + 1]
                    flag.zero_()
                    dpk = torch.empty((n, cols // 2), dtype=torch.uint8, device=device)
                    dsc = torch.empty((n, cols // 32), dtype=torch.uint8, device=device)
                    _core.quantize_into(weight, dpk, dsc, scale_percentile=cfg.scale_percentile, gamma=g, hessian=h,
                                        method=cfg.method, mse_clip_depth=cfg.mse_clip_depth, flags=flag,
                                        stream=R.compute)
                done = torch.cuda.Event()
                done.record(R.compute)
                R.input_free[slot] = done
                R.d2h.wait_event(done)
                with torch.cuda.stream(R.d2h):
                    packed.copy_(dpk, non_blocking=True)
                    scales.copy_(dsc, non_blocking=True)
                    R.host_flags[slot : slot + 1].copy_(flag, non_blocking=True)
                    dpk.record_stream(R.d2h)
                    dsc.record_stream(R.d2h)
                out = torch.cuda.Event()
                out.record(R.d2h)
                pending.append((i, a, b, packed, scales, out))
                next_slab += 1

            while next_slab < len(slabs) and len(pending) < _DEPTH - 1:
                enqueue()
            while pending:
                i, a, b, packed, scales, out = pending.pop(0)
                if next_slab < len(slabs):
                    enqueue()  # keep the pipeline busy while this slab is written
                out.synchronize()
                word = int(R.host_flags[i % _DEPTH].item())
                if word & _lib.MXW_FLAG_TIMEOUT:
                    raise RuntimeError("mxwave_b200: a device wait timed out; outputs are invalid")
                bad_chunk = _first_nonfinite_chunk(shard, name, a, b, chunk_rows, dtype, cols) \
                    if word & _lib.MXW_FLAG_NONFINITE else None
                for s in range(a, b, chunk_rows):
                    e = min(s + chunk_rows, b)
                    if bad_chunk == s:
                        raise ValueError(f"Tensor contains NaN or infinity in rows [{s}, {e}): {name}")
                    yield s, e, packed[s - a : e - a], scales[s - a : e - a]
    finally:
        stop.set()
        # Drain the slots the reader may be blocked on, then wait for it.
        for _ in range(_DEPTH):
            slots_free.release()
        thread.join()
        with torch.cuda.device(device):
            R.d2h.synchronize()


def _first_nonfinite_chunk(shard, name, a, b, chunk_rows, dtype, cols) -> int | None:
    """Row offset of the first reference chunk in [a, b) holding a NaN/inf (error path only)."""
    from safetensors import safe_open

    with safe_open(str(shard.path), framework="pt", device="cpu") as sf:
        rows = sf.get_slice(name)[a:b]
    bad = (~torch.isfinite(rows.to(torch.float32))).any(dim=1).nonzero()
    if bad.numel() == 0:
        return None
    first = a + int(bad[0, 0])
    return a + (first - a) // chunk_rows * chunk_rows


def _check_gamma(cols: int, gamma: torch.Tensor) -> None:
    if gamma.shape != (cols,):
        raise ValueError(f"gamma must have shape {(cols,)}, got {tuple(gamma.shape)}")
    if not _core._gamma_ok.ok(gamma):
        if not torch.isfinite(gamma).all() or (gamma < 0).any():
            raise ValueError("gamma must contain finite, non-negative magnitudes")
        _core._gamma_ok.add(gamma)


def _check_hessian(cols: int, hessian: torch.Tensor) -> None:
    if hessian.shape != (cols // 32, 32, 32):
        raise ValueError(f"hessian must have shape {(cols // 32, 32, 32)}, got {tuple(hessian.shape)}")
    if not _core._hessian_ok.ok(hessian):
        if not torch.isfinite(hessian).all():
            raise ValueError("hessian contains NaN or infinity")
        _core._hessian_ok.add(hessian)


def set_original(fn: Callable[..., Any] | None) -> None:
    """Record the engine's own _quantized_chunks (done by mxwave_b200.install)."""
    global _original
    _original = fn


__all__ = ["quantized_chunks", "set_original"]
