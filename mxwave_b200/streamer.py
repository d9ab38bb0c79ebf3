"""Host -> HBM -> host MXFP4 quantization pipeline (the chunked checkpoint engine).

A weight held in host memory (pinned for asynchronous copies) is cut into row
slabs.  Three CUDA streams overlap the stages of consecutive slabs:

    h2d stream     copy slab i      host -> device input ring slot i % depth
    compute stream quantize slab i  (sm_100a kernel, fused NaN/inf flag)
    d2h stream     copy slab i      packed + scales -> host outputs

with CUDA events between the stages and before every ring slot is reused.
The host thread only enqueues work; nothing blocks until ``finish``.  Output
bytes do not depend on the slab size (rows are independent), so slabs are far
larger than the reference's 1,048,576-element chunks (mxwave/checkpoint.py:20),
which are an artefact of its synchronous loop.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .core import BLOCK_SIZE, _gamma_ok, _hessian_ok, quantize_into


@dataclass
class _Slot:
    weight: torch.Tensor
    packed: torch.Tensor
    scales: torch.Tensor
    in_free: torch.cuda.Event
    out_free: torch.cuda.Event


class ChunkStreamer:
    """Reusable device rings for streaming many host tensors through the quantizer."""

    def __init__(self, device: torch.device | str | None = None, slab_bytes: int = 64 << 20, depth: int = 2) -> None:
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise RuntimeError("ChunkStreamer streams to a CUDA device (no CPU fallback)")
        self.slab_bytes = int(slab_bytes)
        self.depth = int(depth)
        with torch.cuda.device(self.device):
            self.h2d = torch.cuda.Stream(self.device)
            self.compute = torch.cuda.Stream(self.device)
            self.d2h = torch.cuda.Stream(self.device)
        # One flag word per enqueued slab (NaN/inf, wait timeout), read by finish().
        self._flag_pages: list[torch.Tensor] = []
        self._pending: list[tuple[str, int, int]] = []  # (name, first row, last row + 1) per slab
        self._slots: list[_Slot] = []
        self._shape_key: tuple | None = None

    _FLAG_PAGE = 1024

    def _next_flag(self) -> torch.Tensor:
        i = len(self._pending)
        page, slot = divmod(i, self._FLAG_PAGE)
        if page == len(self._flag_pages):
            # Zeroed on the current stream, which the compute stream waits on before use.
            self._flag_pages.append(torch.zeros(self._FLAG_PAGE, dtype=torch.int32, device=self.device))
        return self._flag_pages[page][slot : slot + 1]

    def _ensure(self, rows: int, cols: int, dtype: torch.dtype) -> None:
        key = (rows, cols, dtype)
        if self._shape_key == key:
            return
        with torch.cuda.device(self.device):
            self._slots = []
            for _ in range(self.depth):
                ev_in, ev_out = torch.cuda.Event(), torch.cuda.Event()
                ev_in.record(self.compute)
                ev_out.record(self.d2h)
                self._slots.append(
                    _Slot(
                        torch.empty((rows, cols), dtype=dtype, device=self.device),
                        torch.empty((rows, cols // 2), dtype=torch.uint8, device=self.device),
                        torch.empty((rows, cols // BLOCK_SIZE), dtype=torch.uint8, device=self.device),
                        ev_in,
                        ev_out,
                    )
                )
        self._shape_key = key

    @torch.no_grad()
    def quantize(
        self,
        weight: torch.Tensor,
        packed_out: torch.Tensor | None = None,
        scales_out: torch.Tensor | None = None,
        *,
        scale_percentile: float = 99.5,
        gamma: torch.Tensor | None = None,
        hessian: torch.Tensor | None = None,
        method: str = "mse",
        mse_clip_depth: int = 1,
        name: str = "weight",
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """Quantize a host [rows, cols] tensor; returns host (packed, scales).

        Outputs are written into `packed_out` / `scales_out` when given (pinned
        host tensors keep the copies asynchronous).  Raises ValueError, with the
        reference's message, if the weight holds a NaN or infinity.  gamma and
        hessian are validated as the reference validates them.
        """
        if weight.ndim != 2 or weight.shape[1] % BLOCK_SIZE != 0:
            raise ValueError(f"Expected a 2D weight tensor with a multiple of {BLOCK_SIZE} columns")
        if weight.device.type != "cpu":
            raise ValueError("ChunkStreamer.quantize takes a host tensor")
        rows, cols = weight.shape
        if packed_out is None:
            packed_out = torch.empty((rows, cols // 2), dtype=torch.uint8, pin_memory=True)
        if scales_out is None:
            scales_out = torch.empty((rows, cols // BLOCK_SIZE), dtype=torch.uint8, pin_memory=True)
        g = h = None
        with torch.cuda.device(self.device):
            # Validated once per unchanged statistic tensor (a host sync each
            # time otherwise, which would serialise the copy pipeline).
            if gamma is not None:
                if gamma.shape != (cols,):
                    raise ValueError(f"gamma must have shape {(cols,)}, got {tuple(gamma.shape)}")
                if not _gamma_ok.ok(gamma):
                    if not torch.isfinite(gamma).all() or (gamma < 0).any():
                        raise ValueError("gamma must contain finite, non-negative magnitudes")
                    _gamma_ok.add(gamma)
                g = gamma.to(device=self.device, dtype=torch.float32).contiguous()
            if hessian is not None:
                if hessian.shape != (cols // BLOCK_SIZE, BLOCK_SIZE, BLOCK_SIZE):
                    raise ValueError(
                        f"hessian must have shape {(cols // BLOCK_SIZE, BLOCK_SIZE, BLOCK_SIZE)}, "
                        f"got {tuple(hessian.shape)}"
                    )
                if not _hessian_ok.ok(hessian):
                    if not torch.isfinite(hessian).all():
                        raise ValueError("hessian contains NaN or infinity")
                    _hessian_ok.add(hessian)
                h = hessian.to(device=self.device, dtype=torch.float32).contiguous()
            slab_rows = max(1, min(rows, self.slab_bytes // max(1, cols * weight.element_size())))
            self._ensure(slab_rows, cols, weight.dtype)
            flags = [self._next_flag_for(name, start, min(start + slab_rows, rows)) for start in range(0, rows, slab_rows)]
            self.compute.wait_stream(torch.cuda.current_stream(self.device))
            for i, start in enumerate(range(0, rows, slab_rows)):
                stop = min(start + slab_rows, rows)
                n = stop - start
                slot = self._slots[i % self.depth]
                # h2d: slab -> input ring slot (free once its previous quantize ran)
                self.h2d.wait_event(slot.in_free)
                with torch.cuda.stream(self.h2d):
                    slot.weight[:n].copy_(weight[start:stop], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(self.h2d)
                # compute: quantize into the output ring slot (free once copied out)
                self.compute.wait_event(ready)
                self.compute.wait_event(slot.out_free)
                quantize_into(slot.weight[:n], slot.packed[:n], slot.scales[:n], scale_percentile=scale_percentile,
                              gamma=g, hessian=h, method=method, mse_clip_depth=mse_clip_depth, flags=flags[i],
                              stream=self.compute)
                slot.in_free.record(self.compute)
                done = torch.cuda.Event()
                done.record(self.compute)
                # d2h: outputs -> host
                self.d2h.wait_event(done)
                with torch.cuda.stream(self.d2h):
                    packed_out[start:stop].copy_(slot.packed[:n], non_blocking=True)
                    scales_out[start:stop].copy_(slot.scales[:n], non_blocking=True)
                slot.out_free.record(self.d2h)
            torch.cuda.current_stream(self.device).wait_stream(self.d2h)
        return packed_out, scales_out

    def _next_flag_for(self, name: str, start: int, stop: int) -> torch.Tensor:
        flag = self._next_flag()
        self._pending.append((name, start, stop))
        return flag

    def finish(self) -> None:
        """Wait for every enqueued slab; raise if any quantized input held a NaN/inf.

        The error names the first offending slab (tensor name and row range),
        in enqueue order, with the reference's message.
        """
        self.d2h.synchronize()
        self.compute.synchronize()
        pending, self._pending = self._pending, []
        if not pending:
            return
        words = torch.cat([p for p in self._flag_pages]).cpu()[: len(pending)].tolist()
        for page in self._flag_pages:
            page.zero_()
        torch.cuda.current_stream(self.device).synchronize()
        for (name, start, stop), word in zip(pending, words):
            if word & _lib.MXW_FLAG_TIMEOUT:
                raise RuntimeError("mxwave_b200: a device wait timed out; outputs are invalid")
            if word & _lib.MXW_FLAG_NONFINITE:
                raise ValueError(f"Tensor contains NaN or infinity in rows [{start}, {stop}): {name}")


def quantize_host(weight: torch.Tensor, **kwargs) -> tuple[torch.Tensor, torch.Tensor]:
    """One-shot convenience: stream a host tensor through the quantizer and wait."""
    streamer = ChunkStreamer(kwargs.pop("device", None))
    packed, scales = streamer.quantize(weight, **kwargs)
    streamer.finish()
    return packed, scales


__all__ = ["ChunkStreamer", "quantize_host"]
