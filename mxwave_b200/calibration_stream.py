"""Drop-in for ``mxwave.calibration_stream.calibrate_decoder_sequentially`` on B200.

Same signature, validation and result type as the reference
(mxwave/calibration_stream.py:296-466).  What changes:

* hidden states stay in HBM between layers (two device buffers of
  [sequences, length, hidden]) instead of a CPU copy with an H2D/D2H round
  trip per batch per layer (calibration_stream.py:339-349, 409, 441); when
  they do not fit the given budget they live in pinned host memory and move
  with asynchronous copies;
* statistics are accumulated by ``mxwave_b200.calibration.ActivationCollector``
  (sm_100a kernel, one read per distinct input: q/k/v and gate/up share one);
  layers run under ``torch.no_grad`` rather than inference mode so that the
  shared inputs keep the version counter that proves them unchanged;
* with ``process_group`` set, sequences are split across ranks (contiguous,
  equal slices) and each layer's fp32 accumulators and counts are summed with
  one all-reduce before finalisation, so every rank returns the statistics of
  the whole corpus.

The model-structure helpers (layout inference, module loading from
safetensors, attention masks, rotary embeddings, calling a layer) are the
reference's own functions, imported from ``mxwave.calibration_stream``; they
are not on the hot path.
"""

from __future__ import annotations

import copy
import importlib
from collections.abc import Callable, Mapping, Sequence
from pathlib import Path
from typing import Any, cast

import torch

from .calibration import ActivationCollector, attach_activation_hooks


def _reference() -> Any:
    return importlib.import_module("mxwave.calibration_stream")


def _shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    return n * rank // world, n * (rank + 1) // world


def calibrate_decoder_sequentially(
    model: torch.nn.Module,
    target_widths: Mapping[str, int],
    objectives: Sequence[str],
    sequences: Sequence[Sequence[int]],
    checkpoint_files: Mapping[str, Path],
    *,
    device: torch.device,
    dtype: torch.dtype,
    batch_size: int,
    hessian_damp: float,
    hessian_damp_mode: str = "absolute",
    skip_first_tokens: int = 0,
    progress: Callable[[int, int], None] | None = None,
    process_group: Any = None,
    hidden_budget_bytes: int | None = None,
) -> Any:
    """Capture statistics while keeping at most one decoder layer resident."""
    ref = _reference()
    if not sequences:
        raise ValueError("Sequential calibration requires at least one sequence")
    if batch_size <= 0:
        raise ValueError("batch_size must be positive")
    sequence_length = len(sequences[0])
    if sequence_length == 0 or any(len(sequence) != sequence_length for sequence in sequences):
        raise ValueError("Sequential calibration requires equal non-empty sequence lengths")
    if not 0 <= skip_first_tokens < sequence_length:
        raise ValueError("skip_first_tokens must be in [0, sequence_length)")
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("mxwave_b200 calibrates on CUDA devices only (no CPU fallback)")

    world, rank = 1, 0
    if process_group is not None:
        import torch.distributed as dist

        world, rank = dist.get_world_size(process_group), dist.get_rank(process_group)
    lo, hi = _shard_bounds(len(sequences), rank, world)
    local = sequences[lo:hi]

    layout = ref.infer_sequential_decoder_layout(model, target_widths, checkpoint_files)
    base = ref._module_at(model, layout.base_prefix)
    stack = cast(torch.nn.ModuleList, ref._module_at(model, layout.stack_prefix))
    embedding = ref._load_module_from_checkpoint(
        copy.deepcopy(ref._module_at(model, layout.embedding_prefix)),
        layout.embedding_prefix,
        checkpoint_files,
        device=device,
        dtype=dtype,
    )
    embedding.eval()
    first_parameter = next(embedding.parameters(), None)
    if first_parameter is None or first_parameter.ndim != 2:
        raise ValueError("Sequential calibration embedding has no matrix parameter")
    hidden_width = first_parameter.shape[-1]

    n_local = len(local)
    element = torch.empty((), dtype=dtype).element_size()
    hidden_bytes = 2 * max(n_local, 1) * sequence_length * hidden_width * element
    if hidden_budget_bytes is None:
        free, _total = torch.cuda.mem_get_info(device)
        hidden_budget_bytes = free // 2
    on_device = hidden_bytes <= hidden_budget_bytes
    store_device = device if on_device else torch.device("cpu")

    def new_hidden() -> torch.Tensor:
        return torch.empty(
            (n_local, sequence_length, hidden_width), dtype=dtype, device=store_device,
            pin_memory=not on_device,
        )

    hidden = new_hidden()
    with torch.no_grad():
        for start in range(0, n_local, batch_size):
            rows = local[start : start + batch_size]
            input_ids = torch.tensor(rows, dtype=torch.long, device=device)
            hidden[start : start + len(rows)].copy_(embedding(input_ids), non_blocking=True)
    del embedding
    ref._advise_prefix_unused(checkpoint_files, layout.embedding_prefix)

    rotary = ref._new_rotary(
        ref._module_at(base, "rotary_emb"), base.config, f"{layout.base_prefix}.rotary_emb",
        checkpoint_files, device=device, dtype=dtype,
    )
    position_ids = torch.arange(sequence_length, dtype=torch.long, device=device).unsqueeze(0)
    statistics: dict[str, dict[str, torch.Tensor]] = {objective: {} for objective in objectives}
    counts: dict[str, int] = {}
    next_hidden = new_hidden()

    with torch.no_grad():
        for layer_index in range(layout.layer_count):
            layer_prefix = f"{layout.stack_prefix}.{layer_index}"
            layer = ref._load_module_from_checkpoint(
                copy.deepcopy(stack[layer_index]), layer_prefix, checkpoint_files, device=device, dtype=dtype,
            )
            layer.eval()
            layer_widths = {n: w for n, w in target_widths.items() if n.startswith(f"{layer_prefix}.")}
            collector = (
                ActivationCollector(
                    layer_widths, objectives, hessian_damp=hessian_damp,
                    hessian_damp_mode=hessian_damp_mode, skip_first_tokens=skip_first_tokens,
                )
                if layer_widths
                else None
            )
            handles = attach_activation_hooks(layer, collector, module_prefix=layer_prefix) if collector else []
            try:
                for start in range(0, n_local, batch_size):
                    stop = min(start + batch_size, n_local)
                    batch = hidden[start:stop]
                    if not on_device:
                        batch = batch.to(device, non_blocking=True)
                    ones = torch.ones((stop - start, sequence_length), dtype=torch.long, device=device)
                    layer_mask = ref._attention_mask_for_layer(base, batch, ones, position_ids, layer_index)
                    raw = rotary(batch, position_ids)
                    if not isinstance(raw, tuple) or len(raw) != 2 or not all(isinstance(t, torch.Tensor) for t in raw):
                        raise TypeError("rotary_emb must return a (cos, sin) tensor tuple")
                    output = ref._run_layer(
                        layer, batch, position_embeddings=cast(tuple[torch.Tensor, torch.Tensor], raw),
                        attention_mask=layer_mask, position_ids=position_ids,
                    )
                    next_hidden[start:stop].copy_(output, non_blocking=True)
            finally:
                for handle in handles:
                    handle.remove()
            if collector is not None:
                if process_group is not None:
                    collector.all_reduce(process_group)
                layer_statistics = collector.finalize()
                for objective, values in layer_statistics.items():
                    statistics[objective].update(values)
                counts.update(collector.observation_counts)
            hidden, next_hidden = next_hidden, hidden
            del layer, collector
            ref._advise_prefix_unused(checkpoint_files, layer_prefix)
            if progress is not None:
                progress(layer_index + 1, layout.layer_count)

    if set(counts) != set(target_widths):
        missing = sorted(set(target_widths).difference(counts))
        raise ValueError(f"Sequential calibration missed {len(missing)} target(s): {missing[:5]}")
    return ref.StreamingCalibrationResult(
        statistics=statistics, observation_counts=counts, layer_count=layout.layer_count
    )


__all__ = ["calibrate_decoder_sequentially"]
