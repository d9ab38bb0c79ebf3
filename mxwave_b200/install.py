"""Install the B200 hot path behind MxWave's own Python API.

``install()`` replaces, in the already importable ``mxwave`` package, exactly
the names its engines look up at call time:

=====================================  ============================================
reference name (file:line of use)      replacement
=====================================  ============================================
mxwave.core.quantize_mxfp4             mxwave_b200.core.quantize_mxfp4
  engine.py:33,382  expert_engine.py:42,533
mxwave.core.dequant_mxfp4              mxwave_b200.core.dequant_mxfp4
  engine.py:442,565  expert_engine.py:615,771
mxwave.core.compute_block_hessian      mxwave_b200.core.compute_block_hessian
mxwave.checkpoint.iter_quantized_row_chunks
  engine.py:379  expert_engine.py:530  mxwave_b200.checkpoint.iter_quantized_row_chunks
mxwave.shard.read_tensor_row_range     mxwave_b200.checkpoint.read_tensor_row_range
  engine.py:380
mxwave.calibration.ActivationCollector mxwave_b200.calibration.ActivationCollector
mxwave.calibration.attach_activation_hooks
  calibration_stream.py:385-404        mxwave_b200.calibration.attach_activation_hooks
mxwave.calibration_stream.calibrate_decoder_sequentially
  calibration_cli.py                   mxwave_b200.calibration_stream.calibrate_decoder_sequentially
mxwave.verify.sqnr / channel_weighted_sqnr / block_hessian_weighted_sqnr
  engine.py:447-458,565-585            mxwave_b200.verify (same names)
  expert_engine.py:620,776
mxwave.routed_calibration.RoutedLayerMoments
                                       mxwave_b200.routed_calibration.RoutedLayerMoments
mxwave.gguf.repack_mxfp4_blocks        mxwave_b200.gguf.repack_mxfp4_blocks
  gguf.py:349  kolibri_gguf.py:279
mxwave.calibration.save_calibration_data / open_calibration_data
  calibration_cli.py:474  engine.py:500
                                       mxwave_b200.calibration_artifact (device hand-off)
mxwave.engine._quantized_chunks        mxwave_b200.engine_stream.quantized_chunks
  engine.py:428,630                    (file -> pinned -> HBM -> pinned pipeline per tensor)
=====================================  ============================================

The engines keep their planning, durability, manifests and CLI; only the
numeric hot path and its chunk loop move to the GPU.  ``cfg.device`` must
be a CUDA device (there is no CPU fallback).  ``uninstall()`` restores the
originals.  Test suites that monkeypatch ``mxwave.engine.quantize_mxfp4``
keep working: the engines still resolve the module attribute at call time.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from typing import Any


@dataclass
class Installation:
    """Record of replaced attributes, for uninstall()."""

    saved: list[tuple[Any, str, Any]] = field(default_factory=list)

    def uninstall(self) -> None:
        for module, name, value in reversed(self.saved):
            setattr(module, name, value)
        self.saved.clear()
        from . import engine_stream

        engine_stream.set_original(None)


def _replacements() -> dict[str, dict[str, Any]]:
    from . import (calibration, calibration_artifact, calibration_stream, checkpoint, core, engine_stream, gguf,
                   routed_calibration, verify)

    return {
        "mxwave.core": {
            "quantize_mxfp4": core.quantize_mxfp4,
            "dequant_mxfp4": core.dequant_mxfp4,
            "compute_block_hessian": core.compute_block_hessian,
        },
        "mxwave.engine": {
            "quantize_mxfp4": core.quantize_mxfp4,
            "dequant_mxfp4": core.dequant_mxfp4,
            "iter_quantized_row_chunks": checkpoint.iter_quantized_row_chunks,
            "read_tensor_row_range": checkpoint.read_tensor_row_range,
            "sqnr": verify.sqnr,
            "channel_weighted_sqnr": verify.channel_weighted_sqnr,
            "block_hessian_weighted_sqnr": verify.block_hessian_weighted_sqnr,
            "open_calibration_data": calibration_artifact.open_calibration_data,
            "_quantized_chunks": engine_stream.quantized_chunks,
        },
        "mxwave.expert_engine": {
            "quantize_mxfp4": core.quantize_mxfp4,
            "dequant_mxfp4": core.dequant_mxfp4,
            "iter_quantized_row_chunks": checkpoint.iter_quantized_row_chunks,
            "sqnr": verify.sqnr,
        },
        "mxwave.verify": {
            "sqnr": verify.sqnr,
            "channel_weighted_sqnr": verify.channel_weighted_sqnr,
            "block_hessian_weighted_sqnr": verify.block_hessian_weighted_sqnr,
        },
        "mxwave.routed_calibration": {"RoutedLayerMoments": routed_calibration.RoutedLayerMoments},
        "mxwave.gguf": {"repack_mxfp4_blocks": gguf.repack_mxfp4_blocks},
        "mxwave.kolibri_gguf": {"repack_mxfp4_blocks": gguf.repack_mxfp4_blocks},
        "mxwave": {"repack_mxfp4_blocks": gguf.repack_mxfp4_blocks},
        "mxwave.checkpoint": {"iter_quantized_row_chunks": checkpoint.iter_quantized_row_chunks},
        "mxwave.shard": {"read_tensor_row_range": checkpoint.read_tensor_row_range},
        "mxwave.calibration": {
            "ActivationCollector": calibration.ActivationCollector,
            "attach_activation_hooks": calibration.attach_activation_hooks,
            "save_calibration_data": calibration_artifact.save_calibration_data,
            "open_calibration_data": calibration_artifact.open_calibration_data,
        },
        "mxwave.calibration_stream": {
            "ActivationCollector": calibration.ActivationCollector,
            "attach_activation_hooks": calibration.attach_activation_hooks,
            "calibrate_decoder_sequentially": calibration_stream.calibrate_decoder_sequentially,
        },
        "mxwave.calibration_cli": {
            "calibrate_decoder_sequentially": calibration_stream.calibrate_decoder_sequentially,
            "save_calibration_data": calibration_artifact.save_calibration_data,
        },
    }


def install() -> Installation:
    """Patch the importable ``mxwave`` package; returns a handle for uninstall()."""
    from . import _lib

    _lib.load()  # fail loudly now, not at the first chunk, if the library is missing
    record = Installation()
    # Import every target before patching any: a module imported after another
    # was patched would bind the replacement through its own `from .x import`
    # and record it as the original.
    modules = {}
    for module_name in _replacements():
        try:
            modules[module_name] = importlib.import_module(module_name)
        except ImportError:
            continue
    if "mxwave.calibration" in modules:
        from . import calibration_artifact

        calibration_artifact._capture_originals()  # it calls the reference's own writer/reader
    if "mxwave.engine" in modules:
        from . import engine_stream

        # Tensors the stream does not take (another quantizer patched in, a CPU
        # device) go through the engine's own chunk loop.
        engine_stream.set_original(getattr(modules["mxwave.engine"], "_quantized_chunks", None))
    for module_name, names in _replacements().items():
        module = modules.get(module_name)
        if module is None:
            continue
        for name, value in names.items():
            if hasattr(module, name):
                record.saved.append((module, name, getattr(module, name)))
                setattr(module, name, value)
    return record


__all__ = ["Installation", "install"]
