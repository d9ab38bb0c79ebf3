"""The reference run live on this machine's host cores against the GPU.

The golden hashes were produced by the reference under one torch CPU build.
The kernel's exponent arithmetic assumes that torch's fp32 ``log2`` rounds as
``(float)log2((double)x)`` near powers of two, and the error replay assumes
torch's CPU reduction order; a different vector-math dispatch on another host
could change either.  These tests run where the GPU is:

* torch's CPU ``log2`` near every power of two in fp32 range, against the
  float64 definition the kernel implements (the same check as the CPU suite's
  oracle test, repeated on this host);
* the reference's own ``quantize_mxfp4`` (mxwave/core.py:114-232, installed in
  baseline/_ref) on this host's cores, on config-size inputs, against this
  package's kernel on the GPU; bar: identical bytes.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mxwave_b200 import synthetic as syn
from mxwave_b200.core import quantize_mxfp4
from tests.golden.fixtures import load_config_stats
from tests.reference_pkg import import_reference

pytestmark = pytest.mark.gpu


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


def _compare(w: torch.Tensor, dev, **kw) -> None:
    ref = import_reference("mxwave.core")
    host_kw = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    p_ref, s_ref = ref.quantize_mxfp4(w, **host_kw)
    p, s = quantize_mxfp4(w.to(dev), **kw)
    torch.cuda.synchronize(dev)
    p, s = p.cpu(), s.cpu()
    bad_s = int((s != s_ref).sum())
    bad_p = int((p != p_ref).sum())
    assert bad_s == 0 and bad_p == 0, f"{bad_s} scale and {bad_p} packed byte mismatches ({kw.keys()})"


def test_host_log2_matches_float64_definition() -> None:
    from tests import test_oracle

    test_oracle.test_oracle_log2_floor_ceil_match_torch_near_powers_of_two()


def test_dense4096_unweighted_depth4_on_this_host(cuda_device) -> None:
    w = _bf16(syn.det_dense_weight(4096, 4096, seed=0))
    _compare(w, cuda_device, mse_clip_depth=4)


def test_mlp_gamma_depth1_on_this_host(cuda_device) -> None:
    stats = load_config_stats()
    if "mlp_rms" not in stats:
        pytest.skip("config statistics not generated")
    w = _bf16(syn.det_dense_weight(17408, 5120, seed=20, sigma=0.015, outlier_fraction=0.0))
    _compare(w, cuda_device, gamma=torch.from_numpy(stats["mlp_rms"]).to(cuda_device), mse_clip_depth=1)


def test_block_hessian_depth4_slice_on_this_host(cuda_device) -> None:
    stats = load_config_stats()
    if "hess5120" not in stats:
        pytest.skip("config statistics not generated")
    w = _bf16(syn.det_dense_weight(17408, 5120, seed=31, sigma=0.015)[:1024])
    _compare(w, cuda_device, hessian=torch.from_numpy(stats["hess5120"]).to(cuda_device), mse_clip_depth=4)
