"""The torch operator layer (mxwave_b200.ops) over the C ABI.

CPU: every operator is registered under ``mxwave_b200::`` with the expected
schema, and its fake implementation propagates shapes and dtypes (FakeTensor
needs no GPU).  GPU: ``torch.library.opcheck`` on every operator, a
``torch.compile``d caller of the quantize operator gives the eager bytes, and
the default flag word of ``quantize_mxfp4`` does not keep a stale rare-block
bit from one call to the next.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from mxwave_b200 import ops  # noqa: F401  -- registers the operators
from mxwave_b200 import synthetic as syn

SCHEMAS = {
    "quantize_mxfp4": "mxwave_b200::quantize_mxfp4(Tensor weight, float scale_percentile, Tensor? gamma, "
                      "Tensor? hessian, SymInt method, SymInt mse_clip_depth, Tensor(a6!) flags) -> (Tensor, Tensor)",
    "dequant_mxfp4": "mxwave_b200::dequant_mxfp4(Tensor packed, Tensor scales, SymInt rows, SymInt cols) -> Tensor",
    "accumulate_moments_": "mxwave_b200::accumulate_moments_(Tensor x, Tensor(a1!) sum_abs, Tensor(a2!) sum_sq) -> ()",
    "accumulate_activation_stats_": "mxwave_b200::accumulate_activation_stats_(Tensor x, Tensor(a1!)? sum_abs, "
                                    "Tensor(a2!)? sum_sq, Tensor(a3!)? gram_blocks) -> ()",
    "accumulate_xtx_": "mxwave_b200::accumulate_xtx_(Tensor x, Tensor(a1!) gram) -> ()",
    "finalize_moments": "mxwave_b200::finalize_moments(Tensor sums, SymInt count, bool root) -> Tensor",
    "finalize_block_hessian": "mxwave_b200::finalize_block_hessian(Tensor gram, bool full, SymInt count, float damp, "
                              "SymInt mode) -> Tensor",
}


@pytest.mark.parametrize("name", sorted(SCHEMAS))
def test_schema(name: str) -> None:
    op = getattr(torch.ops.mxwave_b200, name).default
    assert str(op._schema) == SCHEMAS[name]


def test_fake_shapes() -> None:
    with FakeTensorMode():
        w = torch.empty(96, 160, dtype=torch.bfloat16, device="cuda")
        flags = torch.zeros(1, dtype=torch.int32, device="cuda")
        p, s = torch.ops.mxwave_b200.quantize_mxfp4(w, 99.5, None, None, 0, 1, flags)
        assert p.shape == (96, 80) and s.shape == (96, 5) and p.dtype == s.dtype == torch.uint8
        d = torch.ops.mxwave_b200.dequant_mxfp4(p, s, 96, 160)
        assert d.shape == (96, 160) and d.dtype == torch.float32
        g = torch.empty(5, 32, 32, device="cuda")
        h = torch.ops.mxwave_b200.finalize_block_hessian(g, False, 10, 1e-6, 0)
        assert h.shape == (5, 32, 32)
        full = torch.empty(160, 160, device="cuda")
        assert torch.ops.mxwave_b200.finalize_block_hessian(full, True, 10, 1e-6, 0).shape == (5, 32, 32)
        m = torch.ops.mxwave_b200.finalize_moments(torch.empty(160, device="cuda"), 7, True)
        assert m.shape == (160,) and m.dtype == torch.float32


def _weight(rows: int, cols: int, seed: int, device) -> torch.Tensor:
    bits = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.01)
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)


@pytest.mark.gpu
def test_opcheck_every_operator(cuda_device) -> None:
    dev = cuda_device
    w = _weight(64, 256, 1, dev)
    gamma = torch.rand(256, device=dev) + 0.1
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    x = (torch.randn(300, 256, device=dev) * 3).to(torch.bfloat16)
    checks = [
        (torch.ops.mxwave_b200.quantize_mxfp4.default, (w, 99.5, None, None, 0, 1, flags)),
        (torch.ops.mxwave_b200.quantize_mxfp4.default, (w, 99.5, gamma, None, 0, 4, flags)),
        (torch.ops.mxwave_b200.accumulate_moments_.default,
         (x, torch.zeros(256, device=dev), torch.zeros(256, device=dev))),
        (torch.ops.mxwave_b200.accumulate_activation_stats_.default,
         (x, None, torch.zeros(256, device=dev), torch.zeros(8, 32, 32, device=dev))),
        (torch.ops.mxwave_b200.accumulate_xtx_.default, (x, torch.zeros(256, 256, device=dev))),
        (torch.ops.mxwave_b200.finalize_moments.default, (torch.rand(256, device=dev), 300, True)),
        (torch.ops.mxwave_b200.finalize_block_hessian.default, (torch.rand(8, 32, 32, device=dev), False, 300, 1e-6, 0)),
    ]
    p, s = torch.ops.mxwave_b200.quantize_mxfp4(w, 99.5, None, None, 0, 1, flags)
    checks.append((torch.ops.mxwave_b200.dequant_mxfp4.default, (p, s, 64, 256)))
    for op, args in checks:
        torch.library.opcheck(op, args)


@pytest.mark.gpu
@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_compiled_caller_gives_eager_bytes(cuda_device, backend) -> None:
    from mxwave_b200.core import quantize_mxfp4

    w = _weight(256, 512, 2, cuda_device)
    gamma = torch.rand(512, device=cuda_device) + 0.1

    def step(weight: torch.Tensor, g: torch.Tensor, flags: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return torch.ops.mxwave_b200.quantize_mxfp4(weight, 99.5, g, None, 0, 1, flags)

    compiled = torch.compile(step, fullgraph=True, backend=backend)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    cp, cs = compiled(w, gamma, flags)
    ep, es = quantize_mxfp4(w, gamma=gamma)
    assert torch.equal(cp, ep) and torch.equal(cs, es)
    torch._dynamo.reset()


@pytest.mark.gpu
def test_default_flag_word_is_cleared_between_calls(cuda_device) -> None:
    from mxwave_b200 import _lib
    from mxwave_b200.core import _DEVICE_FLAGS, quantize_mxfp4

    normal = _weight(64, 256, 3, cuda_device)
    rare = normal.clone()
    rare[5, :32] = 1.0e6  # block scale 2^17: outside the fast path, finished by the rare-block pass
    key = (cuda_device.index if cuda_device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(cuda_device).cuda_stream)
    quantize_mxfp4(rare)
    torch.cuda.synchronize()
    assert int(_DEVICE_FLAGS[key].item()) & _lib.MXW_FLAG_RARE
    p, s = quantize_mxfp4(normal)
    torch.cuda.synchronize()
    assert int(_DEVICE_FLAGS[key].item()) == 0  # the later call's rare-block pass returned at once
    p2, s2 = quantize_mxfp4(normal.clone())
    assert torch.equal(p, p2) and torch.equal(s, s2)
