"""GPU parity of the calibration statistics kernels (through the C ABI)
against the float64 oracle.  Bar: 1e-5 relative (fp32 accumulation)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mxwave_b200 import _lib
from mxwave_b200 import synthetic as syn
from mxwave_b200.core import compute_block_hessian
from oracle import oracle

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _gram_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |dG_ij| / sqrt(G_ii G_jj) over each 32x32 block (Cauchy-Schwarz scale)."""
    d = np.einsum("bii->bi", ref)
    scale = np.sqrt(np.maximum(d[:, :, None] * d[:, None, :], 1e-300))
    return float(np.max(np.abs(got - ref) / scale))


def _x(tokens: int, cols: int, seed: int, dev, dtype=torch.bfloat16):
    bits = syn.det_activations(tokens, cols, seed)
    xf = syn.bf16_bits_to_f32(bits)
    t = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)
    if dtype != torch.bfloat16:
        t = t.to(dtype)
        xf = t.float().cpu().numpy()
    return t, xf.astype(np.float64)


SIZES = [(1, 32), (7, 64), (300, 96), (1000, 160), (8192, 5120), (4097, 544)]


@pytest.mark.parametrize("tokens,cols", SIZES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_moments_and_block_gram(tokens, cols, dtype, cuda_device) -> None:
    if dtype != torch.bfloat16 and tokens > 5000:
        pytest.skip("large case covered in bf16")
    lib = _lib.load()
    x, xf = _x(tokens, cols, tokens + cols, cuda_device, dtype)
    s1 = torch.zeros(cols, device=cuda_device)
    s2 = torch.zeros(cols, device=cuda_device)
    g = torch.zeros(cols // 32, 32, 32, device=cuda_device)
    code = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}[dtype]
    st = lib.mxw_accumulate_activation_stats(x.data_ptr(), code, tokens, cols, cols, s1.data_ptr(),
                                             s2.data_ptr(), g.data_ptr(), None, _stream(cuda_device))
    assert st == _lib.MXW_OK
    torch.cuda.synchronize()
    r1, r2 = oracle.moments(xf)
    np.testing.assert_allclose(s1.cpu().numpy(), r1, rtol=RTOL)
    np.testing.assert_allclose(s2.cpu().numpy(), r2, rtol=RTOL)
    assert _gram_err(g.cpu().numpy(), oracle.block_gram(xf)) < RTOL


# Moments without the block Gram take the vector-load pass when the width is a
# multiple of 4 and the rows are 8-byte aligned (16-byte for fp32): 128-channel
# strips (the last one ragged below), one to eight token slices per strip.
@pytest.mark.parametrize("tokens,cols", [(1, 4), (513, 100), (9000, 644), (4096, 5120)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("which", ["abs", "sq", "both"])
def test_moments_only_pass(tokens, cols, dtype, which, cuda_device) -> None:
    lib = _lib.load()
    x, xf = _x(tokens, cols, 7 * tokens + cols, cuda_device, dtype)
    code = {torch.bfloat16: _lib.MXW_BF16, torch.float16: _lib.MXW_F16, torch.float32: _lib.MXW_F32}[dtype]
    r1, r2 = oracle.moments(xf)
    runs = []
    for _ in range(2):
        s1 = torch.full((cols,), 0.5, device=cuda_device) if which != "sq" else None
        s2 = torch.full((cols,), 0.25, device=cuda_device) if which != "abs" else None
        st = lib.mxw_accumulate_moments(x.data_ptr(), code, tokens, cols, cols,
                                        None if s1 is None else s1.data_ptr(),
                                        None if s2 is None else s2.data_ptr(), _stream(cuda_device))
        assert st == _lib.MXW_OK
        torch.cuda.synchronize()
        if s1 is not None:
            np.testing.assert_allclose(s1.cpu().numpy(), r1 + 0.5, rtol=RTOL)
        if s2 is not None:
            np.testing.assert_allclose(s2.cpu().numpy(), r2 + 0.25, rtol=RTOL)
        runs.append([t.cpu() for t in (s1, s2) if t is not None])
    for a, b in zip(*runs):
        assert torch.equal(a, b)  # fixed summation order: identical bits run to run


# Widths that are multiples of 128 with 2-byte activations take the tensor-core
# block Gram (xtx.cu block_gram_tc_kernel): one to eight token slices per
# 128-channel strip, and more than one launch past 262,144 tokens.
TC_SIZES = [(1, 128), (63, 256), (300, 384), (4097, 640), (70001, 256), (262200, 128)]


@pytest.mark.parametrize("tokens,cols", TC_SIZES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_block_gram_on_tensor_cores(tokens, cols, dtype, cuda_device) -> None:
    lib = _lib.load()
    x, xf = _x(tokens, cols, 3 * tokens + cols, cuda_device, dtype)
    code = _lib.MXW_BF16 if dtype == torch.bfloat16 else _lib.MXW_F16
    ref = oracle.block_gram(xf)
    grams = []
    for _ in range(2):
        g = torch.zeros(cols // 32, 32, 32, device=cuda_device)
        s2 = torch.zeros(cols, device=cuda_device)
        assert lib.mxw_accumulate_activation_stats(x.data_ptr(), code, tokens, cols, cols, None, s2.data_ptr(),
                                                   g.data_ptr(), None, _stream(cuda_device)) == 0
        torch.cuda.synchronize()
        assert _gram_err(g.cpu().numpy(), ref) < RTOL
        np.testing.assert_allclose(s2.cpu().numpy(), oracle.moments(xf)[1], rtol=RTOL)
        grams.append(g.cpu())
    assert torch.equal(grams[0], grams[1])  # deterministic run to run


def test_accumulation_across_calls_and_ragged_width(cuda_device) -> None:
    lib = _lib.load()
    x, xf = _x(3000, 5120, 5, cuda_device)
    s2 = torch.zeros(5120, device=cuda_device)
    g = torch.zeros(160, 32, 32, device=cuda_device)
    for a, b in ((0, 1000), (1000, 1001), (1001, 3000)):
        part = x[a:b]
        assert lib.mxw_accumulate_activation_stats(part.data_ptr(), _lib.MXW_BF16, b - a, 5120, 5120, None,
                                                   s2.data_ptr(), g.data_ptr(), None, _stream(cuda_device)) == 0
    torch.cuda.synchronize()
    np.testing.assert_allclose(s2.cpu().numpy(), oracle.moments(xf)[1], rtol=RTOL)
    assert _gram_err(g.cpu().numpy(), oracle.block_gram(xf)) < RTOL
    # Width not divisible by 32 (moments only) and a strided view (plain path).
    y, yf = _x(500, 70, 6, cuda_device)
    s1 = torch.zeros(70, device=cuda_device)
    assert lib.mxw_accumulate_moments(y.data_ptr(), _lib.MXW_BF16, 500, 70, 70, s1.data_ptr(), None,
                                      _stream(cuda_device)) == 0
    z = x[:, 1:1025]
    sz = torch.zeros(1024, device=cuda_device)
    assert lib.mxw_accumulate_moments(z.data_ptr(), _lib.MXW_BF16, 3000, 1024, z.stride(0), None, sz.data_ptr(),
                                      _stream(cuda_device)) == 0
    torch.cuda.synchronize()
    np.testing.assert_allclose(s1.cpu().numpy(), oracle.moments(yf)[0], rtol=RTOL)
    np.testing.assert_allclose(sz.cpu().numpy(), oracle.moments(xf[:, 1:1025])[1], rtol=RTOL)


@pytest.mark.parametrize("mode", ["absolute", "relative"])
def test_compute_block_hessian_matches_oracle(mode, cuda_device) -> None:
    x, xf = _x(2048, 1024, 9, cuda_device)
    h = compute_block_hessian(x, damp=1e-3, damp_mode=mode).cpu().numpy()
    ref = oracle.finalize_block_hessian(oracle.block_gram(xf), 2048, 1e-3, mode)
    assert _gram_err(h, ref) < RTOL


def test_finalize_moments(cuda_device) -> None:
    lib = _lib.load()
    s1 = torch.rand(333, device=cuda_device) * 100
    s2 = torch.rand(333, device=cuda_device) * 100
    ma = torch.empty(333, device=cuda_device)
    rms = torch.empty(333, device=cuda_device)
    assert lib.mxw_finalize_moments(s1.data_ptr(), s2.data_ptr(), 333, 77, ma.data_ptr(), rms.data_ptr(),
                                    _stream(cuda_device)) == 0
    torch.cuda.synchronize()
    # Same fp32 operations as the reference's CPU finalize (calibration.py:
    # 262-266): IEEE division by the count, then an IEEE square root.
    c1, c2 = s1.cpu(), s2.cpu()
    assert torch.equal(ma.cpu(), c1 / 77)
    # torch's vectorised CPU sqrt may differ from the IEEE square root by 1 ulp.
    torch.testing.assert_close(rms.cpu(), torch.sqrt(c2 / 77), rtol=2e-7, atol=0)


def test_dequant_matches_oracle(cuda_device) -> None:
    from mxwave_b200.core import dequant_mxfp4, quantize_mxfp4

    w = syn.det_dense_weight(33, 256, 4, outlier_fraction=0.05)
    wt = torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16).to(cuda_device)
    p, s = quantize_mxfp4(wt)
    d = dequant_mxfp4(p, s, (33, 256)).cpu().numpy()
    ref = oracle.dequant_mxfp4(p.cpu().numpy(), s.cpu().numpy(), 256)
    np.testing.assert_array_equal(d, ref)


# ------------------------------------------------------------- full X^T X


def _full_err(got: np.ndarray, ref: np.ndarray) -> float:
    d = np.diag(ref)
    scale = np.sqrt(np.maximum(np.outer(d, d), 1e-300))
    return float(np.max(np.abs(got - ref) / scale))


# 262,200 tokens: two launches (at most 262,144 tokens each) and a ragged last
# 1024-token TMEM chunk.
@pytest.mark.parametrize("tokens,cols", [(1, 128), (64, 128), (1000, 256), (300, 384), (4097, 640), (65536, 1024),
                                         (262200, 128)])
def test_xtx_matches_fp64(tokens, cols, cuda_device) -> None:
    lib = _lib.load()
    x, xf = _x(tokens, cols, tokens * 3 + cols, cuda_device)
    g = torch.zeros(cols, cols, device=cuda_device)
    st = lib.mxw_accumulate_xtx(x.data_ptr(), tokens, cols, cols, g.data_ptr(), cols, None, _stream(cuda_device))
    assert st == _lib.MXW_OK
    torch.cuda.synchronize()
    ref = oracle.gram(xf)
    got = g.cpu().numpy()
    assert _full_err(got.astype(np.float64), ref) < RTOL
    # Only the upper triangle's tiles are computed; the lower one is their mirror.
    assert np.array_equal(got, got.T)


@pytest.mark.parametrize("cols", [384, 512, 640, 1024])
def test_xtx_packed_then_unpacked_equals_direct(cols, cuda_device) -> None:
    """Two token slices accumulated in the packed tile form and unpacked give
    the direct path's Gram bit for bit (the all-reduce path of the bench), at
    widths with and without a ragged last 256-column tile."""
    lib = _lib.load()
    x, _ = _x(3000, cols, cols + 5, cuda_device)
    direct = torch.zeros(cols, cols, device=cuda_device)
    n_packed = lib.mxw_xtx_packed_floats(cols)
    n_tiles = sum((cols + 255) // 256 - (by >> 1) for by in range(cols // 128))
    assert n_packed == n_tiles * 128 * 256
    packed = torch.zeros(n_packed, device=cuda_device)
    for a, b in ((0, 1234), (1234, 3000)):
        part = x[a:b]
        assert lib.mxw_accumulate_xtx(part.data_ptr(), b - a, cols, cols, direct.data_ptr(), cols, None,
                                      _stream(cuda_device)) == 0
        assert lib.mxw_accumulate_xtx_packed(part.data_ptr(), b - a, cols, cols, packed.data_ptr(), None,
                                             _stream(cuda_device)) == 0
    unpacked = torch.zeros(cols, cols, device=cuda_device)
    assert lib.mxw_xtx_unpack(packed.data_ptr(), cols, unpacked.data_ptr(), cols, _stream(cuda_device)) == 0
    torch.cuda.synchronize()
    assert torch.equal(direct, unpacked)
    assert lib.mxw_xtx_packed_floats(100) == 0


def test_xtx_accumulates_with_strides(cuda_device) -> None:
    lib = _lib.load()
    x, xf = _x(3000, 520, 12, cuda_device)
    xs = x[:, :512]  # row stride 520 elements (1040 bytes, 16-byte multiple)
    g = torch.zeros(512, 520, device=cuda_device)  # Gram row stride 520
    g[:, :512] = torch.eye(512, device=cuda_device)
    for a, b in ((0, 1234), (1234, 3000)):
        part = xs[a:b]
        assert lib.mxw_accumulate_xtx(part.data_ptr(), b - a, 512, 520, g.data_ptr(), 520, None,
                                      _stream(cuda_device)) == 0
    torch.cuda.synchronize()
    ref = oracle.gram(xf[:, :512]) + np.eye(512)
    assert _full_err(g[:, :512].cpu().numpy().astype(np.float64), ref) < RTOL
    assert float(g[:, 512:].abs().max()) == 0.0  # padding columns untouched


@pytest.mark.parametrize("tokens", [300, 4097, 8192, 65536])
def test_statistics_are_deterministic_run_to_run(tokens, cuda_device) -> None:
    """The strip totals are folded in a fixed order: two runs give identical bits."""
    lib = _lib.load()
    x, _ = _x(tokens, 640, 11, cuda_device, torch.bfloat16)
    outs = []
    for _ in range(2):
        s1 = torch.zeros(640, device=cuda_device)
        s2 = torch.zeros(640, device=cuda_device)
        g = torch.zeros(20, 32, 32, device=cuda_device)
        st = lib.mxw_accumulate_activation_stats(x.data_ptr(), _lib.MXW_BF16, tokens, 640, 640, s1.data_ptr(),
                                                 s2.data_ptr(), g.data_ptr(), None, _stream(cuda_device))
        assert st == _lib.MXW_OK
        outs.append((s1, s2, g))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
