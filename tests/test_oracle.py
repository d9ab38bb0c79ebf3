"""CPU tests: the oracle is pinned against the reference's golden vectors and
against the torch arithmetic it restates (no GPU needed)."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from mxwave_b200 import synthetic as syn
from oracle import oracle
from tests.golden.fixtures import load_cases, load_configs

CASES = load_cases()


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference_golden_case(case) -> None:
    p, s = oracle.quantize_mxfp4(case.weight, gamma=case.gamma, hessian=case.hessian, dtype=case.dtype,
                                 **case.kwargs)
    np.testing.assert_array_equal(s, case.scales)
    np.testing.assert_array_equal(p, case.packed)


def test_reference_known_answers_through_oracle() -> None:
    # tests/test_core.py:115-124 of the reference: RTN E8M0 bytes of block maxima.
    case = next(c for c in CASES if c.name == "kat_rtn_edges")
    p, s = oracle.quantize_mxfp4(case.weight, method="rtn", dtype="f32")
    assert s[:, 0].tolist() == [0, 101, 105, 127, 127, 128, 128]
    # tests/test_core.py:132-145: tie-to-even codes and nibble order.
    case = next(c for c in CASES if c.name == "kat_midpoints_mse")
    p, s = oracle.quantize_mxfp4(case.weight, scale_percentile=100, dtype="f32")
    codes = np.stack([p & 15, p >> 4], axis=-1).reshape(-1)
    assert s.item() == 127
    assert codes[:14].tolist() == [0, 2, 2, 4, 4, 6, 6, 8, 10, 10, 12, 12, 14, 14]
    # tests/test_core.py:91-95: the no-clipping candidate protects an outlier.
    case = next(c for c in CASES if c.name == "kat_no_clip_outlier_d8")
    _, s = oracle.quantize_mxfp4(case.weight, mse_clip_depth=8, dtype="f32")
    assert s[0, 0] == 128


def test_zero_block_known_answer() -> None:
    # An all-zero block takes the first candidate: byte 127 - 23 - depth.
    w = np.zeros((1, 32), np.uint16)
    for depth, byte in ((0, 104), (1, 103), (4, 100)):
        p, s = oracle.quantize_mxfp4(w, mse_clip_depth=depth)
        assert s.item() == byte and not p.any()
    _, s = oracle.quantize_mxfp4(w, method="rtn")
    assert s.item() == 0


def test_oracle_sum_order_matches_torch_cpu() -> None:
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(4000, 32, generator=g) * torch.exp(torch.randn(4000, 32, generator=g) * 3)).float()
    ref = x.sum(dim=-1).numpy()
    got = np.array([oracle.sum32(row) for row in x.numpy()], np.float32)
    np.testing.assert_array_equal(got, ref)
    np.testing.assert_array_equal((got / np.float32(32)).astype(np.float32), x.mean(dim=-1).numpy())


def test_oracle_log2_floor_ceil_match_torch_near_powers_of_two() -> None:
    # Every fp32 value within +-512 ulps of 2^k (k in [-130, 127]) plus 6*2^k edges.
    vals = []
    for k in range(-126, 128):
        base = np.float32(2.0 ** k).view(np.uint32).astype(np.int64)
        vals.append((base + np.arange(-512, 513)).astype(np.uint32))
    q = np.concatenate(vals).view(np.float32)
    q = q[np.isfinite(q) & (q > 0)]
    t = torch.from_numpy(q)
    lg = torch.log2(t)
    ref_floor = torch.floor(lg).numpy()
    ref_ceil = torch.ceil(lg).numpy()
    ours = (np.log2(q.astype(np.float64))).astype(np.float32)
    np.testing.assert_array_equal(np.floor(ours), ref_floor)
    np.testing.assert_array_equal(np.ceil(ours), ref_ceil)
    sample = q[:: max(1, q.size // 2000)]
    got = np.array([oracle.log2_f32(float(v)) for v in sample], np.float32)
    np.testing.assert_array_equal(got, np.log2(sample.astype(np.float64)).astype(np.float32))


@pytest.mark.parametrize("pct", [99.5, 50.0, 3.0, 90.0, 99.99, 12.3])
def test_oracle_quantile_matches_torch(pct: float) -> None:
    g = torch.Generator().manual_seed(7)
    x = torch.randn(3000, 32, generator=g).abs()
    ref = torch.quantile(x, pct / 100.0, dim=-1).numpy()
    got = np.array([oracle.block_quantile(row, pct) for row in x.numpy()], np.float32)
    np.testing.assert_array_equal(got, ref)


def test_oracle_row_chunking_invariant() -> None:
    w = syn.det_dense_weight(300, 512, seed=9, outlier_fraction=0.01)
    full = oracle.quantize_mxfp4(w, mse_clip_depth=4)
    parts = [oracle.quantize_mxfp4(w[a : a + 61], mse_clip_depth=4) for a in range(0, 300, 61)]
    np.testing.assert_array_equal(full[0], np.concatenate([p for p, _ in parts]))
    np.testing.assert_array_equal(full[1], np.concatenate([s for _, s in parts]))


def test_oracle_thread_count_invariant() -> None:
    w = syn.det_dense_weight(257, 1024, seed=10, outlier_fraction=0.01)
    a = oracle.quantize_mxfp4(w, threads=1)
    b = oracle.quantize_mxfp4(w, threads=7)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])


def test_oracle_dense4096_matches_reference_sha() -> None:
    cfg = load_configs()
    if "dense4096_mse_d1" not in cfg:
        pytest.skip("full-size golden hashes not generated")
    w = syn.det_dense_weight(4096, 4096, seed=0)
    assert _sha(w) == cfg["dense4096_mse_d1"]["input_sha256"]
    for name, kw in (("dense4096_mse_d1", {}), ("dense4096_mse_d4", {"mse_clip_depth": 4}),
                     ("dense4096_rtn", {"method": "rtn"}), ("dense4096_pct100_d1", {"scale_percentile": 100.0})):
        p, s = oracle.quantize_mxfp4(w, **kw)
        assert _sha(p) == cfg[name]["packed_sha256"], name
        assert _sha(s) == cfg[name]["scales_sha256"], name


def test_oracle_rejects_bad_arguments() -> None:
    w = np.zeros((2, 32), np.uint16)
    with pytest.raises(ValueError):
        oracle.quantize_mxfp4(w, mse_clip_depth=9)
    with pytest.raises(ValueError):
        oracle.quantize_mxfp4(w, scale_percentile=0.0)
    with pytest.raises(ValueError):
        oracle.quantize_mxfp4(w, method="rtn", gamma=np.ones(32, np.float32))


def test_moment_and_gram_oracles_match_reference_collector() -> None:
    import sys

    ref = "/root/reference"
    from pathlib import Path

    if not Path(ref).exists():
        pytest.skip("reference checkout not present")
    sys.path.insert(0, ref)
    from mxwave.calibration import ActivationCollector

    x = syn.det_activations(512, 256, seed=77)
    xt = torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16)
    col = ActivationCollector({"p.weight": 256}, ("mean-abs", "rms", "block-hessian"), hessian_damp=1e-6)
    col.update("p.weight", xt)
    st = col.finalize()
    xf = syn.bf16_bits_to_f32(x)
    s1, s2 = oracle.moments(xf)
    np.testing.assert_allclose(st["mean-abs"]["p.weight"].numpy(), s1 / 512, rtol=1e-5)
    np.testing.assert_allclose(st["rms"]["p.weight"].numpy(), np.sqrt(s2 / 512), rtol=1e-5)
    h = oracle.finalize_block_hessian(oracle.block_gram(xf), 512, 1e-6, "absolute")
    scale = np.sqrt(np.einsum("bii->bi", h)[:, :, None] * np.einsum("bii->bi", h)[:, None, :])
    assert np.max(np.abs(st["block-hessian"]["p.weight"].numpy() - h) / scale) < 1e-5


@pytest.mark.parametrize("short,objective", [("self_attn.k_proj", "hess"), ("self_attn.k_proj", "rms"),
                                             ("self_attn.o_proj", "hess"), ("self_attn.v_proj", "hess")])
def test_oracle_matches_decoder_layer_reference_sha(short, objective) -> None:
    """The oracle reproduces the reference's hashes on linears of the decoder
    layer quantized with the statistics of the reference's own sequential
    calibration (tests/golden/layer_golden.py)."""
    from tests.golden.fixtures import load_layer_stats
    from tests.golden.layer_specs import LAYER_INPUT_GROUP, LAYER_LINEARS, layer_seed

    stats = load_layer_stats()
    cfg = load_configs()
    key = f"layer_{short}_{objective}_d1"
    if key not in cfg or not stats:
        pytest.skip("layer fixtures not generated")
    rows, cols = LAYER_LINEARS[short]
    bits = syn.det_dense_weight(rows, cols, seed=layer_seed(short), outlier_fraction=0.0)
    group = LAYER_INPUT_GROUP[short]
    kw = {"hessian": stats[f"layer_hess_{group}"]} if objective == "hess" else {"gamma": stats[f"layer_rms_{group}"]}
    p, s = oracle.quantize_mxfp4(bits, mse_clip_depth=1, **kw)
    assert _sha(p) == cfg[key]["packed_sha256"]
    assert _sha(s) == cfg[key]["scales_sha256"]


def _nonfinite_cases():
    from pathlib import Path

    from tests.golden import nonfinite_golden

    here = Path(__file__).resolve().parent / "golden"
    if not (here / "nonfinite.json").exists():
        return []
    return nonfinite_golden.load(here)[0]


NONFINITE = _nonfinite_cases()


@pytest.mark.parametrize("case", NONFINITE, ids=[c["name"] for c in NONFINITE])
def test_oracle_matches_nonfinite_golden(case) -> None:
    """Blocks holding NaN or infinity, against the reference's own bytes (nonfinite_golden.py)."""
    p, s = oracle.quantize_mxfp4(case["weight"], **case["kwargs"])
    np.testing.assert_array_equal(s, case["scales"])
    np.testing.assert_array_equal(p, case["packed"])

