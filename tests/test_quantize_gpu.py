"""GPU parity of the MXFP4 quantize kernel (through the C ABI) against the
reference's golden bytes and the oracle.  Bar: bit-exact packed and scales."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from mxwave_b200 import _lib
from mxwave_b200 import synthetic as syn
from mxwave_b200.core import quantize_mxfp4
from oracle import oracle
from tests.golden.fixtures import load_cases, load_config_stats, load_configs

pytestmark = pytest.mark.gpu

CASES = load_cases()


def _sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.cpu().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _to_device(w: np.ndarray, dev, dtype: str = "bf16") -> torch.Tensor:
    if w.dtype == np.float32:
        t = torch.from_numpy(w.copy())
        return t.to(dev) if dtype == "f32" else t.to(dev)
    return torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _gpu(w, dev, **kw):
    p, s = quantize_mxfp4(w, **kw)
    torch.cuda.synchronize(dev)
    return p.cpu().numpy(), s.cpu().numpy()


def assert_same_bytes(weight: np.ndarray, p, s, p_ref, s_ref) -> None:
    """Bit-exact comparison with a readable report of the first mismatches."""
    bad_s = np.argwhere(s != s_ref)
    bad_p = np.argwhere(p != p_ref)
    if bad_s.size == 0 and bad_p.size == 0:
        return
    lines = [f"{len(bad_s)} scale and {len(bad_p)} packed byte mismatches"]
    w = weight if weight.dtype == np.float32 else syn.bf16_bits_to_f32(weight)
    for r, b in bad_s[:5]:
        blk = w[r, 32 * b: 32 * b + 32]
        lines.append(f"scale[{r},{b}] got {s[r, b]} want {s_ref[r, b]} block {blk.tolist()}")
    for r, c in bad_p[:8]:
        vals = "" if w is None else f" inputs {w[r, 2 * c]!r}, {w[r, 2 * c + 1]!r}"
        lines.append(f"packed[{r},{c}] got {p[r, c]:#04x} want {p_ref[r, c]:#04x} scale {s_ref[r, (2 * c) // 32]}{vals}")
    raise AssertionError("\n".join(lines))


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_golden_case_bit_exact(case, cuda_device) -> None:
    w = _to_device(case.weight, cuda_device)
    kw = dict(case.kwargs)
    if case.gamma is not None:
        kw["gamma"] = torch.from_numpy(case.gamma).to(cuda_device)
    if case.hessian is not None:
        kw["hessian"] = torch.from_numpy(case.hessian).to(cuda_device)
    p, s = _gpu(w, cuda_device, **kw)
    assert_same_bytes(case.weight, p, s, case.packed, case.scales)


def _bf16_all_finite_blocks() -> np.ndarray:
    """Every finite bf16 bit pattern once, 32 per block (2040 blocks)."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    exp = (bits >> 7) & 0xFF
    bits = bits[exp != 0xFF]
    pad = (-bits.size) % 32
    bits = np.concatenate([bits, np.zeros(pad, np.uint16)])
    return bits.reshape(-1, 32)


@pytest.mark.parametrize("kw", [{}, {"method": "rtn"}, {"mse_clip_depth": 4}, {"scale_percentile": 100.0},
                                {"scale_percentile": 40.0}])
def test_every_bf16_value_matches_oracle(kw, cuda_device) -> None:
    w = _bf16_all_finite_blocks()
    # Mix the ordering so blocks see very different scales.
    rng = np.random.default_rng(3)
    shuffled = w.reshape(-1)[rng.permutation(w.size)].reshape(w.shape)
    for arr in (w, shuffled):
        p, s = _gpu(_to_device(arr, cuda_device), cuda_device, **kw)
        po, so = oracle.quantize_mxfp4(arr, **kw)
        assert_same_bytes(syn.bf16_bits_to_f32(arr), p, s, po, so)


SHAPES = [(1, 32), (7, 64), (31, 96), (33, 160), (64, 544), (100, 2048), (257, 768), (40, 5120)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{r}x{c}" for r, c in SHAPES])
@pytest.mark.parametrize("objective", ["none", "gamma", "hessian", "rtn"])
@pytest.mark.parametrize("depth", [0, 1, 4, 8])
def test_random_shapes_match_oracle(shape, objective, depth, cuda_device) -> None:
    rows, cols = shape
    if objective == "rtn" and depth != 1:
        pytest.skip("rtn has no depth")
    seed = rows * 7919 + cols + depth
    w = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.01)
    kw: dict = {"mse_clip_depth": depth}
    okw: dict = {"mse_clip_depth": depth}
    if objective == "rtn":
        kw = {"method": "rtn"}
        okw = {"method": "rtn"}
    elif objective == "gamma":
        g = syn.det_channel_scales(cols, seed + 1).astype(np.float32)
        kw["gamma"] = torch.from_numpy(g).to(cuda_device)
        okw["gamma"] = g
    elif objective == "hessian":
        x = syn.bf16_bits_to_f32(syn.det_activations(128, cols, seed + 2)).astype(np.float64)
        h = oracle.finalize_block_hessian(oracle.block_gram(x), 128, 1e-6, "absolute").astype(np.float32)
        kw["hessian"] = torch.from_numpy(h).to(cuda_device)
        okw["hessian"] = h
    p, s = _gpu(_to_device(w, cuda_device), cuda_device, **kw)
    po, so = oracle.quantize_mxfp4(w, **okw)
    np.testing.assert_array_equal(s, so)
    np.testing.assert_array_equal(p, po)


@pytest.mark.parametrize("pct", [99.5, 100.0, 50.0, 3.0, 90.0, 99.99, 97.0])
@pytest.mark.parametrize("objective", ["none", "gamma"])
def test_percentiles_match_oracle(pct, objective, cuda_device) -> None:
    w = syn.det_dense_weight(65, 1024, 500, outlier_fraction=0.02)
    kw: dict = {"scale_percentile": pct}
    okw = dict(kw)
    if objective == "gamma":
        g = syn.det_channel_scales(1024, 501).astype(np.float32)
        kw["gamma"] = torch.from_numpy(g).to(cuda_device)
        okw["gamma"] = g
    p, s = _gpu(_to_device(w, cuda_device), cuda_device, **kw)
    po, so = oracle.quantize_mxfp4(w, **okw)
    np.testing.assert_array_equal(s, so)
    np.testing.assert_array_equal(p, po)


@pytest.mark.parametrize("dtype", ["f16", "f32"])
@pytest.mark.parametrize("objective", ["none", "gamma", "hessian", "rtn"])
def test_f16_f32_inputs_match_oracle(dtype, objective, cuda_device) -> None:
    rows, cols = 45, 512
    rng = np.random.default_rng(11)
    w32 = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w32[rng.random((rows, cols)) < 0.01] *= 20
    if dtype == "f16":
        host = w32.astype(np.float16)
        wt = torch.from_numpy(host).to(cuda_device)
        oarr, odt = host.view(np.uint16), "f16"
    else:
        wt = torch.from_numpy(w32).to(cuda_device)
        oarr, odt = w32, "f32"
    kw: dict = {}
    okw: dict = {}
    if objective == "rtn":
        kw = okw = {"method": "rtn"}
    elif objective == "gamma":
        g = np.abs(rng.standard_normal(cols)).astype(np.float32)
        kw, okw = {"gamma": torch.from_numpy(g).to(cuda_device)}, {"gamma": g}
    elif objective == "hessian":
        x = rng.standard_normal((64, cols))
        h = oracle.finalize_block_hessian(oracle.block_gram(x), 64, 1e-6, "absolute").astype(np.float32)
        kw, okw = {"hessian": torch.from_numpy(h).to(cuda_device)}, {"hessian": h}
    p, s = _gpu(wt, cuda_device, **kw)
    po, so = oracle.quantize_mxfp4(oarr, dtype=odt, **okw)
    np.testing.assert_array_equal(s, so)
    np.testing.assert_array_equal(p, po)


def test_strided_and_unaligned_inputs(cuda_device) -> None:
    base = syn.det_dense_weight(40, 1100, 77, outlier_fraction=0.01)
    full = _to_device(base, cuda_device)
    # TMA-describable stride (1100 * 2 bytes is 16-byte aligned? no: 2200 % 16 == 8) -> plain path.
    view = full[:, :1024]
    p, s = _gpu(view, cuda_device)
    po, so = oracle.quantize_mxfp4(np.ascontiguousarray(base[:, :1024]))
    np.testing.assert_array_equal(p, po)
    np.testing.assert_array_equal(s, so)
    # 16-byte aligned stride (1104 * 2 = 2208 = 16 * 138): TMA path with ld > cols.
    padded = torch.zeros((40, 1104), dtype=torch.bfloat16, device=cuda_device)
    padded[:, :1100] = full
    p, s = _gpu(padded[:, :1024], cuda_device)
    np.testing.assert_array_equal(p, po)
    np.testing.assert_array_equal(s, so)
    # Misaligned base pointer (offset by one element).
    p, s = _gpu(full[:, 1:1025], cuda_device)
    po, so = oracle.quantize_mxfp4(np.ascontiguousarray(base[:, 1:1025]))
    np.testing.assert_array_equal(p, po)
    np.testing.assert_array_equal(s, so)


def test_nonfinite_input_sets_flag(cuda_device) -> None:
    w = torch.zeros((70, 256), dtype=torch.bfloat16, device=cuda_device)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    quantize_mxfp4(w, _flags=flags)
    assert int(flags.item()) == 0
    w[65, 200] = float("nan")
    quantize_mxfp4(w, _flags=flags)
    assert int(flags.item()) & _lib.MXW_FLAG_NONFINITE
    flags.zero_()
    w[65, 200] = float("inf")
    quantize_mxfp4(w, gamma=torch.ones(256, device=cuda_device), _flags=flags)
    assert int(flags.item()) & _lib.MXW_FLAG_NONFINITE


def _nonfinite_cases():
    from pathlib import Path

    from tests.golden import nonfinite_golden

    here = Path(__file__).resolve().parent / "golden"
    if not (here / "nonfinite.json").exists():
        return []
    return nonfinite_golden.load(here)[0]


NONFINITE = _nonfinite_cases()


@pytest.mark.parametrize("case", NONFINITE, ids=[c["name"] for c in NONFINITE])
def test_nonfinite_blocks_match_reference(case, cuda_device) -> None:
    """NaN / infinity blocks through every kernel path (fast-path rare marker, Hessian
    screening, rtn, fp32 inputs), against the reference's own bytes."""
    w = case["weight"]
    kw = {k: (torch.from_numpy(v).to(cuda_device) if isinstance(v, np.ndarray) else v)
          for k, v in case["kwargs"].items()}
    p, s = _gpu(_to_device(w, cuda_device, "f32" if w.dtype == np.float32 else "bf16"), cuda_device, **kw)
    ref_w = w if w.dtype == np.float32 else syn.bf16_bits_to_f32(w)
    assert_same_bytes(ref_w, p, s, case["packed"], case["scales"])


def test_empty_and_argument_errors(cuda_device) -> None:
    p, s = quantize_mxfp4(torch.zeros((0, 64), dtype=torch.bfloat16, device=cuda_device))
    assert p.shape == (0, 32) and s.shape == (0, 2)
    w = torch.zeros((4, 64), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="mutually exclusive"):
        quantize_mxfp4(w, gamma=torch.ones(64, device=cuda_device), hessian=torch.zeros(2, 32, 32, device=cuda_device))
    with pytest.raises(ValueError, match="gamma must contain finite"):
        quantize_mxfp4(w, gamma=-torch.ones(64, device=cuda_device))
    with pytest.raises(ValueError, match="hessian must have shape"):
        quantize_mxfp4(w, hessian=torch.zeros(3, 32, 32, device=cuda_device))
    with pytest.raises(ValueError, match="hessian contains NaN"):
        quantize_mxfp4(w, hessian=torch.full((2, 32, 32), float("nan"), device=cuda_device))
    with pytest.raises(AssertionError):
        quantize_mxfp4(torch.zeros((4, 48), dtype=torch.bfloat16, device=cuda_device))


# ------------------------------------------------------- full-size workloads


def _config_case(name: str):
    cfg = load_configs()
    if name not in cfg:
        pytest.skip(f"golden hash {name} not generated")
    return cfg[name]


@pytest.mark.parametrize("name,kw", [("dense4096_mse_d1", {}), ("dense4096_mse_d4", {"mse_clip_depth": 4}),
                                     ("dense4096_rtn", {"method": "rtn"}),
                                     ("dense4096_pct100_d1", {"scale_percentile": 100.0})])
def test_dense4096_reference_sha(name, kw, cuda_device) -> None:
    c = _config_case(name)
    w = syn.det_dense_weight(4096, 4096, seed=0)
    assert _sha(w) == c["input_sha256"]
    p, s = quantize_mxfp4(_to_device(w, cuda_device), **kw)
    assert _sha(p) == c["packed_sha256"]
    assert _sha(s) == c["scales_sha256"]


def test_mlp_gamma_reference_sha(cuda_device) -> None:
    stats = load_config_stats()
    if "mlp_rms" not in stats:
        pytest.skip("config statistics not generated")
    gamma = torch.from_numpy(stats["mlp_rms"]).to(cuda_device)
    for idx, name in enumerate(("gate", "up")):
        w = syn.det_dense_weight(17408, 5120, seed=20 + idx, sigma=0.015, outlier_fraction=0.0)
        wt = _to_device(w, cuda_device)
        depths = (1, 4) if name == "gate" else (1,)
        for d in depths:
            c = _config_case(f"mlp_{name}_gamma_d{d}")
            assert _sha(w) == c["input_sha256"]
            p, s = quantize_mxfp4(wt, gamma=gamma, mse_clip_depth=d)
            assert _sha(p) == c["packed_sha256"], f"{name} d{d}"
            assert _sha(s) == c["scales_sha256"], f"{name} d{d}"


def test_block_hessian_reference_sha(cuda_device) -> None:
    stats = load_config_stats()
    if "hess5120" not in stats:
        pytest.skip("config statistics not generated")
    h = torch.from_numpy(stats["hess5120"]).to(cuda_device)
    w = syn.det_dense_weight(17408, 5120, seed=31, sigma=0.015)
    wt = _to_device(w, cuda_device)
    for d in (1, 4):
        c = _config_case(f"hess5120_w17408x5120_d{d}")
        p, s = quantize_mxfp4(wt, hessian=h, mse_clip_depth=d)
        assert _sha(p) == c["packed_sha256"], d
        assert _sha(s) == c["scales_sha256"], d
    h4 = torch.from_numpy(stats["hess17408"]).to(cuda_device)
    w4 = syn.det_dense_weight(5120, 17408, seed=41, sigma=0.015)
    c = _config_case("hess17408_w5120x17408_d1")
    p, s = quantize_mxfp4(_to_device(w4, cuda_device), hessian=h4, mse_clip_depth=1)
    assert _sha(p) == c["packed_sha256"]
    assert _sha(s) == c["scales_sha256"]


@pytest.mark.parametrize("objective", ["none", "gamma"])
@pytest.mark.parametrize("depth", [1, 4])
def test_near_flt_max_blocks_in_a_large_tensor(objective, depth, cuda_device) -> None:
    """Blocks whose candidates reach e >= 126 (magnitudes near FLT_MAX) are
    finished by the rare-block pass; the rest of the tensor takes the fast
    path.  Bytes must match the oracle everywhere."""
    rows, cols = 96, 2048
    w = syn.det_dense_weight(rows, cols, 77 + depth, outlier_fraction=0.01)
    f = syn.bf16_bits_to_f32(w).copy()
    rng = np.random.default_rng(5)
    for r, b in zip(rng.integers(0, rows, 40), rng.integers(0, cols // 32, 40)):
        mag = rng.uniform(0.3e38, 1.6e38)  # block maxima from ~1e38 up to the bf16 limit
        f[r, 32 * b: 32 * b + 32] = np.clip(rng.standard_normal(32) * mag, -3.3e38, 3.3e38).astype(np.float32)
    bits = syn.f32_to_bf16_bits(f)
    kw: dict = {"mse_clip_depth": depth}
    okw: dict = {"mse_clip_depth": depth}
    if objective == "gamma":
        g = syn.det_channel_scales(cols, 9).astype(np.float32)
        kw["gamma"], okw["gamma"] = torch.from_numpy(g).to(cuda_device), g
    p, s = _gpu(_to_device(bits, cuda_device), cuda_device, **kw)
    po, so = oracle.quantize_mxfp4(bits, **okw)
    block_max = np.abs(syn.bf16_bits_to_f32(bits)).reshape(rows, cols // 32, 32).max(axis=-1)
    assert (block_max > 6.0 * 2.0 ** 125).any(), "the case must contain blocks with e >= 126 candidates"
    assert_same_bytes(bits, p, s, po, so)


@pytest.mark.parametrize("pct", [99.5, 97.0, 100.0])
@pytest.mark.parametrize("depth", [0, 1, 2, 4, 8])
@pytest.mark.parametrize("objective", ["none", "gamma"])
def test_close_call_blocks_match_oracle(objective, depth, pct, cuda_device) -> None:
    """Inputs that push many blocks off the kernel's two-candidate fast path:
    extreme per-channel gamma (clipping candidates below the anchor exponent
    win or come close, so their lower bound does not decide and the warp
    evaluates them exactly) and dense outliers (the no-clipping exponent is
    two above the anchor's).  Bytes must match the oracle everywhere."""
    rows, cols = 192, 2048
    seed = 900 + 10 * depth + int(pct)
    w = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.03)
    kw: dict = {"mse_clip_depth": depth, "scale_percentile": pct}
    okw = dict(kw)
    if objective == "gamma":
        z = syn.det_normal(cols, seed + 1)
        g = np.exp(3.0 * z).astype(np.float32)  # channel weights over ~8 decades
        g[::97] = 0.0
        kw["gamma"], okw["gamma"] = torch.from_numpy(g).to(cuda_device), g
    p, s = _gpu(_to_device(w, cuda_device), cuda_device, **kw)
    po, so = oracle.quantize_mxfp4(w, **okw)
    assert_same_bytes(w, p, s, po, so)


def test_rare_block_pass_runs_only_when_flagged(cuda_device) -> None:
    """With a flag word, the main pass reports whether it marked any block for
    the exact second pass (MXW_FLAG_RARE); the second pass skips its scan when
    the bit is clear.  Bytes must match the oracle in both cases, and a bit
    left set by an earlier call only makes later calls scan."""
    rows, cols = 64, 1024
    plain = syn.det_dense_weight(rows, cols, 31, outlier_fraction=0.01)
    f = syn.bf16_bits_to_f32(plain).copy()
    f[5, 64:96] = np.linspace(-3.0e38, 3.0e38, 32, dtype=np.float32)  # e >= 126 candidates: a rare block
    rare = syn.f32_to_bf16_bits(f)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for arr, expect_rare in ((plain, False), (rare, True), (plain, True)):
        p, s = quantize_mxfp4(_to_device(arr, cuda_device), _flags=flags)
        torch.cuda.synchronize(cuda_device)
        assert bool(int(flags.item()) & _lib.MXW_FLAG_RARE) == expect_rare
        po, so = oracle.quantize_mxfp4(arr)
        assert_same_bytes(arr, p.cpu().numpy(), s.cpu().numpy(), po, so)


@pytest.mark.parametrize("kind", ["psd_few_tokens", "indefinite", "negative_diagonal", "pct100"])
@pytest.mark.parametrize("depth", [0, 1, 4, 8])
def test_block_hessian_screening_matches_oracle(kind, depth, cuda_device) -> None:
    """The block-Hessian objective's tensor-core screening (bf16 weights):
    Hessians from few tokens (many close calls, exact ties included through
    dense outliers), indefinite and negative-diagonal matrices (the bound
    without the Cauchy-Schwarz property), and the amax anchor.  Blocks the
    screening cannot decide are re-quantized exactly; bytes must match the
    oracle everywhere."""
    rows, cols = 300, 2048 + 96  # a ragged last 128-row tile and an odd number of block columns
    seed = 4000 + 17 * depth + len(kind)
    w = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.05)
    rng = np.random.default_rng(seed)
    if kind in ("psd_few_tokens", "pct100"):
        x = syn.bf16_bits_to_f32(syn.det_activations(8, cols, seed + 1)).astype(np.float64)
        h = oracle.finalize_block_hessian(oracle.block_gram(x), 8, 1e-6, "absolute").astype(np.float32)
    else:
        a = rng.standard_normal((cols // 32, 32, 32)).astype(np.float32)
        h = ((a + a.transpose(0, 2, 1)) * 0.5).astype(np.float32)
        if kind == "indefinite":
            h += np.eye(32, dtype=np.float32)[None] * 2.0  # symmetric, some negative eigenvalues
        else:
            h[:, np.arange(32), np.arange(32)] = -np.abs(h[:, np.arange(32), np.arange(32)])
    kw: dict = {"mse_clip_depth": depth, "hessian": torch.from_numpy(h).to(cuda_device)}
    okw: dict = {"mse_clip_depth": depth, "hessian": h}
    if kind == "pct100":
        kw["scale_percentile"] = okw["scale_percentile"] = 100.0
    p, s = _gpu(_to_device(w, cuda_device), cuda_device, **kw)
    po, so = oracle.quantize_mxfp4(w, **okw)
    assert_same_bytes(w, p, s, po, so)
