"""Generate the golden fixtures of the quantization hot path from the reference.

Run in a container where the reference MxWave checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/MxWave
    python tests/golden/make_golden.py --reference /path/to/MxWave --only-layers
    python tests/golden/make_golden.py --reference /path/to/MxWave --only-nonfinite

It imports the reference's own ``mxwave.core.quantize_mxfp4`` and
``mxwave.calibration.ActivationCollector`` (CPU, fp32) and records:

* ``cases.npz`` + ``cases.json``: small inputs stored verbatim with the
  reference's packed/scale bytes -- the reference's known-answer tests
  (tests/test_core.py in the reference), edge-value blocks and random shapes
  over every objective, depth and percentile;
* ``configs.json``: SHA-256 of the packed and scale bytes for the full-size
  benchmark workloads, whose inputs are regenerated bit-exactly from
  ``mxwave_b200.synthetic`` (platform-independent); the reference's gamma and
  block Hessians for them are stored in ``config_stats.npz`` so the check does
  not depend on fp32 accumulation order.

Weights are quantized through the reference's ``iter_quantized_row_chunks``
with its default 1,048,576-element chunks, as its engine does.

``--only-nonfinite`` runs ``nonfinite_golden.py``: blocks holding NaN or
infinity, every objective.

``--only-layers`` runs ``layer_golden.py``: the decoder-layer workload (the
reference's sequential calibration of a random-init layer, then all seven
linears) and the whole-checkpoint workload (one more layer plus a 128-expert
stack, block-Hessian weighted).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1]))

from mxwave_b200 import synthetic as syn  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_quantize_chunked(torch, ref_core, ref_ckpt, w_bits: np.ndarray, **kw):
    """Reference quantization through its own chunk iterator (engine.py:372-394)."""
    w = torch.from_numpy(w_bits.view(np.int16).copy()).view(torch.bfloat16)
    rows, cols = w.shape
    packed = np.empty((rows, cols // 2), np.uint8)
    scales = np.empty((rows, cols // 32), np.uint8)

    def quantize(chunk):
        return ref_core.quantize_mxfp4(chunk, **kw)

    for start, stop, p, s in ref_ckpt.iter_quantized_row_chunks(
        lambda a, b: w[a:b], quantize, rows=rows, columns=cols, max_rows=1024,
        max_elements=ref_ckpt.DEFAULT_TENSOR_CHUNK_MAX_ELEMENTS, name="w",
    ):
        packed[start:stop] = p.numpy()
        scales[start:stop] = s.numpy()
    return packed, scales


def edge_blocks() -> np.ndarray:
    """Hand-built fp32 blocks hitting the arithmetic corner cases (float32)."""
    rows = []

    def add(vals):
        v = np.zeros(32, np.float32)
        v[: len(vals)] = vals
        rows.append(v)

    add([])  # all zero
    add([-0.0] * 32)  # negative zeros
    add([-1e-7, 3e-7, -5e-7])  # near-zero block (max < 1e-6)
    add([1e-6, -1e-6])  # exactly at the near-zero threshold (bf16-rounded)
    add([6.0, -6.0, 3.0])  # anchor / 6 an exact power of two
    add([12.0, 0.75, -0.25, 0.25])
    add([2.0 ** -126, 2.0 ** -130, -(2.0 ** -133)])  # subnormal and tiny bf16
    add([3.0e38, -1.0, 2.0e38])  # huge: exponents near 127, overflowing errors
    add([1.0e38, 1e-30, -1e-35])
    add([0.1] * 31 + [8.0])  # reference outlier test block
    add([-0.01, 1.0, -0.3])  # negative values rounding to zero
    add(list(np.linspace(-7, 7, 32)))
    add([2.0 ** k for k in range(-20, 12)])
    add([6 * 2.0 ** k * (1 - 2.0 ** -8) for k in range(-8, 24)])  # just below 6 * 2^k
    add([6 * 2.0 ** k * (1 + 2.0 ** -7) for k in range(-8, 24)])  # just above 6 * 2^k
    add([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0] + [6.0] * 18)
    add([1e-5] * 32)
    add([7.0, -7.0, 6.99])
    return np.stack(rows).astype(np.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference MxWave checkout")
    ap.add_argument("--skip-configs", action="store_true")
    ap.add_argument("--only-layers", action="store_true",
                    help="only (re)generate the decoder-layer and expert-stack fixtures (configs 4 and 5)")
    ap.add_argument("--only-nonfinite", action="store_true",
                    help="only (re)generate the fixtures of blocks holding NaN or infinity")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    if args.only_nonfinite:
        import nonfinite_golden

        nonfinite_golden.main(HERE)
        return
    if args.only_layers:
        import layer_golden

        layer_golden.main(HERE)
        return
    import torch
    from mxwave import calibration as ref_cal
    from mxwave import checkpoint as ref_ckpt
    from mxwave import core as ref_core

    torch.set_num_threads(8)
    cases: list[dict] = []
    arrays: dict[str, np.ndarray] = {}

    stored: dict[int, str] = {}

    def share(prefix: str, a) -> str:
        """Store an input array once and return its key (inputs are reused across cases)."""
        key = stored.get(id(a))
        if key is None:
            key = f"{prefix}{len(stored)}"
            stored[id(a)] = key
            arrays[key] = np.asarray(a)
        return key

    def record(name: str, w_bits: np.ndarray, gamma=None, hessian=None, **kw):
        # uint16 arrays are bf16 bit patterns; float32 arrays are fp32 weights.
        if w_bits.dtype == np.float32:
            t = torch.from_numpy(w_bits.copy())
        else:
            t = torch.from_numpy(w_bits.view(np.int16).copy()).view(torch.bfloat16)
        g = None if gamma is None else torch.from_numpy(np.asarray(gamma, np.float32))
        h = None if hessian is None else torch.from_numpy(np.asarray(hessian, np.float32))
        p, s = ref_core.quantize_mxfp4(t, gamma=g, hessian=h, **kw)
        i = len(cases)
        arrays[f"p{i}"] = p.numpy()
        arrays[f"s{i}"] = s.numpy()
        cases.append({"name": name, "index": i, "kwargs": kw, "weight": share("w", w_bits),
                      "dtype": "f32" if w_bits.dtype == np.float32 else "bf16",
                      "gamma": None if gamma is None else share("g", gamma),
                      "hessian": None if hessian is None else share("h", hessian)})

    # -- the reference's own known-answer tests (tests/test_core.py) ----------
    maxima = np.array([0.0, 1e-7, 1e-6, 6.0, 6.99, 7.0, 10.0], np.float32)
    w = np.zeros((len(maxima), 32), np.float32)
    w[:, 0] = maxima
    record("kat_rtn_edges", w, method="rtn")
    mid = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    w = np.full((1, 32), 6.0, np.float32)
    w[0, :7] = mid
    w[0, 7:14] = -mid
    for m in ("rtn", "mse"):
        record(f"kat_midpoints_{m}", w.copy(), method=m, scale_percentile=100)
    w = np.full((1, 32), 0.1, np.float32)
    w[0, 0] = 8.0
    record("kat_no_clip_outlier_d8", w, mse_clip_depth=8)
    mags = np.ones(32, np.float32)
    mags[0] = 1e-4
    for d in (1, 4):
        record(f"kat_clip_unimportant_d{d}", w, gamma=mags, mse_clip_depth=d)
    gen = torch.Generator().manual_seed(123)
    weight = torch.randn(8, 64, generator=gen)
    rms = torch.rand(64, generator=gen).add(0.1)
    hdiag = torch.diag_embed(rms.reshape(2, 32).square())
    wb = weight.numpy()
    record("kat_diag_hessian_as_gamma_g", wb, gamma=rms.numpy(), mse_clip_depth=4)
    record("kat_diag_hessian_as_gamma_h", wb, hessian=hdiag.numpy(), mse_clip_depth=4)

    # -- edge-value blocks, every objective ----------------------------------
    eb32 = edge_blocks()
    record("edge_f32_mse_d1", eb32)
    record("edge_f32_mse_d4", eb32, mse_clip_depth=4)
    record("edge_f32_rtn", eb32, method="rtn")
    eb = syn.f32_to_bf16_bits(eb32)
    eg = syn.det_channel_scales(32, seed=11).astype(np.float32)
    ex = syn.bf16_bits_to_f32(syn.det_activations(64, 32, seed=12)).astype(np.float64)
    eh = (ex.T @ ex / 64).astype(np.float32)[None] + np.eye(32, dtype=np.float32)[None] * 1e-6
    for d in (0, 1, 4, 8):
        record(f"edge_mse_d{d}", eb, mse_clip_depth=d)
        record(f"edge_gamma_d{d}", eb, gamma=eg, mse_clip_depth=d)
        record(f"edge_hessian_d{d}", eb, hessian=eh, mse_clip_depth=d)
    for pct in (100.0, 50.0, 3.0, 90.0, 99.99):
        record(f"edge_pct{pct}", eb, scale_percentile=pct)
    record("edge_rtn", eb, method="rtn")

    # -- random shapes -------------------------------------------------------
    seed = 100
    for rows, cols in ((1, 32), (3, 96), (37, 160), (64, 1024), (33, 2048), (5, 5120)):
        seed += 1
        wr = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.01)
        gx = syn.bf16_bits_to_f32(syn.det_activations(256, cols, seed + 1000)).astype(np.float64)
        gam = np.sqrt((gx ** 2).mean(0)).astype(np.float32)
        hb = gx.reshape(256, cols // 32, 32)
        hes = (np.einsum("nbi,nbj->bij", hb, hb) / 256).astype(np.float32)
        hes += np.eye(32, dtype=np.float32)[None] * 1e-6
        for d in (0, 1, 4, 8):
            record(f"rand_{rows}x{cols}_mse_d{d}", wr, mse_clip_depth=d)
            record(f"rand_{rows}x{cols}_gamma_d{d}", wr, gamma=gam, mse_clip_depth=d)
            record(f"rand_{rows}x{cols}_hess_d{d}", wr, hessian=hes, mse_clip_depth=d)
        for pct in (100.0, 50.0, 97.0):
            record(f"rand_{rows}x{cols}_pct{pct}", wr, scale_percentile=pct)
            record(f"rand_{rows}x{cols}_gamma_pct{pct}", wr, gamma=gam, scale_percentile=pct)
        record(f"rand_{rows}x{cols}_rtn", wr, method="rtn")

    np.savez_compressed(HERE / "cases.npz", **arrays)
    (HERE / "cases.json").write_text(json.dumps({"cases": cases}, indent=1) + "\n")
    print(f"{len(cases)} small cases written")
    if args.skip_configs:
        return

    # -- full-size workloads -------------------------------------------------
    configs: dict[str, dict] = {}
    stats: dict[str, np.ndarray] = {}

    def run(name, w_bits, **kw):
        t0 = time.time()
        p, s = ref_quantize_chunked(torch, ref_core, ref_ckpt, w_bits, **kw)
        configs[name] = {"packed_sha256": sha(p), "scales_sha256": sha(s), "input_sha256": sha(w_bits),
                         "shape": list(w_bits.shape), "seconds": round(time.time() - t0, 2)}
        print(name, configs[name], flush=True)

    # Dense 4096x4096, N(0, 0.02^2) + 0.1% outliers x20, seed 0.
    w1 = syn.det_dense_weight(4096, 4096, seed=0)
    for d in (1, 4):
        run(f"dense4096_mse_d{d}", w1, mse_clip_depth=d)
    run("dense4096_rtn", w1, method="rtn")
    run("dense4096_pct100_d1", w1, scale_percentile=100.0)
    del w1

    # Gamma-weighted MLP up/gate: X 8192x5120 heavy-channel -> rms (reference collector).
    x2 = syn.det_activations(8192, 5120, seed=2)
    col = ref_cal.ActivationCollector({"mlp.weight": 5120}, ("rms",))
    col.update("mlp.weight", torch.from_numpy(x2.view(np.int16).copy()).view(torch.bfloat16))
    gamma2 = col.finalize()["rms"]["mlp.weight"].numpy()
    stats["mlp_rms"] = gamma2
    configs["mlp_activations"] = {"input_sha256": sha(x2), "rms_sha256": sha(gamma2)}
    del x2
    for idx, name in enumerate(("gate", "up")):
        w2 = syn.det_dense_weight(17408, 5120, seed=20 + idx, sigma=0.015, outlier_fraction=0.0)
        run(f"mlp_{name}_gamma_d1", w2, gamma=torch.from_numpy(gamma2), mse_clip_depth=1)
        if name == "gate":
            run(f"mlp_{name}_gamma_d4", w2, gamma=torch.from_numpy(gamma2), mse_clip_depth=4)
        del w2

    # Block-Hessian: X 65536x5120 -> reference block Hessian (damp 1e-6 absolute).
    col = ref_cal.ActivationCollector({"down.weight": 5120}, ("block-hessian",), hessian_damp=1e-6)
    for lo in range(0, 65536, 8192):
        xs = syn.det_activations(8192, 5120, seed=300 + lo // 8192, scales_seed=3)
        col.update("down.weight", torch.from_numpy(xs.view(np.int16).copy()).view(torch.bfloat16))
    h3 = col.finalize()["block-hessian"]["down.weight"].numpy()
    stats["hess5120"] = h3
    w3 = syn.det_dense_weight(17408, 5120, seed=31, sigma=0.015)
    for d in (1, 4):
        run(f"hess5120_w17408x5120_d{d}", w3, hessian=torch.from_numpy(h3), mse_clip_depth=d)
    del w3
    # The reference's [out, in] down_proj 5120x17408 needs 17408-wide blocks:
    # a Hessian from 8192 tokens of a 17408-wide heavy-channel activation set.
    x4 = syn.det_activations(8192, 17408, seed=4)
    col = ref_cal.ActivationCollector({"down.weight": 17408}, ("block-hessian",), hessian_damp=1e-6)
    col.update("down.weight", torch.from_numpy(x4.view(np.int16).copy()).view(torch.bfloat16))
    h4 = col.finalize()["block-hessian"]["down.weight"].numpy()
    stats["hess17408"] = h4
    del x4
    w4 = syn.det_dense_weight(5120, 17408, seed=41, sigma=0.015)
    run("hess17408_w5120x17408_d1", w4, hessian=torch.from_numpy(h4), mse_clip_depth=1)
    del w4

    np.savez_compressed(HERE / "config_stats.npz", **stats)
    (HERE / "configs.json").write_text(json.dumps(configs, indent=1) + "\n")
    print("configs written")


if __name__ == "__main__":
    main()
