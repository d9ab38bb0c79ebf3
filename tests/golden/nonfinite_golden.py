"""Golden vectors for blocks holding NaN or infinity, made by the reference.

Run through ``make_golden.py --reference <checkout> --only-nonfinite``.  The
reference's ``quantize_mxfp4`` (mxwave/core.py:114-251) is called on CPU in
fp32; its packed and scale bytes are stored beside the inputs in
``nonfinite.npz`` / ``nonfinite.json``.  The cases cover NaN (both signs),
+-inf, several non-finite values in one block, a non-finite value beside
zeros or a subnormal, every objective (unweighted, gamma, block Hessian, rtn)
and percentiles on both sides of the interpolation weight 0.5.

The bytes of such blocks follow from the reference's float arithmetic:
torch.quantile is NaN when a block holds a NaN and its lerp turns an infinity
into NaN for weights >= 0.5; a NaN exponent is stored as the x86 float->uint8
conversion of NaN (0) with every code 7; an infinite anchor clamps every
candidate to 127.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

NAN, NEG_NAN, POS_INF, NEG_INF = 0x7FC0, 0xFFC0, 0x7F80, 0xFF80


def planted_bf16(seed: int) -> np.ndarray:
    """A [48, 256] bf16 weight (bit patterns) with non-finite values planted in some blocks."""
    from mxwave_b200 import synthetic as syn

    w = syn.det_dense_weight(48, 256, seed=seed).copy()
    w[3, 10] = NAN
    w[4, 70] = NEG_NAN
    w[10, 40] = POS_INF
    w[20, 100] = NEG_INF
    w[30, 0:32] = NAN
    w[31, 32:64] = POS_INF
    w[32, 64], w[32, 65] = POS_INF, NEG_INF
    w[33, 96], w[33, 97] = NAN, POS_INF
    w[34, 128:160] = 0
    w[34, 130] = POS_INF
    w[35, 160:192] = 0
    w[35, 161] = NAN
    w[36, 192], w[36, 193] = 0x0001, POS_INF  # the smallest bf16 subnormal beside an infinity
    w[40, 224:256] = NEG_INF
    return w


def settings(gamma: np.ndarray, hessian: np.ndarray) -> list[tuple[str, dict]]:
    return [
        ("mse_d1", {}),
        ("mse_d0", {"mse_clip_depth": 0}),
        ("mse_d4", {"mse_clip_depth": 4}),
        ("pct100_d1", {"scale_percentile": 100.0}),
        ("pct100_d4", {"scale_percentile": 100.0, "mse_clip_depth": 4}),
        ("pct40_d1", {"scale_percentile": 40.0}),
        ("pct50_d2", {"scale_percentile": 50.0, "mse_clip_depth": 2}),
        ("rtn", {"method": "rtn"}),
        ("gamma_d1", {"gamma": gamma}),
        ("gamma_pct3_d1", {"gamma": gamma, "scale_percentile": 3.0}),
        ("hess_d1", {"hessian": hessian}),
        ("hess_pct100_d4", {"hessian": hessian, "scale_percentile": 100.0, "mse_clip_depth": 4}),
    ]


def inputs() -> tuple[dict[str, np.ndarray], np.ndarray, np.ndarray]:
    rng = np.random.default_rng(1)
    gamma = (np.abs(rng.standard_normal(256)) + 0.1).astype(np.float32)
    hessian = np.stack([np.eye(32, dtype=np.float32) * (1 + i) + 0.01 for i in range(8)]).astype(np.float32)
    w16 = planted_bf16(3)
    from mxwave_b200 import synthetic as syn

    w32 = syn.bf16_bits_to_f32(planted_bf16(4)).astype(np.float32)
    return {"bf16": w16, "f32": w32}, gamma, hessian


def main(here: Path) -> None:
    import torch
    from mxwave import core as ref_core

    weights, gamma, hessian = inputs()
    arrays: dict[str, np.ndarray] = {"gamma": gamma, "hessian": hessian}
    cases = []
    for wname, w in weights.items():
        arrays[f"w_{wname}"] = w
        if w.dtype == np.float32:
            t = torch.from_numpy(w.copy())
        else:
            t = torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16)
        for sname, kw in settings(gamma, hessian):
            tkw = {k: (torch.from_numpy(v) if isinstance(v, np.ndarray) else v) for k, v in kw.items()}
            p, s = ref_core.quantize_mxfp4(t, **tkw)
            name = f"{wname}_{sname}"
            arrays[f"p_{name}"] = p.numpy()
            arrays[f"s_{name}"] = s.numpy()
            cases.append({"name": name, "weight": f"w_{wname}", "setting": sname})
    np.savez_compressed(here / "nonfinite.npz", **arrays)
    (here / "nonfinite.json").write_text(json.dumps({"cases": cases}, indent=1) + "\n")
    print(f"{len(cases)} non-finite cases written")


def load(here: Path) -> tuple[list[dict], dict[str, np.ndarray]]:
    """The recorded cases with their keyword arguments rebuilt from the stored gamma/Hessian."""
    meta = json.loads((here / "nonfinite.json").read_text())["cases"]
    arr = dict(np.load(here / "nonfinite.npz"))
    kwargs = dict(settings(arr["gamma"], arr["hessian"]))
    out = []
    for c in meta:
        out.append({"name": c["name"], "weight": arr[c["weight"]], "kwargs": kwargs[c["setting"]],
                    "packed": arr[f"p_{c['name']}"], "scales": arr[f"s_{c['name']}"]})
    return out, arr
