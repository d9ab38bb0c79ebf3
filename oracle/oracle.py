"""Oracle for the MxWave hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, and only as the checker.  The product package
``mxwave_b200`` never imports it.

* ``quantize_mxfp4`` wraps ``liboracle.so``, the C restatement of MxWave's
  ``quantize_mxfp4`` (mxwave/core.py:114-251), bit-exact against the reference
  run on CPU (pinned by ``tests/golden``).
* ``moments`` / ``gram`` / ``finalize_block_hessian`` restate the calibration
  collector (mxwave/calibration.py:206-274, mxwave/core.py:61-69) in float64
  numpy: the reference accumulates in fp32, so these are the exact-arithmetic
  targets that both the reference and the CUDA path are held to within a
  relative tolerance.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib: ctypes.CDLL | None = None

DTYPE_CODES = {"bf16": 0, "f16": 1, "f32": 2}
METHOD_CODES = {"mse": 0, "rtn": 1}


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        lib.oracle_quantize_mxfp4.restype = ctypes.c_int
        lib.oracle_quantize_mxfp4.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_double, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ]
        lib.oracle_dequant_mxfp4.restype = None
        lib.oracle_dequant_mxfp4.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ]
        lib.oracle_log2_f32.restype = ctypes.c_float
        lib.oracle_log2_f32.argtypes = [ctypes.c_float]
        lib.oracle_sum32.restype = ctypes.c_float
        lib.oracle_sum32.argtypes = [ctypes.c_void_p]
        lib.oracle_block_quantile.restype = ctypes.c_float
        lib.oracle_block_quantile.argtypes = [ctypes.c_void_p, ctypes.c_double]
        _lib = lib
    return _lib


def default_threads() -> int:
    return len(os.sched_getaffinity(0))


def quantize_mxfp4(
    weight: np.ndarray,
    scale_percentile: float = 99.5,
    gamma: np.ndarray | None = None,
    hessian: np.ndarray | None = None,
    method: str = "mse",
    mse_clip_depth: int = 1,
    *,
    dtype: str | None = None,
    threads: int | None = None,
) -> tuple[np.ndarray, np.ndarray]:
    """Oracle quantize.  ``weight`` is uint16 bf16/f16 bits or float32, [R, K].

    ``dtype`` defaults to "f32" for a float32 array and "bf16" for uint16 bits
    (f16 bits need ``dtype="f16"``)."""
    lib = _load()
    w = np.ascontiguousarray(weight)
    if dtype is None:
        dtype = "f32" if w.dtype == np.float32 else "bf16"
    if (dtype == "f32") != (w.dtype == np.float32):
        raise ValueError(f"weight dtype {w.dtype} does not match dtype={dtype!r}")
    if w.ndim != 2:
        raise ValueError("oracle expects a 2-D weight")
    rows, cols = w.shape
    packed = np.empty((rows, cols // 2), dtype=np.uint8)
    scales = np.empty((rows, cols // 32), dtype=np.uint8)
    g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32)
    h = None if hessian is None else np.ascontiguousarray(hessian, dtype=np.float32)
    status = lib.oracle_quantize_mxfp4(
        w.ctypes.data, DTYPE_CODES[dtype], rows, cols, cols, float(scale_percentile),
        None if g is None else g.ctypes.data, None if h is None else h.ctypes.data,
        METHOD_CODES[method], int(mse_clip_depth), packed.ctypes.data, scales.ctypes.data,
        int(threads if threads is not None else default_threads()),
    )
    if status != 0:
        raise ValueError(f"oracle rejected the arguments (status {status})")
    return packed, scales


def dequant_mxfp4(packed: np.ndarray, scales: np.ndarray, cols: int) -> np.ndarray:
    lib = _load()
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    s = np.ascontiguousarray(scales, dtype=np.uint8)
    out = np.empty((p.shape[0], cols), dtype=np.float32)
    lib.oracle_dequant_mxfp4(p.ctypes.data, s.ctypes.data, p.shape[0], cols, out.ctypes.data)
    return out


def log2_f32(q: float) -> float:
    return float(_load().oracle_log2_f32(q))


def sum32(v: np.ndarray) -> float:
    a = np.ascontiguousarray(v, dtype=np.float32)
    return float(_load().oracle_sum32(a.ctypes.data))


def block_quantile(absv: np.ndarray, pct: float) -> float:
    a = np.ascontiguousarray(absv, dtype=np.float32)
    return float(_load().oracle_block_quantile(a.ctypes.data, float(pct)))


# ---------------------------------------------------------------- calibration


def moments(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Exact-arithmetic (float64) sum|x| and sum x^2 per channel, calibration.py:227-232."""
    v = np.asarray(x, dtype=np.float64).reshape(-1, x.shape[-1])
    return np.abs(v).sum(axis=0), np.square(v).sum(axis=0)


def gram(x: np.ndarray) -> np.ndarray:
    """Full X^T X in float64 (the reference computes only its 32x32 diagonal blocks)."""
    v = np.asarray(x, dtype=np.float64).reshape(-1, x.shape[-1])
    return v.T @ v


def block_gram(x: np.ndarray) -> np.ndarray:
    """Diagonal 32x32 blocks of X^T X, float64: einsum nbi,nbj->bij, calibration.py:233-236."""
    v = np.asarray(x, dtype=np.float64).reshape(-1, x.shape[-1])
    b = v.reshape(v.shape[0], -1, 32)
    return np.einsum("nbi,nbj->bij", b, b)


def finalize_block_hessian(block_sums: np.ndarray, count: int, damp: float, mode: str) -> np.ndarray:
    """calibration.py:268-270 + core.py:61-69: G/N, then diagonal damping."""
    h = np.array(block_sums, dtype=np.float64) / count
    idx = np.arange(h.shape[-1])
    if mode == "absolute":
        h[..., idx, idx] += damp
    else:
        h[..., idx, idx] += h[..., idx, idx].mean(axis=-1, keepdims=True) * damp
    return h


def error_sums(
    original: np.ndarray,
    reconstructed: np.ndarray,
    gamma: np.ndarray | None = None,
    hessian: np.ndarray | None = None,
) -> np.ndarray:
    """float64 sums behind the SQNR family, verify.py:24-86.

    [sum o^2, sum (o - r)^2, weighted signal, weighted noise]; the difference
    o - r is formed in fp32 as the reference forms it, the rest in float64.
    Weighted: gamma^2 per input channel, or the 32x32 block quadratic form.
    """
    o32 = np.asarray(original, dtype=np.float32)
    d32 = (o32 - np.asarray(reconstructed, dtype=np.float32)).astype(np.float32)
    o, d = o32.astype(np.float64), d32.astype(np.float64)
    out = np.zeros(4)
    out[0], out[1] = (o * o).sum(), (d * d).sum()
    if gamma is not None:
        g2 = np.asarray(gamma, dtype=np.float64) ** 2
        out[2], out[3] = (o * o * g2).sum(), (d * d * g2).sum()
    elif hessian is not None:
        h = np.asarray(hessian, dtype=np.float64)
        ob, db = o.reshape(o.shape[0], -1, 32), d.reshape(d.shape[0], -1, 32)
        out[2] = np.einsum("rbi,bij,rbj->", ob, h, ob)
        out[3] = np.einsum("rbi,bij,rbj->", db, h, db)
    return out


def sqnr_db(signal: float, noise: float) -> float:
    """10 log10(signal / noise) with both clamped below at fp32(1e-12), as verify.py does."""
    floor = float(np.float32(1e-12))
    return float(10.0 * np.log10(max(signal, floor) / max(noise, floor)))


def routed_squares(inputs: np.ndarray, ids: np.ndarray, weights: np.ndarray, experts: int,
                   token_major: bool) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """routed_calibration.py:104-141: per-expert sums of fl(fl(x^2) * fl(w^2)), float64.

    token_major=False: route (t, k) reads row t (update_inputs); True: row r of
    the flattened routes (update_down).  Returns (squares, mass, counts).
    """
    x = np.asarray(inputs, dtype=np.float32)
    flat_ids = np.asarray(ids).reshape(-1).astype(np.int64)
    w2 = np.square(np.asarray(weights, dtype=np.float32).reshape(-1))
    top_k = np.asarray(ids).shape[1]
    squares = np.zeros((experts, x.shape[1]))
    mass = np.zeros(experts)
    for r, e in enumerate(flat_ids):
        row = x[r if token_major else r // top_k]
        squares[e] += (np.square(row) * w2[r]).astype(np.float32)
        mass[e] += w2[r]
    return squares, mass, np.bincount(flat_ids, minlength=experts)


def gguf_repack(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """gguf.py:134-150: per block the scale byte, then code j | code j+16 << 4."""
    p = np.asarray(packed, dtype=np.uint8)
    rows, half = p.shape
    blocks = half * 2 // 32
    codes = np.empty((rows, half * 2), dtype=np.uint8)
    codes[:, 0::2] = p & 0x0F
    codes[:, 1::2] = p >> 4
    codes = codes.reshape(rows, blocks, 32)
    body = codes[:, :, :16] | (codes[:, :, 16:] << 4)
    out = np.concatenate([np.asarray(scales, dtype=np.uint8).reshape(rows, blocks, 1), body], axis=-1)
    return out.reshape(rows, blocks * 17)
