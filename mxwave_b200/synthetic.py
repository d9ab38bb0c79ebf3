"""Seeded synthetic inputs with the benchmark shapes and value laws.

No checkpoint or calibration corpus is available offline, so weights and
activations are synthetic.  Two generators are provided:

* ``det_*`` functions: platform-independent numpy generators built only from
  integer hashing and IEEE-exact basic float64 operations (+, -, *, /, sqrt,
  frexp/ldexp), so the same seed gives the same bits on any x86 host whatever
  its SIMD dispatch.  Golden fixtures are keyed on these.
* ``torch_*`` functions: fast on-device generators with the same laws, for
  benchmarks where bit-reproducibility across hosts is not needed.

Laws (one per workload):
* dense weight: N(0, sigma^2), a fraction of uniformly chosen positions x20;
* heavy-channel activations: N(0,1) * s_c with s_c = exp(N(0,1)) per channel
  and 16 random channels boosted x50.
"""

from __future__ import annotations

import numpy as np

_LN2 = 0.6931471805599453
_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(counter: np.ndarray, seed: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = counter.astype(np.uint64) + np.uint64((seed * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF)
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def det_uniform(n: int, seed: int, stream: int = 0) -> np.ndarray:
    """Uniform float64 in (0, 1), 53-bit, from a counter-based hash."""
    counter = np.arange(n, dtype=np.uint64) + np.uint64(stream) * np.uint64(1 << 32)
    bits = _splitmix64(counter, seed) >> np.uint64(11)
    return (bits.astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def _det_log(x: np.ndarray) -> np.ndarray:
    """ln(x) for x > 0 from frexp and an atanh series (basic ops only)."""
    m, e = np.frexp(x)  # x = m * 2^e, m in [0.5, 1)
    small = m < 0.7071067811865476
    m = np.where(small, m * 2.0, m)
    e = np.where(small, e - 1, e)
    s = (m - 1.0) / (m + 1.0)
    s2 = s * s
    acc = np.full_like(s, 1.0 / 27.0)
    for k in range(13, 0, -1):
        acc = acc * s2 + 1.0 / (2 * k - 1)
    return e.astype(np.float64) * _LN2 + 2.0 * s * acc


def _det_exp(x: np.ndarray) -> np.ndarray:
    """exp(x) from 2^k * Taylor(r) (basic ops only)."""
    k = np.floor(x / _LN2 + 0.5)
    r = x - k * _LN2
    acc = np.ones_like(r)
    for j in range(20, 0, -1):
        acc = acc * (r / j) + 1.0
    return np.ldexp(acc, k.astype(np.int64))


_CHUNK = 1 << 20


def _normal_chunk(n: int, seed: int, stream: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float64)
    filled, rnd = 0, 0
    while filled < n:
        need = n - filled
        m = int(need * 0.66) + 64
        u = det_uniform(2 * m, seed, stream * 64 + rnd) * 2.0 - 1.0
        a, b = u[:m], u[m:]
        s = a * a + b * b
        ok = (s > 0.0) & (s < 1.0)
        a, b, s = a[ok], b[ok], s[ok]
        f = np.sqrt(-2.0 * _det_log(s) / s)
        z = np.concatenate([a * f, b * f])[:need]
        out[filled : filled + z.size] = z
        filled += z.size
        rnd += 1
    return out


def det_normal(n: int, seed: int, stream: int = 0) -> np.ndarray:
    """Standard normal float64 by the Marsaglia polar method.

    The sequence is cut into fixed 2^20-element chunks, each with its own
    counter stream, so chunks are generated on a thread pool and the result
    does not depend on the number of threads.
    """
    import os
    from concurrent.futures import ThreadPoolExecutor

    out = np.empty(n, dtype=np.float64)
    starts = list(range(0, n, _CHUNK))

    def fill(i: int) -> None:
        lo = starts[i]
        hi = min(lo + _CHUNK, n)
        out[lo:hi] = _normal_chunk(hi - lo, seed, (stream << 20) + i)

    workers = max(1, min(len(starts), len(os.sched_getaffinity(0))))
    if workers == 1:
        for i in range(len(starts)):
            fill(i)
    else:
        with ThreadPoolExecutor(workers) as pool:
            list(pool.map(fill, range(len(starts))))
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (round-to-nearest-even), returned as uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    with np.errstate(over="ignore"):
        return ((u + rounding) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def det_dense_weight(rows: int, cols: int, seed: int, sigma: float = 0.02,
                     outlier_fraction: float = 0.001, outlier_scale: float = 20.0) -> np.ndarray:
    """Dense [rows, cols] bf16 bits: N(0, sigma^2) with outliers x outlier_scale."""
    n = rows * cols
    w = det_normal(n, seed, stream=1) * sigma
    if outlier_fraction > 0:
        count = int(round(n * outlier_fraction))
        keys = det_uniform(n, seed, stream=2)
        idx = np.argpartition(keys, count)[:count] if count < n else np.arange(n)
        w[idx] *= outlier_scale
    return f32_to_bf16_bits(w.astype(np.float32)).reshape(rows, cols)


def det_channel_scales(cols: int, seed: int, sigma: float = 1.0, boosted: int = 16,
                       boost: float = 50.0) -> np.ndarray:
    """Per-channel scale s_c = exp(N(0, sigma^2)), `boosted` channels x boost (float64)."""
    s = _det_exp(det_normal(cols, seed, stream=3) * sigma)
    if boosted:
        keys = det_uniform(cols, seed, stream=4)
        s[np.argsort(keys, kind="stable")[:boosted]] *= boost
    return s


def det_activations(tokens: int, cols: int, seed: int, scales_seed: int | None = None) -> np.ndarray:
    """Heavy-channel activations [tokens, cols] as bf16 bits."""
    s = det_channel_scales(cols, seed if scales_seed is None else scales_seed)
    x = det_normal(tokens * cols, seed, stream=5).reshape(tokens, cols) * s[None, :]
    return f32_to_bf16_bits(x.astype(np.float32))


# ------------------------------------------------------------------ on device


def torch_dense_weight(rows: int, cols: int, seed: int, device, sigma: float = 0.02,
                       outlier_fraction: float = 0.001, outlier_scale: float = 20.0):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(rows, cols, generator=g, device=device) * sigma
    if outlier_fraction > 0:
        mask = torch.rand(rows, cols, generator=g, device=device) < outlier_fraction
        w = torch.where(mask, w * outlier_scale, w)
    return w.to(torch.bfloat16)


def torch_activations(tokens: int, cols: int, seed: int, device):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    s = torch.exp(torch.randn(cols, generator=g, device=device))
    boost = torch.randperm(cols, generator=g, device=device)[:16]
    s[boost] *= 50.0
    x = torch.randn(tokens, cols, generator=g, device=device) * s
    return x.to(torch.bfloat16)


# Decoder layer of the calibration workload: hidden 5120, 40 query / 8 KV heads
# of 128 (gated q_proj: 40 * 128 * 2 outputs), SwiGLU intermediate 17408.
DECODER_SHAPE = {"hidden": 5120, "heads": 40, "kv_heads": 8, "head_dim": 128, "intermediate": 17408,
                 "vocab": 151936}


def decoder_config(layers: int, vocab: int | None = None):
    """transformers Qwen3.5 text config of the calibration workload's decoder (full attention)."""
    from transformers.models.qwen3_5 import configuration_qwen3_5 as qc

    d = DECODER_SHAPE
    return qc.Qwen3_5TextConfig(hidden_size=d["hidden"], num_attention_heads=d["heads"],
                                num_key_value_heads=d["kv_heads"], head_dim=d["head_dim"],
                                intermediate_size=d["intermediate"], num_hidden_layers=layers,
                                vocab_size=vocab or d["vocab"], layer_types=["full_attention"] * layers)


def meta_decoder(config):
    """The model skeleton on the meta device (weights come from the checkpoint)."""
    import torch
    from transformers.models.qwen3_5 import modeling_qwen3_5 as qm

    with torch.device("meta"):
        return qm.Qwen3_5ForCausalLM(config)


def write_decoder_checkpoint(path, config, seed: int, device) -> dict:
    """Random-init weights of `config` (N(0, 0.02^2) matrices, zero RMSNorm offsets) as one
    safetensors file; returns the tensor name -> path map calibration takes."""
    import torch
    from safetensors.torch import save_file

    tensors = {}
    for i, (name, param) in enumerate(meta_decoder(config).named_parameters()):
        if name == "lm_head.weight":
            continue
        if param.ndim == 2:
            tensors[name] = torch_dense_weight(*param.shape, seed=seed + i, device=device,
                                               outlier_fraction=0.0).cpu()
        else:
            tensors[name] = torch.zeros(tuple(param.shape), dtype=torch.bfloat16)
    save_file(tensors, str(path))
    return {k: path for k in tensors}


__all__ = [
    "DECODER_SHAPE",
    "bf16_bits_to_f32",
    "decoder_config",
    "det_activations",
    "det_channel_scales",
    "det_dense_weight",
    "det_normal",
    "det_uniform",
    "f32_to_bf16_bits",
    "meta_decoder",
    "torch_activations",
    "torch_dense_weight",
    "write_decoder_checkpoint",
]
