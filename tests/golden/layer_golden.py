"""Golden fixtures for the decoder-layer and whole-checkpoint workloads.

Run through ``make_golden.py --reference <checkout> --only-layers`` (the
reference package must be importable; this container's CPU torch runs it).

Decoder layer (hidden 5120, 40 query / 8 KV heads of 128, gated q_proj,
SwiGLU 17408): the layer's seven linears are seeded synthetic N(0, 0.02^2)
bf16 weights (``mxwave_b200.synthetic``, platform-independent).  The
reference's own ``calibrate_decoder_sequentially`` (mxwave/calibration_stream.py
296-466) runs the transformers Qwen3.5 layer on CPU in bf16 over 4 x 256
uniformly random token ids and returns per-target rms and damped block
Hessians.  Those statistics are stored verbatim (``layer_stats.npz``), and
the reference's ``quantize_mxfp4`` through ``iter_quantized_row_chunks``
quantizes all seven linears with them (block Hessian and rms weighting,
depth 1).  The SHA-256 of every packed / scale tensor goes to configs.json.
The embedding uses a 2,048-token vocabulary instead of 151,936: the
statistics only see the embedded rows, and the smaller table keeps the
fixture run short.

Whole checkpoint: one more layer of the same shapes (other seeds) and the
128-expert MoE stack (gate/up 768 x 2048, down 2048 x 768 per expert), all
block-Hessian weighted at depth 1 with Hessians per input width synthesized
from the heavy-channel activation law through the reference's collector
(5120 and 17408 are the block-Hessian workload's; 2048 and 768 are new).
The expert stack is recorded as one SHA-256 over the concatenated packed
bytes of every expert (gate, up, down, expert by expert) and one over the
scales.
"""

from __future__ import annotations

import hashlib
import json
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from mxwave_b200 import synthetic as syn  # noqa: E402
from tests.golden.layer_specs import (  # noqa: E402
    EXPERT_COUNT,
    EXPERT_LINEARS,
    LAYER_INPUT_GROUP,
    LAYER_LINEARS,
    ckpt_layer_seed,
    expert_seed,
    layer_seed,
)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _bf16(torch, bits: np.ndarray):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


def _quantize_chunked(torch, ref_core, ref_ckpt, w_bits: np.ndarray, **kw):
    w = _bf16(torch, w_bits)
    rows, cols = w.shape
    packed = np.empty((rows, cols // 2), np.uint8)
    scales = np.empty((rows, cols // 32), np.uint8)
    for start, stop, p, s in ref_ckpt.iter_quantized_row_chunks(
        lambda a, b: w[a:b], lambda chunk: ref_core.quantize_mxfp4(chunk, **kw), rows=rows, columns=cols,
        max_rows=1024, max_elements=ref_ckpt.DEFAULT_TENSOR_CHUNK_MAX_ELEMENTS, name="w",
    ):
        packed[start:stop] = p.numpy()
        scales[start:stop] = s.numpy()
    return packed, scales


def _calibrate_layer(torch, ref_stream, weights: dict[str, np.ndarray]):
    """The reference's sequential calibration of one random-init Qwen3.5 layer on CPU (bf16)."""
    from safetensors.torch import save_file
    from transformers.models.qwen3_5 import configuration_qwen3_5 as qc
    from transformers.models.qwen3_5 import modeling_qwen3_5 as qm

    vocab, seqs, length = 2048, 4, 256
    cfg = qc.Qwen3_5TextConfig(hidden_size=5120, num_attention_heads=40, num_key_value_heads=8, head_dim=128,
                               intermediate_size=17408, num_hidden_layers=1, vocab_size=vocab,
                               layer_types=["full_attention"])
    with torch.device("meta"):
        model = qm.Qwen3_5ForCausalLM(cfg)
    tensors = {}
    for name, param in model.named_parameters():
        short = name.removeprefix("model.layers.0.").removesuffix(".weight")
        if short in weights:
            tensors[name] = _bf16(torch, weights[short])
        elif name == "model.embed_tokens.weight":
            tensors[name] = _bf16(torch, syn.det_dense_weight(vocab, 5120, seed=420, outlier_fraction=0.0))
        elif name != "lm_head.weight":
            tensors[name] = torch.zeros(tuple(param.shape), dtype=torch.bfloat16)  # (1 + w) RMSNorm gains
    ids = np.floor(syn.det_uniform(seqs * length, seed=430) * vocab).astype(np.int64).reshape(seqs, length)
    targets = {f"model.layers.0.{short}.weight": shape[1] for short, shape in LAYER_LINEARS.items()}
    with tempfile.TemporaryDirectory() as tmp:
        ckpt = Path(tmp) / "model.safetensors"
        save_file(tensors, str(ckpt))
        files = {k: ckpt for k in tensors}
        result = ref_stream.calibrate_decoder_sequentially(
            model, targets, ("rms", "block-hessian"), ids.tolist(), files, device=torch.device("cpu"),
            dtype=torch.bfloat16, batch_size=4, hessian_damp=1e-6,
        )
    return result


def _heavy_hessian(torch, ref_cal, width: int, seed: int) -> np.ndarray:
    x = syn.det_activations(8192, width, seed=seed)
    col = ref_cal.ActivationCollector({"expert.weight": width}, ("block-hessian",), hessian_damp=1e-6)
    col.update("expert.weight", _bf16(torch, x))
    return col.finalize()["block-hessian"]["expert.weight"].numpy()


def main(out_dir: Path) -> None:
    import torch
    from mxwave import calibration as ref_cal
    from mxwave import calibration_stream as ref_stream
    from mxwave import checkpoint as ref_ckpt
    from mxwave import core as ref_core

    torch.set_num_threads(8)
    configs = json.loads((out_dir / "configs.json").read_text())
    stats: dict[str, np.ndarray] = {}

    def record(key: str, w_bits: np.ndarray, **kw) -> None:
        t0 = time.time()
        p, s = _quantize_chunked(torch, ref_core, ref_ckpt, w_bits, **kw)
        configs[key] = {"packed_sha256": sha(p), "scales_sha256": sha(s), "input_sha256": sha(w_bits),
                        "shape": list(w_bits.shape), "seconds": round(time.time() - t0, 2)}
        print(key, configs[key], flush=True)

    # -- decoder layer: reference calibration, then all seven linears --------
    weights = {short: syn.det_dense_weight(r, c, seed=layer_seed(short), outlier_fraction=0.0)
               for short, (r, c) in LAYER_LINEARS.items()}
    t0 = time.time()
    cal = _calibrate_layer(torch, ref_stream, weights)
    print(f"layer calibration {time.time() - t0:.1f}s", flush=True)
    for short, group in LAYER_INPUT_GROUP.items():
        name = f"model.layers.0.{short}.weight"
        h = cal.statistics["block-hessian"][name].numpy()
        r = cal.statistics["rms"][name].numpy()
        if f"layer_hess_{group}" in stats:  # targets sharing one input see identical statistics
            assert np.array_equal(stats[f"layer_hess_{group}"], h) and np.array_equal(stats[f"layer_rms_{group}"], r)
        stats[f"layer_hess_{group}"] = h
        stats[f"layer_rms_{group}"] = r
    configs["layer_calibration"] = {"observation_counts": sorted(set(cal.observation_counts.values())),
                                    "tokens": 4 * 256, "vocab": 2048}
    for short, w in weights.items():
        group = LAYER_INPUT_GROUP[short]
        record(f"layer_{short}_hess_d1", w, hessian=torch.from_numpy(stats[f"layer_hess_{group}"]), mse_clip_depth=1)
        record(f"layer_{short}_rms_d1", w, gamma=torch.from_numpy(stats[f"layer_rms_{group}"]), mse_clip_depth=1)
    del weights

    # -- whole checkpoint: one more layer + the 128-expert stack -------------
    old = dict(np.load(out_dir / "config_stats.npz"))
    hess = {5120: old["hess5120"], 17408: old["hess17408"]}
    hess[2048] = stats["ckpt_hess2048"] = _heavy_hessian(torch, ref_cal, 2048, seed=520)
    hess[768] = stats["ckpt_hess768"] = _heavy_hessian(torch, ref_cal, 768, seed=521)
    for short, (r, c) in LAYER_LINEARS.items():
        w = syn.det_dense_weight(r, c, seed=ckpt_layer_seed(short), outlier_fraction=0.0)
        record(f"ckpt_layer_{short}_hess_d1", w, hessian=torch.from_numpy(hess[c]), mse_clip_depth=1)
    t0 = time.time()
    hp, hs = hashlib.sha256(), hashlib.sha256()
    for e in range(EXPERT_COUNT):
        for short, (r, c) in EXPERT_LINEARS.items():
            w = syn.det_dense_weight(r, c, seed=expert_seed(e, short), outlier_fraction=0.0)
            p, s = _quantize_chunked(torch, ref_core, ref_ckpt, w, hessian=torch.from_numpy(hess[c]),
                                     mse_clip_depth=1)
            hp.update(np.ascontiguousarray(p).tobytes())
            hs.update(np.ascontiguousarray(s).tobytes())
    configs["ckpt_experts_hess_d1"] = {"packed_sha256": hp.hexdigest(), "scales_sha256": hs.hexdigest(),
                                       "experts": EXPERT_COUNT, "seconds": round(time.time() - t0, 2)}
    print("ckpt_experts_hess_d1", configs["ckpt_experts_hess_d1"], flush=True)

    np.savez_compressed(out_dir / "layer_stats.npz", **stats)
    (out_dir / "configs.json").write_text(json.dumps(configs, indent=1) + "\n")
    print("layer fixtures written")
