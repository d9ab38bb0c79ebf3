"""GPU parity on the decoder-layer and whole-checkpoint workloads.

* Decoder layer (hidden 5120, gated q_proj, GQA 40/8, SwiGLU 17408): all seven
  linears quantized with the statistics the reference's own sequential
  calibration produced (tests/golden/layer_golden.py), block-Hessian and rms
  weighted; bar: SHA-256 of packed and scales equal to the reference's.
* Whole checkpoint: one more layer and the 128-expert MoE stack
  (gate/up 768 x 2048, down 2048 x 768), block-Hessian weighted; the expert
  stack is one SHA-256 over every expert's bytes in order.
* The sequential calibration of a two-layer model of the decoder-layer shape:
  this package on the GPU against the reference on the CPU, both in fp32 on
  the same checkpoint and tokens; bar: rtol 1e-5 with an absolute floor of
  1e-5 x the statistic's largest magnitude (fp32 forwards on two devices
  differ in the last bits).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from mxwave_b200 import synthetic as syn
from mxwave_b200.core import quantize_mxfp4
from tests.golden.fixtures import load_config_stats, load_configs, load_layer_stats
from tests.golden.layer_specs import (
    EXPERT_COUNT,
    EXPERT_LINEARS,
    LAYER_INPUT_GROUP,
    LAYER_LINEARS,
    ckpt_layer_seed,
    expert_seed,
    layer_seed,
)
from tests.reference_pkg import import_reference

pytestmark = pytest.mark.gpu


def _sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.cpu().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _bf16(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _golden(key: str) -> dict:
    cfg = load_configs()
    if key not in cfg:
        pytest.skip(f"golden hash {key} not generated")
    return cfg[key]


@pytest.mark.parametrize("short", list(LAYER_LINEARS))
def test_decoder_layer_linears_match_reference(short, cuda_device) -> None:
    stats = load_layer_stats()
    group = LAYER_INPUT_GROUP[short]
    if f"layer_hess_{group}" not in stats:
        pytest.skip("layer statistics not generated")
    rows, cols = LAYER_LINEARS[short]
    bits = syn.det_dense_weight(rows, cols, seed=layer_seed(short), outlier_fraction=0.0)
    w = _bf16(bits, cuda_device)
    for objective, kw in (("hess", {"hessian": torch.from_numpy(stats[f"layer_hess_{group}"]).to(cuda_device)}),
                          ("rms", {"gamma": torch.from_numpy(stats[f"layer_rms_{group}"]).to(cuda_device)})):
        c = _golden(f"layer_{short}_{objective}_d1")
        assert _sha(bits) == c["input_sha256"]
        p, s = quantize_mxfp4(w, mse_clip_depth=1, **kw)
        assert _sha(p) == c["packed_sha256"], objective
        assert _sha(s) == c["scales_sha256"], objective


@pytest.mark.parametrize("short", list(LAYER_LINEARS))
def test_checkpoint_layer_linears_match_reference(short, cuda_device) -> None:
    old = load_config_stats()
    if "hess5120" not in old:
        pytest.skip("config statistics not generated")
    hess = {5120: old["hess5120"], 17408: old["hess17408"]}
    rows, cols = LAYER_LINEARS[short]
    c = _golden(f"ckpt_layer_{short}_hess_d1")
    bits = syn.det_dense_weight(rows, cols, seed=ckpt_layer_seed(short), outlier_fraction=0.0)
    assert _sha(bits) == c["input_sha256"]
    p, s = quantize_mxfp4(_bf16(bits, cuda_device), hessian=torch.from_numpy(hess[cols]).to(cuda_device),
                          mse_clip_depth=1)
    assert _sha(p) == c["packed_sha256"]
    assert _sha(s) == c["scales_sha256"]


def test_expert_stack_matches_reference(cuda_device) -> None:
    stats = load_layer_stats()
    if "ckpt_hess2048" not in stats:
        pytest.skip("expert statistics not generated")
    c = _golden("ckpt_experts_hess_d1")
    hess = {2048: torch.from_numpy(stats["ckpt_hess2048"]).to(cuda_device),
            768: torch.from_numpy(stats["ckpt_hess768"]).to(cuda_device)}
    hp, hs = hashlib.sha256(), hashlib.sha256()
    for e in range(EXPERT_COUNT):
        for short, (rows, cols) in EXPERT_LINEARS.items():
            bits = syn.det_dense_weight(rows, cols, seed=expert_seed(e, short), outlier_fraction=0.0)
            p, s = quantize_mxfp4(_bf16(bits, cuda_device), hessian=hess[cols], mse_clip_depth=1)
            hp.update(p.cpu().numpy().tobytes())
            hs.update(s.cpu().numpy().tobytes())
    assert hp.hexdigest() == c["packed_sha256"]
    assert hs.hexdigest() == c["scales_sha256"]


def _decoder_checkpoint(tmp_path, layers: int, vocab: int):
    """A random-init Qwen3.5 model of the decoder-layer shape, written to safetensors."""
    from safetensors.torch import save_file
    from transformers.models.qwen3_5 import configuration_qwen3_5 as qc
    from transformers.models.qwen3_5 import modeling_qwen3_5 as qm

    cfg = qc.Qwen3_5TextConfig(hidden_size=5120, num_attention_heads=40, num_key_value_heads=8, head_dim=128,
                               intermediate_size=17408, num_hidden_layers=layers, vocab_size=vocab,
                               layer_types=["full_attention"] * layers)
    with torch.device("meta"):
        model = qm.Qwen3_5ForCausalLM(cfg)
    tensors = {}
    for name, param in model.named_parameters():
        if name == "lm_head.weight":
            continue
        if param.ndim == 2:
            seed = 7000 + len(tensors)
            tensors[name] = _bf16(syn.det_dense_weight(*param.shape, seed=seed, outlier_fraction=0.0), "cpu")
        else:
            tensors[name] = torch.full(tuple(param.shape), 0.05, dtype=torch.bfloat16)  # (1 + w) RMSNorm gains
    ckpt = tmp_path / "model.safetensors"
    save_file(tensors, str(ckpt))
    return (lambda: _meta_model(qm, cfg)), {k: ckpt for k in tensors}


def _meta_model(qm, cfg):
    with torch.device("meta"):
        return qm.Qwen3_5ForCausalLM(cfg)


def test_decoder_layer_calibration_matches_reference(tmp_path, cuda_device) -> None:
    ref = import_reference("mxwave.calibration_stream")
    from mxwave_b200.calibration_stream import calibrate_decoder_sequentially

    make_model, files = _decoder_checkpoint(tmp_path, layers=2, vocab=512)
    targets = {f"model.layers.{i}.{short}.weight": shape[1] for i in range(2) for short, shape in LAYER_LINEARS.items()}
    ids = np.floor(syn.det_uniform(2 * 48, seed=77) * 512).astype(np.int64).reshape(2, 48).tolist()
    kw = dict(dtype=torch.float32, batch_size=2, hessian_damp=1e-6, skip_first_tokens=1)
    objectives = ("mean-abs", "rms", "block-hessian")
    want = ref.calibrate_decoder_sequentially(make_model(), targets, objectives, ids, files,
                                              device=torch.device("cpu"), **kw)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        got = calibrate_decoder_sequentially(make_model(), targets, objectives, ids, files, device=cuda_device, **kw)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert got.observation_counts == want.observation_counts
    assert got.layer_count == want.layer_count == 2
    for objective in objectives:
        for name in targets:
            g, w = got.statistics[objective][name], want.statistics[objective][name]
            floor = 1e-5 * float(w.abs().max())
            torch.testing.assert_close(g, w, rtol=1e-5, atol=floor, msg=f"{objective} {name}")
