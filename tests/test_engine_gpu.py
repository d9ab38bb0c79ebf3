"""GPU integration: the reference's own engines with the B200 hot path
installed produce byte-identical checkpoints to the reference on CPU; the
streamer and sequential calibration match their references."""

from __future__ import annotations

import json
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from mxwave_b200 import synthetic as syn
from tests.reference_pkg import import_reference

pytestmark = pytest.mark.gpu


def _write_model(root: Path) -> Path:
    from safetensors.torch import save_file

    model = root / "model"
    model.mkdir()

    def w(rows: int, cols: int, seed: int) -> torch.Tensor:
        bits = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.01)
        return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)

    shard1 = {
        "model.layers.0.mlp.gate_proj.weight": w(300, 512, 1),
        "model.layers.0.mlp.down_proj.weight": w(128, 1024, 2),
        "model.embed_tokens.weight": w(16, 512, 3),
    }
    shard2 = {
        "model.layers.1.mlp.gate_proj.weight": w(77, 512, 4),
        "model.layers.1.input_layernorm.weight": torch.ones(512, dtype=torch.bfloat16),
    }
    save_file(shard1, str(model / "model-00001-of-00002.safetensors"))
    save_file(shard2, str(model / "model-00002-of-00002.safetensors"))
    weight_map = {k: "model-00001-of-00002.safetensors" for k in shard1}
    weight_map.update({k: "model-00002-of-00002.safetensors" for k in shard2})
    (model / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    (model / "config.json").write_text(json.dumps({"model_type": "test"}))
    (model / "tokenizer.json").write_text('{"version":"1.0"}')
    return model


def _shards(out: Path) -> dict[str, bytes]:
    return {p.name: p.read_bytes() for p in sorted(out.glob("*.safetensors"))}


@pytest.mark.parametrize("method,depth", [("mse", 1), ("mse", 4), ("rtn", 1)])
def test_reference_engine_with_b200_hot_path_is_byte_identical(tmp_path, method, depth, cuda_device) -> None:
    engine = import_reference("mxwave.engine")
    from mxwave_b200.install import install

    model = _write_model(tmp_path)
    common = dict(model_dir=model, policy="all-linear", verbose=False, method=method, mse_clip_depth=depth,
                  tensor_row_chunk_size=7, tensor_chunk_max_elements=4096, verify_sqnr=True)
    engine.quantize_model(engine.QuantizeConfig(output_dir=tmp_path / "cpu", device="cpu", **common))
    handle = install()
    try:
        # The installed module attribute is what the engine resolves at call time.
        engine_mod = sys.modules["mxwave.engine"]
        engine_mod.quantize_model(engine_mod.QuantizeConfig(output_dir=tmp_path / "gpu", device="cuda:0", **common))
    finally:
        handle.uninstall()
    cpu, gpu = _shards(tmp_path / "cpu"), _shards(tmp_path / "gpu")
    assert cpu.keys() == gpu.keys() and cpu
    for name in cpu:
        assert cpu[name] == gpu[name], name


def test_streamer_matches_device_quantizer(cuda_device) -> None:
    from mxwave_b200.core import quantize_mxfp4
    from mxwave_b200.streamer import ChunkStreamer

    bits = syn.det_dense_weight(1000, 2048, 5, outlier_fraction=0.01)
    host = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).pin_memory()
    gamma = torch.rand(2048) + 0.25
    streamer = ChunkStreamer(cuda_device, slab_bytes=300 * 2048 * 2)  # 4 slabs, ragged last one
    for kw in ({}, {"gamma": gamma}, {"method": "rtn"}, {"mse_clip_depth": 4}):
        p, s = streamer.quantize(host, **kw)
        streamer.finish()
        dkw = dict(kw)
        if "gamma" in dkw:
            dkw["gamma"] = dkw["gamma"].to(cuda_device)
        rp, rs = quantize_mxfp4(host.to(cuda_device), **dkw)
        assert torch.equal(p, rp.cpu()) and torch.equal(s, rs.cpu())
    bad = host.clone()
    bad[700, 3] = float("inf")
    streamer.quantize(bad)
    with pytest.raises(ValueError, match="NaN or infinity"):
        streamer.finish()


# ------------------------------------------------ sequential calibration


def create_causal_mask(**kwargs):
    """Explicit causal mask for the toy decoder (looked up in this module)."""
    hidden = kwargs["inputs_embeds"]
    n = hidden.shape[1]
    return torch.full((n, n), -torch.inf, device=hidden.device).triu(1)[None, None]


class _Rotary(torch.nn.Module):
    def __init__(self, config, device=None) -> None:
        super().__init__()

    def forward(self, values, position_ids):
        shape = (1, position_ids.shape[-1], values.shape[-1])
        z = torch.zeros(shape, dtype=values.dtype, device=values.device)
        return z, z


class _Layer(torch.nn.Module):
    def __init__(self, width: int) -> None:
        super().__init__()
        self.q_proj = torch.nn.Linear(width, width, bias=False)
        self.k_proj = torch.nn.Linear(width, width, bias=False)
        self.v_proj = torch.nn.Linear(width, width, bias=False)
        self.o_proj = torch.nn.Linear(width, width, bias=False)

    def forward(self, hidden_states, **_kwargs):
        mixed = self.q_proj(hidden_states) + self.k_proj(hidden_states) + self.v_proj(hidden_states)
        return hidden_states + 0.1 * self.o_proj(torch.tanh(mixed))


class _Decoder(torch.nn.Module):
    def __init__(self, width: int, layers: int) -> None:
        super().__init__()
        self.config = SimpleNamespace(model_type="qwen3_5_text", layer_types=["full_attention"] * layers,
                                      _attn_implementation="eager")
        self.embed_tokens = torch.nn.Embedding(50, width)
        self.layers = torch.nn.ModuleList([_Layer(width) for _ in range(layers)])
        self.rotary_emb = _Rotary(self.config)


class _CausalLM(torch.nn.Module):
    def __init__(self, width: int = 64, layers: int = 2) -> None:
        super().__init__()
        self.model = _Decoder(width, layers)


def test_sequential_calibration_matches_reference(tmp_path, cuda_device) -> None:
    ref = import_reference("mxwave.calibration_stream")
    from safetensors.torch import save_file

    from mxwave_b200.calibration_stream import calibrate_decoder_sequentially

    torch.manual_seed(3)
    source = _CausalLM()
    tensors = {k: v.detach().clone().contiguous() for k, v in source.state_dict().items()}
    ckpt = tmp_path / "model.safetensors"
    save_file(tensors, str(ckpt))
    files = {k: ckpt for k in tensors}
    targets = {f"model.layers.{i}.{p}.weight": 64 for i in range(2) for p in ("q_proj", "k_proj", "v_proj", "o_proj")}
    g = torch.Generator().manual_seed(9)
    sequences = torch.randint(0, 50, (6, 17), generator=g).tolist()
    kw = dict(device=None, dtype=torch.float32, batch_size=4, hessian_damp=1e-6, skip_first_tokens=1)
    objectives = ("mean-abs", "rms", "block-hessian")
    want = ref.calibrate_decoder_sequentially(_CausalLM(), targets, objectives, sequences, files,
                                              **dict(kw, device=torch.device("cpu")))
    got = calibrate_decoder_sequentially(_CausalLM(), targets, objectives, sequences, files,
                                         **dict(kw, device=cuda_device))
    assert got.observation_counts == want.observation_counts
    assert got.layer_count == want.layer_count == 2
    for objective in objectives:
        for name in targets:
            torch.testing.assert_close(got.statistics[objective][name], want.statistics[objective][name],
                                       rtol=1e-5, atol=1e-6)


# ------------------------------------------------ engine chunk stream


def _engine_chunks(engine, shard, info, cfg, gamma=None, hessian=None):
    out, err = [], None
    try:
        for start, stop, p, s in engine._quantized_chunks(shard, info, cfg, gamma, hessian):
            out.append((start, stop, p.cpu().clone(), s.cpu().clone(), p.device.type))
    except ValueError as exc:
        err = str(exc)
    return out, err


def test_engine_stream_chunks_match_reference_loop(tmp_path, cuda_device) -> None:
    """The installed _quantized_chunks yields the reference's chunks, bytes and NaN error."""
    from safetensors.torch import save_file

    engine = import_reference("mxwave.engine")
    shard_mod = import_reference("mxwave.shard")
    from mxwave_b200.install import install

    bits = syn.det_dense_weight(1000, 1024, 21, outlier_fraction=0.01)
    good = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    bad = good.clone()
    bad[613, 77] = float("nan")
    path = tmp_path / "w.safetensors"
    save_file({"a.weight": good, "b.weight": bad, "c.weight": good[:, :992].contiguous()}, str(path))
    shard = shard_mod.ShardFile(path=path, weight_map={})
    infos = shard_mod.shard_tensor_info(shard)
    gamma = torch.rand(1024) + 0.25
    errors = {}
    for name, kw in (("a.weight", {}), ("a.weight", {"gamma": gamma}), ("b.weight", {}), ("c.weight", {})):
        base = dict(model_dir=tmp_path, output_dir=tmp_path / "o", policy="all-linear", verbose=False,
                    tensor_row_chunk_size=96, tensor_chunk_max_elements=1 << 20)
        cpu_cfg = engine.QuantizeConfig(device="cpu", **base)
        want = _engine_chunks(engine, shard, infos[name], cpu_cfg, **kw)
        handle = install()
        try:
            eng = sys.modules["mxwave.engine"]
            gpu_cfg = eng.QuantizeConfig(device="cuda:0", **base)
            dkw = {k: v.to(cuda_device) for k, v in kw.items()}
            got = _engine_chunks(eng, shard, infos[name], gpu_cfg, **dkw)
        finally:
            handle.uninstall()
        assert [(a, b) for a, b, *_ in got[0]] == [(a, b) for a, b, *_ in want[0]], name
        assert got[1] == want[1], name
        for (_, _, gp, gs, dev), (_, _, wp, ws, _) in zip(got[0], want[0]):
            assert dev == "cpu"  # host chunks: the writer's .cpu() is a no-op
            assert torch.equal(gp, wp) and torch.equal(gs, ws)
        errors[name] = want[1]
    assert errors["b.weight"] is not None and "rows [576, 672)" in errors["b.weight"]
    assert errors["a.weight"] is None and errors["c.weight"] is None


def test_engine_stream_defers_to_a_patched_quantizer(tmp_path, cuda_device) -> None:
    from safetensors.torch import save_file

    import_reference("mxwave.engine")
    shard_mod = import_reference("mxwave.shard")
    from mxwave_b200.install import install

    bits = syn.det_dense_weight(64, 256, 22)
    path = tmp_path / "w.safetensors"
    save_file({"a.weight": torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)}, str(path))
    shard = shard_mod.ShardFile(path=path, weight_map={})
    info = shard_mod.shard_tensor_info(shard)["a.weight"]
    calls = []

    def fake(chunk, **_kw):
        calls.append(tuple(chunk.shape))
        return (torch.zeros(chunk.shape[0], chunk.shape[1] // 2, dtype=torch.uint8, device=chunk.device),
                torch.zeros(chunk.shape[0], chunk.shape[1] // 32, dtype=torch.uint8, device=chunk.device))

    handle = install()
    try:
        eng = sys.modules["mxwave.engine"]
        saved = eng.quantize_mxfp4
        eng.quantize_mxfp4 = fake
        try:
            cfg = eng.QuantizeConfig(model_dir=tmp_path, output_dir=tmp_path / "o", device="cuda:0", verbose=False,
                                     tensor_row_chunk_size=16, tensor_chunk_max_elements=1 << 20)
            chunks = list(eng._quantized_chunks(shard, info, cfg, None, None))
        finally:
            eng.quantize_mxfp4 = saved
    finally:
        handle.uninstall()
    assert len(chunks) == 4 and calls == [(16, 256)] * 4
