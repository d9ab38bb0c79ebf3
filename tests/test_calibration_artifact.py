"""Calibration artefact hand-off: files match the reference's (header entries,
metadata and data bytes),
and a same-process open serves the device statistics (GPU part) instead of
re-reading the file."""

from __future__ import annotations

import json
import os
import struct

import pytest
import torch

from tests.reference_pkg import import_reference

META = {"policy": "all-linear", "num_sequences": "4", "sequence_length": "16", "num_tokens": "64"}
WIDTHS = {"a.weight": 64, "b.weight": 32}


def _same_artifact(a, b) -> None:
    """Same header entries and metadata (safetensors writes metadata keys in hash
    order, which differs between calls even for the reference), same data bytes."""
    da, db = a.read_bytes(), b.read_bytes()
    na, nb = struct.unpack("<Q", da[:8])[0], struct.unpack("<Q", db[:8])[0]
    assert json.loads(da[8 : 8 + na]) == json.loads(db[8 : 8 + nb])
    assert da[8 + na :] == db[8 + nb :]


def _stats(device) -> dict[str, dict[str, torch.Tensor]]:
    g = torch.Generator().manual_seed(3)
    rms = {n: (torch.rand(w, generator=g) + 0.1).to(device) for n, w in WIDTHS.items()}
    hess = {}
    for n, w in WIDTHS.items():
        x = torch.randn(16, w, generator=g)
        h = torch.einsum("nbi,nbj->bij", x.view(16, -1, 32), x.view(16, -1, 32)) / 16 + 1e-3 * torch.eye(32)
        hess[n] = h.to(device)
    return {"rms": rms, "block-hessian": hess}


def test_cpu_statistics_write_the_reference_bytes(tmp_path) -> None:
    ref = import_reference("mxwave.calibration")
    from mxwave_b200.calibration_artifact import open_calibration_data, save_calibration_data

    stats = _stats("cpu")
    save_calibration_data(tmp_path / "ours.safetensors", stats, META)
    ref.save_calibration_data(tmp_path / "ref.safetensors", stats, META)
    _same_artifact(tmp_path / "ours.safetensors", tmp_path / "ref.safetensors")
    art = open_calibration_data(tmp_path / "ours.safetensors", "rms", WIDTHS, expected_policy="all-linear")
    assert torch.equal(art.tensors["a.weight"], stats["rms"]["a.weight"])


@pytest.mark.gpu
def test_device_statistics_hand_off(tmp_path, cuda_device) -> None:
    ref = import_reference("mxwave.calibration")
    from mxwave_b200.calibration_artifact import (
        open_calibration_data,
        release_device_statistics,
        save_calibration_data,
    )

    stats = _stats(cuda_device)
    path = tmp_path / "stats.safetensors"
    save_calibration_data(path, stats, META)
    cpu = {o: {n: v.cpu() for n, v in vals.items()} for o, vals in stats.items()}
    ref.save_calibration_data(tmp_path / "ref.safetensors", cpu, META)
    _same_artifact(path, tmp_path / "ref.safetensors")

    for objective in ("rms", "block-hessian"):
        art = open_calibration_data(path, objective, WIDTHS, expected_policy="all-linear")
        art.validate_all()
        for name in WIDTHS:
            got = art.tensors[name]
            assert got.device.type == "cuda"
            assert torch.equal(got, stats[objective][name])
        assert art.file_sha256 == ref.open_calibration_data(path, objective, WIDTHS,
                                                            expected_policy="all-linear").file_sha256
    # A file changed after saving is read from disk again, as the reference reads it.
    data = path.read_bytes()
    path.unlink()
    path.write_bytes(data)
    os.utime(path, ns=(1, 1))
    art = open_calibration_data(path, "rms", WIDTHS, expected_policy="all-linear")
    assert art.tensors["a.weight"].device.type == "cpu"
    release_device_statistics(path)


@pytest.mark.gpu
def test_device_statistics_are_validated_like_the_file(tmp_path, cuda_device) -> None:
    from mxwave_b200.calibration_artifact import open_calibration_data, save_calibration_data

    stats = _stats(cuda_device)
    stats["rms"]["b.weight"][3] = -1.0  # invalid magnitude: the reference rejects it when read
    path = tmp_path / "bad.safetensors"
    save_calibration_data(path, stats, META)
    art = open_calibration_data(path, "rms", WIDTHS, expected_policy="all-linear")
    with pytest.raises(ValueError, match="non-negative and nonzero"):
        art.tensors["b.weight"]


def test_installed_functions_call_the_reference_not_themselves(tmp_path) -> None:
    import_reference("mxwave.calibration")
    import sys

    from mxwave_b200 import _lib
    from mxwave_b200.install import install

    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    handle = install()
    try:
        mod = sys.modules["mxwave.calibration"]
        stats = _stats("cpu")
        mod.save_calibration_data(tmp_path / "x.safetensors", stats, META)
        art = mod.open_calibration_data(tmp_path / "x.safetensors", "rms", WIDTHS, expected_policy="all-linear")
        assert torch.equal(art.tensors["b.weight"], stats["rms"]["b.weight"])
    finally:
        handle.uninstall()
