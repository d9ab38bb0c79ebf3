"""CPU tests of the chunk loop and the install boundary (no GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mxwave_b200 import checkpoint as ours
from oracle import oracle
from tests.reference_pkg import import_reference


def _oracle_quantize(weight: torch.Tensor):
    p, s = oracle.quantize_mxfp4(weight.float().numpy(), dtype="f32")
    return torch.from_numpy(p), torch.from_numpy(s)


@pytest.mark.parametrize("columns", [32, 96, 768, 2048, 5120, 17408])
@pytest.mark.parametrize("max_rows", [1, 60, 1024])
@pytest.mark.parametrize("max_elements", [1024, 1_048_576, 33_554_432])
def test_chunk_rows_match_reference(columns, max_rows, max_elements) -> None:
    ref = import_reference("mxwave.checkpoint")
    try:
        expected = ref.tensor_chunk_rows(columns, max_rows, max_elements)
    except ValueError as exc:
        with pytest.raises(ValueError, match=str(exc)):
            ours.tensor_chunk_rows(columns, max_rows, max_elements)
        return
    assert ours.tensor_chunk_rows(columns, max_rows, max_elements) == expected


@pytest.mark.parametrize("prefetch", [0, 2])
def test_chunk_iteration_matches_reference(prefetch) -> None:
    ref = import_reference("mxwave.checkpoint")
    g = torch.Generator().manual_seed(0)
    w = torch.randn(203, 96, generator=g)
    kwargs = dict(rows=203, columns=96, max_rows=1024, max_elements=96 * 17, name="w")
    got = list(ours.iter_quantized_row_chunks(lambda a, b: w[a:b], _oracle_quantize, prefetch=prefetch, **kwargs))
    want = list(ref.iter_quantized_row_chunks(lambda a, b: w[a:b], _oracle_quantize, **kwargs))
    assert [(a, b) for a, b, _, _ in got] == [(a, b) for a, b, _, _ in want]
    for (_, _, p, s), (_, _, rp, rs) in zip(got, want):
        assert torch.equal(p, rp) and torch.equal(s, rs)


def test_chunk_errors_match_reference() -> None:
    ref = import_reference("mxwave.checkpoint")
    w = torch.zeros(100, 64)
    w[57, 3] = float("nan")
    kwargs = dict(rows=100, columns=64, max_rows=20, max_elements=1 << 20, name="layer.weight")
    with pytest.raises(ValueError) as ref_exc:
        list(ref.iter_quantized_row_chunks(lambda a, b: w[a:b], _oracle_quantize, **kwargs))
    with pytest.raises(ValueError) as our_exc:
        list(ours.iter_quantized_row_chunks(lambda a, b: w[a:b], _oracle_quantize, **kwargs))
    assert str(our_exc.value) == str(ref_exc.value)
    bad_shape = dict(kwargs, columns=32)
    with pytest.raises(ValueError) as ref_exc:
        list(ref.iter_quantized_row_chunks(lambda a, b: w[a:b], _oracle_quantize, **bad_shape))
    with pytest.raises(ValueError) as our_exc:
        list(ours.iter_quantized_row_chunks(lambda a, b: w[a:b], _oracle_quantize, **bad_shape))
    assert str(our_exc.value) == str(ref_exc.value)


def test_install_replaces_and_restores_reference_names() -> None:
    import_reference("mxwave.engine")
    import sys

    from mxwave_b200 import core as our_core
    from mxwave_b200.install import install

    engine = sys.modules["mxwave.engine"]
    original = engine.quantize_mxfp4
    handle = install()
    try:
        assert engine.quantize_mxfp4 is our_core.quantize_mxfp4
        assert sys.modules["mxwave.core"].quantize_mxfp4 is our_core.quantize_mxfp4
        assert engine.iter_quantized_row_chunks is ours.iter_quantized_row_chunks
    finally:
        handle.uninstall()
    assert engine.quantize_mxfp4 is original


def test_install_then_uninstall_restores_every_module_in_a_fresh_interpreter() -> None:
    """No module first imported during install() may keep a replacement after uninstall()."""
    import subprocess
    import sys
    from pathlib import Path

    import_reference("mxwave")
    from tests.reference_pkg import REF_DIR

    root = Path(__file__).resolve().parents[1]
    code = f"""
import sys
sys.path[:0] = [{str(REF_DIR)!r}, {str(root)!r}]
import mxwave_b200._lib as lib
lib.load = lambda: None  # the CPU container has no GPU library to bind
from mxwave_b200.install import install, _replacements
h = install()
h.uninstall()
bad = []
for mod, names in _replacements().items():
    m = sys.modules.get(mod)
    for n, v in names.items():
        if m is not None and getattr(m, n, None) is v:
            bad.append(mod + "." + n)
print("BAD", bad)
"""
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert "BAD []" in out.stdout, out.stdout


def test_oracle_chunk_helper_is_consistent() -> None:
    w = torch.randn(5, 64)
    p, s = _oracle_quantize(w)
    assert p.shape == (5, 32) and s.shape == (5, 2)
    assert np.array_equal(p.numpy(), oracle.quantize_mxfp4(w.numpy(), dtype="f32")[0])
