"""The quantize kernel's division-free block exponents (floor/ceil of
log2(x / 6), mxwave/core.py:199-206) agree with the division-based definition
for every fp32 value in range: an exhaustive CPU run of
oracle/check_exponents.c (a few seconds)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_division_free_exponents_match_definition(tmp_path) -> None:
    exe = tmp_path / "check_exponents"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", str(exe), str(ROOT / "oracle" / "check_exponents.c")],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 disagreements" in out.stdout
