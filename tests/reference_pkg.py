"""Access to the reference MxWave package installed into baseline/_ref.

Integration tests run the reference's own engines (planning, chunk loop,
safetensors writer) with and without the B200 hot path installed.  When the
package is not installed they skip.
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

REF_DIR = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def reference_available() -> bool:
    return (REF_DIR / "mxwave" / "__init__.py").exists()


def import_reference(module: str = "mxwave"):
    if not reference_available():
        pytest.skip("reference package not installed in baseline/_ref")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    return importlib.import_module(module)
