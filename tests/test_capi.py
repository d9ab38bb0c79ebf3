"""CPU tests of the C ABI: the library loads, exports every declared symbol,
and rejects bad arguments on the host before touching a GPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from mxwave_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "mxwave_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"MXW_API\s+[\w\s\*]+?\b(mxw_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    if not _lib.LIB_PATH.exists():
        pytest.fail(f"{_lib.LIB_PATH} not built (run __graft_entry__.build())")
    return _lib.load()


def test_header_declares_the_entry_points() -> None:
    names = declared_functions()
    for required in ("mxw_quantize_mxfp4", "mxw_accumulate_moments", "mxw_accumulate_block_gram",
                     "mxw_finalize_block_hessian", "mxw_dequant_mxfp4"):
        assert required in names


def test_every_declared_symbol_is_exported(lib: ctypes.CDLL) -> None:
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"


def test_python_binding_covers_the_header() -> None:
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_status_strings_and_version(lib: ctypes.CDLL) -> None:
    assert lib.mxw_status_string(_lib.MXW_OK) == b"ok"
    assert lib.mxw_status_string(_lib.MXW_EINVAL) == b"invalid argument"
    assert b"sm_100a" in lib.mxw_version()


@pytest.mark.parametrize(
    "kwargs",
    [
        {"cols": 48},  # not a multiple of 32
        {"depth": 9},
        {"depth": -1},
        {"pct": 0.0},
        {"pct": 100.5},
        {"method": 7},
        {"dtype": 9},
        {"ld": 16},  # ld < cols
        {"both": True},  # gamma and hessian together
        {"rtn_weighted": True},
    ],
)
def test_quantize_rejects_bad_arguments_on_host(lib: ctypes.CDLL, kwargs: dict) -> None:
    cols = kwargs.get("cols", 64)
    g = ctypes.c_void_p(16) if kwargs.get("both") or kwargs.get("rtn_weighted") else None
    h = ctypes.c_void_p(16) if kwargs.get("both") else None
    status = lib.mxw_quantize_mxfp4(
        ctypes.c_void_p(16), kwargs.get("dtype", _lib.MXW_BF16), 4, cols, kwargs.get("ld", cols),
        kwargs.get("pct", 99.5), g, h,
        _lib.MXW_METHOD_RTN if kwargs.get("rtn_weighted") else kwargs.get("method", _lib.MXW_METHOD_MSE),
        kwargs.get("depth", 1), ctypes.c_void_p(16), ctypes.c_void_p(16), None, None,
    )
    assert status == _lib.MXW_EINVAL


def test_zero_rows_is_a_no_op(lib: ctypes.CDLL) -> None:
    status = lib.mxw_quantize_mxfp4(None, _lib.MXW_BF16, 0, 64, 64, 99.5, None, None, 0, 1, None, None, None, None)
    assert status == _lib.MXW_OK


def test_stats_reject_bad_arguments_on_host(lib: ctypes.CDLL) -> None:
    # block Gram needs widths divisible by 32; moments accept any width.
    assert lib.mxw_accumulate_block_gram(ctypes.c_void_p(16), _lib.MXW_BF16, 8, 40, 40, ctypes.c_void_p(16), None) \
        == _lib.MXW_EINVAL
    assert lib.mxw_accumulate_moments(ctypes.c_void_p(16), _lib.MXW_BF16, 8, 40, 39, None, None, None) \
        == _lib.MXW_EINVAL
    assert lib.mxw_finalize_block_hessian(ctypes.c_void_p(16), 0, 64, 64, 10, -1.0, 0, ctypes.c_void_p(16), None) \
        == _lib.MXW_EINVAL
    assert lib.mxw_finalize_block_hessian(ctypes.c_void_p(16), 0, 64, 64, 10, 1e-6, 5, ctypes.c_void_p(16), None) \
        == _lib.MXW_EINVAL


def test_product_path_fails_loudly_without_cuda_tensors() -> None:
    import torch

    from mxwave_b200.core import quantize_mxfp4

    with pytest.raises(RuntimeError, match="CUDA devices only"):
        quantize_mxfp4(torch.zeros(2, 32))
