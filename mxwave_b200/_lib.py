"""ctypes binding of the C ABI declared in include/mxwave_b200.h.

The shared library is built in-tree (``mxwave_b200/_native/libmxwave_b200.so``)
by ``mxwave_b200.build`` / ``__graft_entry__.build()``.  There is no CPU
fallback: importing a compute entry point without the library raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_native" / "libmxwave_b200.so"

MXW_OK = 0
MXW_EINVAL = 1
MXW_ENONFINITE = 2
MXW_ECUDA = 3
MXW_ETIMEOUT = 4
MXW_EUNSUPPORTED = 5

MXW_BF16 = 0
MXW_F16 = 1
MXW_F32 = 2

MXW_METHOD_MSE = 0
MXW_METHOD_RTN = 1

MXW_DAMP_ABSOLUTE = 0
MXW_DAMP_RELATIVE = 1

MXW_FLAG_NONFINITE = 1
MXW_FLAG_TIMEOUT = 2
MXW_FLAG_RARE = 4

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_int = ctypes.c_int

# name -> (restype, argtypes).  Must list every symbol of include/mxwave_b200.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "mxw_status_string": (ctypes.c_char_p, [_int]),
    "mxw_last_cuda_error": (_int, []),
    "mxw_version": (ctypes.c_char_p, []),
    "mxw_quantize_mxfp4": (
        _int,
        [_vp, _int, _i64, _i64, _i64, ctypes.c_double, _vp, _vp, _int, _int, _vp, _vp, _vp, _vp],
    ),
    "mxw_dequant_mxfp4": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "mxw_accumulate_moments": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _vp]),
    "mxw_accumulate_block_gram": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp]),
    "mxw_accumulate_activation_stats": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "mxw_accumulate_xtx": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "mxw_xtx_packed_floats": (ctypes.c_size_t, [_i64]),
    "mxw_accumulate_xtx_packed": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "mxw_xtx_unpack": (_int, [_vp, _i64, _vp, _i64, _vp]),
    "mxw_xtx_packed_tiles": (_i64, [_i64]),
    "mxw_xtx_unpack_tiles": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "mxw_finalize_moments": (_int, [_vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "mxw_finalize_block_hessian": (_int, [_vp, _int, _i64, _i64, _i64, ctypes.c_double, _int, _vp, _vp]),
    "mxw_error_sums_workspace_size": (ctypes.c_size_t, [_i64, _i64]),
    "mxw_error_sums": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _int, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                              ctypes.c_size_t, _vp]),
    "mxw_accumulate_routed_squares": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp,
                                             _vp]),
    "mxw_repack_gguf_mxfp4": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "mxw_error_sums_noalloc": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _int, _i64, _vp, _vp, _vp, _vp, _vp,
                                      _vp]),
}

_lib: ctypes.CDLL | None = None


class NativeLibraryMissing(RuntimeError):
    """The sm_100a library has not been built; there is no fallback."""


class MxwCudaError(RuntimeError):
    """A CUDA runtime call inside the library failed."""


def load() -> ctypes.CDLL:
    """Load the native library (once), binding every C-ABI signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise NativeLibraryMissing(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(mxwave_b200 has no CPU fallback)"
        )
    import torch  # noqa: F401  -- initialise torch's CUDA runtime before ours

    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    """Map a non-OK status to an exception."""
    if status == MXW_OK:
        return
    lib = load()
    name = lib.mxw_status_string(status).decode()
    if status == MXW_ECUDA:
        raise MxwCudaError(f"{what}: {name} (cudaError {lib.mxw_last_cuda_error()})")
    if status == MXW_EINVAL:
        raise ValueError(f"{what}: {name}")
    raise RuntimeError(f"{what}: {name}")
