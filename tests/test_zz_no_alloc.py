"""GPU: the allocation-free error-sum entry point (mxw_error_sums_noalloc).

Some callers cannot allocate device memory when they call: a process that
reserves its whole device memory budget at start-up and forbids later
allocations, or a health check that must still run on a device that is out
of memory.  mxw_error_sums_noalloc serves them from a fixed device array in
the library instead of a caller workspace.  This file checks, through the C
ABI, that two calls in a row (different inputs and modes, then a repeat) give
the same sums as mxw_error_sums with a workspace.  It is collected last, and
it passes alone in a fresh process (where its first call does the one-time
set-up) as well as after the other tests.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mxwave_b200 import _lib
from mxwave_b200 import synthetic as syn
from mxwave_b200.core import dequant_mxfp4, quantize_mxfp4
from oracle import oracle

pytestmark = pytest.mark.gpu

RTOL = 1e-12  # the two entry points run the same kernel and grid: the sums should agree to the last bit
DB_TOL = 1e-4  # dB, the tolerance of the SQNR tests


def _inputs(rows: int, cols: int, seed: int, device):
    bits = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.01)
    w = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)
    g = torch.Generator().manual_seed(seed)
    gamma = (torch.rand(cols, generator=g) + 0.1).to(device)
    x = torch.randn(64, cols, generator=g)
    h = torch.einsum("nbi,nbj->bij", x.view(64, -1, 32), x.view(64, -1, 32)) / 64 + 1e-3 * torch.eye(32)
    return w, gamma, h.to(device)


def _with_workspace(lib, w, *, recon=None, packed=None, scales=None, gamma=None, hessian=None) -> torch.Tensor:
    rows, cols = w.shape
    need = lib.mxw_error_sums_workspace_size(rows, cols)
    ws = torch.zeros(need, dtype=torch.uint8, device=w.device)
    sums = torch.empty(4, dtype=torch.float64, device=w.device)
    st = lib.mxw_error_sums(
        w.data_ptr(), _lib.MXW_BF16, rows, cols, cols,
        None if recon is None else recon.data_ptr(), _lib.MXW_F32, cols,
        None if packed is None else packed.data_ptr(), None if scales is None else scales.data_ptr(),
        None if gamma is None else gamma.data_ptr(), None if hessian is None else hessian.data_ptr(),
        sums.data_ptr(), ws.data_ptr(), need, torch.cuda.current_stream().cuda_stream,
    )
    assert st == _lib.MXW_OK
    return sums


def _no_alloc(lib, w, *, recon=None, packed=None, scales=None, gamma=None, hessian=None) -> torch.Tensor:
    rows, cols = w.shape
    sums = torch.empty(4, dtype=torch.float64, device=w.device)
    st = lib.mxw_error_sums_noalloc(
        w.data_ptr(), _lib.MXW_BF16, rows, cols, cols,
        None if recon is None else recon.data_ptr(), _lib.MXW_F32, cols,
        None if packed is None else packed.data_ptr(), None if scales is None else scales.data_ptr(),
        None if gamma is None else gamma.data_ptr(), None if hessian is None else hessian.data_ptr(),
        sums.data_ptr(), torch.cuda.current_stream().cuda_stream,
    )
    assert st == _lib.MXW_OK, lib.mxw_status_string(st)
    return sums


def test_no_alloc_entry_point_matches_the_workspace_one_on_consecutive_calls(cuda_device) -> None:
    lib = _lib.load()
    w1, gamma1, _ = _inputs(512, 5120, 31, cuda_device)
    p1, s1 = quantize_mxfp4(w1, gamma=gamma1)
    w2, _, h2 = _inputs(96, 2048, 32, cuda_device)
    p2, s2 = quantize_mxfp4(w2, hessian=h2)
    recon2 = dequant_mxfp4(p2, s2, (96, 2048))

    # Call 1: packed input, gamma weighting.
    want1 = _with_workspace(lib, w1, packed=p1, scales=s1, gamma=gamma1)
    got1 = _no_alloc(lib, w1, packed=p1, scales=s1, gamma=gamma1)
    # Call 2, right after: another shape, a dense reconstruction, Hessian weighting.
    want2 = _with_workspace(lib, w2, recon=recon2, hessian=h2)
    got2 = _no_alloc(lib, w2, recon=recon2, hessian=h2)
    # Call 3: call 1 again -- the shared array keeps the last call's contents.
    got3 = _no_alloc(lib, w1, packed=p1, scales=s1, gamma=gamma1)
    torch.cuda.synchronize()

    for got, want in ((got1, want1), (got2, want2), (got3, want1)):
        torch.testing.assert_close(got, want, rtol=RTOL, atol=0.0)
    # And the same values as the float64 oracle, in the units the SQNR tests use.
    ref = oracle.error_sums(w2.float().cpu().numpy(), recon2.cpu().numpy(), hessian=h2.cpu().numpy())
    got = got2.cpu().tolist()
    assert abs(oracle.sqnr_db(got[0], got[1]) - oracle.sqnr_db(ref[0], ref[1])) < DB_TOL
    assert abs(oracle.sqnr_db(got[2], got[3]) - oracle.sqnr_db(ref[2], ref[3])) < DB_TOL


def test_no_alloc_entry_point_rejects_bad_arguments(cuda_device) -> None:
    lib = _lib.load()
    sums = torch.empty(4, dtype=torch.float64, device=cuda_device)
    w = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda_device)
    # neither a reconstruction nor packed bytes
    st = lib.mxw_error_sums_noalloc(w.data_ptr(), _lib.MXW_BF16, 4, 64, 64, None, 0, 0, None, None, None, None,
                                    sums.data_ptr(), None)
    assert st == _lib.MXW_EINVAL
    st = lib.mxw_error_sums_noalloc(w.data_ptr(), _lib.MXW_BF16, -1, 64, 64, w.data_ptr(), _lib.MXW_BF16, 64,
                                    None, None, None, None, sums.data_ptr(), None)
    assert st == _lib.MXW_EINVAL
