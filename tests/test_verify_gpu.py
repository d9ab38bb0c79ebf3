"""GPU: the fused error-sum kernel behind the SQNR family, against the
float64 oracle, the reference's own functions, and the dequantized path."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mxwave_b200 import _lib, synthetic as syn
from mxwave_b200.core import dequant_mxfp4, quantize_mxfp4
from mxwave_b200.verify import block_hessian_weighted_sqnr, channel_weighted_sqnr, sqnr, sqnr_packed
from oracle import oracle
from tests.reference_pkg import import_reference

pytestmark = pytest.mark.gpu

DB_TOL = 1e-4  # dB: the reference sums in fp32 (about 1e-6 relative), the kernel in fp64


def _inputs(rows: int, cols: int, seed: int, device):
    bits = syn.det_dense_weight(rows, cols, seed, outlier_fraction=0.01)
    w = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)
    g = torch.Generator().manual_seed(seed)
    gamma = (torch.rand(cols, generator=g) + 0.1).to(device)
    x = torch.randn(128, cols, generator=g)
    h = (torch.einsum("nbi,nbj->bij", x.view(128, -1, 32), x.view(128, -1, 32)) / 128 + 1e-3 * torch.eye(32)).to(device)
    return w, gamma, h


@pytest.mark.parametrize("rows,cols", [(16, 5120), (16, 17408), (300, 2048), (1, 32), (1000, 96)])
def test_sqnr_family_matches_oracle_and_reference(rows, cols, cuda_device) -> None:
    ver = import_reference("mxwave.verify")
    w, gamma, h = _inputs(rows, cols, rows * 7 + cols, cuda_device)
    p, s = quantize_mxfp4(w)
    recon = dequant_mxfp4(p, s, (rows, cols))
    on, rn = w.float().cpu().numpy(), recon.cpu().numpy()
    want = oracle.error_sums(on, rn)
    assert abs(sqnr(w, recon) - oracle.sqnr_db(want[0], want[1])) < DB_TOL
    assert abs(sqnr(w, recon) - ver.sqnr(w.cpu(), recon.cpu())) < DB_TOL
    want_g = oracle.error_sums(on, rn, gamma=gamma.cpu().numpy())
    got_g = channel_weighted_sqnr(w, recon, gamma)
    assert abs(got_g - oracle.sqnr_db(want_g[2], want_g[3])) < DB_TOL
    assert abs(got_g - ver.channel_weighted_sqnr(w.cpu(), recon.cpu(), gamma.cpu())) < DB_TOL
    want_h = oracle.error_sums(on, rn, hessian=h.cpu().numpy())
    got_h = block_hessian_weighted_sqnr(w, recon, h)
    assert abs(got_h - oracle.sqnr_db(want_h[2], want_h[3])) < DB_TOL
    assert abs(got_h - ver.block_hessian_weighted_sqnr(w.cpu(), recon.cpu(), h.cpu())) < DB_TOL


def test_packed_path_equals_the_dequantized_path_bit_for_bit(cuda_device) -> None:
    w, gamma, h = _inputs(64, 5120, 3, cuda_device)
    p, s = quantize_mxfp4(w, gamma=gamma)
    recon = dequant_mxfp4(p, s, (64, 5120))
    plain, weighted = sqnr_packed(w, p, s, gamma=gamma)
    assert plain == sqnr(w, recon)
    assert weighted == channel_weighted_sqnr(w, recon, gamma)
    plain_h, weighted_h = sqnr_packed(w, p, s, hessian=h)
    assert plain_h == plain and weighted_h == block_hessian_weighted_sqnr(w, recon, h)
    assert sqnr_packed(w, p, s) == (plain, None)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_other_dtypes_and_ragged_widths(dtype, cuda_device) -> None:
    g = torch.Generator().manual_seed(5)
    o = torch.randn(7, 77, generator=g).to(dtype).to(cuda_device)
    r = (o.float() + 1e-2 * torch.randn(7, 77, generator=g).to(cuda_device)).to(dtype)
    want = oracle.error_sums(o.float().cpu().numpy(), r.float().cpu().numpy())
    assert abs(sqnr(o, r) - oracle.sqnr_db(want[0], want[1])) < DB_TOL
    # any shape with the same number of elements, as the reference flattens
    assert abs(sqnr(o.reshape(-1), r.reshape(7, 77)) - sqnr(o, r)) < 1e-9


def test_repeatable_bits_and_zero_noise(cuda_device) -> None:
    w, gamma, _ = _inputs(256, 4096, 9, cuda_device)
    p, s = quantize_mxfp4(w)
    first = sqnr_packed(w, p, s, gamma=gamma)
    for _ in range(3):
        assert sqnr_packed(w, p, s, gamma=gamma) == first
    ver = import_reference("mxwave.verify")
    assert sqnr(w, w.float()) == pytest.approx(ver.sqnr(w.cpu(), w.cpu().float()), abs=DB_TOL)


def test_validation_messages_match_the_reference(cuda_device) -> None:
    ver = import_reference("mxwave.verify")
    o = torch.zeros(2, 64, device=cuda_device)
    for fn, ref_fn, args in (
        (block_hessian_weighted_sqnr, ver.block_hessian_weighted_sqnr, (o, o[:, :32], torch.zeros(2, 32, 32))),
        (block_hessian_weighted_sqnr, ver.block_hessian_weighted_sqnr, (o, o, torch.zeros(3, 32, 32))),
        (channel_weighted_sqnr, ver.channel_weighted_sqnr, (o, o[:1], torch.ones(64))),
        (channel_weighted_sqnr, ver.channel_weighted_sqnr, (o, o, torch.ones(63))),
    ):
        with pytest.raises(ValueError) as ref_exc:
            ref_fn(*[a.cpu() for a in args])
        with pytest.raises(ValueError, match=str(ref_exc.value).replace("(", r"\(").replace(")", r"\)")):
            fn(*args)


def test_c_abi_rejects_bad_workspace(cuda_device) -> None:
    lib = _lib.load()
    o = torch.zeros(4, 64, device=cuda_device)
    sums = torch.empty(4, dtype=torch.float64, device=cuda_device)
    need = lib.mxw_error_sums_workspace_size(4, 64)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    st = lib.mxw_error_sums(o.data_ptr(), _lib.MXW_F32, 4, 64, 64, o.data_ptr(), _lib.MXW_F32, 64, None, None,
                            None, None, sums.data_ptr(), ws.data_ptr(), need - 1, None)
    assert st == _lib.MXW_EINVAL
    st = lib.mxw_error_sums(o.data_ptr(), _lib.MXW_F32, 4, 64, 64, o.data_ptr(), _lib.MXW_F32, 64, None, None,
                            None, None, sums.data_ptr(), ws.data_ptr(), need, None)
    assert st == _lib.MXW_OK
    torch.cuda.synchronize()
    assert sums.tolist() == [0.0, 0.0, 0.0, 0.0]
    assert int(ws[:16].sum()) == 0  # the ticket is left at zero
