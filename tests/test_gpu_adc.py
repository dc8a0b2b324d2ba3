"""Density control on the B200 (gsx_b200_provider's default ADC over libgsx_b200's gsx_b200_adc_*,
gather and clamp kernels), through GSX's public API, vs the oracle and vs the reference CUDA backend;
plus the structural kernels through the C ABI.

Bars: counts and row order exact; rows that no split offset touched bit-identical; split rows
(hashed offsets through CUDA's expf/logf and the rotation) within 1e-5 relative; optimizer moments
carried with the rows (checked through one more Adam step) within 1e-5 relative.
"""
import ctypes

import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200._capi import GsxError, check, lib
from oracle import pyoracle as po
from tests.test_adc_oracle import CASES, FIELDS, _state

pytestmark = pytest.mark.gpu


def _need(kind):
    if not po.ref_available(kind):
        pytest.skip(f"GSX library for '{kind}' not built")


def _close(a, b, what):
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6, err_msg=what)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"s{c['seed']}_n{c['n']}_step{c['ip'][6]}")
def test_adc_matches_oracle(case):
    _need("b200")
    g, aux, zeros = _state(case["seed"], case["n"])
    res, g2, a2, origin, split_rows = po.adc_step(g, aux, case["fp"], case["ip"])
    r, fa, ff, fx = po.ref_adc_run("b200", g, aux, zeros, case["fp"], case["ip"])
    assert r == res
    plain = np.setdiff1d(np.arange(res["after"]), split_rows)
    for k in FIELDS:
        np.testing.assert_array_equal(fa[k][plain], g2[k][plain], err_msg=k)
        _close(fa[k][split_rows], g2[k][split_rows], k)
    for k in ("grad_acc", "visible_counter", "max_screen_radius"):
        np.testing.assert_array_equal(fx[k], a2[k], err_msg=k)


@pytest.mark.parametrize("case", CASES[:4], ids=lambda c: f"s{c['seed']}_n{c['n']}_step{c['ip'][6]}")
def test_adc_matches_reference_cuda_backend(case):
    """The same public-API sequence (Adam step, ADC step, Adam step) on the reference CUDA backend
    and on gsx-b200: identical decisions and rows, the optimizer moments moved with the rows."""
    _need("b200")
    _need("cuda")
    g, aux, _ = _state(case["seed"], case["n"])
    rng = np.random.default_rng(100 + case["seed"])
    grads = {k: rng.normal(0, 0.1, v.shape).astype(np.float32) for k, v in g.items()}
    r_ref, fa_ref, ff_ref, fx_ref = po.ref_adc_run("cuda", g, aux, grads, case["fp"], case["ip"])
    r, fa, ff, fx = po.ref_adc_run("b200", g, aux, grads, case["fp"], case["ip"])
    assert r == r_ref
    for k in FIELDS:
        _close(fa[k], fa_ref[k], k)
        _close(ff[k], ff_ref[k], k)
    for k in fx:
        np.testing.assert_array_equal(fx[k], fx_ref[k], err_msg=k)


def _dptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("row_bytes,offset", [(48, 0), (12, 0), (16, 0), (7, 0), (12, 4), (48, 16)])
def test_gather_rows(cuda_device, row_bytes, offset):
    rng = np.random.default_rng(row_bytes + offset)
    src_rows, out_rows = 1000, 1500
    src = torch.from_numpy(rng.integers(0, 256, src_rows * row_bytes + 64, dtype=np.uint8)).cuda()
    idx = rng.integers(0, src_rows, out_rows).astype(np.int32)
    dst = torch.zeros(out_rows * row_bytes + 64, dtype=torch.uint8, device="cuda:0")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    s = src[offset:offset + src_rows * row_bytes]
    d = dst[offset:offset + out_rows * row_bytes]
    check(lib().gsx_b200_gather_rows(_dptr(s), src_rows, row_bytes, _dptr(torch.from_numpy(idx).cuda()), out_rows, _dptr(d),
                                     _dptr(flag), None))
    torch.cuda.synchronize()
    exp = s.cpu().numpy().reshape(src_rows, row_bytes)[idx]
    np.testing.assert_array_equal(d.cpu().numpy().reshape(out_rows, row_bytes), exp)
    assert int(flag.item()) == 0


def test_gather_rows_out_of_range_flags_and_skips(cuda_device):
    src = torch.arange(40, dtype=torch.float32, device="cuda:0")
    idx = torch.tensor([0, 9, 10, -1, 3], dtype=torch.int32, device="cuda:0")
    dst = torch.full((5 * 4,), -7.0, device="cuda:0")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    check(lib().gsx_b200_gather_rows(_dptr(src), 10, 16, _dptr(idx), 5, _dptr(dst), _dptr(flag), None))
    torch.cuda.synchronize()
    out = dst.view(5, 4).cpu().numpy()
    assert int(flag.item()) == 1
    np.testing.assert_array_equal(out[0], [0, 1, 2, 3])
    np.testing.assert_array_equal(out[1], [36, 37, 38, 39])
    np.testing.assert_array_equal(out[2], [-7] * 4)
    np.testing.assert_array_equal(out[3], [-7] * 4)
    np.testing.assert_array_equal(out[4], [12, 13, 14, 15])


def test_clamp_inplace(cuda_device):
    x = torch.tensor([-5.0, -1.0, 0.5, 2.0, float("nan"), float("inf")], device="cuda:0")
    lo, hi = ctypes.c_float(-1.0), ctypes.c_float(1.0)
    check(lib().gsx_b200_clamp_inplace(_dptr(x), 0, 6, ctypes.byref(lo), ctypes.byref(hi), None))
    y = torch.tensor([-5, 0, 9], dtype=torch.int32, device="cuda:0")
    li, hi_ = ctypes.c_int32(-1), ctypes.c_int32(3)
    check(lib().gsx_b200_clamp_inplace(_dptr(y), 12, 3, ctypes.byref(li), ctypes.byref(hi_), None))
    torch.cuda.synchronize()
    xs = x.cpu().numpy()
    np.testing.assert_array_equal(xs[[0, 1, 2, 3, 5]], [-1, -1, 0.5, 1, 1])
    assert np.isnan(xs[4])
    assert y.cpu().tolist() == [-1, 0, 3]
    with pytest.raises(GsxError):
        check(lib().gsx_b200_clamp_inplace(_dptr(x), 1, 6, ctypes.byref(lo), ctypes.byref(hi), None))
