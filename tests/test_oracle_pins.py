"""The CPU oracle pinned against the reference itself (no GPU needed).

Golden vectors in tests/golden/reference_cpu.npz were produced by the UNMODIFIED reference GSX
library's CPU backend (tests/golden/make_golden.py).  SSIM, L1, MSE and Adam are tight pins; the
reference CPU renderer follows different culling rules from the CUDA renderer the oracle restates
(3-sigma box with a power cut vs the opacity-aware extent, no Jacobian frustum clamp), so the
render pin is the 1-pixel known answer (exact) plus a loose whole-image comparison.
"""
import math
import os

import numpy as np
import pytest

from gsx_b200 import scenes
from oracle import pyoracle as po

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_cpu.npz"))


def _ulp_diff(a, b):
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


def test_ssim_reference_test_inputs():
    """tests/cuda_loss_runtime.cpp:388-391 inputs: every pixel is in the 5-px border -> all zero."""
    lm, g = po.ssim(GOLD["ssim_a_pred"], GOLD["ssim_a_target"], 0.7, np.float32(0.7) / np.float32(180))
    np.testing.assert_array_equal(lm, GOLD["ssim_a_loss"])
    np.testing.assert_allclose(g, GOLD["ssim_a_grad"], atol=1e-9)


def test_ssim_interior_matches_reference_cpu():
    p, t = GOLD["ssim_b_pred"], GOLD["ssim_b_target"]
    lm, g = po.ssim(p, t, 0.2, np.float32(0.2) / np.float32(p.size))
    np.testing.assert_allclose(lm, GOLD["ssim_b_loss"], rtol=0, atol=2e-7)
    np.testing.assert_allclose(g, GOLD["ssim_b_grad"], rtol=1e-5, atol=1e-10)


def test_pointwise_losses_match_reference_cpu():
    p, t = GOLD["ssim_b_pred"], GOLD["ssim_b_target"]
    n = p.size
    d = (p - t).astype(np.float32)
    np.testing.assert_array_equal(np.float32(0.8) * np.abs(d), GOLD["l1_loss"])
    np.testing.assert_array_equal(np.sign(d) * (np.float32(0.8) / np.float32(n)), GOLD["l1_grad"])
    np.testing.assert_allclose(np.float32(0.8) * d * d, GOLD["mse_loss"], rtol=1e-6)


@pytest.mark.parametrize("key,wd,mg", [("adam_plain", 0.0, 0.0), ("adam_wd_clamp", 0.01, 5e-4)])
def test_adam_bit_exact_vs_reference_cpu(key, wd, mg):
    x = GOLD["adam_x"].copy()
    m1 = np.zeros_like(x)
    m2 = np.zeros_like(x)
    for step in range(1, 6):
        po.adam(x, GOLD["adam_g"], m1, m2, step, 1e-2, weight_decay=wd, max_grad=mg)
    np.testing.assert_array_equal(x, GOLD[key])


def test_render_one_pixel_known_answer():
    g = dict(mean3d=np.array([[0, 0, 4]], np.float32), rotation=np.array([[0, 0, 0, 1]], np.float32),
             logscale=np.zeros((1, 3), np.float32), opacity=np.zeros(1, np.float32),
             sh0=np.array([[1, 0, 0]], np.float32))
    f = po.render_forward(g, po.Camera(1, 1, 1.0, 1.0, 0.5, 0.5, near=0.1, far=10.0))
    np.testing.assert_allclose(f["rgb"].ravel(), [0.3910474, 0.25, 0.25], atol=1e-5)
    np.testing.assert_allclose(f["rgb"], GOLD["render_1px"], atol=1e-7)


def test_render_close_to_reference_cpu_renderer():
    g, cam = scenes.small_scene(0, 2000, 96, 80)
    oc = po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl,
                   cam.near_plane, cam.far_plane)
    f = po.render_forward(g, oc)
    d = np.abs(f["rgb"] - GOLD["render_small_cpu"])
    assert d.max() < 2e-2 and d.mean() < 2e-3


def test_detmath_exp_log_within_two_ulp():
    xs = np.concatenate([np.linspace(-87.0, 88.0, 200001, dtype=np.float32),
                         -np.logspace(-8, 1, 20001).astype(np.float32)])
    L = po.lib()
    import ctypes
    # the oracle shares the product's deterministic exp/log; check them through the oracle's sigmoid-free path
    got = np.array([_exp(L, float(x)) for x in xs[::37]], np.float32)
    exp = np.exp(xs[::37].astype(np.float64)).astype(np.float32)
    assert _ulp_diff(got, exp).max() <= 2
    ys = np.logspace(-30, 30, 40001).astype(np.float32)
    got = np.array([_log(L, float(y)) for y in ys[::13]], np.float32)
    exp = np.log(ys[::13].astype(np.float64)).astype(np.float32)
    assert _ulp_diff(got, exp).max() <= 2


def _exp(L, x):
    import ctypes
    f = L.orc_expf
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_float]
    return f(x)


def _log(L, x):
    import ctypes
    f = L.orc_logf
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_float]
    return f(x)


def test_oracle_sort_is_stable():
    rng = np.random.default_rng(0)
    k = rng.integers(0, 50, 10000).astype(np.uint64)
    v = np.arange(10000, dtype=np.uint32)
    sk, sv = po.sort_pairs(k, v)
    order = np.argsort(k, kind="stable")
    np.testing.assert_array_equal(sk, k[order])
    np.testing.assert_array_equal(sv, v[order])
    assert not math.isnan(float(sk[0]))


def test_pack_hwc_to_chw_pinned_to_reference_test():
    """Known answer of the reference's DataRuntime.NextExProducesFixedCHWOutputAndPreservesMetadata
    (tests/data_runtime.cpp:386-428): a 2x2 u8 RGB sample with alpha, packed to f32 CHW."""
    rgb = np.array([0, 10, 20, 40, 50, 60, 80, 90, 100, 120, 130, 140], np.uint8).reshape(2, 2, 3)
    alpha = np.array([10, 30, 50, 70], np.uint8).reshape(2, 2)
    np.testing.assert_array_equal(po.pack_hwc_to_chw(rgb).ravel(),
                                  np.array([0, 40, 80, 120, 10, 50, 90, 130, 20, 60, 100, 140], np.float32))
    np.testing.assert_array_equal(po.pack_hwc_to_chw(alpha).ravel(), np.array([10, 30, 50, 70], np.float32))
