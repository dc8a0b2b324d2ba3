"""Density-control statistics (gs_visible_counter, gs_max_screen_radius, gs_grad_acc, gs_absgrad_acc)
on the B200 vs the oracle, through the C ABI and through GSX's public API (the provider).

The reference's CUDA backend fills none of them; the semantics followed are its Metal backend's
(gsx-metal/kernels/render.metal:425-439, render_backward.metal:700-714), restated in the oracle
(orc_preprocess_aux, orc_blend_backward_abs, pyoracle.aux_forward/aux_backward).  Bars: the
forward statistics bit-exact (same arithmetic contract as the preprocess); the backward ones
rel-L2 <= 1e-3 (atomic accumulation order).
"""
import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200 import scenes
from oracle import pyoracle as po
from tests.gpu_helpers import rel_l2, render, to_dev, zeros_like_fields

pytestmark = pytest.mark.gpu


def _ocam(cam):
    return po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl, cam.near_plane,
                     cam.far_plane)


@pytest.fixture(scope="module")
def ctx(cuda_device):
    c = gb.RenderContext(0)
    yield c
    c.close()


@pytest.mark.parametrize("seed,n,w,h,sh", [(0, 3000, 96, 80, 0), (1, 4000, 120, 77, 2), (2, 20000, 200, 150, 0)])
def test_aux_statistics_match_oracle(ctx, seed, n, w, h, sh):
    g, cam = scenes.small_scene(seed, n, w, h, sh, scale_mu=-2.8)
    oc = _ocam(cam)
    rng = np.random.default_rng(50 + seed)
    start = [rng.integers(0, 4, n).astype(np.float32), rng.uniform(0, 6, n).astype(np.float32),
             rng.uniform(0, 1, n).astype(np.float32), rng.uniform(0, 1, n).astype(np.float32)]
    exp = [a.copy() for a in start]
    dev = [torch.from_numpy(a.copy()).cuda() for a in start]
    gd = to_dev(g)
    ctx.bind_aux(*dev)
    renderer = gb.Renderer(cam.width, cam.height)
    for view in range(2):  # two TRAIN forward+backward rounds accumulate
        grad_rgb = rng.normal(0, 1, (3, cam.height, cam.width)).astype(np.float32)
        f = po.render_forward(g, oc, sh)
        b = po.render_backward(g, oc, f, grad_rgb, sh)
        po.aux_forward(f, exp[0], exp[1])
        po.aux_backward(b, oc, exp[2], exp[3])
        render(ctx, gd, cam, sh)
        renderer.backward(ctx, torch.from_numpy(grad_rgb).cuda(), zeros_like_fields(gd))
        ctx.check()
    got = [t.cpu().numpy() for t in dev]
    np.testing.assert_array_equal(got[0], exp[0])
    np.testing.assert_array_equal(got[1], exp[1])
    assert rel_l2(got[2] - start[2], exp[2] - start[2]) <= 1e-3
    assert rel_l2(got[3] - start[3], exp[3] - start[3]) <= 1e-3
    # absolute per-pixel gradients dominate the signed sum
    assert np.all(got[3] - start[3] >= (got[2] - start[2]) - 1e-4 * (1 + np.abs(got[2])))
    ctx.bind_aux()


def test_inference_and_unbound_leave_statistics_alone(ctx):
    g, cam = scenes.small_scene(3, 2000, 80, 64, 0)
    gd = to_dev(g)
    dev = [torch.full((2000,), 7.0, device="cuda:0") for _ in range(4)]
    ctx.bind_aux(*dev)
    render(ctx, gd, cam, 0, train=False)
    ctx.check()
    for t in dev[:2]:
        assert float((t - 7.0).abs().max()) == 0.0
    ctx.bind_aux()
    render(ctx, gd, cam, 0, train=True)
    gb.Renderer(cam.width, cam.height).backward(ctx, torch.ones((3, cam.height, cam.width), device="cuda:0"),
                                                zeros_like_fields(gd))
    ctx.check()
    for t in dev:
        assert float((t - 7.0).abs().max()) == 0.0


def test_absgrad_variant_leaves_gradients_unchanged(ctx):
    """Binding absgrad_acc selects another backward kernel; the parameter gradients stay within the
    atomic-order tolerance of the plain kernel's."""
    g, cam = scenes.small_scene(4, 3000, 96, 80, 1)
    gd = to_dev(g)
    grad_rgb = torch.from_numpy(np.random.default_rng(3).normal(0, 1, (3, 80, 96)).astype(np.float32)).cuda()
    r = gb.Renderer(cam.width, cam.height)
    out = []
    for bind in (False, True):
        ctx.bind_aux(absgrad_acc=torch.zeros(3000, device="cuda:0") if bind else None)
        render(ctx, gd, cam, 1)
        gr = zeros_like_fields(gd)
        r.backward(ctx, grad_rgb, gr)
        ctx.check()
        out.append({k: v.cpu().numpy() for k, v in gr.items()})
    ctx.bind_aux()
    for k in out[0]:
        assert rel_l2(out[1][k], out[0][k]) <= 1e-5, k


def test_public_api_aux_statistics():
    """GSX's gs_visible_counter / gs_max_screen_radius / gs_grad_acc / gs_absgrad_acc request fields
    through the provider."""
    if not po.ref_available("b200"):
        pytest.skip("GSX library for 'b200' not built")
    g, cam = scenes.small_scene(6, 3000, 96, 80, 0, scale_mu=-2.8)
    oc = _ocam(cam)
    grad_rgb = np.random.default_rng(11).normal(0, 1, (3, cam.height, cam.width)).astype(np.float32)
    sess = po.RefSession("b200", g, oc, np.zeros((3, cam.height, cam.width), np.float32))
    sess.enable_aux(True)
    sess.render_backward(grad_rgb)
    got = sess.aux()
    n = 3000
    exp = [np.zeros(n, np.float32) for _ in range(4)]
    f = po.render_forward(g, oc)
    b = po.render_backward(g, oc, f, grad_rgb)
    po.aux_forward(f, exp[0], exp[1])
    po.aux_backward(b, oc, exp[2], exp[3])
    np.testing.assert_array_equal(got[0], exp[0])
    np.testing.assert_array_equal(got[1], exp[1])
    assert rel_l2(got[2], exp[2]) <= 1e-3
    assert rel_l2(got[3], exp[3]) <= 1e-3
