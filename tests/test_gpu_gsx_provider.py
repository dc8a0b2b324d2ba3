"""The drop-in: GSX's own public C API, core and front-ends (built from the reference sources),
with the gsx_b200 GSX provider (gsx_b200/provider/) as its CUDA backend.

oracle/Makefile.ref (target b200) links the reference core (compiled with GSX_HAS_CUDA=1) with the
provider and libgsx_b200.so instead of the reference's gsx-cuda sources; oracle/ref_driver.c drives
it through gsx_renderer_render / gsx_renderer_backward / gsx_loss_* / gsx_optim_step exactly as it
drives the reference CPU and CUDA backends.  The same bars as the direct C-ABI tests apply: RGB
bit-identical to the oracle, gradients rel-L2 <= 1e-3, losses as the reference CPU backend, Adam
bit-exact.
"""
import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200 import scenes
from oracle import pyoracle as po
from tests.gpu_helpers import rel_l2, render, to_dev, zeros_like_fields

pytestmark = pytest.mark.gpu


def _need(kind="b200"):
    if not po.ref_available(kind):
        pytest.skip(f"GSX library for '{kind}' not built (oracle/_ref/libgsx_refdrv_{kind}.so)")


def _ocam(cam):
    return po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl, cam.near_plane,
                     cam.far_plane)


CASES = [
    dict(seed=0, n=2000, width=96, height=80, sh=0),
    dict(seed=1, n=3000, width=77, height=53, sh=1),
    dict(seed=3, n=2500, width=65, height=33, sh=3),
    dict(seed=5, n=20000, width=200, height=150, sh=0, scale_mu=-3.5),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"s{c['seed']}_{c['width']}x{c['height']}_sh{c['sh']}")
def test_public_api_render_and_backward(case):
    _need()
    g, cam = scenes.small_scene(case["seed"], case["n"], case["width"], case["height"], case["sh"],
                                scale_mu=case.get("scale_mu", -3.0))
    oc = _ocam(cam)
    grad_rgb = np.random.default_rng(9 + case["seed"]).normal(0, 1, (3, cam.height, cam.width)).astype(np.float32)
    sess = po.RefSession("b200", g, oc, np.zeros((3, cam.height, cam.width), np.float32), sh_degree=case["sh"])
    rgb, grads = sess.render_backward(grad_rgb)
    f = po.render_forward(g, oc, case["sh"])
    b = po.render_backward(g, oc, f, grad_rgb, case["sh"])
    assert np.array_equal(rgb, f["rgb"]), f"max-abs {np.abs(rgb - f['rgb']).max():.3e}"
    for k, v in grads.items():
        assert rel_l2(v, b[k]) <= 1e-3, k


def test_public_api_matches_direct_c_abi(cuda_device):
    """The provider adds no arithmetic of its own: the same kernels as the direct C-ABI path."""
    _need()
    g, cam = scenes.small_scene(2, 4000, 120, 90, 2)
    grad_rgb = np.random.default_rng(3).normal(0, 1, (3, 90, 120)).astype(np.float32)
    sess = po.RefSession("b200", g, _ocam(cam), np.zeros((3, 90, 120), np.float32), sh_degree=2)
    rgb, grads = sess.render_backward(grad_rgb)
    ctx = gb.RenderContext(0)
    gd = to_dev(g)
    out = render(ctx, gd, cam, 2)
    dg = zeros_like_fields(gd)
    gb.Renderer(120, 90).backward(ctx, torch.from_numpy(grad_rgb).cuda(), dg)
    ctx.check()
    np.testing.assert_array_equal(rgb, out.cpu().numpy())
    for k, v in grads.items():
        assert rel_l2(v, dg[k].cpu().numpy().ravel()) <= 1e-5, k
    ctx.close()


@pytest.mark.parametrize("algorithm,name", [(0, "l1"), (1, "mse"), (2, "ssim")])
@pytest.mark.parametrize("normalization", [0, 1], ids=["mean", "sum"])
def test_public_api_losses_match_reference_cpu(algorithm, name, normalization):
    """gsx_loss_forward / gsx_loss_backward through the provider vs the reference CPU backend,
    with accumulation into non-zero loss maps and gradients."""
    _need()
    _need("cpu")
    rng = np.random.default_rng(40 + algorithm)
    pred = rng.uniform(0, 1, (2, 3, 37, 45)).astype(np.float32)
    target = rng.uniform(0, 1, (2, 3, 37, 45)).astype(np.float32)
    lm0 = rng.normal(0, 0.1, pred.shape).astype(np.float32)
    g0 = rng.normal(0, 0.1, pred.shape).astype(np.float32)
    lm, gr = po.ref_loss("b200", algorithm, pred, target, 0.7, normalization, lm0, g0)
    elm, egr = po.ref_loss("cpu", algorithm, pred, target, 0.7, normalization, lm0, g0)
    assert np.abs(lm - elm).max() <= 2e-5, name
    assert rel_l2(gr - g0, egr - g0) <= 1e-4, name


def test_public_api_adam_bit_exact_vs_reference_cpu():
    _need()
    _need("cpu")
    rng = np.random.default_rng(8)
    p = rng.normal(0, 1, 10007).astype(np.float32)
    g = rng.normal(0, 1e-2, 10007).astype(np.float32)
    for kw in (dict(), dict(weight_decay=0.01, max_grad=0.005)):
        got = po.ref_adam("b200", p, g, 5, 1e-2, **kw)
        exp = po.ref_adam("cpu", p, g, 5, 1e-2, **kw)
        np.testing.assert_array_equal(got, exp)


def test_public_api_training_step_matches_oracle_step():
    """One GSX training step through the public API on the provider (render TRAIN, L1 and SSIM
    forward/backward with weights 0.8/0.2, render backward, Adam on every role), against the same
    step restated on the oracle.  The loss map and image gradient must match the oracle's; Adam's
    first step moves an element by about lr times the sign of its gradient, so an element whose
    gradient is at rounding level may flip: the updates must agree as a whole and nearly everywhere."""
    _need()
    g, cam = scenes.small_scene(4, 3000, 80, 64, 0)
    oc = _ocam(cam)
    target = np.random.default_rng(2).uniform(0, 1, (3, 64, 80)).astype(np.float32)
    sess = po.RefSession("b200", g, oc, target)
    sess.step()
    P = 3 * 64 * 80
    f = po.render_forward(g, oc)
    lm, grad = po.l1_ssim_train(f["rgb"], target, 0.8, 0.2)
    assert np.abs(sess.download(9, P) - lm.ravel()).max() <= 1e-5
    assert rel_l2(sess.download(10, P), grad.ravel()) <= 1e-4
    b = po.render_backward(g, oc, f, grad)
    fields = ("mean3d", "logscale", "rotation", "opacity", "sh0")
    lrs = (1e-3, 1e-2, 1e-2, 1e-2, 1e-2)
    for i, (k, lr) in enumerate(zip(fields, lrs)):
        p = g[k].ravel().astype(np.float32).copy()
        p0 = p.copy()
        m1, m2 = np.zeros_like(p), np.zeros_like(p)
        po.adam(p, b[k].ravel(), m1, m2, 1, lr)
        got = sess.download(i, p.size)
        du, do = got - p0, p - p0
        assert rel_l2(du, do) <= 1e-3, k
        assert (np.abs(du - do) > lr).mean() <= 1e-3, k


def test_public_api_training_step_at_config3():
    """The drop-in at the benchmarked size: GSX's own training step (gsx-runtime.c:1413-1536 order: zero
    grads, render TRAIN, L1 and SSIM forward and backward, render backward, Adam on every role) through the
    public API on the provider, config 3 (3M Gaussians, 1245x825, teacher target).  Checks the loss map
    against the fused direct path's on the same render, and prints the step's wall time (the driver syncs
    the backend's stream at the end of each step) for the integration notes."""
    _need()
    import time
    g = scenes.config3_scene(0)
    cam = scenes.config3_cameras()[0]
    oc = _ocam(cam)
    ctx = gb.RenderContext(0)
    target = render(ctx, to_dev(scenes.teacher(g)), cam, train=False)
    ctx.check()
    sess = po.RefSession("b200", g, oc, target.cpu().numpy())
    sess.step()
    P = 3 * cam.width * cam.height
    lm_api = sess.download(9, P)
    # the same step's loss map on the direct path (fused L1 + SSIM on the same render)
    out = render(ctx, to_dev(g), cam, train=True)
    lm = torch.zeros_like(out)
    grad = torch.zeros_like(out)
    gb.l1_ssim(out, target, lm, grad, 0.8, 0.2)
    torch.cuda.synchronize()
    assert np.abs(lm.cpu().numpy().ravel() - lm_api).max() <= 1e-4
    secs = [sess.step() for _ in range(10)]
    print(f"\nGSX public-API training step at config 3 on the provider: median {1e3 * sorted(secs)[5]:.3f} ms "
          f"(min {1e3 * min(secs):.3f} ms) over 10 steps")
    ctx.close()
