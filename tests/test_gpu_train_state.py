"""TRAIN-state contract between a forward and its backward when the caller changes the Gaussians in between.

The reference keeps either a cloned copy of the inputs (borrow_train_state = false) or borrows them
and re-renders at backward (borrow_train_state = true), gsx-cuda/render.c:481-756.  Its tests:
- BackwardUsesRetainedTrainState (tests/cuda_render_runtime.cpp:601-639): cloned state, inputs
  overwritten after the forward, the backward still gives the gradients of the original inputs (1e-5);
- BackwardBorrowedTrainStateTracksInputMutations (:641-689): borrowed state, the same mutation, the
  gradients differ from the original ones.
Both are ported through GSX's public API on the gsx_b200 provider, with a stronger check for the borrowed
case: the gradients equal a fresh TRAIN forward + backward of the mutated inputs (oracle, rel-L2 1e-3).
The direct C-ABI mode (gsx_b200_context_set_train_state) is checked for the refresh count, for the
unchanged-input path (no refresh, the retained result) and for the caller's image.
"""
import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200 import scenes
from oracle import pyoracle as po
from tests.gpu_helpers import rel_l2, render, to_dev, zeros_like_fields

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3


def _ocam(cam):
    return po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl, cam.near_plane,
                     cam.far_plane)


def _scene():
    g, cam = scenes.small_scene(31, 3000, 96, 72, 1, scale_mu=-2.8)
    rng = np.random.default_rng(77)
    mutated = dict(mean3d=(g["mean3d"] + rng.normal(0, 0.05, g["mean3d"].shape)).astype(np.float32),
                   logscale=(g["logscale"] + 0.2).astype(np.float32),
                   opacity=(g["opacity"] - 0.5).astype(np.float32),
                   sh0=rng.uniform(0, 1, g["sh0"].shape).astype(np.float32))
    grad_rgb = np.random.default_rng(78).normal(0, 1, (3, cam.height, cam.width)).astype(np.float32)
    return g, cam, mutated, grad_rgb


def _oracle_grads(g, cam, grad_rgb, sh=1):
    f = po.render_forward(g, _ocam(cam), sh)
    return po.render_backward(g, _ocam(cam), f, grad_rgb, sh)


def _need(kind):
    if not po.ref_available(kind):
        pytest.skip(f"GSX library for '{kind}' not built")


def test_provider_cloned_state_keeps_the_forward_inputs():
    _need("b200")
    g, cam, mutated, grad_rgb = _scene()
    ref = po.RefSession("b200", g, _ocam(cam), np.zeros((3, cam.height, cam.width), np.float32), sh_degree=1)
    _, base = ref.render_backward(grad_rgb)
    sess = po.RefSession("b200", g, _ocam(cam), np.zeros((3, cam.height, cam.width), np.float32), sh_degree=1)
    sess.set_borrow(False)
    got = sess.mutate_backward(grad_rgb, mutated)
    exp = _oracle_grads(g, cam, grad_rgb)
    for k in ("mean3d", "logscale", "sh0", "opacity"):
        # the reference's bar is 1e-5 absolute; the two backwards here add their atomic contributions
        # in different orders, which moves a gradient of magnitude ~20 by a few f32 ulps, so the bar
        # also allows 1e-5 relative
        np.testing.assert_allclose(got[k], base[k], rtol=1e-5, atol=1e-5, err_msg=k)
        assert rel_l2(got[k], exp[k]) <= GRAD_TOL, k


def test_provider_borrowed_state_tracks_input_mutations():
    _need("b200")
    g, cam, mutated, grad_rgb = _scene()
    ref = po.RefSession("b200", g, _ocam(cam), np.zeros((3, cam.height, cam.width), np.float32), sh_degree=1)
    _, base = ref.render_backward(grad_rgb)
    sess = po.RefSession("b200", g, _ocam(cam), np.zeros((3, cam.height, cam.width), np.float32), sh_degree=1)
    sess.set_borrow(True)
    got = sess.mutate_backward(grad_rgb, mutated)
    # the reference test's assertion: the gradients moved with the inputs
    assert np.abs(got["mean3d"] - base["mean3d"]).max() > 1e-3
    assert np.abs(got["logscale"] - base["logscale"]).max() > 1e-4
    assert np.abs(got["opacity"] - base["opacity"]).max() > 1e-3
    # stronger: they are the gradients of a fresh TRAIN forward + backward of the mutated inputs
    g2 = dict(g, **mutated)
    exp = _oracle_grads(g2, cam, grad_rgb)
    for k, v in got.items():
        assert rel_l2(v, exp[k]) <= GRAD_TOL, f"{k}: rel-L2 {rel_l2(v, exp[k]):.3e}"


def test_provider_borrowed_state_matches_reference_cuda_backend():
    """The reference CUDA backend's own borrowed refresh, same inputs and mutation."""
    _need("b200")
    _need("cuda")
    g, cam, mutated, grad_rgb = _scene()
    out = {}
    for kind in ("b200", "cuda"):
        sess = po.RefSession(kind, g, _ocam(cam), np.zeros((3, cam.height, cam.width), np.float32), sh_degree=1)
        sess.set_borrow(True)
        out[kind] = sess.mutate_backward(grad_rgb, mutated)
    for k, v in out["b200"].items():
        assert rel_l2(v, out["cuda"][k]) <= GRAD_TOL, k


def test_c_abi_borrowed_mode_refreshes_only_on_change(cuda_device):
    g, cam, mutated, grad_rgb = _scene()
    gd = to_dev(g)
    gr = torch.from_numpy(grad_rgb).cuda()
    rend = gb.Renderer(cam.width, cam.height)
    # retained mode, no mutation: the baseline
    ctx = gb.RenderContext(0)
    render(ctx, gd, cam, 1)
    base = zeros_like_fields(gd)
    rend.backward(ctx, gr, base)
    ctx.check()
    # borrowed mode, no mutation: no refresh, the same gradients (up to the order of the blend
    # backward's atomic additions)
    ctx.set_train_state(True)
    render(ctx, gd, cam, 1)
    same = zeros_like_fields(gd)
    rend.backward(ctx, gr, same)
    ctx.check()
    assert ctx.train_refreshes() == 0
    for k in gd:
        assert rel_l2(same[k].cpu().numpy(), base[k].cpu().numpy()) <= 1e-5, k
    # borrowed mode, mutation after the forward: one refresh, gradients of the mutated inputs
    out = render(ctx, gd, cam, 1)
    out_before = out.clone()
    for k, v in mutated.items():
        gd[k].copy_(torch.from_numpy(v))
    moved = zeros_like_fields(gd)
    rend.backward(ctx, gr, moved)
    ctx.check()
    assert ctx.train_refreshes() == 1
    exp = _oracle_grads(dict(g, **mutated), cam, grad_rgb)
    for k in gd:
        err = rel_l2(moved[k].cpu().numpy(), exp[k])
        assert err <= GRAD_TOL, f"{k}: rel-L2 {err:.3e}"
    # the refresh renders privately: the caller's image is the one its forward wrote
    assert torch.equal(out, out_before)
    # retained mode after a mutation uses the forward's screen-space state: the documented contract is
    # that the caller does not mutate; switching modes drops the retained forward
    ctx.set_train_state(False)
    with pytest.raises(gb.GsxError) as e:
        rend.backward(ctx, gr, moved)
    assert e.value.code == gb.INVALID_STATE
    ctx.close()
