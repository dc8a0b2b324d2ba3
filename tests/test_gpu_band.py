"""Band rendering (rows [r0, r1) of a full frame, the frame-split path of a large frame over several
GPUs) and bf16 output, through the C ABI.

A band uses full-frame coordinates for every projection, clip, tile test and pixel position, so:
band RGB == the same rows of the full-frame render, bit for bit; the band's keys/values are the
full frame's keys of the band's tile rows (tile index shifted by the band's first tile row) in the
same order; the band backward equals the full-frame backward of an upstream gradient that is zero
outside the band (rel-L2 <= 1e-3, atomic order).  bf16 output == round-to-nearest-even of the f32
output.
"""
import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200 import scenes
from oracle import pyoracle as po
from tests.gpu_helpers import fetch_view, rel_l2, render, to_dev, zeros_like_fields

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3


def _ocam(cam):
    return po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl, cam.near_plane,
                     cam.far_plane)


@pytest.fixture(scope="module")
def ctx(cuda_device):
    c = gb.RenderContext(0)
    yield c
    c.close()


def _band(ctx, gd, cam, r0, r1, sh=0, bg=(0.0, 0.0, 0.0), train=False, dtype=torch.float32):
    out = torch.empty((3, r1 - r0, cam.width), dtype=dtype, device="cuda:0")
    gb.Renderer(cam.width, cam.height).render_rows(ctx, gd, cam, r0, r1, out, background=bg, sh_degree=sh,
                                                   forward_type=gb.FORWARD_TRAIN if train else gb.FORWARD_INFERENCE)
    return out


@pytest.mark.parametrize("world", [1, 2, 3, 5])
@pytest.mark.parametrize("case", [dict(seed=11, n=4000, width=120, height=101, sh=1, bg=(0.1, 0.2, 0.3)),
                                  dict(seed=12, n=3000, width=64, height=64, sh=0, bg=(0.0, 0.0, 0.0))],
                         ids=lambda c: f"{c['width']}x{c['height']}")
def test_bands_equal_full_frame_rows(ctx, case, world):
    g, cam = scenes.small_scene(case["seed"], case["n"], case["width"], case["height"], case["sh"], scale_mu=-2.5)
    gd = to_dev(g)
    full = render(ctx, gd, cam, case["sh"], case["bg"], train=False)
    ctx.check()
    fv = fetch_view(ctx, case["n"])
    full_np = full.cpu().numpy()
    gw = (cam.width + 15) // 16
    covered = 0
    for r in range(world):
        r0, r1 = gb.band_rows(cam.height, r, world)
        if r0 == r1:
            continue
        out = _band(ctx, gd, cam, r0, r1, case["sh"], case["bg"])
        ctx.check()
        np.testing.assert_array_equal(out.cpu().numpy(), full_np[:, r0:r1, :])
        v = fetch_view(ctx, case["n"])
        t0, t1 = r0 // 16, (r1 + 15) // 16
        tiles = (fv["keys"] >> np.uint64(32)).astype(np.int64)
        sel = (tiles >= t0 * gw) & (tiles < t1 * gw)
        exp_keys = fv["keys"][sel] - (np.uint64(t0 * gw) << np.uint64(32))
        np.testing.assert_array_equal(v["keys"], exp_keys)
        np.testing.assert_array_equal(v["vals"], fv["vals"][sel])
        covered += r1 - r0
    assert covered == cam.height


def test_band_matches_oracle_rows(ctx):
    g, cam = scenes.small_scene(21, 2500, 80, 72, 2, scale_mu=-2.5)
    ref = po.render_forward(g, _ocam(cam), 2, (0.3, 0.3, 0.3))
    out = _band(ctx, to_dev(g), cam, 32, 72, 2, (0.3, 0.3, 0.3))
    ctx.check()
    np.testing.assert_array_equal(out.cpu().numpy(), ref["rgb"][:, 32:72, :])


@pytest.mark.parametrize("r0,r1", [(0, 48), (16, 53), (48, 77)])
def test_band_backward_matches_masked_full_frame(ctx, r0, r1):
    sh = 1
    g, cam = scenes.small_scene(31, 3000, 90, 77, sh, scale_mu=-2.5)
    rng = np.random.default_rng(5)
    grad_full = rng.normal(0, 1, (3, cam.height, cam.width)).astype(np.float32)
    grad_full[:, :r0, :] = 0.0
    grad_full[:, r1:, :] = 0.0
    ref_f = po.render_forward(g, _ocam(cam), sh, (0, 0, 0))
    ref_b = po.render_backward(g, _ocam(cam), ref_f, grad_full, sh)
    gd = to_dev(g)
    out = _band(ctx, gd, cam, r0, r1, sh, train=True)
    np.testing.assert_array_equal(out.cpu().numpy(), ref_f["rgb"][:, r0:r1, :])
    grads = zeros_like_fields(gd)
    gb.Renderer(cam.width, cam.height).backward(ctx, torch.from_numpy(np.ascontiguousarray(grad_full[:, r0:r1, :])).cuda(),
                                                grads)
    ctx.check()
    for k in gd:
        err = rel_l2(grads[k].cpu().numpy(), ref_b[k])
        assert err <= GRAD_TOL, f"{k}: rel-L2 {err:.3e}"


def test_bf16_output_is_rne_of_f32(ctx):
    g, cam = scenes.small_scene(41, 3000, 100, 70, 0, scale_mu=-2.5)
    gd = to_dev(g)
    f32 = _band(ctx, gd, cam, 0, cam.height, 0, (0.2, 0.1, 0.0))
    b16 = _band(ctx, gd, cam, 0, cam.height, 0, (0.2, 0.1, 0.0), dtype=torch.bfloat16)
    ctx.check()
    assert torch.equal(b16.view(torch.int16), f32.to(torch.bfloat16).view(torch.int16))
    b16b = _band(ctx, gd, cam, 16, 70, 0, (0.2, 0.1, 0.0), dtype=torch.bfloat16)
    ctx.check()
    assert torch.equal(b16b.view(torch.int16), f32[:, 16:70].to(torch.bfloat16).view(torch.int16))


def test_band_argument_checks(ctx):
    g, cam = scenes.small_scene(1, 100, 64, 48)
    gd = to_dev(g)
    r = gb.Renderer(cam.width, cam.height)
    for r0, r1 in ((8, 48), (0, 0), (32, 16), (0, 49), (-16, 16)):
        out = torch.empty((3, max(r1 - r0, 1), cam.width), device="cuda:0")
        with pytest.raises(gb.GsxError):
            r.render_rows(ctx, gd, cam, r0, r1, out)


def test_row_costs_are_deterministic_and_cut_into_bands(ctx):
    """gsx_b200_render_row_costs: integer per-tile-row work estimates, identical on repeated calls (every
    rank of a frame split derives the same bands from them), zero for rows no Gaussian reaches; the
    equal-work bands they give render bit-identically to the full frame's rows."""
    g, cam = scenes.small_scene(13, 6000, 96, 200, 0, scale_mu=-2.5)
    gd = to_dev(g)
    a = ctx.row_costs(gd, cam)
    b = ctx.row_costs(gd, cam)
    assert a.shape == ((cam.height + 15) // 16,) and a.sum() > 0
    np.testing.assert_array_equal(a, b)
    full = render(ctx, gd, cam, 0, (0.0, 0.0, 0.0), train=False).cpu().numpy()
    pos = 0
    for r in range(3):
        r0, r1 = gb.balanced_band_rows(a, cam.height, r, 3)
        assert r0 == pos
        pos = r1
        if r1 > r0:
            out = _band(ctx, gd, cam, r0, r1)
            ctx.check()
            np.testing.assert_array_equal(out.cpu().numpy(), full[:, r0:r1, :])
    assert pos == cam.height
