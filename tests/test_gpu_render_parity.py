"""Render forward/backward on the B200 vs the CPU oracle (oracle/gsx_oracle.c), through the C ABI.

Bars: tile keys, sort order, tile ranges and per-Gaussian offsets bit-exact;
RGB max-abs <= 1e-4 (the arithmetic contract makes it bit-exact in practice; both are checked);
parameter gradients rel-L2 <= 1e-3 per field (atomic accumulation order differs).
"""
import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200 import scenes
from oracle import pyoracle as po
from tests.gpu_helpers import fetch_view, rel_l2, render, to_dev, zeros_like_fields

pytestmark = pytest.mark.gpu

RGB_TOL = 1e-4
GRAD_TOL = 1e-3

CASES = [
    dict(seed=0, n=2000, width=96, height=80, sh=0, bg=(0.0, 0.0, 0.0)),
    dict(seed=1, n=3000, width=77, height=53, sh=1, bg=(0.2, 0.5, 0.9)),
    dict(seed=2, n=1500, width=128, height=128, sh=2, bg=(1.0, 1.0, 1.0)),
    dict(seed=3, n=2500, width=65, height=33, sh=3, bg=(0.0, 0.3, 0.0)),
    dict(seed=4, n=6000, width=160, height=96, sh=0, bg=(0.0, 0.0, 0.0), scale_mu=-2.0),
]


def _ocam(cam):
    return po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl, cam.near_plane,
                     cam.far_plane)


@pytest.fixture(scope="module")
def ctx(cuda_device):
    c = gb.RenderContext(0)
    yield c
    c.close()


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"s{c['seed']}_{c['width']}x{c['height']}_sh{c['sh']}")
def test_forward_bit_exact(ctx, case):
    g, cam = scenes.small_scene(case["seed"], case["n"], case["width"], case["height"], case["sh"],
                                scale_mu=case.get("scale_mu", -3.0))
    ref = po.render_forward(g, _ocam(cam), case["sh"], case["bg"])
    assert ref["n_instances"] > 0
    gd = to_dev(g)
    out = render(ctx, gd, cam, case["sh"], case["bg"])
    ctx.check()
    v = fetch_view(ctx, case["n"])
    exp_offsets = np.concatenate([[0], np.cumsum(ref["n_touched"].astype(np.uint64))]).astype(np.uint32)
    np.testing.assert_array_equal(v["offsets"], exp_offsets)
    np.testing.assert_array_equal(v["keys"], ref["keys"])
    np.testing.assert_array_equal(v["vals"], ref["vals"])
    np.testing.assert_array_equal(v["ranges"], ref["ranges"])
    np.testing.assert_array_equal(v["tile_max"], ref["tile_max"])
    rgb = out.cpu().numpy()
    assert np.abs(rgb - ref["rgb"]).max() <= RGB_TOL
    assert np.array_equal(rgb, ref["rgb"]), "arithmetic contract: expected bit-identical RGB"


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"s{c['seed']}_{c['width']}x{c['height']}_sh{c['sh']}")
def test_backward_matches_oracle(ctx, case):
    g, cam = scenes.small_scene(case["seed"], case["n"], case["width"], case["height"], case["sh"],
                                scale_mu=case.get("scale_mu", -3.0))
    rng = np.random.default_rng(100 + case["seed"])
    grad_rgb = rng.normal(0, 1, (3, cam.height, cam.width)).astype(np.float32)
    ref_f = po.render_forward(g, _ocam(cam), case["sh"], case["bg"])
    ref_b = po.render_backward(g, _ocam(cam), ref_f, grad_rgb, case["sh"])
    gd = to_dev(g)
    render(ctx, gd, cam, case["sh"], case["bg"])
    grads = zeros_like_fields(gd)
    for k in grads:
        grads[k].fill_(123.0)  # must be overwritten, not accumulated
    gb.Renderer(cam.width, cam.height).backward(ctx, torch.from_numpy(grad_rgb).cuda(), grads)
    ctx.check()
    for k in gd:
        got = grads[k].cpu().numpy()
        exp = ref_b[k]
        assert np.isfinite(got).all(), k
        err = rel_l2(got, exp)
        assert err <= GRAD_TOL, f"{k}: rel-L2 {err:.3e}"


def test_empty_scene_is_background(ctx):
    cam = gb.Camera(40, 24, 30.0, 30.0, 20.0, 12.0)
    g = {k: torch.zeros((0,) + s, device="cuda:0") for k, s in
         (("mean3d", (3,)), ("rotation", (4,)), ("logscale", (3,)), ("opacity", ()), ("sh0", (3,)))}
    out = render(ctx, g, cam, 0, (0.25, 0.5, 0.75))
    ctx.check()
    exp = np.broadcast_to(np.array([0.25, 0.5, 0.75], np.float32)[:, None, None], (3, 24, 40))
    np.testing.assert_array_equal(out.cpu().numpy(), exp)


def test_all_culled_scene(ctx):
    g, cam = scenes.small_scene(7, 500, 48, 48)
    g["mean3d"][:, 2] = -3.0  # all behind the camera
    gd = to_dev(g)
    out = render(ctx, gd, cam, 0, (0.1, 0.2, 0.3))
    ctx.check()
    assert ctx.stats()["n_instances"] == 0
    exp = np.broadcast_to(np.array([0.1, 0.2, 0.3], np.float32)[:, None, None], (3, 48, 48))
    np.testing.assert_array_equal(out.cpu().numpy(), exp)
    grads = zeros_like_fields(gd)
    gb.Renderer(48, 48).backward(ctx, torch.ones((3, 48, 48), device="cuda:0"), grads)
    ctx.check()
    for k in grads:
        assert float(grads[k].abs().max()) == 0.0


def test_one_gaussian_covering_every_tile(ctx):
    W, H = 200, 150
    g = dict(mean3d=np.array([[0.05, -0.02, 1.0]], np.float32), rotation=np.array([[0.1, 0.2, 0.3, 0.9]], np.float32),
             logscale=np.array([[0.5, 0.3, 0.1]], np.float32), opacity=np.array([2.0], np.float32),
             sh0=np.array([[0.4, 0.1, 0.9]], np.float32))
    cam = gb.Camera(W, H, 150.0, 150.0, W / 2, H / 2)
    ref = po.render_forward(g, _ocam(cam), 0, (0, 0, 0))
    gd = to_dev(g)
    out = render(ctx, gd, cam)
    ctx.check()
    v = fetch_view(ctx, 1)
    n_tiles = ((W + 15) // 16) * ((H + 15) // 16)
    assert ref["n_instances"] == n_tiles
    np.testing.assert_array_equal(v["keys"], ref["keys"])
    np.testing.assert_array_equal(out.cpu().numpy(), ref["rgb"])


def test_one_pixel_known_answer(ctx):
    """tests/render_runtime.cpp:671-722 of the reference: 1 Gaussian, 1x1 image -> (0.3910474, 0.25, 0.25)."""
    g = dict(mean3d=np.array([[0, 0, 4]], np.float32), rotation=np.array([[0, 0, 0, 1]], np.float32),
             logscale=np.zeros((1, 3), np.float32), opacity=np.zeros(1, np.float32), sh0=np.array([[1, 0, 0]], np.float32))
    cam = gb.Camera(1, 1, 1.0, 1.0, 0.5, 0.5, near_plane=0.1, far_plane=10.0)
    out = render(ctx, to_dev(g), cam, train=False)
    np.testing.assert_allclose(out.cpu().numpy().ravel(), [0.3910474, 0.25, 0.25], atol=1e-5)


def test_backward_requires_train_forward(ctx):
    g, cam = scenes.small_scene(9, 100, 32, 32)
    gd = to_dev(g)
    render(ctx, gd, cam, train=False)
    with pytest.raises(gb.GsxError) as e:
        gb.Renderer(32, 32).backward(ctx, torch.zeros((3, 32, 32), device="cuda:0"), zeros_like_fields(gd))
    assert e.value.code == gb.INVALID_STATE


def test_invalid_arguments(ctx):
    g, cam = scenes.small_scene(9, 100, 32, 32)
    gd = to_dev(g)
    out = torch.empty((3, 32, 32), device="cuda:0")
    with pytest.raises(gb.GsxError) as e:
        gb.Renderer(32, 32).render(ctx, gd, cam, out, sh_degree=4)
    assert e.value.code == gb.OUT_OF_RANGE
    bad = gb.Camera(32, 32, 30.0, 30.0, 16.0, 16.0, near_plane=-1.0)
    with pytest.raises(gb.GsxError) as e:
        gb.Renderer(32, 32).render(ctx, gd, bad, out)
    assert e.value.code == gb.INVALID_ARGUMENT
    with pytest.raises(gb.GsxError) as e:
        gb.Renderer(32, 32).render(ctx, gd, cam, out, sh_degree=1)  # sh1 missing
    assert e.value.code == gb.INVALID_ARGUMENT


def test_repeated_forward_is_deterministic(ctx):
    g, cam = scenes.small_scene(11, 4000, 100, 70)
    gd = to_dev(g)
    a = render(ctx, gd, cam).clone()
    b = render(ctx, gd, cam).clone()
    assert torch.equal(a, b)


def _cluster_scene(seed, n, width, height, z_levels=None):
    """n small Gaussians packed into a width x height view (every tile holds thousands of
    instances); with z_levels, depths take only that many distinct values (ties broken by index)."""
    rng = np.random.default_rng(seed)
    z = rng.uniform(2.0, 6.0, n) if z_levels is None else rng.choice(np.linspace(2.0, 6.0, z_levels), n)
    g = dict(mean3d=np.stack([rng.uniform(-0.5, 0.5, n) * z, rng.uniform(-0.5, 0.5, n) * z, z], 1).astype(np.float32),
             rotation=scenes._unit_quats(rng, n), logscale=rng.normal(-2.5, 0.3, (n, 3)).astype(np.float32),
             opacity=rng.normal(-1.0, 1.0, n).astype(np.float32), sh0=rng.uniform(0.0, 1.0, (n, 3)).astype(np.float32))
    cam = gb.Camera(width, height, float(width), float(width), width / 2.0, height / 2.0, near_plane=0.2, far_plane=100.0)
    return g, cam


@pytest.mark.parametrize("n,size,z_levels", [(5000, 16, None), (3000, 24, 7), (60000, 32, None)],
                         ids=["one_tile_5k", "depth_ties", "tiles_over_16384_global_sort"])
def test_dense_tiles_order_and_gradients(ctx, n, size, z_levels):
    """Dense tiles: the shared-memory per-tile sort (segments up to 16384, heavy depth ties) and the
    global radix sort fallback (a tile above 16384) give the oracle's exact order and results."""
    g, cam = _cluster_scene(21, n, size, size, z_levels)
    ref = po.render_forward(g, _ocam(cam), 0, (0, 0, 0))
    seg = ref["ranges"][:, 1] - ref["ranges"][:, 0]
    if size == 32:
        assert seg.max() > 16384
    gd = to_dev(g)
    out = render(ctx, gd, cam)
    ctx.check()
    v = fetch_view(ctx, n)
    np.testing.assert_array_equal(v["keys"], ref["keys"])
    np.testing.assert_array_equal(v["vals"], ref["vals"])
    np.testing.assert_array_equal(v["ranges"], ref["ranges"])
    np.testing.assert_array_equal(out.cpu().numpy(), ref["rgb"])
    grad_rgb = np.random.default_rng(5).normal(0, 1, (3, size, size)).astype(np.float32)
    ref_b = po.render_backward(g, _ocam(cam), ref, grad_rgb, 0)
    grads = zeros_like_fields(gd)
    gb.Renderer(size, size).backward(ctx, torch.from_numpy(grad_rgb).cuda(), grads)
    ctx.check()
    for k in gd:
        err = rel_l2(grads[k].cpu().numpy(), ref_b[k])
        assert err <= GRAD_TOL, f"{k}: rel-L2 {err:.3e}"


@pytest.mark.parametrize("n", [1_100_003, 2_500_000])
def test_instance_total_over_many_scan_chunks(ctx, n):
    """More 256-Gaussian blocks than the block-total scan takes in one pass (4096 per chunk, a ragged
    last chunk): the instance total read back to the host (the scan's last word) equals the last
    per-Gaussian offset (the emission's in-block scans over the same totals) and the number of keys,
    and the keys come out sorted."""
    g, cam = scenes.small_scene(5, n, 640, 480, 0, scale_mu=-3.5)
    gd = to_dev(g)
    render(ctx, gd, cam, train=False)
    ctx.check()
    v = fetch_view(ctx, n)
    off = v["offsets"].astype(np.int64)
    assert off[0] == 0 and np.all(np.diff(off) >= 0)
    assert int(ctx.stats()["n_instances"]) == int(off[-1]) == v["keys"].shape[0]
    assert off[-1] > 0
    assert np.all(v["keys"][1:] >= v["keys"][:-1])
    # a second forward of the same scene gives the same total (the scan's last word is rewritten)
    render(ctx, gd, cam, train=False)
    ctx.check()
    assert int(ctx.stats()["n_instances"]) == int(off[-1])
