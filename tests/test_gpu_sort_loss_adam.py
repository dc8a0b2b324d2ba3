"""Radix sort, fused L1+SSIM and fused Adam on the B200 vs the oracle, through the C ABI."""
import math

import numpy as np
import pytest
import torch

import gsx_b200 as gb
from oracle import pyoracle as po
from tests.gpu_helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx(cuda_device):
    c = gb.RenderContext(0)
    yield c
    c.close()


def _tile_depth_keys(rng, n, tiles=8160):
    """Config-5 key distribution: tile uniform over `tiles`, depth = f32 bits of log-uniform [0.1, 100]."""
    tile = rng.integers(0, tiles, n, dtype=np.uint64)
    depth = np.exp(rng.uniform(np.log(0.1), np.log(100.0), n)).astype(np.float32)
    return (tile << np.uint64(32)) | depth.view(np.uint32).astype(np.uint64)


def _sort_gpu(ctx, keys, vals, begin, end):
    k = torch.from_numpy(keys.view(np.int64)).cuda()
    v = torch.from_numpy(vals.view(np.int32)).cuda()
    gb.sort_pairs(ctx, k, v, begin, end)
    ctx.check()
    return k.cpu().numpy().view(np.uint64), v.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("n", [1, 2, 31, 4095, 4096, 4097, 100_003, 1_000_000])
def test_sort_matches_stable_sort(ctx, n):
    rng = np.random.default_rng(n)
    keys = _tile_depth_keys(rng, n)
    vals = np.arange(n, dtype=np.uint32)
    gk, gv = _sort_gpu(ctx, keys, vals, 0, 45)
    ek, ev = po.sort_pairs(keys, vals)
    np.testing.assert_array_equal(gk, ek)
    np.testing.assert_array_equal(gv, ev)


def test_sort_stability_with_many_duplicates(ctx):
    rng = np.random.default_rng(5)
    n = 300_000
    keys = rng.integers(0, 7, n).astype(np.uint64) << np.uint64(40)
    vals = np.arange(n, dtype=np.uint32)
    gk, gv = _sort_gpu(ctx, keys, vals, 0, 64)
    order = np.argsort(keys, kind="stable")
    np.testing.assert_array_equal(gk, keys[order])
    np.testing.assert_array_equal(gv, vals[order])


@pytest.mark.parametrize("bits", [(0, 8), (8, 24), (0, 64), (13, 51)])
def test_sort_bit_ranges(ctx, bits):
    rng = np.random.default_rng(sum(bits))
    n = 50_000
    keys = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
    vals = np.arange(n, dtype=np.uint32)
    gk, gv = _sort_gpu(ctx, keys, vals, *bits)
    b0, b1 = bits
    mask = np.uint64((1 << (b1 - b0)) - 1) if b1 - b0 < 64 else np.uint64(0xFFFFFFFFFFFFFFFF)
    sub = (keys >> np.uint64(b0)) & mask
    order = np.argsort(sub, kind="stable")
    np.testing.assert_array_equal(gk, keys[order])
    np.testing.assert_array_equal(gv, vals[order])


def test_sort_empty(ctx):
    k = torch.zeros(0, dtype=torch.int64, device="cuda:0")
    v = torch.zeros(0, dtype=torch.int32, device="cuda:0")
    gb.sort_pairs(ctx, k, v, 0, 64)


def test_sort_large_properties(ctx):
    """Full-size property check (30M config-5 pairs): sorted, and every pair is an input pair."""
    rng = np.random.default_rng(77)
    n = 30_000_000
    keys = _tile_depth_keys(rng, n)
    kd = torch.from_numpy(keys.view(np.int64)).cuda()
    vd = torch.arange(n, dtype=torch.int32, device="cuda:0")
    gb.sort_pairs(ctx, kd, vd, 0, 45)
    ctx.check()
    ku = kd.view(torch.int64)
    # unsigned order == signed order here (keys < 2^63)
    assert bool((ku[1:] >= ku[:-1]).all())
    orig = torch.from_numpy(keys.view(np.int64)).cuda()
    assert torch.equal(orig[vd.long()], kd)
    # stability: equal keys keep increasing original index
    eq = ku[1:] == ku[:-1]
    assert bool((vd[1:][eq] > vd[:-1][eq]).all())


def _images(seed, shape):
    rng = np.random.default_rng(seed)
    p = rng.uniform(0, 1, shape).astype(np.float32)
    t = np.clip(p + rng.normal(0, 0.2, shape), 0, 1).astype(np.float32)
    return p, t


@pytest.mark.parametrize("shape", [(3, 64, 48), (3, 37, 70), (2, 3, 40, 33), (1, 11, 11), (3, 8, 9)])
def test_fused_l1_ssim_matches_oracle(shape):
    p, t = _images(sum(shape), shape)
    rng = np.random.default_rng(3)
    lm0 = rng.uniform(0, 0.1, shape).astype(np.float32)
    g0 = rng.normal(0, 1e-4, shape).astype(np.float32)
    ref_lm, ref_g = po.l1_ssim_train(p, t, 0.8, 0.2, loss_map=lm0, grad=g0)
    P, T = torch.from_numpy(p).cuda(), torch.from_numpy(t).cuda()
    lm = torch.from_numpy(lm0).cuda()
    g = torch.from_numpy(g0).cuda()
    s = torch.zeros(1, device="cuda:0")
    gb.l1_ssim(P, T, lm, g, 0.8, 0.2, loss_sum=s)
    torch.cuda.synchronize()
    assert np.abs(lm.cpu().numpy() - ref_lm).max() <= 2e-5
    assert rel_l2(g.cpu().numpy(), ref_g) <= 1e-4
    assert abs(float(s) - float(lm.cpu().numpy().sum())) <= 1e-3 * max(1.0, abs(float(s)))


def test_standalone_losses_match_oracle():
    shape = (3, 50, 41)
    p, t = _images(9, shape)
    n = p.size
    P, T = torch.from_numpy(p).cuda(), torch.from_numpy(t).cuda()
    for algo in ("l1", "mse", "ssim"):
        loss = gb.Loss(algo, "mean")
        lm = torch.zeros_like(P)
        g = torch.zeros_like(P)
        loss.forward(P, T, lm, scale=0.7)
        loss.backward(g, scale=0.7)
        torch.cuda.synchronize()
        if algo == "ssim":
            elm, eg = po.ssim(p, t, 0.7, np.float32(0.7) / np.float32(n))
            assert np.abs(lm.cpu().numpy() - elm).max() <= 2e-5
            assert rel_l2(g.cpu().numpy(), eg) <= 1e-4
        else:
            d = p - t
            elm = 0.7 * (np.abs(d) if algo == "l1" else d * d)
            gs = np.float32(0.7) / np.float32(n)
            eg = np.sign(d) * gs if algo == "l1" else 2.0 * d * gs
            np.testing.assert_allclose(lm.cpu().numpy(), elm, rtol=1e-6, atol=1e-7)
            np.testing.assert_allclose(g.cpu().numpy(), eg, rtol=1e-6, atol=1e-12)
    with pytest.raises(gb.GsxError) as e:
        gb.Loss("ssim").backward(torch.zeros_like(P))
    assert e.value.code == gb.INVALID_STATE


def test_adam_bit_exact_vs_oracle():
    rng = np.random.default_rng(0)
    sizes = [(1001, 1e-3, 0.0, 0.0), (4096 * 3 + 5, 1e-2, 0.01, 0.0), (777, 5e-3, 0.0, 1e-3)]
    params = [rng.standard_normal(n).astype(np.float32) for n, *_ in sizes]
    groups, ref = [], []
    for (n, lr, wd, mg), p in zip(sizes, params):
        pt = torch.from_numpy(p.copy()).cuda()
        gt = torch.zeros_like(pt)
        groups.append(gb.ParamGroup("custom", pt, gt, lr, weight_decay=wd, max_grad=mg))
        ref.append(dict(p=p.copy(), m1=np.zeros_like(p), m2=np.zeros_like(p), lr=lr, wd=wd, mg=mg))
    opt = gb.Adam(groups)
    for step in range(1, 6):
        for g, r in zip(groups, ref):
            gr = (rng.standard_normal(r["p"].size) * 1e-3).astype(np.float32)
            g.gradient.copy_(torch.from_numpy(gr))
            po.adam(r["p"], gr, r["m1"], r["m2"], step, r["lr"], weight_decay=r["wd"], max_grad=r["mg"])
        opt.step(force_all=True)
    torch.cuda.synchronize()
    for g, r in zip(groups, ref):
        np.testing.assert_array_equal(g.parameter.cpu().numpy(), r["p"])


def test_adam_role_selection():
    pa = torch.ones(10, device="cuda:0")
    pb = torch.ones(10, device="cuda:0")
    ga = torch.full_like(pa, 0.5)
    gbb = torch.full_like(pb, 0.5)
    opt = gb.Adam([gb.ParamGroup("mean3d", pa, ga, 0.1), gb.ParamGroup("opacity", pb, gbb, 0.1)])
    opt.step(roles={"mean3d"}, force_all=False)
    torch.cuda.synchronize()
    assert float(pa[0]) < 1.0 and float(pb[0]) == 1.0
    assert opt.steps == [1, 0]
    expect = 1.0 - 0.1 * (0.05 / (1 - 0.9)) / (math.sqrt(0.00025 / (1 - 0.999)) + 1e-8)
    assert abs(float(pa[0]) - expect) < 1e-6
