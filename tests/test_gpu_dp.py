"""The fused data-parallel exchange (gsx_b200_dp_reduce_adam_gather) on one GPU: `world` ranks
emulated by `world` buffer sets on the same device, each rank's call made in turn (the kernel never
waits on another rank, and every flat element is written by exactly one rank, so the emulation runs
the same arithmetic as the multi-GPU run).  Bar: every rank's parameters bit-identical to one
all-reduce-average (sum in rank order, times 1/world) followed by the single-GPU Adam kernel, over
several steps; replicas identical."""
import ctypes
import math

import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200._capi import check, lib
from gsx_b200.dp import Segment, shard_bounds, shard_segments

pytestmark = pytest.mark.gpu


def _fields(n):
    cols = {"mean3d": 3, "logscale": 3, "rotation": 4, "opacity": 1, "sh0": 3}
    ranges, o = {}, 0
    for f, c in cols.items():
        cnt = n * c
        ranges[f] = (o, o + (cnt + 3) // 4 * 4)
        o += (cnt + 3) // 4 * 4
    return ranges, o


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_fused_exchange_equals_allreduce_then_adam(cuda_device, world):
    n = 12345
    ranges, numel = _fields(n)
    lr = {"mean3d": 1e-3, "logscale": 1e-2, "rotation": 2e-2, "opacity": 5e-2, "sh0": 3e-3}
    rng = np.random.default_rng(world)
    p0 = torch.from_numpy(rng.normal(size=numel).astype(np.float32)).cuda()
    params = [p0.clone() for _ in range(world)]
    grads = [torch.zeros(numel, device="cuda:0") for _ in range(world)]
    shards = [shard_bounds(numel, world, r) for r in range(world)]
    moments = [(torch.zeros(max(e - b, 4), device="cuda:0"), torch.zeros(max(e - b, 4), device="cuda:0")) for b, e in shards]
    # reference: one flat parameter copy, averaged gradients, the single-GPU Adam per field
    ref = p0.clone()
    rgrad = torch.zeros(numel, device="cuda:0")
    opt = gb.Adam([gb.ParamGroup(f, ref[a:b], rgrad[a:b], lr[f]) for f, (a, b) in ranges.items()])
    P = ctypes.c_void_p * world
    pp = P(*[t.data_ptr() for t in params])
    gp = P(*[t.data_ptr() for t in grads])
    for step in range(1, 4):
        for r in range(world):
            grads[r].copy_(torch.from_numpy(rng.normal(0, 0.1, numel).astype(np.float32)))
        acc = grads[0].clone()
        for r in range(1, world):
            acc += grads[r]
        rgrad.copy_(acc * np.float32(1.0 / world))
        opt.step(force_all=True)
        for r in range(world):
            b, e = shards[r]
            runs = shard_segments(ranges, b, e)
            segs = (Segment * max(len(runs), 1))()
            for k, (f, a, z) in enumerate(runs):
                s = segs[k]
                s.begin, s.end, s.learning_rate, s.beta1, s.beta2, s.epsilon = a, z, lr[f], 0.9, 0.999, 1e-8
                s.inv_bias_correction1 = 1.0 / (1.0 - math.pow(float(np.float32(0.9)), step))
                s.inv_bias_correction2 = 1.0 / (1.0 - math.pow(float(np.float32(0.999)), step))
            check(lib().gsx_b200_dp_reduce_adam_gather(world, r, pp, gp, ctypes.c_void_p(moments[r][0].data_ptr()),
                                                       ctypes.c_void_p(moments[r][1].data_ptr()), b, e, segs, len(runs),
                                                       None))
        torch.cuda.synchronize()
        want = ref.cpu().numpy()
        for r in range(world):
            np.testing.assert_array_equal(params[r].cpu().numpy(), want, err_msg=f"rank {r} step {step}")
