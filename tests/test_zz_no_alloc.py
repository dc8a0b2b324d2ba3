"""The allocation-free sort entry point, checked against the regular one through the C ABI.

gsx_b200_sort_pairs_noalloc is for callers that must not allocate device memory themselves: a host
that hands out every device buffer from its own arenas (GSX's model), or a plugin host with a fixed
GPU memory budget that forbids hidden cudaMalloc calls.  Its scratch is one static device array,
so it sorts at most GSX_B200_NOALLOC_SORT_MAX_PAIRS pairs per call.  This file is named to be
collected last: it must pass alone in a fresh process and after every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import gsx_b200 as gb
from gsx_b200 import _capi

pytestmark = pytest.mark.gpu


def _keys(seed, n):
    rng = np.random.default_rng(seed)
    tile = rng.integers(0, 8160, n, dtype=np.uint64)
    depth = np.exp(rng.uniform(np.log(0.1), np.log(100.0), n)).astype(np.float32)
    return (tile << np.uint64(32)) | depth.view(np.uint32).astype(np.uint64)


def test_noalloc_sort_matches_context_sort_on_two_calls_in_a_row(cuda_device):
    lib = _capi.lib()
    ctx = gb.RenderContext(0)
    stream = torch.cuda.current_stream()
    for call, n in enumerate((300_007, _capi.NOALLOC_SORT_MAX_PAIRS)):
        keys = _keys(call, n)
        # the existing entry point (context scratch)
        k_ref = torch.from_numpy(keys.view(np.int64)).cuda()
        v_ref = torch.arange(n, dtype=torch.int32, device="cuda:0")
        gb.sort_pairs(ctx, k_ref, v_ref, 0, 45)
        # the allocation-free entry point, straight through the C ABI
        k = torch.from_numpy(keys.view(np.int64)).cuda()
        v = torch.arange(n, dtype=torch.int32, device="cuda:0")
        rc = lib.gsx_b200_sort_pairs_noalloc(ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()), n, 0, 45,
                                             ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, lib.gsx_b200_last_error()
        torch.cuda.synchronize()
        # the sort is exact: the tolerance used for it everywhere is bit equality
        assert torch.equal(k, k_ref), f"call {call}: keys differ"
        assert torch.equal(v, v_ref), f"call {call}: values differ"
    ctx.close()


def test_noalloc_sort_rejects_more_than_the_static_capacity(cuda_device):
    lib = _capi.lib()
    n = _capi.NOALLOC_SORT_MAX_PAIRS + 1
    k = torch.zeros(n, dtype=torch.int64, device="cuda:0")
    v = torch.zeros(n, dtype=torch.int32, device="cuda:0")
    rc = lib.gsx_b200_sort_pairs_noalloc(ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()), n, 0, 64, None)
    assert rc == gb.OUT_OF_RANGE
    assert b"GSX_B200_NOALLOC_SORT_MAX_PAIRS" in lib.gsx_b200_last_error()
