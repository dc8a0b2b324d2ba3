"""Dataloader layout conversion (HWC u8/f32 -> CHW f32) on the B200 vs the oracle's restatement of
gsx_dataloader_pack_hwc_to_chw (bit-exact: a permutation and an exact u8 -> f32 conversion)."""
import numpy as np
import pytest
import torch

import gsx_b200 as gb
from oracle import pyoracle as po

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("h,w", [(1, 1), (3, 5), (7, 13), (64, 64), (825, 1245), (1080, 1920), (2160, 3840)])
@pytest.mark.parametrize("dtype", ["u8", "f32"])
@pytest.mark.parametrize("c", [3, 1])
def test_hwc_to_chw_matches_packer(cuda_device, h, w, dtype, c):
    rng = np.random.default_rng(h * 7919 + w + c)
    shape = (h, w, c) if c == 3 else (h, w)
    src = rng.integers(0, 256, shape, dtype=np.uint8) if dtype == "u8" else rng.normal(0, 10, shape).astype(np.float32)
    out = gb.hwc_to_chw(torch.from_numpy(src).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), po.pack_hwc_to_chw(src))


@pytest.mark.parametrize("offset", [1, 3, 5])
def test_unaligned_source_and_sizes(cuda_device, offset):
    """A source that starts off a 16-byte boundary takes the element path; same result."""
    h, w = 37, 41
    rng = np.random.default_rng(offset)
    buf = torch.from_numpy(rng.integers(0, 256, h * w * 3 + 64, dtype=np.uint8)).cuda()
    src = buf[offset:offset + h * w * 3].view(h, w, 3)
    out = gb.hwc_to_chw(src)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), po.pack_hwc_to_chw(src.cpu().numpy()))


def test_bad_arguments(cuda_device):
    import ctypes
    from gsx_b200._capi import lib, check, GsxError
    x = torch.zeros((4, 4, 3), dtype=torch.uint8, device="cuda:0")
    y = torch.zeros((3, 4, 4), device="cuda:0")
    for st, ch in ((3, 3), (8, 2)):
        with pytest.raises(GsxError):
            check(lib().gsx_b200_hwc_to_chw_f32(ctypes.c_void_p(x.data_ptr()), st, ch, 16,
                                                ctypes.c_void_p(y.data_ptr()), None))


def test_reference_known_answer(cuda_device):
    """tests/data_runtime.cpp:399-427 of the reference: the packed f32 CHW of a 2x2 u8 sample."""
    rgb = torch.tensor([0, 10, 20, 40, 50, 60, 80, 90, 100, 120, 130, 140], dtype=torch.uint8).view(2, 2, 3).cuda()
    alpha = torch.tensor([10, 30, 50, 70], dtype=torch.uint8).view(2, 2).cuda()
    assert gb.hwc_to_chw(rgb).flatten().tolist() == [0, 40, 80, 120, 10, 50, 90, 130, 20, 60, 100, 140]
    assert gb.hwc_to_chw(alpha).flatten().tolist() == [10, 30, 50, 70]
