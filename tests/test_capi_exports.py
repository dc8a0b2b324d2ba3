"""The C-ABI library loads without a GPU and exports every function include/gsx_b200.h declares."""
import ctypes
import os
import re

import gsx_b200
from gsx_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            names += re.findall(r"GSX_B200_API\s+[^;(]*?\b(gsx_b200_\w+)\s*\(", src)
    return names


def test_header_declares_the_binding_table():
    declared = set(_declared())
    assert declared, "no declarations found"
    assert declared == set(_capi.SIGNATURES), declared ^ set(_capi.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_capi.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), name


def test_version_and_error_strings_without_gpu():
    L = _capi.lib()
    assert b"sm_100a" in L.gsx_b200_version()
    # no device here: context creation must fail loudly, never fall back to the CPU
    import torch
    if not torch.cuda.is_available():
        h = ctypes.c_void_p()
        rc = L.gsx_b200_context_create(0, ctypes.byref(h))
        assert rc != 0
        assert L.gsx_b200_last_error()


def test_host_side_validation_without_gpu():
    import pytest
    with pytest.raises(gsx_b200.GsxError) as e:
        gsx_b200.Loss("huber")
    assert e.value.code == gsx_b200.OUT_OF_RANGE
    with pytest.raises(gsx_b200.GsxError):
        gsx_b200.Renderer(0, 10)
    L = _capi.lib()
    assert L.gsx_b200_adam_step(None, 17, None) == gsx_b200.OUT_OF_RANGE
    assert L.gsx_b200_loss_l1_ssim(4, None, None, None, None, None, 1, 1, 1, 0, 0, 0, 0, None) == gsx_b200.INVALID_ARGUMENT


def test_gsx_provider_links_into_gsx_without_gpu():
    """The GSX library built with the gsx_b200 provider as its CUDA backend (oracle/Makefile.ref,
    target b200) exports the provider bootstrap, resolves every gsx_b200 symbol, and on a machine
    without a GPU lets GSX start with the CUDA backend reported as unavailable."""
    import pytest
    from oracle import pyoracle as po
    path = os.path.join(ROOT, "oracle", "_ref", "libgsx_ref_b200.so")
    if not os.path.exists(path) or not po.ref_available("b200"):
        pytest.skip("GSX + gsx_b200 provider library not built")
    L = ctypes.CDLL(path)
    assert hasattr(L, "gsx_cuda_backend_provider_bootstrap")
    import torch
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="device"):
            po.ref("b200")
