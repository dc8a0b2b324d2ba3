"""ctypes binding of the gsx-b200 C ABI (include/gsx_b200.h).

The shared library is built in-tree (gsx_b200/libgsx_b200.so, see gsx_b200/csrc/Makefile).  If it is
missing or cannot be loaded, every call raises: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgsx_b200.so")

STAGES = ("preprocess", "emit", "sort", "ranges", "blend_forward", "blend_backward", "preprocess_backward")
SUCCESS, OUT_OF_MEMORY, INVALID_ARGUMENT, OUT_OF_RANGE, INVALID_STATE, NOT_SUPPORTED, UNKNOWN = 0, 1, 2, 3, 4, 5, 255
ERROR_NAMES = {0: "SUCCESS", 1: "OUT_OF_MEMORY", 2: "INVALID_ARGUMENT", 3: "OUT_OF_RANGE", 4: "INVALID_STATE",
               5: "NOT_SUPPORTED", 255: "UNKNOWN"}


class GsxError(RuntimeError):
    """A gsx_error returned by the library: `.code` is the gsx_error_code value."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class Camera(ctypes.Structure):
    _fields_ = [("width", ctypes.c_int32), ("height", ctypes.c_int32), ("fx", ctypes.c_float), ("fy", ctypes.c_float),
                ("cx", ctypes.c_float), ("cy", ctypes.c_float), ("rot_xyzw", ctypes.c_float * 4),
                ("transl", ctypes.c_float * 3), ("near_plane", ctypes.c_float), ("far_plane", ctypes.c_float)]


class Gaussians(ctypes.Structure):
    _fields_ = [("count", ctypes.c_int64)] + [(k, ctypes.c_void_p) for k in
                                               ("mean3d", "rotation", "logscale", "opacity", "sh0", "sh1", "sh2", "sh3")]


class GaussianGrads(ctypes.Structure):
    _fields_ = [(k, ctypes.c_void_p) for k in ("mean3d", "rotation", "logscale", "opacity", "sh0", "sh1", "sh2", "sh3")]


class RenderView(ctypes.Structure):
    _fields_ = [("keys", ctypes.c_void_p), ("values", ctypes.c_void_p), ("ranges", ctypes.c_void_p),
                ("offsets", ctypes.c_void_p), ("tile_max", ctypes.c_void_p), ("pixel_state", ctypes.c_void_p),
                ("n_instances", ctypes.c_uint64), ("n_tiles", ctypes.c_int32), ("grid_width", ctypes.c_int32)]


class AdamGroup(ctypes.Structure):
    _fields_ = [("parameter", ctypes.c_void_p), ("gradient", ctypes.c_void_p), ("first_moment", ctypes.c_void_p),
                ("second_moment", ctypes.c_void_p), ("count", ctypes.c_uint64), ("learning_rate", ctypes.c_float),
                ("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("epsilon", ctypes.c_float),
                ("weight_decay", ctypes.c_float), ("max_grad", ctypes.c_float),
                ("inv_bias_correction1", ctypes.c_double), ("inv_bias_correction2", ctypes.c_double)]


# every exported symbol with its argument types (also the list the export test checks)
SIGNATURES = {
    "gsx_b200_last_error": (ctypes.c_char_p, []),
    "gsx_b200_version": (ctypes.c_char_p, []),
    "gsx_b200_context_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "gsx_b200_context_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "gsx_b200_render_forward": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(Gaussians), ctypes.c_int,
                                               ctypes.POINTER(Camera), ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                                               ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_render_forward_rows": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(Gaussians), ctypes.c_int,
                                                    ctypes.POINTER(Camera), ctypes.c_int, ctypes.c_int,
                                                    ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_void_p,
                                                    ctypes.c_int, ctypes.c_void_p]),
    "gsx_b200_render_bind_aux": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_void_p]),
    "gsx_b200_hwc_to_chw_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                               ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_gather_rows": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_clamp_inplace": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_iota_i32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
    "gsx_b200_adc_scratch_words": (ctypes.c_uint64, [ctypes.c_uint64]),
    "gsx_b200_adc_select_growth": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_adc_apply_split": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_adc_select_keep": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_dp_reduce_adam_gather": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "gsx_b200_dp_nvls_reduce_adam_broadcast": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "gsx_b200_device_alloc": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    "gsx_b200_device_free": (ctypes.c_int, [ctypes.c_void_p]),
    "gsx_b200_ipc_handle": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_ipc_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "gsx_b200_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "gsx_b200_render_backward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(GaussianGrads),
                                                ctypes.c_void_p]),
    "gsx_b200_render_stats": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64),
                                             ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                             ctypes.c_void_p]),
    "gsx_b200_render_get_view": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(RenderView)]),
    "gsx_b200_context_check": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "gsx_b200_context_launch_count": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]),
    "gsx_b200_context_set_train_state": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "gsx_b200_render_row_costs": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]),
    "gsx_b200_context_train_refreshes": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]),
    "gsx_b200_context_set_profiling": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "gsx_b200_context_read_profile": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_float),
                                                     ctypes.POINTER(ctypes.c_int32)]),
    "gsx_b200_loss_l1_ssim": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                                             ctypes.c_int32, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                             ctypes.c_float, ctypes.c_void_p]),
    "gsx_b200_loss_pointwise": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_uint64, ctypes.c_float, ctypes.c_void_p]),
    "gsx_b200_adam_step": (ctypes.c_int, [ctypes.POINTER(AdamGroup), ctypes.c_int32, ctypes.c_void_p]),
    "gsx_b200_sort_pairs": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                                           ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]),
    "gsx_b200_sort_pairs_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int32,
                                                   ctypes.c_int32, ctypes.c_void_p]),
    "gsx_b200_fill_pattern": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint32,
                                             ctypes.c_void_p]),
    "gsx_b200_count_nonfinite_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]),
}
NOALLOC_SORT_MAX_PAIRS = 1 << 20

_lib = None


def lib() -> ctypes.CDLL:
    """Load libgsx_b200.so (raises if it is absent: build it with gsx_b200.build())."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise GsxError(NOT_SUPPORTED, f"{LIB_PATH} is missing; build the CUDA library first (gsx_b200.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int):
    if rc != 0:
        raise GsxError(rc, lib().gsx_b200_last_error().decode(errors="replace"))
