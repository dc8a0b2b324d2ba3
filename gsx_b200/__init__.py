"""gsx_b200: a B200-native (sm_100a) backend for the GSX Gaussian-splatting hot path.

Host-side mirror of GSX's renderer / render-context / loss / optimizer interface
(gsx/include/gsx/gsx-render.h, gsx-loss.h, gsx-optim.h) over the C ABI in include/gsx_b200.h.
Tensors are torch CUDA tensors (device memory and streams only; every computation runs in the
library's own kernels).  Errors raise GsxError with the gsx_error_code of the failing call.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass, field

from ._capi import (AdamGroup, Camera as _CCamera, GaussianGrads as _CGrads, Gaussians as _CGaussians, GsxError,
                    RenderView, check, lib)
from ._capi import INVALID_ARGUMENT, INVALID_STATE, NOT_SUPPORTED, OUT_OF_RANGE  # noqa: F401

__all__ = ["GsxError", "Camera", "RenderContext", "Renderer", "Loss", "Adam", "ParamGroup", "l1_ssim",
           "sort_pairs", "build", "FORWARD_INFERENCE", "FORWARD_TRAIN", "FIELDS"]

FORWARD_INFERENCE = 0
FORWARD_TRAIN = 1
FIELDS = ("mean3d", "rotation", "logscale", "opacity", "sh0", "sh1", "sh2", "sh3")

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build(jobs: int = 8) -> None:
    """Compile libgsx_b200.so for sm_100a in-tree (nvcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-f", "gsx_b200/csrc/Makefile", f"-j{jobs}"], cwd=_ROOT, check=True)


def _stream_handle(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise GsxError(INVALID_ARGUMENT, "tensor must be on a CUDA device")
    if not t.is_contiguous():
        raise GsxError(INVALID_ARGUMENT, "tensor must be contiguous")
    import torch
    if t.dtype not in (torch.float32, torch.bfloat16, torch.uint8, torch.int64, torch.int32, torch.uint64, torch.uint32):
        raise GsxError(NOT_SUPPORTED, f"unsupported dtype {t.dtype}")
    return ctypes.c_void_p(t.data_ptr())


@dataclass
class Camera:
    """Pinhole camera (gsx_camera_intrinsics + gsx_camera_pose, world->camera, quaternion xyzw)."""
    width: int
    height: int
    fx: float
    fy: float
    cx: float
    cy: float
    rot_xyzw: tuple = (0.0, 0.0, 0.0, 1.0)
    transl: tuple = (0.0, 0.0, 0.0)
    near_plane: float = 0.01
    far_plane: float = 1000.0

    def c_struct(self) -> _CCamera:
        c = _CCamera()
        c.width, c.height = int(self.width), int(self.height)
        c.fx, c.fy, c.cx, c.cy = self.fx, self.fy, self.cx, self.cy
        c.rot_xyzw[:] = [float(v) for v in self.rot_xyzw]
        c.transl[:] = [float(v) for v in self.transl]
        c.near_plane, c.far_plane = self.near_plane, self.far_plane
        return c


class RenderContext:
    """gsx_render_context: owns the device scratch of one render stream (grown on demand)."""

    def __init__(self, device: int = 0):
        self.device = device
        h = ctypes.c_void_p()
        check(lib().gsx_b200_context_create(device, ctypes.byref(h)))
        self.handle = h
        self._keep = None

    def close(self):
        if self.handle:
            lib().gsx_b200_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, stream=None):
        """Synchronise and raise on device-side failures (timed-out waits, overflows)."""
        check(lib().gsx_b200_context_check(self.handle, _stream_handle(stream)))

    def stats(self, stream=None):
        v, i, b = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().gsx_b200_render_stats(self.handle, ctypes.byref(v), ctypes.byref(i), ctypes.byref(b),
                                          _stream_handle(stream)))
        return dict(n_visible=v.value, n_instances=i.value, n_buckets=b.value)

    def bind_aux(self, visible_counter=None, max_screen_radius=None, grad_acc=None, absgrad_acc=None):
        """Bind the [N] f32 density-control accumulators (None = unbound) for later TRAIN renders
        (visible_counter, max_screen_radius) and backwards (grad_acc, absgrad_acc)."""
        self._aux = (visible_counter, max_screen_radius, grad_acc, absgrad_acc)
        check(lib().gsx_b200_render_bind_aux(self.handle, _ptr(visible_counter), _ptr(max_screen_radius),
                                             _ptr(grad_acc), _ptr(absgrad_acc)))

    def set_train_state(self, borrowed: bool):
        """False (default): the TRAIN forward's state is retained and the caller must not change the
        Gaussians before the backward.  True: GSX's borrowed train state; the backward re-renders if the
        Gaussians changed since the forward (gsx_b200_context_set_train_state)."""
        check(lib().gsx_b200_context_set_train_state(self.handle, 1 if borrowed else 0))

    def train_refreshes(self) -> int:
        c = ctypes.c_uint64()
        check(lib().gsx_b200_context_train_refreshes(self.handle, ctypes.byref(c)))
        return int(c.value)

    def row_costs(self, gaussians: dict, camera: "Camera", stream=None):
        """Per tile row of the full frame, the integer work estimate of gsx_b200_render_row_costs
        (numpy uint32 array of ceil(height / 16) entries; waits for the stream)."""
        import numpy as np
        rows = (camera.height + 15) // 16
        out = np.zeros(rows, np.uint32)
        g = _c_gaussians(gaussians)
        cam = camera.c_struct()
        check(lib().gsx_b200_render_row_costs(self.handle, ctypes.byref(g), ctypes.byref(cam),
                                              out.ctypes.data_as(ctypes.c_void_p), rows, _stream_handle(stream)))
        return out

    def launch_count(self) -> int:
        """Kernels this context has launched since it was created (host-side count)."""
        c = ctypes.c_uint64()
        check(lib().gsx_b200_context_launch_count(self.handle, ctypes.byref(c)))
        return c.value

    def set_profiling(self, enable: bool = True):
        """Record per-stage CUDA events on the launching stream (see read_profile)."""
        check(lib().gsx_b200_context_set_profiling(self.handle, 1 if enable else 0))

    def read_profile(self) -> dict:
        """{stage: (total_ms, launches)} since the last read; synchronises."""
        from ._capi import STAGES
        ms = (ctypes.c_float * len(STAGES))()
        cnt = (ctypes.c_int32 * len(STAGES))()
        check(lib().gsx_b200_context_read_profile(self.handle, ms, cnt))
        return {s: (float(ms[i]), int(cnt[i])) for i, s in enumerate(STAGES)}

    def view(self) -> RenderView:
        v = RenderView()
        check(lib().gsx_b200_render_get_view(self.handle, ctypes.byref(v)))
        return v


def _c_gaussians(gaussians: dict):
    g = _CGaussians()
    g.count = int(gaussians["mean3d"].shape[0])
    for k in FIELDS:
        t = gaussians.get(k)
        setattr(g, k, _ptr(t).value if t is not None else None)
    return g


def hwc_to_chw(src, out=None, stream=None):
    """Dataloader layout conversion: a [H, W, 3] (or [H, W]) u8/f32 CUDA image to a [3, H, W] (or
    [1, H, W]) f32 tensor, values unchanged (gsx_b200_hwc_to_chw_f32)."""
    import torch
    if src.dim() not in (2, 3) or (src.dim() == 3 and src.shape[2] not in (1, 3)):
        raise GsxError(INVALID_ARGUMENT, "src must be [H, W, 3], [H, W, 1] or [H, W]")
    if src.dtype not in (torch.uint8, torch.float32):
        raise GsxError(NOT_SUPPORTED, "src must be uint8 or float32")
    c = 1 if src.dim() == 2 else int(src.shape[2])
    H, W = int(src.shape[0]), int(src.shape[1])
    if out is None:
        out = torch.empty((c, H, W), dtype=torch.float32, device=src.device)
    if tuple(out.shape) != (c, H, W) or out.dtype != torch.float32:
        raise GsxError(INVALID_ARGUMENT, "out must be a [C, H, W] float32 tensor")
    check(lib().gsx_b200_hwc_to_chw_f32(_ptr(src), 8 if src.dtype == torch.uint8 else 0, c, H * W, _ptr(out),
                                        _stream_handle(stream)))
    return out


def band_rows(height: int, rank: int, world_size: int):
    """Rows [begin, end) of a frame of `height` rows that rank `rank` of `world_size` renders: whole
    16-row tile rows dealt out as evenly as possible (earlier ranks take the remainder), so every
    band starts on a tile row; a rank with no tile row gets an empty band (begin == end)."""
    if height <= 0 or world_size <= 0 or not 0 <= rank < world_size:
        raise GsxError(INVALID_ARGUMENT, "band_rows: height, world_size positive and 0 <= rank < world_size")
    tiles = (height + 15) // 16
    base, extra = divmod(tiles, world_size)
    t0 = rank * base + min(rank, extra)
    t1 = t0 + base + (1 if rank < extra else 0)
    return min(16 * t0, height), min(16 * t1, height)


def balanced_band_rows(row_costs, height: int, rank: int, world_size: int):
    """Rows [begin, end) of rank `rank`'s band when the frame's tile rows are cut where the running sum
    of `row_costs` (one work estimate per tile row, RenderContext.row_costs) crosses k/world_size of the
    total, so the bands carry about equal work; whole tile rows, in order, covering [0, height).  Every
    rank that passes the same costs gets the same cut (integer arithmetic)."""
    if height <= 0 or world_size <= 0 or not 0 <= rank < world_size:
        raise GsxError(INVALID_ARGUMENT, "balanced_band_rows: height, world_size positive and 0 <= rank < world_size")
    tiles = (height + 15) // 16
    costs = [int(c) for c in row_costs]
    if len(costs) != tiles:
        raise GsxError(INVALID_ARGUMENT, "one cost per tile row")
    total = sum(costs)
    if total == 0:
        return band_rows(height, rank, world_size)
    cuts, run, k = [0], 0, 1
    for t, c in enumerate(costs):
        run += c
        while k < world_size and run * world_size >= k * total:
            cuts.append(t + 1)
            k += 1
    while len(cuts) < world_size:
        cuts.append(tiles)
    cuts.append(tiles)
    t0, t1 = cuts[rank], cuts[rank + 1]
    return min(16 * t0, height), min(16 * t1, height)


class Renderer:
    """gsx_renderer: a fixed output size; render()/backward() run on a RenderContext."""

    def __init__(self, width: int, height: int):
        if width <= 0 or height <= 0:
            raise GsxError(INVALID_ARGUMENT, "renderer size must be positive")
        self.width, self.height = int(width), int(height)

    def render(self, context: RenderContext, gaussians: dict, camera: Camera, out_rgb, background=(0.0, 0.0, 0.0),
               sh_degree: int = 0, forward_type: int = FORWARD_TRAIN, stream=None):
        """Forward render into out_rgb ([3,H,W] f32 CUDA tensor).  TRAIN retains state for backward()."""
        if camera.width != self.width or camera.height != self.height:
            raise GsxError(INVALID_ARGUMENT, "camera size must match the renderer size")
        if tuple(out_rgb.shape) != (3, self.height, self.width):
            raise GsxError(INVALID_ARGUMENT, "out_rgb must be [3, H, W]")
        g = _c_gaussians(gaussians)
        bg = (ctypes.c_float * 3)(*[float(v) for v in background])
        cam = camera.c_struct()
        context._keep = gaussians
        check(lib().gsx_b200_render_forward(context.handle, ctypes.byref(g), int(sh_degree), ctypes.byref(cam), bg,
                                            int(forward_type), _ptr(out_rgb), _stream_handle(stream)))
        return out_rgb

    def render_rows(self, context: RenderContext, gaussians: dict, camera: Camera, row_begin: int, row_end: int,
                    out, background=(0.0, 0.0, 0.0), sh_degree: int = 0, forward_type: int = FORWARD_TRAIN,
                    stream=None):
        """Rows [row_begin, row_end) of the full frame into out ([3, rows, W], f32 or bf16 CUDA tensor);
        bit-identical to those rows of render().  row_begin must be a multiple of 16."""
        import torch
        if camera.width != self.width or camera.height != self.height:
            raise GsxError(INVALID_ARGUMENT, "camera size must match the renderer size")
        if tuple(out.shape) != (3, int(row_end) - int(row_begin), self.width):
            raise GsxError(INVALID_ARGUMENT, "out must be [3, row_end - row_begin, W]")
        if out.dtype not in (torch.float32, torch.bfloat16):
            raise GsxError(INVALID_ARGUMENT, "out must be float32 or bfloat16")
        g = _c_gaussians(gaussians)
        bg = (ctypes.c_float * 3)(*[float(v) for v in background])
        cam = camera.c_struct()
        context._keep = gaussians
        check(lib().gsx_b200_render_forward_rows(context.handle, ctypes.byref(g), int(sh_degree), ctypes.byref(cam),
                                                 int(row_begin), int(row_end), bg, int(forward_type), _ptr(out),
                                                 1 if out.dtype == torch.bfloat16 else 0, _stream_handle(stream)))
        return out

    def backward(self, context: RenderContext, grad_rgb, grads: dict, stream=None):
        """Parameter gradients of the last TRAIN render on `context` (written, not accumulated)."""
        gr = _CGrads()
        for k in FIELDS:
            t = grads.get(k)
            setattr(gr, k, _ptr(t).value if t is not None else None)
        check(lib().gsx_b200_render_backward(context.handle, _ptr(grad_rgb), ctypes.byref(gr), _stream_handle(stream)))
        return grads


def l1_ssim(prediction, target, loss_map, grad, l1_weight=0.8, ssim_weight=0.2, normalization="mean",
            loss_sum=None, overwrite=False, stream=None):
    """The fused training loss: L1 and SSIM forward and backward in one kernel.

    Same result as GSX's L1 loss then SSIM loss forward, then L1 then SSIM backward
    (gsx-runtime.c:1496-1510): loss_map and grad are accumulated into (written when overwrite=True).  MEAN normalisation divides
    the gradient scales by numel(prediction) (gsx-tensor-helpers.h:236-244)."""
    n = prediction.numel()
    gs = (1.0 / n) if normalization == "mean" else 1.0
    planes = n // (prediction.shape[-1] * prediction.shape[-2])
    mode = 1 | (2 if grad is not None else 0) | 4 | (8 if overwrite else 0)
    l1g = float(_f32(l1_weight) / _f32(n)) if normalization == "mean" else l1_weight
    ssg = float(_f32(ssim_weight) / _f32(n)) if normalization == "mean" else ssim_weight
    del gs
    check(lib().gsx_b200_loss_l1_ssim(mode, _ptr(prediction), _ptr(target), _ptr(loss_map), _ptr(grad),
                                      _ptr(loss_sum), planes, prediction.shape[-2], prediction.shape[-1],
                                      float(l1_weight), float(ssim_weight), l1g, ssg, _stream_handle(stream)))


def _f32(x):
    import numpy as np
    return np.float32(x)


class Loss:
    """gsx_loss: algorithm "l1", "mse" or "ssim"; forward() retains prediction/target for one backward()."""

    ALGORITHMS = ("l1", "mse", "ssim")

    def __init__(self, algorithm: str, grad_normalization: str = "mean"):
        if algorithm not in self.ALGORITHMS:
            raise GsxError(OUT_OF_RANGE, f"loss algorithm must be one of {self.ALGORITHMS}")
        if grad_normalization not in ("mean", "sum"):
            raise GsxError(OUT_OF_RANGE, "grad_normalization must be 'mean' or 'sum'")
        self.algorithm = algorithm
        self.grad_normalization = grad_normalization
        self._retained = None

    def forward(self, prediction, target, loss_map, scale: float = 1.0, train: bool = True, stream=None):
        if prediction.shape != target.shape or prediction.shape != loss_map.shape:
            raise GsxError(INVALID_ARGUMENT, "prediction, target and loss_map must have the same shape")
        if self.algorithm == "ssim":
            if prediction.dim() < 3:
                raise GsxError(NOT_SUPPORTED, "ssim requires rank>=3 tensors")
            planes = prediction.numel() // (prediction.shape[-1] * prediction.shape[-2])
            check(lib().gsx_b200_loss_l1_ssim(1, _ptr(prediction), _ptr(target), _ptr(loss_map), None, None, planes,
                                              prediction.shape[-2], prediction.shape[-1], 0.0, float(scale), 0.0, 0.0,
                                              _stream_handle(stream)))
        else:
            op = 0 if self.algorithm == "l1" else 2
            check(lib().gsx_b200_loss_pointwise(op, _ptr(prediction), _ptr(target), _ptr(loss_map),
                                                prediction.numel(), float(scale), _stream_handle(stream)))
        self._retained = (prediction, target) if train else None

    def backward(self, grad_prediction, scale: float = 1.0, stream=None):
        if self._retained is None:
            raise GsxError(INVALID_STATE, "loss backward requires a retained train forward")
        prediction, target = self._retained
        self._retained = None
        n = prediction.numel()
        gs = float(_f32(scale) / _f32(n)) if self.grad_normalization == "mean" else float(scale)
        if self.algorithm == "ssim":
            planes = n // (prediction.shape[-1] * prediction.shape[-2])
            check(lib().gsx_b200_loss_l1_ssim(2, _ptr(prediction), _ptr(target), None, _ptr(grad_prediction), None,
                                              planes, prediction.shape[-2], prediction.shape[-1], 0.0, 0.0, 0.0, gs,
                                              _stream_handle(stream)))
        else:
            op = 1 if self.algorithm == "l1" else 3
            check(lib().gsx_b200_loss_pointwise(op, _ptr(prediction), _ptr(target), _ptr(grad_prediction), n, gs,
                                                _stream_handle(stream)))


@dataclass
class ParamGroup:
    """gsx_optim_param_group_desc (gsx-optim.h:60-71)."""
    role: str
    parameter: object
    gradient: object
    learning_rate: float
    beta1: float = 0.9
    beta2: float = 0.999
    weight_decay: float = 0.0
    epsilon: float = 1e-8
    max_grad: float = 0.0


class Adam:
    """gsx_optim (Adam): moment state per group; step() updates the selected groups in ONE launch."""

    ROLES = ("mean3d", "logscale", "rotation", "opacity", "sh0", "sh1", "sh2", "sh3")

    def __init__(self, groups: list):
        import torch
        if len(groups) > 16:
            raise GsxError(OUT_OF_RANGE, "at most 16 parameter groups")
        self.groups = list(groups)
        self.m1 = [torch.zeros_like(g.parameter) for g in self.groups]
        self.m2 = [torch.zeros_like(g.parameter) for g in self.groups]
        self.steps = [0] * len(self.groups)

    def reset(self):
        for i in range(len(self.groups)):
            self.m1[i].zero_()
            self.m2[i].zero_()
            self.steps[i] = 0

    def step(self, roles=None, force_all: bool = True, stream=None):
        sel = [i for i, g in enumerate(self.groups) if force_all or (roles is not None and g.role in roles)]
        arr = (AdamGroup * max(len(sel), 1))()
        for j, i in enumerate(sel):
            g = self.groups[i]
            self.steps[i] += 1
            t = self.steps[i]
            b1 = float(_f32(g.beta1))
            b2 = float(_f32(g.beta2))
            a = arr[j]
            a.parameter = _ptr(g.parameter).value
            a.gradient = _ptr(g.gradient).value
            a.first_moment = _ptr(self.m1[i]).value
            a.second_moment = _ptr(self.m2[i]).value
            a.count = g.parameter.numel()
            a.learning_rate, a.beta1, a.beta2 = g.learning_rate, g.beta1, g.beta2
            a.epsilon, a.weight_decay, a.max_grad = g.epsilon, g.weight_decay, g.max_grad
            a.inv_bias_correction1 = 1.0 / (1.0 - math.pow(b1, t))
            a.inv_bias_correction2 = 1.0 / (1.0 - math.pow(b2, t))
        check(lib().gsx_b200_adam_step(arr, len(sel), _stream_handle(stream)))


def sort_pairs(context: RenderContext, keys, values, begin_bit: int = 0, end_bit: int = 64, stream=None):
    """Stable in-place radix sort of int64/uint64 keys with int32/uint32 values by key bits [begin, end)."""
    if keys.numel() != values.numel():
        raise GsxError(INVALID_ARGUMENT, "keys and values must have the same length")
    check(lib().gsx_b200_sort_pairs(context.handle, _ptr(keys), _ptr(values), keys.numel(), begin_bit, end_bit,
                                    _stream_handle(stream)))
