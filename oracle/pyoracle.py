"""numpy front-end for the C oracle (oracle/gsx_oracle.c) and the reference-library driver.

TEST INFRASTRUCTURE ONLY.  Importable from tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs as the checker; the product package never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(_HERE)
_LIB = os.path.join(_HERE, "_build", "libgsx_oracle.so")
_REF_DIR = os.path.join(_HERE, "_ref")

F32P = ctypes.POINTER(ctypes.c_float)
U32P = ctypes.POINTER(ctypes.c_uint32)
U64P = ctypes.POINTER(ctypes.c_uint64)


def _p(a, t=F32P):
    if a is None:
        return None
    return a.ctypes.data_as(t)


class _Camera(ctypes.Structure):
    _fields_ = [("w2c", ctypes.c_float * 12), ("cam_pos", ctypes.c_float * 3),
                ("fx", ctypes.c_float), ("fy", ctypes.c_float), ("cx", ctypes.c_float), ("cy", ctypes.c_float),
                ("width", ctypes.c_int), ("height", ctypes.c_int),
                ("near_plane", ctypes.c_float), ("far_plane", ctypes.c_float)]


_lib = None


def build():
    """Compile the oracle (gcc, -ffp-contract=off) into oracle/_build."""
    subprocess.run(["make", "-s", "-f", "oracle/Makefile"], cwd=_ROOT, check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build()
        L = ctypes.CDLL(_LIB)
        L.orc_preprocess.restype = ctypes.c_uint64
        L.orc_preprocess_aux.restype = ctypes.c_uint64
        L.orc_ssim.restype = ctypes.c_int
        L.orc_sort_pairs.restype = ctypes.c_int
        _lib = L
    return _lib


@dataclass
class Camera:
    """Pinhole camera: world->camera pose (quaternion xyzw + translation) and intrinsics."""
    width: int
    height: int
    fx: float
    fy: float
    cx: float
    cy: float
    q: tuple = (0.0, 0.0, 0.0, 1.0)
    t: tuple = (0.0, 0.0, 0.0)
    near: float = 0.01
    far: float = 1000.0

    def c_struct(self) -> _Camera:
        c = _Camera()
        q = np.asarray(self.q, np.float32)
        t = np.asarray(self.t, np.float32)
        w2c = np.zeros(12, np.float32)
        pos = np.zeros(3, np.float32)
        lib().orc_pose_to_camera(_p(q), _p(t), _p(w2c), _p(pos))
        c.w2c[:] = w2c.tolist()
        c.cam_pos[:] = pos.tolist()
        c.fx, c.fy, c.cx, c.cy = self.fx, self.fy, self.cx, self.cy
        c.width, c.height = self.width, self.height
        c.near_plane, c.far_plane = self.near, self.far
        return c


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def render_forward(g: dict, cam: Camera, sh_degree: int = 0, bg=(0.0, 0.0, 0.0)):
    """Full forward restatement.  Returns a dict with every intermediate the GPU path exposes."""
    L = lib()
    n = int(g["mean3d"].shape[0])
    mean3d, rot, logscale, op, sh0 = (_f32(g[k]) for k in ("mean3d", "rotation", "logscale", "opacity", "sh0"))
    sh = [_f32(g[k]) if sh_degree >= i + 1 else None for i, k in enumerate(("sh1", "sh2", "sh3"))]
    c = cam.c_struct()
    n_touched = np.zeros(n, np.uint32)
    bounds = np.zeros(n * 4, np.uint32)
    mean2d = np.zeros(n * 2, np.float32)
    conic_op = np.zeros(n * 4, np.float32)
    color = np.zeros(n * 3, np.float32)
    depth = np.zeros(n, np.float32)
    screen_radius = np.zeros(n, np.float32)
    total = L.orc_preprocess_aux(ctypes.c_int64(n), _p(mean3d), _p(rot), _p(logscale), _p(op), _p(sh0),
                                 _p(sh[0]), _p(sh[1]), _p(sh[2]), ctypes.c_int(sh_degree), ctypes.byref(c),
                                 _p(n_touched, U32P), _p(bounds, U32P), _p(mean2d), _p(conic_op), _p(color), _p(depth),
                                 _p(screen_radius))
    keys = np.zeros(max(total, 1), np.uint64)
    vals = np.zeros(max(total, 1), np.uint32)
    L.orc_emit(ctypes.c_int64(n), _p(n_touched, U32P), _p(bounds, U32P), _p(mean2d), _p(conic_op), _p(depth),
               ctypes.c_int(cam.width), _p(keys, U64P), _p(vals, U32P))
    keys, vals = keys[:total], vals[:total]
    unsorted_keys, unsorted_vals = keys.copy(), vals.copy()
    L.orc_sort_pairs(ctypes.c_uint64(total), _p(keys, U64P), _p(vals, U32P))
    gw = (cam.width + 15) // 16
    gh = (cam.height + 15) // 16
    n_tiles = gw * gh
    ranges = np.zeros(n_tiles * 2, np.uint32)
    L.orc_tile_ranges(ctypes.c_uint64(total), _p(keys, U64P), ctypes.c_int(n_tiles), _p(ranges, U32P))
    P = cam.width * cam.height
    out_rgb = np.zeros(3 * P, np.float32)
    out_alpha = np.zeros(P, np.float32)
    n_contrib = np.zeros(P, np.uint32)
    tile_max = np.zeros(n_tiles, np.uint32)
    bgv = np.asarray(bg, np.float32)
    L.orc_blend_forward(ctypes.c_int(cam.width), ctypes.c_int(cam.height), _p(ranges, U32P), _p(vals, U32P),
                        _p(mean2d), _p(conic_op), _p(color), _p(bgv), _p(out_rgb), _p(out_alpha),
                        _p(n_contrib, U32P), _p(tile_max, U32P))
    return dict(n_touched=n_touched, bounds=bounds.reshape(n, 4), mean2d=mean2d.reshape(n, 2),
                conic_op=conic_op.reshape(n, 4), color=color.reshape(n, 3), depth=depth, screen_radius=screen_radius,
                n_instances=int(total), unsorted_keys=unsorted_keys, unsorted_vals=unsorted_vals,
                keys=keys, vals=vals, ranges=ranges.reshape(n_tiles, 2),
                rgb=out_rgb.reshape(3, cam.height, cam.width), alpha=out_alpha.reshape(cam.height, cam.width),
                n_contrib=n_contrib.reshape(cam.height, cam.width), tile_max=tile_max, _raw=dict(
                    mean2d=mean2d, conic_op=conic_op, color=color, ranges=ranges, vals=vals, rgb=out_rgb,
                    n_contrib=n_contrib, tile_max=tile_max, n_touched=n_touched))


def render_backward(g: dict, cam: Camera, fwd: dict, grad_rgb, sh_degree: int = 0):
    """Backward restatement; returns the parameter gradients (and the 2-D helper gradients)."""
    L = lib()
    n = int(g["mean3d"].shape[0])
    r = fwd["_raw"]
    grad_rgb = _f32(grad_rgb).reshape(-1)
    d_mean2d = np.zeros(n * 2, np.float32)
    d_conic = np.zeros(n * 3, np.float32)
    d_op = np.zeros(n, np.float32)
    d_color = np.zeros(n * 3, np.float32)
    d_mean2d_abs = np.zeros(n * 2, np.float32)
    L.orc_blend_backward_abs(ctypes.c_int(cam.width), ctypes.c_int(cam.height), _p(r["ranges"], U32P), _p(r["vals"], U32P),
                         _p(r["mean2d"]), _p(r["conic_op"]), _p(r["color"]), _p(r["rgb"]), _p(r["n_contrib"], U32P),
                         _p(r["tile_max"], U32P), _p(grad_rgb), _p(d_mean2d), _p(d_conic), _p(d_op), _p(d_color),
                         _p(d_mean2d_abs))
    c = cam.c_struct()
    mean3d, rot, logscale = (_f32(g[k]) for k in ("mean3d", "rotation", "logscale"))
    sh = [_f32(g[k]) if sh_degree >= i + 1 else None for i, k in enumerate(("sh1", "sh2", "sh3"))]
    out = dict(mean3d=np.zeros((n, 3), np.float32), rotation=np.zeros((n, 4), np.float32),
               logscale=np.zeros((n, 3), np.float32), opacity=np.zeros(n, np.float32), sh0=np.zeros((n, 3), np.float32))
    gsh = [np.zeros((n, k, 3), np.float32) if sh_degree >= i + 1 else None for i, k in enumerate((3, 5, 7))]
    L.orc_preprocess_backward(ctypes.c_int64(n), _p(mean3d), _p(rot), _p(logscale), _p(sh[0]), _p(sh[1]), _p(sh[2]),
                              ctypes.c_int(sh_degree), ctypes.byref(c), _p(r["n_touched"], U32P), _p(d_mean2d),
                              _p(d_conic), _p(d_color), _p(d_op), _p(out["mean3d"]), _p(out["rotation"]),
                              _p(out["logscale"]), _p(out["opacity"]), _p(out["sh0"]), _p(gsh[0]), _p(gsh[1]), _p(gsh[2]))
    for i, k in enumerate(("sh1", "sh2", "sh3")):
        if gsh[i] is not None:
            out[k] = gsh[i]
    out["_helpers"] = dict(mean2d=d_mean2d.reshape(n, 2), conic=d_conic.reshape(n, 3), opacity=d_op,
                           color=d_color.reshape(n, 3), mean2d_abs=d_mean2d_abs.reshape(n, 2))
    return out


def aux_forward(fwd: dict, visible_counter, max_screen_radius):
    """Fold one TRAIN forward into the density-control accumulators (in place, f32):
    visible_counter += 1 and max_screen_radius = max(., radius) for every tile-touching Gaussian
    (gsx-metal/kernels/render.metal:425-439)."""
    vis = fwd["n_touched"] > 0
    visible_counter[vis] += np.float32(1.0)
    max_screen_radius[vis] = np.maximum(max_screen_radius[vis], fwd["screen_radius"][vis])


def aux_backward(bwd: dict, cam: "Camera", grad_acc, absgrad_acc):
    """Fold one backward into grad_acc / absgrad_acc (in place, f32): the norms of the screen-space
    mean gradient and of the per-pixel absolute gradient, scaled by (W/2, H/2)
    (gsx-metal/kernels/render_backward.metal:700-714)."""
    scale = np.array([0.5 * cam.width, 0.5 * cam.height], np.float32)
    g = bwd["_helpers"]["mean2d"].astype(np.float32) * scale
    a = bwd["_helpers"]["mean2d_abs"].astype(np.float32) * scale
    grad_acc += np.sqrt((g * g).sum(1)).astype(np.float32)
    absgrad_acc += np.sqrt((a * a).sum(1)).astype(np.float32)


def sort_pairs(keys, vals):
    keys = np.ascontiguousarray(keys, np.uint64).copy()
    vals = np.ascontiguousarray(vals, np.uint32).copy()
    lib().orc_sort_pairs(ctypes.c_uint64(keys.size), _p(keys, U64P), _p(vals, U32P))
    return keys, vals


def l1_ssim_train(pred, target, l1_weight=0.8, ssim_weight=0.2, loss_map=None, grad=None, normalization="mean"):
    """The training loss pair in the order the reference session issues it (gsx-runtime.c:1496-1510):
    L1 forward, SSIM forward, L1 backward, SSIM backward, MEAN grad normalisation (scale / numel)."""
    pred = _f32(pred)
    target = _f32(target)
    shp = pred.shape
    outer = int(np.prod(shp[:-3])) if len(shp) > 3 else 1
    C, H, W = shp[-3:]
    n = pred.size
    lm = np.zeros(n, np.float32) if loss_map is None else _f32(loss_map).reshape(-1).copy()
    gr = np.zeros(n, np.float32) if grad is None else _f32(grad).reshape(-1).copy()
    L = lib()
    norm = (1.0 / n) if normalization == "mean" else 1.0
    pf, tf = pred.reshape(-1), target.reshape(-1)
    L.orc_l1_forward(ctypes.c_int64(n), _p(pf), _p(tf), _p(lm), ctypes.c_float(l1_weight))
    L.orc_ssim(ctypes.c_int64(outer), C, H, W, _p(pf), _p(tf), _p(lm), ctypes.c_float(ssim_weight), None, ctypes.c_float(0))
    L.orc_l1_backward(ctypes.c_int64(n), _p(pf), _p(tf), _p(gr), ctypes.c_float(np.float32(l1_weight) / np.float32(n) if normalization == "mean" else l1_weight))
    L.orc_ssim(ctypes.c_int64(outer), C, H, W, _p(pf), _p(tf), None, ctypes.c_float(0),
               _p(gr), ctypes.c_float(np.float32(ssim_weight) / np.float32(n) if normalization == "mean" else ssim_weight))
    del norm
    return lm.reshape(shp), gr.reshape(shp)


def ssim(pred, target, loss_scale=1.0, grad_scale=None, loss_map=None, grad=None):
    pred = _f32(pred)
    target = _f32(target)
    shp = pred.shape
    outer = int(np.prod(shp[:-3])) if len(shp) > 3 else 1
    C, H, W = shp[-3:]
    lm = np.zeros(pred.size, np.float32) if loss_map is None else _f32(loss_map).reshape(-1).copy()
    gr = None
    if grad_scale is not None:
        gr = np.zeros(pred.size, np.float32) if grad is None else _f32(grad).reshape(-1).copy()
    lib().orc_ssim(ctypes.c_int64(outer), C, H, W, _p(pred.reshape(-1)), _p(target.reshape(-1)), _p(lm),
                   ctypes.c_float(loss_scale), _p(gr), ctypes.c_float(grad_scale or 0.0))
    return lm.reshape(shp), (gr.reshape(shp) if gr is not None else None)


def adam(param, grad, m1, m2, step, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, max_grad=0.0):
    """One Adam step in place (param, m1, m2 are float32 arrays); `step` is the 1-based step count."""
    inv1 = 1.0 / (1.0 - float(np.float32(beta1)) ** step)
    inv2 = 1.0 / (1.0 - float(np.float32(beta2)) ** step)
    lib().orc_adam(ctypes.c_int64(param.size), _p(param), _p(_f32(grad)), _p(m1), _p(m2), ctypes.c_float(beta1),
                   ctypes.c_float(beta2), ctypes.c_float(lr), ctypes.c_float(weight_decay), ctypes.c_float(eps),
                   ctypes.c_float(max_grad), ctypes.c_double(inv1), ctypes.c_double(inv2))


# ------------------------------------------------------------------ reference library driver
_ref = {}


def ref_available(kind: str = "cpu") -> bool:
    return os.path.exists(os.path.join(_REF_DIR, f"libgsx_refdrv_{kind}.so"))


def ref(kind: str = "cpu"):
    """The reference GSX library built from its own sources (oracle/Makefile.ref), via oracle/ref_driver.c."""
    if kind not in _ref:
        L = ctypes.CDLL(os.path.join(_REF_DIR, f"libgsx_refdrv_{kind}.so"))
        L.refdrv_message.restype = ctypes.c_char_p
        rc = L.refdrv_init(0 if kind == "cpu" else 1)
        if rc != 0:
            raise RuntimeError(f"reference init failed: {L.refdrv_message().decode()}")
        _ref[kind] = L
    return _ref[kind]


def _ref_check(L, rc):
    if rc != 0:
        raise RuntimeError(f"reference call failed ({rc}): {L.refdrv_message().decode()}")


def ref_loss(kind, algorithm, pred, target, scale, normalization=0, loss_map=None, grad=None):
    L = ref(kind)
    pred = _f32(pred)
    shp = pred.shape
    if pred.ndim == 3:
        outer, (C, H, W) = 1, shp
    else:
        outer, C, H, W = shp
    lm = np.zeros(pred.size, np.float32) if loss_map is None else _f32(loss_map).reshape(-1).copy()
    gr = np.zeros(pred.size, np.float32) if grad is None else _f32(grad).reshape(-1).copy()
    _ref_check(L, L.refdrv_loss(algorithm, normalization, outer, C, H, W, _p(pred.reshape(-1)),
                                _p(_f32(target).reshape(-1)), ctypes.c_float(scale), _p(lm), _p(gr)))
    return lm.reshape(shp), gr.reshape(shp)


def ref_adam(kind, param, grad, steps, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, max_grad=0.0):
    L = ref(kind)
    p = _f32(param).copy()
    _ref_check(L, L.refdrv_adam(ctypes.c_int64(p.size), _p(p), _p(_f32(grad)), steps, ctypes.c_float(lr),
                                ctypes.c_float(beta1), ctypes.c_float(beta2), ctypes.c_float(eps),
                                ctypes.c_float(weight_decay), ctypes.c_float(max_grad)))
    return p


class RefSession:
    """A reference-library training session (render + L1/SSIM + Adam) on the CPU or CUDA backend."""

    FIELDS = ("mean3d", "logscale", "rotation", "opacity", "sh0", "sh1", "sh2", "sh3")

    def __init__(self, kind, g, cam: Camera, target, sh_degree=0, bg=(0, 0, 0), lr=(1e-3, 1e-2, 1e-2, 1e-2, 1e-2, 1e-2, 1e-2, 1e-2)):
        self.L = ref(kind)
        self.g = {k: _f32(v) for k, v in g.items()}
        self.cam = cam
        self.sh_degree = sh_degree
        self.n = int(g["mean3d"].shape[0])
        self.h = ctypes.c_void_p()
        sh = [self.g.get(k) if sh_degree >= i + 1 else None for i, k in enumerate(("sh1", "sh2", "sh3"))]
        q = np.asarray(cam.q, np.float32)
        t = np.asarray(cam.t, np.float32)
        bgv = np.asarray(bg, np.float32)
        lrv = np.asarray(lr, np.float32)
        self._keep = (q, t, bgv, lrv, _f32(target))
        _ref_check(self.L, self.L.refdrv_session_create(
            ctypes.byref(self.h), ctypes.c_int64(self.n), _p(self.g["mean3d"]), _p(self.g["rotation"]),
            _p(self.g["logscale"]), _p(self.g["opacity"]), _p(self.g["sh0"]), _p(sh[0]), _p(sh[1]), _p(sh[2]),
            sh_degree, cam.width, cam.height, ctypes.c_float(cam.fx), ctypes.c_float(cam.fy), ctypes.c_float(cam.cx),
            ctypes.c_float(cam.cy), _p(q), _p(t), ctypes.c_float(cam.near), ctypes.c_float(cam.far), _p(bgv),
            _p(self._keep[4]), _p(lrv)))

    def render(self):
        out = np.zeros(3 * self.cam.width * self.cam.height, np.float32)
        _ref_check(self.L, self.L.refdrv_session_render(self.h, _p(out)))
        return out.reshape(3, self.cam.height, self.cam.width)

    def render_backward(self, grad_rgb):
        out = np.zeros(3 * self.cam.width * self.cam.height, np.float32)
        cols = (3, 3, 4, 1, 3, 9, 15, 21)
        nf = 5 + self.sh_degree
        grads = [np.zeros(self.n * cols[f], np.float32) for f in range(nf)]
        arr = (F32P * nf)(*[_p(x) for x in grads])
        _ref_check(self.L, self.L.refdrv_session_render_backward(self.h, _p(_f32(grad_rgb).reshape(-1)), _p(out), arr))
        res = {self.FIELDS[f]: grads[f] for f in range(nf)}
        return out.reshape(3, self.cam.height, self.cam.width), res

    def set_borrow(self, on=True):
        """TRAIN requests borrow the Gaussian tensors (borrow_train_state) instead of cloning them."""
        _ref_check(self.L, self.L.refdrv_session_set_borrow(self.h, 1 if on else 0))

    def mutate_backward(self, grad_rgb, mutated: dict):
        """TRAIN forward, overwrite the fields in `mutated` (numpy arrays), then the backward of grad_rgb;
        returns the parameter gradients (the ordering of the reference's train-state tests)."""
        cols = (3, 3, 4, 1, 3, 9, 15, 21)
        nf = 5 + self.sh_degree
        keep = [_f32(mutated[self.FIELDS[f]]).reshape(-1) if self.FIELDS[f] in mutated else None for f in range(nf)]
        mp = (F32P * nf)(*[_p(x) if x is not None else None for x in keep])
        grads = [np.zeros(self.n * cols[f], np.float32) for f in range(nf)]
        arr = (F32P * nf)(*[_p(x) for x in grads])
        _ref_check(self.L, self.L.refdrv_session_mutate_backward(self.h, _p(_f32(grad_rgb).reshape(-1)), mp, arr))
        return {self.FIELDS[f]: grads[f] for f in range(nf)}

    def step(self, l1_weight=0.8, ssim_weight=0.2):
        sec = ctypes.c_double()
        _ref_check(self.L, self.L.refdrv_session_step(self.h, ctypes.c_float(l1_weight), ctypes.c_float(ssim_weight),
                                                      ctypes.byref(sec)))
        return sec.value

    def enable_aux(self, on=True):
        """Bind the session's [N] density-control accumulators (zero at creation) on later calls."""
        _ref_check(self.L, self.L.refdrv_session_enable_aux(self.h, 1 if on else 0))

    def aux(self):
        """(visible_counter, max_screen_radius, grad_acc, absgrad_acc) as numpy arrays."""
        return tuple(self.download(11 + k, self.n) for k in range(4))

    def download(self, which: int, size: int):
        out = np.zeros(size, np.float32)
        _ref_check(self.L, self.L.refdrv_session_download(self.h, which, _p(out)))
        return out


def pack_hwc_to_chw(src):
    """Dataloader packing to f32 CHW: gsx_dataloader_pack_hwc_to_chw / pack_hw_to_chw with f32 output
    (gsx/src/gsx-data-impl.h:174-182 read_source_value, :212-240, :242-260): element (y, x, c) of the
    HWC source goes to (c, y, x), u8 values converted exactly to float, f32 copied."""
    a = np.asarray(src)
    if a.ndim == 2:
        a = a[:, :, None]
    return np.ascontiguousarray(np.transpose(a, (2, 0, 1)).astype(np.float32))


ADC_FIELDS = ("mean3d", "logscale", "rotation", "opacity", "sh0")
_ADC_COLS = (3, 3, 4, 1, 3)


def ref_adc_run(kind: str, g: dict, aux: dict, grads: dict, fparams, iparams, cap: int = None):
    """One density-control step of the reference GSX library (oracle/ref_driver.c refdrv_adc_run) on
    backend `kind`: returns (result dict, fields after ADC, fields after the following Adam step,
    statistics after ADC)."""
    L = ref(kind)
    n = int(g["mean3d"].shape[0])
    cap = cap or 2 * n + 1
    keep = [_f32(g[k]) for k in ADC_FIELDS] + [_f32(aux[k]) for k in ("grad_acc", "visible_counter", "max_screen_radius")]
    gr = [_f32(grads[k]) for k in ADC_FIELDS]
    fp = np.asarray(fparams, np.float32)
    ip = np.asarray(iparams, np.int64)
    res = np.zeros(7, np.int64)
    after = [np.zeros(cap * c, np.float32) for c in _ADC_COLS]
    final = [np.zeros(cap * c, np.float32) for c in _ADC_COLS]
    aux_out = [np.zeros(cap, np.float32) for _ in range(3)]
    arr = lambda xs: (F32P * len(xs))(*[_p(x) for x in xs])
    L.refdrv_adc_run.argtypes = None
    _ref_check(L, L.refdrv_adc_run(ctypes.c_int64(n), *[_p(x) for x in keep], arr(gr), _p(fp),
                                   ip.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                   res.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), ctypes.c_int64(cap),
                                   arr(after), arr(final), arr(aux_out)))
    m = int(res[1])
    r = dict(zip(("before", "after", "pruned", "duplicated", "grown", "reset", "mutated"), (int(v) for v in res)))
    shape = lambda c: (m, c) if c > 1 else (m,)
    fa = {k: after[i][:m * c].reshape(shape(c)) for i, (k, c) in enumerate(zip(ADC_FIELDS, _ADC_COLS))}
    ff = {k: final[i][:m * c].reshape(shape(c)) for i, (k, c) in enumerate(zip(ADC_FIELDS, _ADC_COLS))}
    fx = {k: aux_out[i][:m] for i, k in enumerate(("grad_acc", "visible_counter", "max_screen_radius"))}
    return r, fa, ff, fx


def _adc_variate(seed, step, grow_index, lane):
    """The split offset variate of gsx-cuda/adc.cu:582-599: a hashed uniform (u32 arithmetic) mapped
    through the logistic quantile, in float32."""
    M = 0xFFFFFFFF
    key = (int(seed) ^ ((int(step) * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF)) & M
    x = (key ^ (int(grow_index) & M) ^ ((lane * 0x9E3779B9 + 0x85EBCA6B) & M)) & M
    x ^= x >> 16
    x = (x * 0x7FEB352D) & M
    x ^= x >> 15
    x = (x * 0x846CA68B) & M
    x ^= x >> 16
    u = (np.float32(x) + np.float32(1.0)) / np.float32(4294967297.0)
    u = min(max(u, np.float32(1e-6)), np.float32(1.0) - np.float32(1e-6))
    return np.float32(np.log(np.float32(u / (np.float32(1.0) - u))))


def adc_step(g: dict, aux: dict, fparams, iparams, grads=None):
    """Restatement of GSX's CUDA default density control step (gsx-cuda/adc.cu:990-1040 with the refine
    pass :707-946 and the reset :292-331), float32 numpy.  g: mean3d/logscale/rotation/opacity/sh0;
    aux: grad_acc/visible_counter/max_screen_radius.  Returns (result dict, new fields, new aux, the
    row index each output row was gathered from (-1 for none: gathering composes), split rows)."""
    f32 = np.float32
    (op_thr, clamp_v, max_ws, max_ss, dup_thr, dup_scale, scene) = [f32(v) for v in fparams]
    refine_every, start, end, max_n, reset_every, seed, step = (int(v) for v in iparams)
    g = {k: np.array(v, np.float32, copy=True) for k, v in g.items()}
    aux = {k: np.array(v, np.float32, copy=True) for k, v in aux.items()}
    n0 = g["mean3d"].shape[0]
    origin = np.arange(n0)
    split_flag = np.zeros(n0, bool)
    res = dict(before=n0, after=n0, pruned=0, duplicated=0, grown=0, reset=0, mutated=0)
    nn = lambda v: max(v, 0)
    refine = refine_every != 0 and step % refine_every == 0 and nn(start) <= step <= nn(end)
    reset = reset_every != 0 and step % reset_every == 0 and nn(start) <= step < nn(end)

    def gather(idx):
        nonlocal origin, split_flag
        for d in (g, aux):
            for k in d:
                d[k] = d[k][idx]
        origin = origin[idx]
        split_flag = split_flag[idx]

    def max_scale(ls):
        return np.exp(ls).max(axis=1)

    if refine and n0 > 0:
        budget = max(nn(max_n) - n0, 0)
        if budget > 0:
            counter = aux["visible_counter"] if "visible_counter" in aux else np.ones(n0, f32)
            grad = aux["grad_acc"] / np.maximum(counter, f32(1.0))
            grow_on = (counter > 0) & (grad > dup_thr)
            split_on = grow_on & (max_scale(g["logscale"]) > f32(dup_scale * scene))
            modes = np.where(split_on, 2, np.where(grow_on, 1, 0))
            cand = np.nonzero(modes)[0]
            grow = min(len(cand), budget)
            if grow > 0:
                cand = cand[:grow]
                nsplit = int((modes[cand] == 2).sum())
                gather(np.concatenate([np.arange(n0), cand]))
                for gi, src in enumerate(cand):
                    if modes[src] != 2:
                        continue
                    dst = n0 + gi
                    s = np.exp(g["logscale"][src]).astype(f32)
                    so = f32(1.0) / (f32(1.0) + np.exp(-g["opacity"][src]))
                    r = [_adc_variate(seed, step, gi, l) for l in range(6)]
                    q = g["rotation"][src].astype(f32)
                    qn = np.sqrt(np.sum(q * q, dtype=f32))
                    if qn > f32(1e-8):
                        q = q * (f32(1.0) / qn)
                    qx, qy, qz, qw = q
                    R = np.array([[1 - 2 * (qy * qy + qz * qz), 2 * (qx * qy - qw * qz), 2 * (qx * qz + qw * qy)],
                                  [2 * (qx * qy + qw * qz), 1 - 2 * (qx * qx + qz * qz), 2 * (qy * qz - qw * qx)],
                                  [2 * (qx * qz - qw * qy), 2 * (qy * qz + qw * qx), 1 - 2 * (qx * qx + qy * qy)]], f32)
                    t1 = np.array(r[:3], f32) * (s + f32(1e-5))
                    t2 = np.array(r[3:], f32) * (s + f32(1e-5))
                    so = min(max(so, f32(0.0)), f32(1.0) - f32(1e-6))
                    sp = f32(1.0) - np.sqrt(f32(1.0) - so)
                    sp = min(max(sp, f32(1e-6)), f32(1.0) - f32(1e-6))
                    nl = np.log(s / f32(1.6)).astype(f32)
                    nop = f32(np.log(f32(sp / (f32(1.0) - sp))))
                    m = g["mean3d"][src].copy()
                    g["mean3d"][dst] = m + R @ t1
                    g["mean3d"][src] = m + R @ t2
                    g["logscale"][dst] = nl
                    g["logscale"][src] = nl
                    g["opacity"][dst] = nop
                    g["opacity"][src] = nop
                    split_flag[src] = split_flag[dst] = True
                res["duplicated"] += grow - nsplit
                res["grown"] += nsplit
                res["mutated"] = 1
        n1 = g["mean3d"].shape[0]
        op = f32(1.0) / (f32(1.0) + np.exp(-g["opacity"]))
        keep = (op > op_thr) & (np.abs(g["rotation"]).sum(1, dtype=f32) > np.finfo(np.float32).eps)
        if step > nn(reset_every):
            if max_ws > 0:
                keep &= max_scale(g["logscale"]) < f32(max_ws * scene)
            if max_ss > 0 and "max_screen_radius" in aux:
                keep &= ~((np.arange(n1) < n0) & ~(aux["max_screen_radius"] < max_ss))
        kept = np.nonzero(keep)[0]
        if len(kept) == 0:
            kept = np.array([0])
        if len(kept) < n1:
            gather(kept)
            res["pruned"] += n1 - len(kept)
            res["mutated"] = 1
        for k in ("grad_acc", "visible_counter", "max_screen_radius"):
            if k in aux:
                aux[k][:] = 0.0
    if reset:
        p = min(max(f32(clamp_v), f32(1e-6)), f32(1.0))
        p = min(max(p, f32(1e-6)), f32(1.0) - f32(1e-6))
        hi = f32(np.log(f32(p / (f32(1.0) - p))))
        g["opacity"] = np.where(g["opacity"] > hi, hi, g["opacity"]).astype(f32)
        res["reset"] = 1
        res["mutated"] = 1
    res["after"] = g["mean3d"].shape[0]
    if res["after"] != res["before"]:
        res["mutated"] = 1
    return res, g, aux, origin, np.nonzero(split_flag)[0]


def ref_session_fit(kind: str, g: dict, target_chw, cam: "Camera", fparams, iparams, steps: int, cap: int = None):
    """GSX's runtime session (gsx_session_step with L1 0.8 + SSIM 0.2, Adam, default ADC) on backend
    `kind` over a one-image dataset (oracle/ref_driver.c refdrv_session_fit).  Returns (mean loss
    per step, Gaussian count per step, final fields)."""
    L = ref(kind)
    n = int(g["mean3d"].shape[0])
    cap = cap or 8 * n
    keep = [_f32(g[k]) for k in ADC_FIELDS]
    hwc = np.ascontiguousarray(np.transpose(_f32(target_chw), (1, 2, 0)))
    c = np.array([cam.fx, cam.fy, cam.cx, cam.cy, *cam.q, *cam.t], np.float32)
    fp = np.asarray(fparams, np.float32)
    ip = np.asarray(iparams, np.int64)
    loss = np.zeros(steps, np.float32)
    count = np.zeros(steps, np.int64)
    out = [np.zeros(cap * k, np.float32) for k in _ADC_COLS]
    L.refdrv_session_fit.argtypes = None
    _ref_check(L, L.refdrv_session_fit(ctypes.c_int64(n), *[_p(x) for x in keep], _p(hwc), ctypes.c_int(cam.width),
                                       ctypes.c_int(cam.height), _p(c), _p(fp),
                                       ip.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), ctypes.c_int64(steps), _p(loss),
                                       count.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), ctypes.c_int64(cap),
                                       (F32P * 5)(*[_p(x) for x in out])))
    m = int(count[-1])
    fields = {k: out[i][:m * cc].reshape((m, cc) if cc > 1 else (m,)) for i, (k, cc) in enumerate(zip(ADC_FIELDS, _ADC_COLS))}
    return loss, count, fields
