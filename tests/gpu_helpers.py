"""Helpers shared by the GPU parity tests: torch device copies of numpy scenes and a one-call render."""
import numpy as np
import torch

import gsx_b200 as gb


def to_dev(g, device="cuda:0"):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in g.items()}


def zeros_like_fields(gd):
    return {k: torch.zeros_like(v) for k, v in gd.items()}


def render(ctx, gd, cam, sh_degree=0, bg=(0.0, 0.0, 0.0), train=True):
    out = torch.empty((3, cam.height, cam.width), dtype=torch.float32, device="cuda:0")
    gb.Renderer(cam.width, cam.height).render(ctx, gd, cam, out, background=bg, sh_degree=sh_degree,
                                              forward_type=gb.FORWARD_TRAIN if train else gb.FORWARD_INFERENCE)
    return out


def fetch_view(ctx, n):
    """Copy the last forward's intermediates (keys, values, ranges, offsets, tile_max, pixel state) to numpy."""
    torch.cuda.synchronize()
    v = ctx.view()
    import ctypes

    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]

    def dev_to_np(ptr, count, dtype):
        out = np.empty(count, dtype)
        if count:
            assert rt.cudaMemcpy(out.ctypes.data, ptr, out.nbytes, 2) == 0
        return out

    I = int(v.n_instances)
    return dict(keys=dev_to_np(v.keys, I, np.uint64), vals=dev_to_np(v.values, I, np.uint32),
                ranges=dev_to_np(v.ranges, 2 * v.n_tiles, np.uint32).reshape(-1, 2),
                offsets=dev_to_np(v.offsets, n + 1, np.uint32), tile_max=dev_to_np(v.tile_max, v.n_tiles, np.uint32))


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))
