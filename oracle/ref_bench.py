"""Timed training steps of the REFERENCE CPU backend (test/baseline infrastructure only).

Used by bench.py for its `cpu_baseline` leg and for `--impl reference`.  The reference library is
built unmodified from the reference sources (oracle/Makefile.ref) and driven through its public C
API (oracle/ref_driver.c), one training step = render TRAIN, L1 + SSIM forward and backward,
render backward, Adam over every group (gsx-runtime.c:1413-1536 without density control).

The reference CPU backend is single-threaded scalar C, so "all host threads" means one independent
process per core, each training on its own view.  Its render backward keeps every
(Gaussian, pixel) contribution in one scratch tensor whose size must stay below 2^31 bytes
(gsx-cpu/render.c:156-169, sized at :1447-1453); the full 3M-Gaussian workload exceeds that, so
each step trains on a seeded 1/`subset` sample of the scene's Gaussians at the full image size,
and throughput is scaled to the full workload as views/s x (sample Gaussians / all Gaussians).
"""
from __future__ import annotations

import multiprocessing as mp
import os
import sys
import time

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def available() -> bool:
    return os.path.exists(os.path.join(_ROOT, "oracle", "_ref", "libgsx_refdrv_cpu.so"))


def _worker(args):
    rank, steps, warmup, subset, seed = args
    if _ROOT not in sys.path:
        sys.path.insert(0, _ROOT)
    import numpy as np

    from gsx_b200 import scenes
    from oracle import pyoracle as po

    full = scenes.config3_scene(seed)
    n_full = full["mean3d"].shape[0]
    pick = np.random.default_rng(seed + 17).permutation(n_full)[: n_full // subset]
    pick.sort()
    g = {k: np.ascontiguousarray(v[pick]) for k, v in full.items()}
    teach = {k: np.ascontiguousarray(v[pick]) for k, v in scenes.teacher(full).items()}
    cams = scenes.config3_cameras()
    c = cams[rank % len(cams)]
    oc = po.Camera(c.width, c.height, c.fx, c.fy, c.cx, c.cy, c.rot_xyzw, c.transl, c.near_plane, c.far_plane)
    devnull = os.open(os.devnull, os.O_WRONLY)
    os.dup2(devnull, 1)  # the reference library logs object creation on stdout
    target = po.RefSession("cpu", teach, oc, np.zeros((3, c.height, c.width), np.float32)).render()
    sess = po.RefSession("cpu", g, oc, target)
    for _ in range(warmup):
        sess.step()
    t0 = time.perf_counter()
    for _ in range(steps):
        sess.step()
    return time.perf_counter() - t0, len(pick), n_full


def run(steps: int, warmup: int, processes: int | None = None, subset: int = 16, seed: int = 0) -> dict:
    """Run `processes` independent reference-CPU trainers; returns views/s scaled to the full workload."""
    processes = processes or os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    t0 = time.perf_counter()
    with ctx.Pool(processes) as pool:
        res = pool.map(_worker, [(r, steps, warmup, subset, seed) for r in range(processes)])
    wall = time.perf_counter() - t0
    slowest = max(r[0] for r in res)
    n_sample, n_full = res[0][1], res[0][2]
    sample_views_per_s = processes * steps / slowest
    import platform
    cpu = platform.processor() or "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return dict(value=sample_views_per_s * n_sample / n_full, sample_views_per_s=sample_views_per_s,
                seconds_per_step=slowest / steps, processes=processes, n_sample=n_sample, n_full=n_full,
                wall_s=wall, cpu=cpu)


if __name__ == "__main__":
    print(run(int(sys.argv[1]) if len(sys.argv) > 1 else 1, 0, int(sys.argv[2]) if len(sys.argv) > 2 else 2))
