"""Timed training steps of the REFERENCE CPU backend (test/baseline infrastructure only).

Used by bench.py for its `cpu_baseline` leg and for `--impl reference`.  The reference library is
built unmodified from the reference sources (oracle/Makefile.ref) and driven through its public C
API (oracle/ref_driver.c), one training step = render TRAIN, L1 + SSIM forward and backward,
render backward, Adam over every group (gsx-runtime.c:1413-1536 without density control).

The reference CPU backend is single-threaded scalar C, so "all host threads" means one independent
process per core, each training on its own view.  Its render backward keeps every
(Gaussian, pixel) contribution in one scratch tensor whose size must stay below 2^31 bytes
(gsx-cpu/render.c:156-169, sized at :1447-1453); the full 3M-Gaussian workload exceeds that, so
each process times steps on seeded samples of 1/64, 1/32 and 1/16 of the scene's Gaussians at the
full image size, and the full-size step time is the least-squares line a + b N through them,
evaluated at N = 3M (a = the per-view image work, b = the per-Gaussian work).
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
    rank, steps, warmup, subsets, seed = args
    if _ROOT not in sys.path:
        sys.path.insert(0, _ROOT)
    import numpy as np

    from gsx_b200 import scenes
    from oracle import pyoracle as po

    full = scenes.config3_scene(seed)
    teacher_full = scenes.teacher(full)
    n_full = full["mean3d"].shape[0]
    cams = scenes.config3_cameras()
    c = cams[rank % len(cams)]
    oc = po.Camera(c.width, c.height, c.fx, c.fy, c.cx, c.cy, c.rot_xyzw, c.transl, c.near_plane, c.far_plane)
    devnull = os.open(os.devnull, os.O_WRONLY)
    os.dup2(devnull, 1)  # the reference library logs object creation on stdout
    perm = np.random.default_rng(seed + 17).permutation(n_full)
    out = []
    for subset in subsets:
        pick = np.sort(perm[: n_full // subset])
        g = {k: np.ascontiguousarray(v[pick]) for k, v in full.items()}
        teach = {k: np.ascontiguousarray(v[pick]) for k, v in teacher_full.items()}
        target = po.RefSession("cpu", teach, oc, np.zeros((3, c.height, c.width), np.float32)).render()
        sess = po.RefSession("cpu", g, oc, target)
        for _ in range(warmup):
            sess.step()
        t0 = time.perf_counter()
        for _ in range(steps):
            sess.step()
        out.append((len(pick), (time.perf_counter() - t0) / steps))
    return out, n_full


def _cpu_name():
    import platform
    cpu = platform.processor() or "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return cpu


def run(steps: int, warmup: int, processes: int | None = None, subsets=(64, 32, 16), seed: int = 0) -> dict:
    """`processes` independent reference-CPU trainers (one per core), each timing `steps` steps on seeded
    1/s samples of the config-3 Gaussians for every s in `subsets` (all below the CPU renderer's 2 GiB
    scratch limit).  The seconds per step of the slowest process are fitted as a + b * N over the sample
    sizes N (least squares) and the fit is evaluated at the full 3M: a per-view cost (image loss, image
    passes) plus a per-Gaussian cost.  Returns views/s of all processes at the full size, and the fit."""
    import numpy as np
    processes = processes or os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    t0 = time.perf_counter()
    with ctx.Pool(processes) as pool:
        res = pool.map(_worker, [(r, steps, warmup, tuple(subsets), seed) for r in range(processes)])
    wall = time.perf_counter() - t0
    n_full = res[0][1]
    sizes = [res[0][0][k][0] for k in range(len(subsets))]
    sec = [max(r[0][k][1] for r in res) for k in range(len(subsets))]
    b, a = np.polyfit(np.asarray(sizes, np.float64), np.asarray(sec, np.float64), 1)
    s_full = a + b * n_full
    return dict(value=processes / s_full, seconds_per_step_full=s_full, fit_a_s=a, fit_b_s_per_gaussian=b,
                samples=[{"gaussians": n, "seconds_per_step": round(t, 4)} for n, t in zip(sizes, sec)],
                processes=processes, n_full=n_full, wall_s=wall, cpu=_cpu_name())


def run_config1(steps: int = 3) -> dict:
    """Reference CPU backend on config 1 (100k Gaussians fit to a 512x512 target, the reference's own
    CPU-runnable case): seconds per training step on one core, `steps` steps of the 100-step run."""
    if _ROOT not in sys.path:
        sys.path.insert(0, _ROOT)
    from gsx_b200 import scenes
    from oracle import pyoracle as po
    g, cam, target = scenes.config1(0)
    oc = po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl, cam.near_plane,
                   cam.far_plane)
    sess = po.RefSession("cpu", g, oc, target)
    sess.step()
    t0 = time.perf_counter()
    for _ in range(steps):
        sess.step()
    return {"seconds_per_step": (time.perf_counter() - t0) / steps, "steps_timed": steps, "cores": 1, "cpu": _cpu_name()}


if __name__ == "__main__":
    print(run(int(sys.argv[1]) if len(sys.argv) > 1 else 1, 0, int(sys.argv[2]) if len(sys.argv) > 2 else 2))
