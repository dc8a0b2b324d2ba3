"""Generate the golden fixtures in tests/golden/ from the REFERENCE GSX library itself.

Run here (where the reference sources are present):
    make -f oracle/Makefile.ref all driver && python tests/golden/make_golden.py
It drives the reference CPU backend (built unmodified from the reference sources by
oracle/Makefile.ref) through its public C API (oracle/ref_driver.c) and stores inputs and outputs.
The reference's own test inputs are used where its tests define them:
  - SSIM: tests/cuda_loss_runtime.cpp:388-391 (shape [2,3,6,5], sin/cos inputs);
  - 1-pixel render: tests/render_runtime.cpp:671-722 (expected 0.3910474, 0.25, 0.25).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import pyoracle as po  # noqa: E402
from gsx_b200 import scenes  # noqa: E402


def main():
    out = {}
    # SSIM on the reference test's own inputs, and a larger random case with real interior pixels
    i = np.arange(2 * 3 * 6 * 5, dtype=np.float64)
    p = (0.6 * np.sin(0.19 * i) + 0.3 * np.cos(0.07 * i) + 0.1).astype(np.float32).reshape(2, 3, 6, 5)
    t = (0.55 * np.sin(0.23 * i + 0.4) - 0.25 * np.cos(0.11 * i) + 0.05).astype(np.float32).reshape(2, 3, 6, 5)
    lm, g = po.ref_loss("cpu", 2, p, t, 0.7)
    out.update(ssim_a_pred=p, ssim_a_target=t, ssim_a_loss=lm, ssim_a_grad=g)
    rng = np.random.default_rng(2024)
    p = rng.uniform(0, 1, (1, 3, 40, 37)).astype(np.float32)
    t = np.clip(p + rng.normal(0, 0.2, p.shape), 0, 1).astype(np.float32)
    lm, g = po.ref_loss("cpu", 2, p, t, 0.2)
    out.update(ssim_b_pred=p, ssim_b_target=t, ssim_b_loss=lm, ssim_b_grad=g)
    for name, algo in (("l1", 0), ("mse", 1)):
        lm, g = po.ref_loss("cpu", algo, p, t, 0.8)
        out[f"{name}_loss"] = lm
        out[f"{name}_grad"] = g
    # Adam: 5 steps with a fixed gradient, plain and with weight decay + clamp
    x = rng.standard_normal(1000).astype(np.float32)
    gr = (rng.standard_normal(1000) * 1e-3).astype(np.float32)
    out.update(adam_x=x, adam_g=gr, adam_plain=po.ref_adam("cpu", x, gr, 5, 1e-2),
               adam_wd_clamp=po.ref_adam("cpu", x, gr, 5, 1e-2, weight_decay=0.01, max_grad=5e-4))
    # renders with the reference CPU renderer: 1-pixel known answer and a small scene (loose pin:
    # the CPU renderer culls and clamps differently from the CUDA one)
    g1 = dict(mean3d=np.array([[0, 0, 4]], np.float32), rotation=np.array([[0, 0, 0, 1]], np.float32),
              logscale=np.zeros((1, 3), np.float32), opacity=np.zeros(1, np.float32),
              sh0=np.array([[1, 0, 0]], np.float32))
    cam1 = po.Camera(1, 1, 1.0, 1.0, 0.5, 0.5, near=0.1, far=10.0)
    out["render_1px"] = po.RefSession("cpu", g1, cam1, np.zeros((3, 1, 1), np.float32)).render()
    g, cam = scenes.small_scene(0, 2000, 96, 80)
    oc = po.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx, cam.cy, cam.rot_xyzw, cam.transl,
                   cam.near_plane, cam.far_plane)
    out["render_small_cpu"] = po.RefSession("cpu", g, oc, np.zeros((3, 80, 96), np.float32)).render()
    np.savez_compressed(os.path.join(HERE, "reference_cpu.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_cpu.npz"), sorted(out))


if __name__ == "__main__":
    main()
