"""A small, self-contained training workload for kernel profiling (ncu) and quick timing.

    python -m gsx_b200.profile_case [--gaussians N] [--steps K] [--config 3|2]

Runs K training steps of the config-3 pipeline (or K forward renders of config 2) on a seeded
scene scaled to N Gaussians (default 1M, ~1 GB on the device), then prints per-stage CUDA-event
times.  Launch order per training step: preprocess, emit, histogram, onesweep x passes, ranges,
bucket_scan, blend_forward, l1_ssim, blend_backward, preprocess_backward, adam.
"""
from __future__ import annotations

import argparse
import json


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gaussians", type=int, default=1_000_000)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--config", type=int, default=3)
    args = ap.parse_args()
    import torch

    import gsx_b200 as gb
    from gsx_b200 import scenes
    from gsx_b200.train import GaussianModel, Trainer

    if args.config == 2:
        g = scenes.config2_scene(0, args.gaussians)
        cams = scenes.config2_cameras(8)
        gd = {k: torch.from_numpy(v).cuda() for k, v in g.items()}
        ctx = gb.RenderContext(0)
        c = cams[0]
        out = torch.empty((3, c.height, c.width), device="cuda")
        ctx.set_profiling(True)
        for s in range(args.steps):
            c = cams[s % len(cams)]
            gb.Renderer(c.width, c.height).render(ctx, gd, c, out, forward_type=gb.FORWARD_INFERENCE)
        ctx.check()
        print(json.dumps({"stats": ctx.stats(), "profile": ctx.read_profile()}))
        return
    frac = args.gaussians / 3_000_000
    g = scenes.config3_scene(0, n_volume=int(2_000_000 * frac), n_slab=int(1_000_000 * frac))
    cams = scenes.config3_cameras()
    model = GaussianModel(g)
    c = cams[0]
    trainer = Trainer(model, c.width, c.height)
    target = torch.rand((3, c.height, c.width), device="cuda")
    trainer.ctx.set_profiling(True)
    for s in range(args.steps):
        trainer.step(cams[s % len(cams)], target)
    trainer.ctx.check()
    print(json.dumps({"stats": trainer.ctx.stats(), "profile": trainer.ctx.read_profile()}))


if __name__ == "__main__":
    main()
