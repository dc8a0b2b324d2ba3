"""Seeded synthetic scenes and cameras for the benchmark configurations (numpy, host side).

No public dataset is used: every configuration is generated from one integer seed with the shapes,
sizes and value distributions its description gives.  Arrays come back as float32 numpy arrays in
GSX's layout (mean3d [N,3], rotation [N,4] xyzw, logscale [N,3], opacity [N] pre-sigmoid, sh0 [N,3]).
"""
from __future__ import annotations

import math

import numpy as np

from . import Camera


def _unit_quats(rng, n):
    q = rng.standard_normal((n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True) + 1e-12
    return q.astype(np.float32)


def _logit(p):
    return float(math.log(p / (1.0 - p)))


def rot_to_quat_xyzw(R):
    """Rotation matrix -> unit quaternion (x, y, z, w), Shepperd's method."""
    R = np.asarray(R, np.float64)
    tr = R[0, 0] + R[1, 1] + R[2, 2]
    if tr > 0:
        s = math.sqrt(tr + 1.0) * 2
        w, x, y, z = 0.25 * s, (R[2, 1] - R[1, 2]) / s, (R[0, 2] - R[2, 0]) / s, (R[1, 0] - R[0, 1]) / s
    elif R[0, 0] > R[1, 1] and R[0, 0] > R[2, 2]:
        s = math.sqrt(1.0 + R[0, 0] - R[1, 1] - R[2, 2]) * 2
        w, x, y, z = (R[2, 1] - R[1, 2]) / s, 0.25 * s, (R[0, 1] + R[1, 0]) / s, (R[0, 2] + R[2, 0]) / s
    elif R[1, 1] > R[2, 2]:
        s = math.sqrt(1.0 + R[1, 1] - R[0, 0] - R[2, 2]) * 2
        w, x, y, z = (R[0, 2] - R[2, 0]) / s, (R[0, 1] + R[1, 0]) / s, 0.25 * s, (R[1, 2] + R[2, 1]) / s
    else:
        s = math.sqrt(1.0 + R[2, 2] - R[0, 0] - R[1, 1]) * 2
        w, x, y, z = (R[1, 0] - R[0, 1]) / s, (R[0, 2] + R[2, 0]) / s, (R[1, 2] + R[2, 1]) / s, 0.25 * s
    q = np.array([x, y, z, w])
    return tuple((q / np.linalg.norm(q)).tolist())


def look_at(pos, target, width, height, f, up=(0.0, 0.0, 1.0), near=0.01, far=1000.0) -> Camera:
    """OpenCV-convention pinhole camera (x right, y down, z forward) at `pos` looking at `target`."""
    pos = np.asarray(pos, np.float64)
    fwd = np.asarray(target, np.float64) - pos
    fwd /= np.linalg.norm(fwd)
    upv = np.asarray(up, np.float64)
    if abs(np.dot(fwd, upv)) > 0.999:
        upv = np.array([0.0, 1.0, 0.0])
    right = np.cross(fwd, upv)
    right /= np.linalg.norm(right)
    down = np.cross(fwd, right)
    R = np.stack([right, down, fwd])
    t = -R @ pos
    return Camera(width, height, f, f, width / 2.0, height / 2.0, rot_to_quat_xyzw(R), tuple(t.tolist()), near, far)


def fibonacci_sphere(n, radius):
    i = np.arange(n) + 0.5
    phi = np.arccos(1 - 2 * i / n)
    theta = math.pi * (1 + 5 ** 0.5) * i
    return np.stack([np.cos(theta) * np.sin(phi), np.sin(theta) * np.sin(phi), np.cos(phi)], 1) * radius


def mixture_scene(rng, n, extent, sigma=0.8, clusters=32, logscale_mu=-4.5, logscale_sd=0.5, opacity_sd=1.5):
    centres = rng.uniform(-extent / 2, extent / 2, (clusters, 3))
    which = rng.integers(0, clusters, n)
    mean3d = (centres[which] + rng.standard_normal((n, 3)) * sigma).astype(np.float32)
    return dict(mean3d=mean3d, rotation=_unit_quats(rng, n),
                logscale=rng.normal(logscale_mu, logscale_sd, (n, 3)).astype(np.float32),
                opacity=rng.normal(0.0, opacity_sd, n).astype(np.float32),
                sh0=rng.uniform(0.0, 1.0, (n, 3)).astype(np.float32))


def config1(seed=0, n=100_000, size=512):
    """Image-fit shape: means U[-1,1]^2 on z=0, camera at z=-2 looking +z, fx=fy=512."""
    rng = np.random.default_rng(seed)
    mean3d = np.zeros((n, 3), np.float32)
    mean3d[:, :2] = rng.uniform(-1, 1, (n, 2))
    g = dict(mean3d=mean3d, rotation=_unit_quats(rng, n), logscale=rng.normal(-4.0, 0.3, (n, 3)).astype(np.float32),
             opacity=np.full(n, _logit(0.1), np.float32), sh0=rng.uniform(0, 1, (n, 3)).astype(np.float32))
    cam = Camera(size, size, 512.0 * size / 512, 512.0 * size / 512, size / 2.0, size / 2.0, (0.0, 0.0, 0.0, 1.0),
                 (0.0, 0.0, 2.0), 0.01, 100.0)
    yy, xx = np.meshgrid(np.linspace(0, 1, size), np.linspace(0, 1, size), indexing="ij")
    img = np.zeros((3, size, size), np.float64)
    for _ in range(16):
        c = rng.integers(0, 3)
        fx_, fy_, ph = rng.uniform(1, 12), rng.uniform(1, 12), rng.uniform(0, 2 * math.pi)
        img[c] += rng.uniform(0.05, 0.2) * np.sin(2 * math.pi * (fx_ * xx + fy_ * yy) + ph)
    coarse = rng.uniform(0, 1, (3, size // 16 + 1, size // 16 + 1))
    img += 0.3 * np.kron(coarse, np.ones((16, 16)))[:, :size, :size]
    target = np.clip(img + 0.2, 0, 1).astype(np.float32)
    return g, cam, target


def config2_scene(seed=0, n=1_000_000):
    return mixture_scene(np.random.default_rng(seed), n, extent=10.0)


def config2_cameras(count=64, width=1920, height=1080, f=1100.0, radius=6.0):
    return [look_at(p, (0, 0, 0), width, height, f) for p in fibonacci_sphere(count, radius)]


def config3_scene(seed=0, n_volume=2_000_000, n_slab=1_000_000, extent=20.0):
    rng = np.random.default_rng(seed)
    g = mixture_scene(rng, n_volume, extent=extent)
    slab = dict(mean3d=np.concatenate([rng.uniform(-extent / 2, extent / 2, (n_slab, 2)),
                                       np.full((n_slab, 1), -extent / 2)], 1).astype(np.float32),
                rotation=np.tile(np.array([[0, 0, 0, 1]], np.float32), (n_slab, 1)),
                logscale=np.concatenate([rng.normal(-3.5, 0.5, (n_slab, 2)), np.full((n_slab, 1), -7.0)], 1).astype(np.float32),
                opacity=rng.normal(0.0, 1.5, n_slab).astype(np.float32),
                sh0=rng.uniform(0, 1, (n_slab, 3)).astype(np.float32))
    return {k: np.concatenate([g[k], slab[k]]) for k in g}


def config3_cameras(count=8, width=1245, height=825, f=1000.0, radius=18.0, elevation_deg=30.0):
    el = math.radians(elevation_deg)
    cams = []
    for k in range(count):
        az = 2 * math.pi * k / count
        pos = (radius * math.cos(el) * math.cos(az), radius * math.cos(el) * math.sin(az), radius * math.sin(el))
        cams.append(look_at(pos, (0, 0, 0), width, height, f))
    return cams


def teacher(g, seed=1, jitter=0.02, colour_sd=0.1):
    """Seeded teacher copy of a scene: means + N(0, jitter), colours perturbed (targets of config 3)."""
    rng = np.random.default_rng(seed)
    t = {k: v.copy() for k, v in g.items()}
    t["mean3d"] = (t["mean3d"] + rng.normal(0, jitter, t["mean3d"].shape)).astype(np.float32)
    t["sh0"] = np.clip(t["sh0"] + rng.normal(0, colour_sd, t["sh0"].shape), 0, 1).astype(np.float32)
    return t


def config4_scene(seed=0, n=10_000_000):
    """Config 4: 10M Gaussians built like config 3 (volume mixture + flat ground slab, 2:1)."""
    n_slab = n // 3
    return config3_scene(seed, n_volume=n - n_slab, n_slab=n_slab)


def config4_cameras(count=16, width=3840, height=2160, f=2200.0, radius=8.0):
    return [look_at((radius * math.cos(2 * math.pi * k / count), radius * math.sin(2 * math.pi * k / count), 2.0),
                    (0, 0, 0), width, height, f) for k in range(count)]


def small_scene(seed=0, n=2000, width=96, height=80, sh_degree=0, spread=1.5, scale_mu=-3.0):
    """A small random scene in front of the camera for parity tests (fits the oracle in seconds)."""
    rng = np.random.default_rng(seed)
    g = dict(mean3d=np.concatenate([rng.uniform(-spread, spread, (n, 2)), rng.uniform(2.0, 6.0, (n, 1))], 1).astype(np.float32),
             rotation=_unit_quats(rng, n), logscale=rng.normal(scale_mu, 0.6, (n, 3)).astype(np.float32),
             opacity=rng.normal(0.0, 1.5, n).astype(np.float32), sh0=rng.uniform(-0.2, 1.2, (n, 3)).astype(np.float32))
    for d, k in ((1, 3), (2, 5), (3, 7)):
        if sh_degree >= d:
            g[f"sh{d}"] = rng.normal(0, 0.3, (n, k, 3)).astype(np.float32)
    cam = Camera(width, height, 0.9 * width, 0.9 * width, width / 2.0 + 0.3, height / 2.0 - 0.2, (0.0, 0.0, 0.0, 1.0),
                 (0.0, 0.0, 0.0), 0.2, 100.0)
    return g, cam
