"""Seeded synthetic scenes of the benchmark configurations (numpy PCG64 generators).

No public dataset is involved: each configuration is a seeded random Gaussian cloud of the
stated size and distributions, a set of cameras, and a "ground truth" cloud (a perturbed
copy) whose render is the training target. Config indices follow the benchmark's list:
  0  20k SH0, 3 views 256x256 on a radius-3 circle (the CPU-runnable loss-curve config)
  1  100k SH0 on a noisy unit sphere, 6 views 512x384 on a 30 degree arc, poses refined
  2  500k SH3, box surface + volume, 24 views 1024x768 on a hemisphere, poses refined
  3  3M SH3, 64 Gaussian clusters, 64 cameras 1920x1080 on a radius-4 orbit (forward only)
  4  6M SH3, same distributions, 128 views 1600x1200 on a sphere (view-sharded training)
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .camera import PinholeCamera, focal_for_fov, look_at
from .gaussians import SH_C0, GaussianCloud, rgb_to_sh_dc

UP = np.array([0.0, 0.0, 1.0])


@dataclass
class Scene:
    name: str
    cloud: GaussianCloud
    truth: GaussianCloud
    cameras: list[PinholeCamera]
    iterations: int
    refine_poses: bool
    seed: int


def random_rotations(rng: np.random.Generator, n: int) -> np.ndarray:
    q = rng.standard_normal((n, 4))
    return q / np.linalg.norm(q, axis=1, keepdims=True)


def _sh(rng: np.random.Generator, n: int, degree: int, rest_sigma: float, single: bool = False) -> np.ndarray:
    """DC from uniform colours, higher bands ~N(0, rest_sigma); `single` draws the higher
    bands in float32 (the multi-million-Gaussian configs, where float64 draws are slow)."""
    sh = np.zeros((n, (degree + 1) ** 2, 3), np.float32)
    sh[:, 0, :] = rgb_to_sh_dc(rng.uniform(0.0, 1.0, (n, 3)))
    if degree > 0:
        shape = (n, (degree + 1) ** 2 - 1, 3)
        if single:
            rest = rng.standard_normal(shape, dtype=np.float32)
            rest *= np.float32(rest_sigma)
            sh[:, 1:, :] = rest
        else:
            sh[:, 1:, :] = rng.normal(0.0, rest_sigma, shape)
    return sh


def _cloud(positions, log_scales, rotations, opacity_logits, sh) -> GaussianCloud:
    return GaussianCloud(positions, log_scales, rotations, opacity_logits, sh)


def perturbed(cloud: GaussianCloud, rng: np.random.Generator, position_sigma=0.02, dc_sigma=0.1) -> GaussianCloud:
    """The ground truth: a copy with jittered positions and colours."""
    sh = cloud.sh.copy()
    sh[:, 0, :] += rng.normal(0.0, dc_sigma, sh[:, 0, :].shape).astype(np.float32)
    return _cloud(
        cloud.positions + rng.normal(0.0, position_sigma, cloud.positions.shape).astype(np.float32),
        cloud.log_scales.copy(),
        cloud.rotations.copy(),
        cloud.opacity_logits.copy(),
        sh,
    )


def circle_cameras(count, radius, width, height, fov=60.0, elevation=0.0, arc_degrees=360.0):
    focal = focal_for_fov(width, fov)
    cams = []
    for i in range(count):
        step = arc_degrees / (count if arc_degrees >= 360.0 else max(count - 1, 1))
        theta = np.radians(i * step)
        eye = np.array([radius * np.cos(theta), radius * np.sin(theta), elevation])
        cams.append(look_at(eye, np.zeros(3), UP, focal, width, height))
    return cams


def sphere_cameras(count, radius, width, height, fov=60.0, hemisphere=False):
    """Fibonacci-sphere placement (upper half for `hemisphere`)."""
    focal = focal_for_fov(width, fov)
    cams = []
    golden = np.pi * (3.0 - np.sqrt(5.0))
    for i in range(count):
        z = (1.0 - (i + 0.5) / count) if hemisphere else 1.0 - 2.0 * (i + 0.5) / count
        if hemisphere:
            z = 0.1 + 0.85 * z
        r = np.sqrt(max(0.0, 1.0 - z * z))
        theta = golden * i
        eye = radius * np.array([r * np.cos(theta), r * np.sin(theta), z])
        cams.append(look_at(eye, np.zeros(3), UP, focal, width, height))
    return cams


def config(index: int, scale: float = 1.0) -> Scene:
    """Benchmark configuration `index` (0-4); `scale` shrinks the Gaussian count (tests)."""
    if index == 0:
        rng = np.random.default_rng(0)
        n = int(20_000 * scale)
        cloud = _cloud(
            rng.uniform(-1.0, 1.0, (n, 3)),
            rng.normal(-4.0, 0.5, (n, 3)),
            random_rotations(rng, n),
            rng.normal(0.0, 1.0, n),
            _sh(rng, n, 0, 0.0),
        )
        cams = circle_cameras(3, 3.0, 256, 256)
        return Scene("20k SH0 256x256 x3", cloud, perturbed(cloud, rng), cams, 100, False, 0)
    if index == 1:
        rng = np.random.default_rng(1)
        n = int(100_000 * scale)
        d = rng.standard_normal((n, 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        positions = d * (1.0 + rng.normal(0.0, 0.02, (n, 1)))
        cloud = _cloud(
            positions,
            rng.normal(-4.5, 0.5, (n, 3)),
            random_rotations(rng, n),
            rng.normal(0.0, 1.0, n),
            _sh(rng, n, 0, 0.0),
        )
        cams = circle_cameras(6, 3.0, 512, 384, arc_degrees=30.0, elevation=0.5)
        return Scene("100k SH0 512x384 x6", cloud, perturbed(cloud, rng), cams, 500, True, 1)
    if index == 2:
        rng = np.random.default_rng(2)
        n = int(500_000 * scale)
        surface = int(0.7 * n)
        face = rng.integers(0, 6, surface)
        pts = rng.uniform(-1.0, 1.0, (surface, 3))
        axis = face // 2
        pts[np.arange(surface), axis] = np.where(face % 2 == 0, -1.0, 1.0)
        positions = np.concatenate([pts, rng.uniform(-1.0, 1.0, (n - surface, 3))])
        cloud = _cloud(
            positions,
            rng.normal(-5.0, 0.7, (n, 3)),
            random_rotations(rng, n),
            rng.normal(0.0, 1.0, n),
            _sh(rng, n, 3, 0.05),
        )
        cams = sphere_cameras(24, 3.5, 1024, 768, hemisphere=True)
        return Scene("500k SH3 1024x768 x24", cloud, perturbed(cloud, rng), cams, 1000, True, 2)
    if index in (3, 4):
        seed = 3 if index == 3 else 4
        rng = np.random.default_rng(seed)
        n = int((3_000_000 if index == 3 else 6_000_000) * scale)
        centres = rng.uniform(-1.5, 1.5, (64, 3))
        positions = centres[rng.integers(0, 64, n)] + rng.normal(0.0, 0.2, (n, 3))
        cloud = _cloud(
            positions,
            rng.normal(-5.5, 0.8, (n, 3)),
            random_rotations(rng, n),
            rng.normal(0.5, 1.5, n),
            _sh(rng, n, 3, 0.05, single=True),
        )
        if index == 3:
            cams = circle_cameras(64, 4.0, 1920, 1080, elevation=0.8)
            return Scene("3M SH3 1920x1080 x64", cloud, cloud, cams, 1, False, seed)
        cams = sphere_cameras(128, 4.0, 1600, 1200)
        return Scene("6M SH3 1600x1200 x128", cloud, perturbed(cloud, rng), cams, 200, False, seed)
    raise ValueError(f"config {index}")


def packed_clustered_device(count: int, seed: int, device, perturb: bool = False):
    """Configs 3-4's distributions (64 Gaussian clusters of sigma 0.2 with centres uniform in
    [-1.5, 1.5]^3, log-scales ~N(-5.5, 0.8), random unit quaternions, opacity logits
    ~N(0.5, 1.5), DC from uniform colours, SH bands 1-3 ~N(0, 0.05)), packed at SH degree 3 (59
    floats per Gaussian), drawn on the GPU with torch's seeded generator: seconds instead of
    minutes for the multi-million-Gaussian benchmark scenes. With `perturb`, returns
    (cloud, truth): the truth a copy with positions + N(0, 0.02) and DC + N(0, 0.1), as
    `perturbed`. Not the numpy stream of `config` (whose scenes the parity tests use)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    f = dict(device=device, dtype=torch.float32, generator=g)
    packed = torch.empty((count, 59), device=device, dtype=torch.float32)
    centres = torch.rand((64, 3), **f) * 3.0 - 1.5
    which = torch.randint(0, 64, (count,), device=device, generator=g)
    packed[:, 0:3] = centres[which] + torch.randn((count, 3), **f) * 0.2
    packed[:, 3:6] = torch.randn((count, 3), **f) * 0.8 - 5.5
    q = torch.randn((count, 4), **f)
    packed[:, 6:10] = q / q.norm(dim=1, keepdim=True)
    packed[:, 10] = torch.randn((count,), **f) * 1.5 + 0.5
    packed[:, 11:14] = (torch.rand((count, 3), **f) - 0.5) / float(SH_C0)
    packed[:, 14:59] = torch.randn((count, 45), **f) * 0.05
    if not perturb:
        return packed.reshape(-1)
    truth = packed.clone()
    truth[:, 0:3] += torch.randn((count, 3), **f) * 0.02
    truth[:, 11:14] += torch.randn((count, 3), **f) * 0.1
    return packed.reshape(-1), truth.reshape(-1)
