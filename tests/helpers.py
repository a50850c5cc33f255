"""Scene builders shared by the tests: the structures of the reference's own GPU tests
(instantsplat-rs/src/rasterizer_tests.rs, loss_tests.rs, pose_tests.rs), re-created with
numpy's seeded PCG64 (the reference's ChaCha12 `StdRng` streams cannot be reproduced here),
and a CPU mirror of the projection in f64 (rasterizer_tests.rs:149-243) that shares no
code with the oracle or the CUDA path."""

from __future__ import annotations

import numpy as np

import splat_b200 as sb
from splat_b200.camera import PinholeCamera
from splat_b200.gaussians import GaussianCloud, logit, rgb_to_sh_dc

TILE = 16


def camera_at_origin(width: int, height: int, focal: float) -> PinholeCamera:
    """rasterizer_tests.rs:16-25."""
    return PinholeCamera(np.eye(3), np.zeros(3), (focal, focal), (width // 2, height // 2), width, height)


def single_gaussian(position, sigma, opacity, rgb) -> GaussianCloud:
    """rasterizer_tests.rs:27-35."""
    return GaussianCloud(
        positions=np.array([position], np.float32),
        log_scales=np.full((1, 3), np.log(np.float32(sigma)), np.float32),
        rotations=np.array([[1.0, 0.0, 0.0, 0.0]], np.float32),
        opacity_logits=np.array([logit(opacity)], np.float32),
        sh=rgb_to_sh_dc(np.array(rgb, np.float32)).reshape(1, 1, 3),
    )


def random_cloud(count: int, rng: np.random.Generator, sh_degree: int = 0) -> GaussianCloud:
    """rasterizer_tests.rs:245-268: depths 3 + 0.01 i shuffled, so that the 20-bit depth keys
    never tie."""
    depths = 3.0 + np.arange(count, dtype=np.float32) * np.float32(0.01)
    rng.shuffle(depths)
    spread = 0.4 * depths
    positions = np.stack(
        [rng.uniform(-spread, spread), rng.uniform(-spread, spread), depths], axis=1
    ).astype(np.float32)
    k = (sh_degree + 1) ** 2
    sh = np.zeros((count, k, 3), np.float32)
    sh[:, 0, :] = rng.uniform(-1.5, 1.5, (count, 3))
    if k > 1:
        sh[:, 1:, :] = rng.normal(0.0, 0.3, (count, k - 1, 3))
    return GaussianCloud(
        positions=positions,
        log_scales=rng.uniform(-3.5, -1.5, (count, 3)),
        rotations=rng.uniform(-1.0, 1.0, (count, 4)),
        opacity_logits=rng.uniform(-2.0, 3.0, count),
        sh=sh,
    )


def gradient_check_cloud(camera: PinholeCamera, rng: np.random.Generator) -> GaussianCloud:
    """rasterizer_tests.rs:297-315: 4 Gaussians along the camera's optical axis."""
    positions = []
    for g in range(4):
        in_camera = np.array([rng.uniform(-0.3, 0.3), rng.uniform(-0.3, 0.3), 3.0 + g * 0.5])
        positions.append(camera.rotation @ in_camera + camera.translation)
    return GaussianCloud(
        positions=np.array(positions, np.float32),
        log_scales=rng.uniform(-2.5, -1.0, (4, 3)),
        rotations=rng.uniform(-1.0, 1.0, (4, 4)),
        opacity_logits=rng.uniform(-0.5, 1.5, 4),
        sh=rng.uniform(-1.0, 1.0, (4, 1, 3)),
    )


def moved_camera() -> PinholeCamera:
    """rasterizer_tests.rs:386-396: Rotation3::from_euler_angles(0.4, -0.7, 1.1)."""
    roll, pitch, yaw = 0.4, -0.7, 1.1
    cr, sr, cp, spi, cy, sy = np.cos(roll), np.sin(roll), np.cos(pitch), np.sin(pitch), np.cos(yaw), np.sin(yaw)
    # nalgebra: R = Rz(yaw) Ry(pitch) Rx(roll).
    rx = np.array([[1, 0, 0], [0, cr, -sr], [0, sr, cr]])
    ry = np.array([[cp, 0, spi], [0, 1, 0], [-spi, 0, cp]])
    rz = np.array([[cy, -sy, 0], [sy, cy, 0], [0, 0, 1]])
    return PinholeCamera(rz @ ry @ rx, np.array([1.5, -2.0, 0.7]), (40.0, 40.0), (16.0, 16.0), 32, 32)


def reference_project(cloud: GaussianCloud, camera: PinholeCamera) -> list[dict]:
    """rasterizer_tests.rs:149-203: the projection in f64 with the shaders' conventions."""
    w, t = camera.world_to_camera()
    out = []
    fx, fy = camera.focal
    for g in range(len(cloud)):
        p = w @ cloud.positions[g].astype(np.float64) + t
        if p[2] < 0.01:
            continue
        scale = np.exp(cloud.log_scales[g].astype(np.float64))
        q = cloud.rotations[g].astype(np.float64)
        q = q / np.linalg.norm(q)
        r0, x, y, z = q
        rot = np.array(
            [
                [1 - 2 * (y * y + z * z), 2 * (x * y - r0 * z), 2 * (x * z + r0 * y)],
                [2 * (x * y + r0 * z), 1 - 2 * (x * x + z * z), 2 * (y * z - r0 * x)],
                [2 * (x * z - r0 * y), 2 * (y * z + r0 * x), 1 - 2 * (x * x + y * y)],
            ]
        )
        m = rot @ np.diag(scale)
        sigma = m @ m.T
        limit_x = 1.3 * camera.width / (2.0 * fx)
        limit_y = 1.3 * camera.height / (2.0 * fy)
        tx = np.clip(p[0] / p[2], -limit_x, limit_x) * p[2]
        ty = np.clip(p[1] / p[2], -limit_y, limit_y) * p[2]
        j = np.array([[fx / p[2], 0.0, -fx * tx / p[2] ** 2], [0.0, fy / p[2], -fy * ty / p[2] ** 2]])
        tm = j @ w
        cov = tm @ sigma @ tm.T
        a, b, c = cov[0, 0] + 0.3, cov[0, 1], cov[1, 1] + 0.3
        det = a * c - b * b
        mid = 0.5 * (a + c)
        radius = np.ceil(3.0 * np.sqrt(mid + np.sqrt(max(mid * mid - det, 0.1))))
        mean = np.array([fx * p[0] / p[2] + camera.principal_point[0], fy * p[1] / p[2] + camera.principal_point[1]])
        tiles = np.array([(camera.width + TILE - 1) // TILE, (camera.height + TILE - 1) // TILE], np.float64)
        tile_min = np.clip(np.floor((mean - radius) / TILE), 0, tiles).astype(np.int64)
        tile_max = np.clip(np.floor((mean + radius) / TILE) + 1.0, 0, tiles).astype(np.int64)
        out.append(
            dict(
                index=g,
                mean=mean.astype(np.float32),
                conic=np.array([c / det, -b / det, a / det], np.float32),
                depth=np.float32(p[2]),
                color=np.maximum(0.0, np.float32(0.28209479) * cloud.sh[g, 0] + np.float32(0.5)).astype(np.float32),
                opacity=np.float32(1.0 / (1.0 + np.exp(-np.float64(cloud.opacity_logits[g])))),
                radius=radius,
                tile_min=tile_min,
                tile_max=tile_max,
            )
        )
    return out


def reference_render(cloud: GaussianCloud, camera: PinholeCamera) -> np.ndarray:
    """rasterizer_tests.rs:205-243: per pixel, every Gaussian in depth order."""
    gaussians = sorted(reference_project(cloud, camera), key=lambda g: g["depth"])
    image = np.zeros((camera.height, camera.width, 4), np.float32)
    for py in range(camera.height):
        for px in range(camera.width):
            tx, ty = px // TILE, py // TILE
            transmittance = np.float32(1.0)
            color = np.zeros(3, np.float32)
            for g in gaussians:
                if not (g["tile_min"][0] <= tx < g["tile_max"][0] and g["tile_min"][1] <= ty < g["tile_max"][1]):
                    continue
                dx = g["mean"][0] - np.float32(px)
                dy = g["mean"][1] - np.float32(py)
                cn = g["conic"]
                power = np.float32(-0.5) * (cn[0] * dx * dx + cn[2] * dy * dy) - cn[1] * dx * dy
                if power > 0:
                    continue
                alpha = min(np.float32(0.99), g["opacity"] * np.float32(np.exp(power)))
                if alpha < np.float32(1.0 / 255.0):
                    continue
                nxt = transmittance * (np.float32(1.0) - alpha)
                if nxt < np.float32(1e-4):
                    break
                color += g["color"] * alpha * transmittance
                transmittance = nxt
            image[py, px, :3] = color
            image[py, px, 3] = transmittance
    return image.reshape(-1)


def scene_buffers(cloud: GaussianCloud, camera: PinholeCamera, ground_truth=None, views: int = 1):
    """Device tensors for a rasterizer over `cloud`: (params, ground_truth)."""
    import torch

    params = torch.from_numpy(cloud.to_packed()).cuda()
    if ground_truth is None:
        ground_truth = np.zeros(camera.width * camera.height * 4 * views, np.float32)
    gt = torch.from_numpy(np.ascontiguousarray(ground_truth, np.float32).reshape(-1)).cuda()
    return params, gt


def make_rasterizer(ctx, cloud: GaussianCloud, camera: PinholeCamera, ground_truth=None, views: int = 1, **options):
    params, gt = scene_buffers(cloud, camera, ground_truth, views)
    opts = sb.default_options(sh_degree=cloud.sh_degree, **options)
    rast = sb.Rasterizer(ctx, params, len(cloud), camera.width, camera.height, gt, views, opts)
    rast.set_camera(camera)
    return rast, params, gt
