"""The reference's own GPU tests (instantsplat-rs/src/rasterizer_tests.rs, loss_tests.rs,
densify_tests.rs, pose_tests.rs), re-created with numpy's PCG64 in place of rand's StdRng
and written against a backend (tests/backends.py), so that each runs on the CPU oracle and
on the CUDA path with the reference's own tolerances."""

from __future__ import annotations

import numpy as np

import splat_b200 as sb
from helpers import (
    TILE,
    camera_at_origin,
    gradient_check_cloud,
    moved_camera,
    random_cloud,
    reference_project,
    reference_render,
)
from splat_b200.pose import PoseCorrection, camera_gradient, corrected_camera, pose_gradient


def forward_matches_the_cpu_reference(make_backend):
    """rasterizer_tests.rs:270-287: 600 random Gaussians, 80 x 48, f = 60, against the
    per-pixel f64-projected renderer; largest pixel difference below 2e-4."""
    rng = np.random.default_rng(7)
    cloud = random_cloud(600, rng)
    camera = camera_at_origin(80, 48, 60.0)
    backend = make_backend(len(cloud), camera)
    rendered = backend.render(cloud.to_packed())
    reference = reference_render(cloud, camera)
    worst = float(np.max(np.abs(rendered - reference)))
    assert worst < 2e-4, f"largest pixel difference {worst}"
    return backend


def gradient_check(make_backend, camera: sb.PinholeCamera, sh_degree: int = 0, seed: int = 3):
    """rasterizer_tests.rs:289-379: the backward pass against central finite differences
    at two step sizes, pixels where the two disagree (discontinuities) left out on both
    sides; tolerance 3e-3 + 1e-2 max(|a|, |n|); more than 40 non-zero gradients."""
    rng = np.random.default_rng(seed)
    cloud = gradient_check_cloud(camera, rng)
    if sh_degree:
        k = (sh_degree + 1) ** 2
        sh = np.zeros((len(cloud), k, 3), np.float32)
        sh[:, 0] = cloud.sh[:, 0]
        sh[:, 1:] = rng.normal(0.0, 0.3, (len(cloud), k - 1, 3))
        cloud = sb.GaussianCloud(cloud.positions, cloud.log_scales, cloud.rotations, cloud.opacity_logits, sh)
    backend = make_backend(len(cloud), camera, sh_degree)
    pixel_count = camera.width * camera.height
    weights = rng.uniform(-1.0, 1.0, pixel_count * 4).astype(np.float32)
    packed = cloud.to_packed()
    base = backend.render(packed).reshape(-1, 4)
    assert np.any(base[:, 3] < 0.5), "scene too transparent"
    stride = sb.param_stride(sh_degree)
    eps = np.float32(1e-3)
    failures, nonzero = [], 0
    for index in range(packed.size):
        samples = []
        for k in (-2.0, -1.0, 1.0, 2.0):
            moved = packed.copy()
            moved[index] = packed[index] + np.float32(k) * eps
            samples.append(backend.render(moved).astype(np.float64).reshape(-1, 4))
        narrow = (samples[2] - samples[1]) / (2.0 * float(eps))
        wide = (samples[3] - samples[0]) / (4.0 * float(eps))
        jumps = np.any(np.abs(narrow - wide) > 2e-2 + 5e-2 * np.abs(narrow), axis=1)
        assert jumps.sum() * 20 < pixel_count, f"param {index}: {jumps.sum()} of {pixel_count} pixels jump"
        smooth = weights.reshape(-1, 4).copy()
        smooth[jumps] = 0.0
        numeric = float(np.sum(smooth.astype(np.float64) * narrow))
        analytic = float(backend.backward(packed, smooth.reshape(-1))[0][index])
        if abs(analytic) > 1e-3:
            nonzero += 1
        tolerance = 3e-3 + 1e-2 * max(abs(numeric), abs(analytic))
        if abs(analytic - numeric) > tolerance:
            failures.append(f"gaussian {index // stride} slot {index % stride}: {analytic:.5f} vs {numeric:.5f}")
    assert nonzero > 40, f"only {nonzero} non-zero gradients"
    assert not failures, "gradient mismatches:\n" + "\n".join(failures)


def random_pair(width, height, rng):
    """loss_tests.rs:50-63: a random photo with a 60 % mask and a random render."""
    pixels = width * height
    mask = (rng.random(pixels) < 0.6).astype(np.float32)
    gt = np.concatenate([rng.random((pixels, 3)).astype(np.float32) * mask[:, None], mask[:, None]], axis=1)
    rgbt = np.concatenate([rng.random((pixels, 3)), rng.uniform(0.1, 0.9, (pixels, 1))], axis=1).astype(np.float32)
    return gt.reshape(-1), rgbt.reshape(-1)


def identical_images_have_zero_loss(make_backend):
    """loss_tests.rs:65-84."""
    width, height = 24, 20
    gt, _ = random_pair(width, height, np.random.default_rng(11))
    g = gt.reshape(-1, 4)
    rgbt = np.concatenate([g[:, :3], 1.0 - g[:, 3:4]], axis=1).astype(np.float32).reshape(-1)
    backend = make_backend(1, camera_at_origin(width, height, 40.0), 0, gt)
    pixel_loss, gradient = backend.loss(rgbt)
    terms = sb.LossTerms.from_pixel_loss(pixel_loss)
    assert terms.l1 == 0.0 and terms.alpha == 0.0
    assert abs(terms.dssim) < 1e-6 and abs(terms.total) < 1e-6
    assert float(np.max(np.abs(gradient))) < 1e-7


def reference_dssim(width, height, rgbt, gt):
    """loss_tests.rs:86-121: 1 - SSIM in f64 on the foreground, averaged over all."""
    taps = np.exp(-np.arange(-5, 6, dtype=np.float64) ** 2 / 4.5)
    taps = (taps / taps.sum()).astype(np.float32).astype(np.float64)
    window = np.outer(taps, taps)
    x = rgbt.reshape(height, width, 4)[..., :3].astype(np.float64)
    y = gt.reshape(height, width, 4)[..., :3].astype(np.float64)
    mask = gt.reshape(height, width, 4)[..., 3].astype(np.float64)

    def conv(img):
        pad = np.pad(img, ((5, 5), (5, 5), (0, 0)))
        out = np.zeros_like(img)
        for dy in range(11):
            for dx in range(11):
                out += window[dy, dx] * pad[dy : dy + height, dx : dx + width]
        return out

    mx, my, exx, eyy, exy = conv(x), conv(y), conv(x * x), conv(y * y), conv(x * y)
    sxx, syy, sxy = exx - mx * mx, eyy - my * my, exy - mx * my
    ssim = ((2 * mx * my + 1e-4) * (2 * sxy + 9e-4)) / ((mx * mx + my * my + 1e-4) * (sxx + syy + 9e-4))
    return float(np.sum(mask[..., None] * (1.0 - ssim)) / (3 * width * height))


def loss_terms_match_the_cpu_reference(make_backend):
    """loss_tests.rs:123-149."""
    width, height = 40, 24
    gt, rgbt = random_pair(width, height, np.random.default_rng(5))
    backend = make_backend(1, camera_at_origin(width, height, 40.0), 0, gt)
    pixel_loss, _ = backend.loss(rgbt)
    terms = sb.LossTerms.from_pixel_loss(pixel_loss)
    g, r = gt.reshape(-1, 4).astype(np.float64), rgbt.reshape(-1, 4).astype(np.float64)
    l1 = float(np.sum(g[:, 3:4] * np.abs(r[:, :3] - g[:, :3])) / (3 * width * height))
    alpha = float(np.mean(np.abs(1.0 - r[:, 3] - g[:, 3])))
    dssim = reference_dssim(width, height, rgbt, gt)
    assert abs(terms.l1 - l1) < 1e-5
    assert abs(terms.alpha - alpha) < 1e-5
    assert abs(terms.dssim - dssim) < 1e-4
    total = 0.8 * l1 + 1.0 * alpha + 0.2 * dssim
    assert abs(terms.total - total) < 1e-4
    assert dssim > 0.3


def loss_gradient_matches_finite_differences(make_backend):
    """loss_tests.rs:151-195: 60 random entries away from the L1 kinks; tolerance
    1e-6 + 1e-2 max(|a|, |n|); at least 4 background colour entries."""
    width, height = 32, 20
    rng = np.random.default_rng(17)
    gt, rgbt = random_pair(width, height, rng)
    backend = make_backend(1, camera_at_origin(width, height, 40.0), 0, gt)
    _, gradient = backend.loss(rgbt)
    eps = np.float32(1e-2)

    def total(values):
        pl = backend.loss(values)[0].reshape(-1, 4).astype(np.float64)
        return float(pl[:, 3].sum() / len(pl))

    failures, checked, background = [], 0, 0
    while checked < 60:
        pixel = int(rng.integers(0, width * height))
        channel = int(rng.integers(0, 4))
        index = pixel * 4 + channel
        diff = rgbt[index] - gt[pixel * 4 + channel]
        if channel < 3 and abs(diff) < 3 * eps:
            continue
        if channel < 3 and gt[pixel * 4 + 3] == 0.0:
            background += 1
        checked += 1
        up, down = rgbt.copy(), rgbt.copy()
        up[index] += eps
        down[index] -= eps
        numeric = (total(up) - total(down)) / (2.0 * float(eps))
        analytic = float(gradient[index])
        if abs(analytic - numeric) > 1e-6 + 1e-2 * max(abs(numeric), abs(analytic)):
            failures.append(f"pixel {pixel} channel {channel}: {analytic:.3e} vs {numeric:.3e}")
    assert not failures, "\n".join(failures)
    assert background >= 4


def densify_stats_match_the_cpu_mean_gradient(make_backend):
    """densify_tests.rs:15-119: two backward passes of the same render and loss gradient
    double the statistics; the mean-gradient sums match an f64 backward of the mean."""
    rng = np.random.default_rng(11)
    cloud = random_cloud(40, rng)
    camera = camera_at_origin(48, 32, 40.0)
    backend = make_backend(len(cloud), camera)
    gaussians = reference_project(cloud, camera)
    assert len(gaussians) == len(cloud)
    weights = rng.uniform(-1.0, 1.0, camera.width * camera.height * 4).astype(np.float32)
    packed = cloud.to_packed()
    backend.backward(packed, weights)
    stats = backend.backward(packed, weights)[2]
    reference = reference_mean_gradients(gaussians, camera.width, camera.height, weights)
    half = np.array([camera.width / 2.0, camera.height / 2.0])
    visible = 0
    for g in gaussians:
        i = g["index"]
        on_screen = g["radius"] > 0 and g["tile_max"][0] > g["tile_min"][0] and g["tile_max"][1] > g["tile_min"][1]
        if not on_screen:
            assert np.all(stats[i] == 0.0)
            continue
        visible += 1
        assert stats[i, 1] == 2.0
        assert stats[i, 2] == np.float32(g["radius"])
        expected = 2.0 * float(np.hypot(reference[i][0] * half[0], reference[i][1] * half[1]))
        assert abs(float(stats[i, 0]) - expected) <= 1e-3 + 2e-3 * expected, (i, stats[i, 0], expected)
    assert visible > 20


def reference_mean_gradients(gaussians, width, height, weights):
    """densify_tests.rs:11-75, in f64."""
    order = sorted(range(len(gaussians)), key=lambda k: gaussians[k]["depth"])
    grads = {g["index"]: np.zeros(2) for g in gaussians}
    w4 = weights.reshape(-1, 4).astype(np.float64)
    for py in range(height):
        for px in range(width):
            tx, ty = px // TILE, py // TILE
            weight = w4[py * width + px]
            contributions = []
            transmittance = 1.0
            for k in order:
                g = gaussians[k]
                if not (g["tile_min"][0] <= tx < g["tile_max"][0] and g["tile_min"][1] <= ty < g["tile_max"][1]):
                    continue
                d = np.array([g["mean"][0] - px, g["mean"][1] - py], np.float64)
                c = g["conic"].astype(np.float64)
                power = -0.5 * (c[0] * d[0] ** 2 + c[2] * d[1] ** 2) - c[1] * d[0] * d[1]
                if power > 0:
                    continue
                unclamped = float(g["opacity"]) * np.exp(power)
                alpha = min(unclamped, 0.99)
                if alpha < 1.0 / 255.0:
                    continue
                nxt = transmittance * (1.0 - alpha)
                if nxt < 1e-4:
                    break
                contributions.append((g, alpha, unclamped if unclamped < 0.99 else 0.0, d, transmittance))
                transmittance = nxt
            behind = np.array([0.0, 0.0, 0.0, transmittance])
            for g, alpha, d_alpha_d_power, d, in_front in reversed(contributions):
                color = np.array([*g["color"].astype(np.float64), 0.0])
                d_alpha = float(np.sum(weight * (color * in_front - behind / (1.0 - alpha))))
                behind += color * alpha * in_front
                c = g["conic"].astype(np.float64)
                d_power = d_alpha * d_alpha_d_power
                grads[g["index"]][0] += -d_power * (c[0] * d[0] + c[1] * d[1])
                grads[g["index"]][1] += -d_power * (c[1] * d[0] + c[2] * d[1])
    return grads


def _euler(roll, pitch, yaw):
    cr, sr, cp, sp, cy, sy = np.cos(roll), np.sin(roll), np.cos(pitch), np.sin(pitch), np.cos(yaw), np.sin(yaw)
    rx = np.array([[1, 0, 0], [0, cr, -sr], [0, sr, cr]])
    ry = np.array([[cp, 0, sp], [0, 1, 0], [-sp, 0, cp]])
    rz = np.array([[cy, -sy, 0], [sy, cy, 0], [0, 0, 1]])
    return rz @ ry @ rx


def pose_test_cameras():
    """pose_tests.rs:18-35."""
    poses = [((0.0, 0.0, 0.0), (0.0, 0.0, 0.0)), ((0.4, -0.7, 1.1), (1.5, -2.0, 0.7)),
             ((-0.2, 0.3, -0.5), (-0.8, 0.4, -1.2))]
    return [sb.PinholeCamera(_euler(*e), np.array(t), (40.0, 42.0), (16.0, 16.0), 32, 32) for e, t in poses]


def pose_gradient_matches_finite_differences(make_backend):
    """pose_tests.rs:77-166: the camera gradient of the backward pass chained to the 7
    pose parameters, against finite differences of the render (epsilon 2.5e-4)."""
    rng = np.random.default_rng(11)
    correction = PoseCorrection(np.array([0.1, -0.05, 0.08]), np.array([0.02, -0.03, 0.01]))
    fls = 0.03
    failures, nonzero = [], 0
    for view, initial in enumerate(pose_test_cameras()):
        camera = corrected_camera(initial, correction, fls)
        cloud = gradient_check_cloud(camera, rng)
        backend = make_backend(len(cloud), camera)
        packed = cloud.to_packed()
        pixel_count = camera.width * camera.height
        weights = rng.uniform(-1.0, 1.0, pixel_count * 4).astype(np.float32)
        assert np.any(backend.render(packed).reshape(-1, 4)[:, 3] < 0.5)
        eps = 2.5e-4
        for index in range(7):
            samples = []
            for k in (-2.0, -1.0, 1.0, 2.0):
                moved = PoseCorrection(correction.rotation.copy(), correction.translation.copy())
                f = fls
                if index < 3:
                    moved.rotation[index] += k * eps
                elif index < 6:
                    moved.translation[index - 3] += k * eps
                else:
                    f += k * eps
                backend.set_camera(corrected_camera(initial, moved, f))
                samples.append(backend.render(packed).astype(np.float64).reshape(-1, 4))
            backend.set_camera(camera)
            narrow = (samples[2] - samples[1]) / (2 * eps)
            wide = (samples[3] - samples[0]) / (4 * eps)
            jumps = np.any(np.abs(narrow - wide) > 2e-2 + 5e-2 * np.abs(narrow), axis=1)
            assert jumps.sum() * 20 < pixel_count
            smooth = weights.reshape(-1, 4).copy()
            smooth[jumps] = 0.0
            numeric = float(np.sum(smooth.astype(np.float64) * narrow))
            cam_grad = backend.backward(packed, smooth.reshape(-1))[1]
            pose = pose_gradient(initial, correction, fls, camera_gradient(cam_grad))
            analytic = [*pose.rotation, *pose.translation, pose.focal_log_scale][index]
            if abs(analytic) > 1e-3:
                nonzero += 1
            if abs(analytic - numeric) > 3e-3 + 1e-2 * max(abs(numeric), abs(analytic)):
                failures.append(f"view {view} param {index}: {analytic:.5f} vs {numeric:.5f}")
    assert nonzero >= 18, f"only {nonzero} non-zero pose gradients of 21"
    assert not failures, "\n".join(failures)


__all__ = [
    "forward_matches_the_cpu_reference",
    "gradient_check",
    "identical_images_have_zero_loss",
    "loss_terms_match_the_cpu_reference",
    "loss_gradient_matches_finite_differences",
    "densify_stats_match_the_cpu_mean_gradient",
    "pose_gradient_matches_finite_differences",
    "camera_at_origin",
    "moved_camera",
]
