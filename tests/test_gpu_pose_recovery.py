"""The reference's pose-recovery test (instantsplat-rs/src/pose_tests.rs:190-330), re-created with
numpy's seeded PCG64 in place of rand's StdRng, on the CUDA path with the host pose refinement
(sp_train_step_host_poses: the camera gradient read back every step, the f64 pose Adam).

400 opaque Gaussians of 1-2 px in a box at depth 2-3; three views from x = -1, 0, 1 turned
towards it, photographed from the true cameras; views 1 and 2 start 1.5 degrees and 0.03 away
from the truth, the Gaussians are held fixed (their rates zero) and the poses must come back:
angle and centre error each below a tenth of the start, view 0 untouched, the loss at least
halved, the focal scale within 1 % of 1.

Along the way the camera gradient of the first steps of the perturbed views is compared with
the oracle's backward of the same state (element-wise 1e-4 relative above 1e-6 of the largest).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import splat_b200 as sb
from splat_b200.pose import PoseCorrection, corrected_camera

pytestmark = pytest.mark.gpu


def _opaque_cloud(rng) -> sb.GaussianCloud:
    """pose_tests.rs:190-215."""
    n = 400
    positions = np.stack([rng.uniform(-0.3, 0.3, n), rng.uniform(-0.3, 0.3, n), rng.uniform(2.0, 3.0, n)], axis=1)
    return sb.GaussianCloud(
        positions=positions,
        log_scales=rng.uniform(-4.6, -3.9, (n, 3)),
        rotations=rng.uniform(-1.0, 1.0, (n, 4)),
        opacity_logits=rng.uniform(3.0, 5.0, n),
        sh=rng.uniform(-1.5, 1.5, (n, 1, 3)),
    )


def _rotation_y(angle: float) -> np.ndarray:
    """Rotation3::from_euler_angles(0, angle, 0)."""
    c, s = np.cos(angle), np.sin(angle)
    return np.array([[c, 0.0, s], [0.0, 1.0, 0.0], [-s, 0.0, c]])


def _pose_distance(a: sb.PinholeCamera, b: sb.PinholeCamera) -> tuple[float, float]:
    """(angle of a's rotation relative to b's in degrees, distance of the centres)."""
    relative = a.rotation.T @ b.rotation
    cosine = np.clip((np.trace(relative) - 1.0) / 2.0, -1.0, 1.0)
    return float(np.degrees(np.arccos(cosine))), float(np.linalg.norm(a.translation - b.translation))


def test_perturbed_cameras_are_recovered(ctx):
    rng = np.random.default_rng(5)
    cloud = _opaque_cloud(rng)
    true_cameras = [
        sb.PinholeCamera(_rotation_y(-np.arctan(x / 2.5)), np.array([x, 0.0, 0.0]), (150.0, 150.0), (32.0, 32.0), 64, 64)
        for x in (-1.0, 0.0, 1.0)
    ]
    perturbed = [true_cameras[0]]
    for camera in true_cameras[1:]:
        axis = rng.uniform(-1.0, 1.0, 3)
        axis /= np.linalg.norm(axis)
        direction = rng.uniform(-1.0, 1.0, 3)
        direction /= np.linalg.norm(direction)
        correction = PoseCorrection(rotation=axis * np.radians(1.5), translation=direction * 0.03)
        perturbed.append(corrected_camera(camera, correction, 0.0))
    # The photos: the scene rendered from the true cameras, masked at coverage 0.5 (synthetic_view).
    painter = sb.Trainer(cloud, true_cameras, np.zeros(3 * 64 * 64 * 4, np.float32), ctx=ctx)
    photos = []
    for view in range(3):
        rgbt = painter.render(view).rgbt.reshape(-1, 4)
        mask = ((1.0 - rgbt[:, 3]) > 0.5).astype(np.float32)
        photos.append(np.concatenate([rgbt[:, :3] * mask[:, None], mask[:, None]], axis=1))
    assert int(photos[0][:, 3].sum()) > 500, "the scene covers too little of the view"
    gt = np.stack(photos).reshape(-1)

    fixed = sb.LearningRates(position=0.0, log_scale=0.0, rotation=0.0, opacity=0.0, sh_dc=0.0,
                             camera_rotation=1e-3, camera_translation=1e-3, camera_focal=1e-3, sh_rest=0.0)
    trainer = sb.Trainer(cloud, perturbed, gt, fixed, refine_poses=True, ctx=ctx)

    def errors():
        return [_pose_distance(trainer.camera(v), true_cameras[v]) for v in (1, 2)]

    def loss_over_views():
        return float(np.mean([trainer.loss(v).total for v in range(3)]))

    before = errors()
    loss_before = loss_over_views()
    for view, (angle, distance) in zip((1, 2), before):
        assert abs(angle - 1.5) < 1e-9 and abs(distance - 0.03) < 1e-9, before

    packed = cloud.to_packed()
    for step in range(600):
        view = step % 3
        if step < 6 and view != 0:
            # (View 0 is at its true pose: its render equals its photo bit for bit on the GPU, so
            # the L1 term's sign there is the oracle's rounding against the GPU's, not a gradient.)
            # The camera gradient the step will consume, against the oracle's backward.
            r = trainer.rasterizer
            camera = trainer.camera(view)
            r.set_camera(camera)
            r.encode_forward()
            r.encode_loss(view)
            r.encode_backward()
            cg = r.read_camera_gradient()
            got = np.array([cg.world_to_camera_rotation_rows[i][j] for i in range(3) for j in range(3)]
                           + list(cg.world_to_camera_translation) + list(cg.focal), np.float64)
            cam = oracle.camera_of(camera)
            fwd = oracle.render(packed, 0, cam)
            partials = oracle.ssim(fwd["image"], gt.reshape(3, -1)[view], 64, 64)
            lg, _ = oracle.loss(fwd["image"], gt.reshape(3, -1)[view], partials, 64, 64)
            want = oracle.backward(packed, 0, cam, fwd, lg)["camera_gradient"].astype(np.float64)
            assert np.all(np.abs(got - want) <= 1e-4 * np.abs(want) + 1e-6 * np.abs(want).max()), (step, got, want)
        trainer.step(view, 1.0)
    after = errors()
    loss_after = loss_over_views()
    assert np.array_equal(trainer.camera(0).rotation, true_cameras[0].rotation), "view 0 is fixed"
    for (a0, d0), (a1, d1) in zip(before, after):
        assert a1 < a0 / 10.0, f"angle {a0:.4f} -> {a1:.4f} deg"
        assert d1 < d0 / 10.0, f"centre {d0:.5f} -> {d1:.5f}"
    assert loss_after < loss_before / 2.0, f"loss {loss_before} -> {loss_after}"
    assert abs(trainer.poses.focal_scale() - 1.0) < 0.01
    # The Gaussians did not move (their rates are zero).
    assert np.array_equal(trainer.params.cpu().numpy(), packed)
