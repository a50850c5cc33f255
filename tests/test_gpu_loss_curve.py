"""Loss-curve parity (the benchmark's config 0): 20k Gaussians, SH degree 0, 3 views of
256 x 256, 100 training steps (forward, loss, backward, Adam with the scale clamp) on the
CUDA path through the C ABI against the CPU oracle's full training step on the same
seeded inputs. Bar: every step's mean total loss within 1e-3 relative."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import splat_b200 as sb
from splat_b200 import scenes

pytestmark = pytest.mark.gpu

STEPS = 100


def ground_truth(scene):
    gts = []
    for cam in scene.cameras:
        rgbt = oracle.render(scene.truth.to_packed(), 0, oracle.camera_array(cam.uniform()))["image"].reshape(-1, 4)
        mask = ((1.0 - rgbt[:, 3]) > 0.5).astype(np.float32)
        gts.append(np.concatenate([rgbt[:, :3] * mask[:, None], mask[:, None]], axis=1))
    return np.stack(gts).astype(np.float32)


@pytest.mark.parametrize("mode", [sb.SP_BWD_DETERMINISTIC, sb.SP_BWD_ATOMIC])
def test_loss_curve_matches_the_oracle(ctx, mode):
    import torch

    scene = scenes.config(0)
    cams = scene.cameras
    gt = ground_truth(scene)
    extent = np.float32(sb.cameras_extent(cams))
    rates = sb.LEARNING_RATES_3DGS

    params = torch.from_numpy(scene.cloud.to_packed()).cuda()
    gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
    rast = sb.Rasterizer(ctx, params, len(scene.cloud), 256, 256, gt_dev, len(cams),
                         sb.default_options(backward_mode=mode))
    adam = sb.Adam(ctx, params, rast, len(scene.cloud), rates, extent)
    gpu_losses = []
    for step in range(STEPS):
        view = step % len(cams)
        rast.set_camera(cams[view])
        rast.encode_forward()
        rast.encode_loss(view)
        rast.encode_backward()
        adam.encode_step(sb.position_rate_factor(step, STEPS))
        gpu_losses.append(rast.read_loss().total)

    packed = scene.cloud.to_packed().copy()
    m, v = np.zeros_like(packed), np.zeros_like(packed)
    max_log = float(np.log(np.float32(0.02) * extent))
    aniso = float(np.log(np.float32(10.0)))
    oracle_losses = []
    for step in range(STEPS):
        view = step % len(cams)
        factor = np.float32(sb.position_rate_factor(step, STEPS))
        lr = oracle.learning_rates_by_slot(rates.to_c(), np.float32(extent * factor), 14)
        loss, _ = oracle.train_step(packed, 0, oracle.camera_array(cams[view].uniform()), gt[view].reshape(-1), m, v, lr,
                                    step + 1, max_log, aniso)
        oracle_losses.append(loss)

    gpu_losses, oracle_losses = np.array(gpu_losses), np.array(oracle_losses)
    rel = np.abs(gpu_losses - oracle_losses) / np.abs(oracle_losses)
    assert rel.max() < 1e-3, f"step {rel.argmax()}: {gpu_losses[rel.argmax()]} vs {oracle_losses[rel.argmax()]}"
    # The run trains: the loss falls.
    assert gpu_losses[-3:].mean() < gpu_losses[:3].mean()


def _camera_gradient(values):
    v = np.asarray(values, np.float32)
    from splat_b200._lib import CameraGradient

    cg = CameraGradient()
    for i in range(3):
        for j in range(3):
            cg.world_to_camera_rotation_rows[i][j] = float(v[3 * i + j])
    for i in range(3):
        cg.world_to_camera_translation[i] = float(v[9 + i])
    cg.focal[0], cg.focal[1] = float(v[12]), float(v[13])
    return cg


@pytest.mark.parametrize("mode", [sb.SP_BWD_DETERMINISTIC, sb.SP_BWD_ATOMIC])
def test_loss_curve_with_pose_refinement_matches_the_oracle(ctx, mode):
    """The same 100 steps with pose refinement on (Trainer::step_async with a PoseRefinement,
    training.rs:197-209): each step's camera from the refinement, the step, the camera gradient
    read back and the f64 pose Adam step. The oracle's leg takes the oracle's render, loss,
    backward and Adam and feeds its own camera gradient to its own refinement (the host pose
    chain, pinned by the reference's known answers, is the same code on both legs). Bars: every
    step's loss within 1e-3 relative; the refined poses of views 1 and 2 (view 0 stays fixed)
    within 1e-3 of how far the refinement moved them (Adam's normalised steps integrate the
    rounding-level differences of the two legs' camera gradients over the run: measured 1.7e-4)."""
    import torch

    scene = scenes.config(0)
    cams = scene.cameras
    gt = ground_truth(scene)
    extent = np.float32(sb.cameras_extent(cams))
    rates = sb.LEARNING_RATES_3DGS

    params = torch.from_numpy(scene.cloud.to_packed()).cuda()
    gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
    rast = sb.Rasterizer(ctx, params, len(scene.cloud), 256, 256, gt_dev, len(cams),
                         sb.default_options(backward_mode=mode))
    adam = sb.Adam(ctx, params, rast, len(scene.cloud), rates, extent)
    poses = sb.PoseRefinement(cams, rates, float(extent))
    gpu_losses = []
    for step in range(STEPS):
        view = step % len(cams)
        factor = sb.position_rate_factor(step, STEPS)
        gradient, loss = rast.train_step(adam, poses.camera(view), view, factor)
        poses.step(view, gradient, factor)
        gpu_losses.append(loss.total)

    packed = scene.cloud.to_packed().copy()
    m, v = np.zeros_like(packed), np.zeros_like(packed)
    max_log = float(np.log(np.float32(0.02) * extent))
    aniso = float(np.log(np.float32(10.0)))
    oracle_poses = sb.PoseRefinement(cams, rates, float(extent))
    oracle_losses = []
    for step in range(STEPS):
        view = step % len(cams)
        factor = sb.position_rate_factor(step, STEPS)
        cam = oracle.camera_of(oracle_poses.camera(view))
        fwd = oracle.render(packed, 0, cam)
        partials = oracle.ssim(fwd["image"], gt[view].reshape(-1), 256, 256)
        loss_gradient, pixel_loss = oracle.loss(fwd["image"], gt[view].reshape(-1), partials, 256, 256)
        bwd = oracle.backward(packed, 0, cam, fwd, loss_gradient)
        lr = oracle.learning_rates_by_slot(rates.to_c(), np.float32(extent * np.float32(factor)), 14)
        oracle.adam_step(packed, bwd["param_gradients"], m, v, 14, lr, step + 1, max_log, aniso)
        oracle_poses.step(view, _camera_gradient(bwd["camera_gradient"]), factor)
        oracle_losses.append(float(np.mean(pixel_loss.reshape(-1, 4)[:, 3].astype(np.float64))))

    gpu_losses, oracle_losses = np.array(gpu_losses), np.array(oracle_losses)
    rel = np.abs(gpu_losses - oracle_losses) / np.abs(oracle_losses)
    assert rel.max() < 1e-3, f"step {rel.argmax()}: {gpu_losses[rel.argmax()]} vs {oracle_losses[rel.argmax()]}"
    assert gpu_losses[-3:].mean() < gpu_losses[:3].mean()
    for view in range(1, len(cams)):
        got, want = poses.camera(view), oracle_poses.camera(view)
        moved = max(np.abs(want.rotation - cams[view].rotation).max(),
                    np.abs(want.translation - cams[view].translation).max())
        assert moved > 0.0, "the refinement moved the pose"
        assert np.abs(got.rotation - want.rotation).max() <= 1e-3 * moved
        assert np.abs(got.translation - want.translation).max() <= 1e-3 * moved


def test_fused_train_step_equals_the_separate_calls(ctx):
    """sp_train_step (one call with its 88-byte read-back) against set_camera, forward, loss,
    backward, Adam and the two reads issued one by one: bit-identical parameters, camera
    gradients and losses over 10 steps (deterministic backward)."""
    import torch

    scene = scenes.config(0)
    cams = scene.cameras
    gt_dev = torch.from_numpy(ground_truth(scene).reshape(-1)).cuda()
    extent = np.float32(sb.cameras_extent(cams))
    runs = []
    for fused in (False, True):
        params = torch.from_numpy(scene.cloud.to_packed()).cuda()
        rast = sb.Rasterizer(ctx, params, len(scene.cloud), 256, 256, gt_dev, len(cams),
                             sb.default_options(backward_mode=sb.SP_BWD_DETERMINISTIC))
        adam = sb.Adam(ctx, params, rast, len(scene.cloud), sb.LEARNING_RATES_3DGS, extent)
        trace = []
        for step in range(10):
            view, factor = step % len(cams), sb.position_rate_factor(step, 10)
            if fused:
                gradient, loss = rast.train_step(adam, cams[view], view, factor)
            else:
                rast.set_camera(cams[view])
                rast.encode_forward()
                rast.encode_loss(view)
                rast.encode_backward()
                adam.encode_step(factor)
                gradient, loss = rast.read_camera_gradient(), rast.read_loss()
            trace.append((bytes(gradient), loss.total, loss.l1, loss.dssim, loss.alpha))
        ctx.sync()
        runs.append((trace, params.cpu().numpy().copy()))
        del adam, rast
    assert runs[0][0] == runs[1][0]
    assert np.array_equal(runs[0][1].view(np.uint32), runs[1][1].view(np.uint32))


def test_device_poses_equal_host_poses(ctx):
    """The pose refinement on the device (sp_device_poses, no host synchronisation per step)
    against the host refinement fed the read-back camera gradient (the reference's
    Trainer::step_async, training.rs:197-209): 20 steps of config 0 with poses refined, the
    deterministic backward. The corrections, the focal scale and every step's loss agree to
    f64 rounding of the math library (1e-9 relative)."""
    import torch

    scene = scenes.config(0)
    cams = scene.cameras
    gt_dev = torch.from_numpy(ground_truth(scene).reshape(-1)).cuda()
    extent = np.float32(sb.cameras_extent(cams))
    rates = sb.LEARNING_RATES_3DGS
    steps = 20
    runs = []
    for device in (False, True):
        params = torch.from_numpy(scene.cloud.to_packed()).cuda()
        rast = sb.Rasterizer(ctx, params, len(scene.cloud), 256, 256, gt_dev, len(cams),
                             sb.default_options(backward_mode=sb.SP_BWD_DETERMINISTIC))
        adam = sb.Adam(ctx, params, rast, len(scene.cloud), rates, extent)
        poses = sb.PoseRefinement(cams, rates, float(extent))
        losses = []
        if device:
            dp = sb.DevicePoses(rast, poses)
            sums = torch.zeros(4, dtype=torch.float64).pin_memory()
            dp.set_camera(0)
            for step in range(steps):
                view, nxt = step % len(cams), (step + 1) % len(cams)
                rast.train_step_device_poses(adam, dp, view, nxt, sb.position_rate_factor(step, steps), sums)
                ctx.sync()
                losses.append(float(sums[3]) / (256 * 256))
            dp.download()
        else:
            for step in range(steps):
                view = step % len(cams)
                factor = sb.position_rate_factor(step, steps)
                gradient, loss = rast.train_step(adam, poses.camera(view), view, factor)
                poses.step(view, gradient, factor)
                losses.append(loss.total)
        corrections = [poses.correction(v) for v in range(len(cams))]
        runs.append((np.array(losses), corrections, poses.focal_scale()))
        del adam, rast
    (l0, c0, f0), (l1, c1, f1) = runs
    np.testing.assert_allclose(l1, l0, rtol=1e-6)
    assert abs(f1 - f0) <= 1e-9 * abs(f0)
    for a, b in zip(c0, c1):
        np.testing.assert_allclose(b.rotation, a.rotation, rtol=1e-9, atol=1e-15)
        np.testing.assert_allclose(b.translation, a.translation, rtol=1e-9, atol=1e-15)
    # The refinement moved the poses of every view but the fixed first one.
    assert np.all(c0[0].rotation == 0.0) and np.any(c0[1].rotation != 0.0)


def test_host_pose_step_in_one_call(ctx):
    """sp_train_step_host_poses (camera from the refinement, step, read-back, host pose step in
    one call) against the same sequence from Python: identical losses and corrections."""
    import torch

    scene = scenes.config(0)
    cams = scene.cameras
    gt_dev = torch.from_numpy(ground_truth(scene).reshape(-1)).cuda()
    extent = np.float32(sb.cameras_extent(cams))
    rates = sb.LEARNING_RATES_3DGS
    runs = []
    for one_call in (False, True):
        params = torch.from_numpy(scene.cloud.to_packed()).cuda()
        rast = sb.Rasterizer(ctx, params, len(scene.cloud), 256, 256, gt_dev, len(cams),
                             sb.default_options(backward_mode=sb.SP_BWD_DETERMINISTIC))
        adam = sb.Adam(ctx, params, rast, len(scene.cloud), rates, extent)
        poses = sb.PoseRefinement(cams, rates, float(extent))
        losses = []
        for step in range(6):
            view, factor = step % len(cams), sb.position_rate_factor(step, 6)
            if one_call:
                losses.append(rast.train_step_host_poses(adam, poses, view, factor).total)
            else:
                gradient, loss = rast.train_step(adam, poses.camera(view), view, factor)
                poses.step(view, gradient, factor)
                losses.append(loss.total)
        runs.append((losses, [poses.correction(v) for v in range(len(cams))], poses.focal_scale()))
        del adam, rast
    assert runs[0][0] == runs[1][0] and runs[0][2] == runs[1][2]
    for a, b in zip(runs[0][1], runs[1][1]):
        assert np.array_equal(a.rotation, b.rotation) and np.array_equal(a.translation, b.translation)
