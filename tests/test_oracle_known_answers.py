"""The oracle and the host logic against the known answers of the reference's own tests
(tests/golden/reference_known_answers.json). CPU only."""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import oracle
import splat_b200 as sb
from helpers import camera_at_origin, single_gaussian
from splat_b200 import _lib
from splat_b200.pose import PoseCorrection, camera_gradient, corrected_camera, pose_gradient

KNOWN = json.loads((Path(__file__).resolve().parent / "golden" / "reference_known_answers.json").read_text())


def oracle_render(cloud, camera):
    return oracle.render(cloud.to_packed(), cloud.sh_degree, oracle.camera_array(camera.uniform()))


def known_scene(section):
    img = section["image"]
    g = section["gaussian"]
    camera = camera_at_origin(img["width"], img["height"], img["focal"])
    return single_gaussian(g["position"], g["sigma"], g["opacity"], g["rgb"]), camera


def test_known_gaussian():
    k = KNOWN["known_gaussian"]
    cloud, camera = known_scene(k)
    rendered = sb.Rendered(camera.width, camera.height, oracle_render(cloud, camera)["image"])
    tol = k["tolerance"]
    for case in k["premultiplied"]:
        assert np.max(np.abs(rendered.premultiplied(*case["pixel"]) - case["rgb"])) <= tol, case
    for case in k["alpha"]:
        assert abs(rendered.alpha(*case["pixel"]) - case["value"]) < tol
    for case in k["transmittance"]:
        assert abs(rendered.transmittance(*case["pixel"]) - case["value"]) < tol
    for case in k["exact_corners"]:
        assert np.array_equal(rendered.premultiplied(*case["pixel"]), case["rgb"])
        assert np.array_equal(rendered.over_background(0, 0), np.array(k["background"], np.float32))
    over = rendered.over_background(16, 16)
    assert np.max(np.abs(over - k["over_background_center"])) < tol
    rgba = rendered.to_rgba8()
    for case in k["rgba8"]:
        x, y = case["pixel"]
        assert list(rgba[y, x]) == case["value"]


def test_culled():
    c = KNOWN["culled"]
    cloud, camera = known_scene(c)
    image = oracle_render(cloud, camera)["image"].reshape(-1, 4)
    assert np.all(image == np.array(c["every_pixel"], np.float32))


def test_ssim_taps():
    k = KNOWN["ssim_taps"]
    # The window the oracle applies: its SSIM of an image against itself shifted by the
    # window recovers the taps; simpler, restate common.wgsl:110-122 with the shared exp.
    taps = np.array([oracle.sp_expf(-(d * d) / np.float32(4.5)) for d in range(-5, 6)], np.float32)
    taps = taps / np.float32(taps.sum(dtype=np.float32))
    assert abs(float(taps.sum()) - k["sum"]) < k["sum_tolerance"]
    assert abs(float(taps[5]) - k["center"]) < k["center_tolerance"]
    assert abs(float(taps[0]) - k["edge"]) < k["edge_tolerance"]
    assert taps[k["symmetric_pair"][0]] == taps[k["symmetric_pair"][1]]


def test_loss_terms_mean():
    k = KNOWN["loss_terms"]
    terms = sb.LossTerms.from_pixel_loss(np.array(k["pixel_loss"], np.float32))
    for name, value in k["expected"].items():
        assert abs(getattr(terms, name) - value) < k["tolerance"]


def test_learning_rates_by_slot():
    k = KNOWN["learning_rates"]
    rates = sb.LearningRates(**k["rates_3dgs"])
    by_slot = rates.by_slot(k["position_scale"], 14)
    from_oracle = oracle.learning_rates_by_slot(rates.to_c(), k["position_scale"], 14)
    assert np.array_equal(by_slot, from_oracle)
    for case in k["by_slot_exact"]:
        assert by_slot[case["slot"]] == np.float32(case["value"])


def test_position_rate_factor():
    for case in KNOWN["position_rate"]["cases"]:
        value = sb.position_rate_factor(case["step"], case["steps"])
        if case.get("exact"):
            assert value == case["value"]
        else:
            assert abs(value - case["value"]) < case["tolerance"]
    with pytest.raises(ValueError):
        sb.position_rate_factor(5, 5)


@pytest.mark.parametrize("index", [0, 1])
def test_scale_clamp(index):
    k = KNOWN["clamp"]
    case = k["cases"][index]
    n = len(k["log_scales"])
    params = np.zeros((n, 14), np.float32)
    params[:, 3:6] = k["log_scales"]
    params[:, 6] = 1.0
    flat = params.reshape(-1).copy()
    zeros = np.zeros_like(flat)
    extent = np.float32(case["extent"])
    oracle.adam_step(flat, zeros, zeros.copy(), zeros.copy(), 14, np.zeros(14, np.float32), 1,
                     float(np.log(np.float32(0.02) * extent)), float(np.log(np.float32(10.0))))
    got = flat.reshape(n, 14)[:, 3:6]
    want = np.array(case["expected"], np.float32)
    if case.get("exact"):
        assert np.array_equal(got, want)
    else:
        assert np.max(np.abs(got - want)) < case["tolerance"]


def test_cameras():
    k = KNOWN["cameras"]
    cams = [sb.PinholeCamera(np.eye(3), np.array([x, 0.0, 0.0]), (1, 1), (0, 0), 1, 1) for x in k["centres_x"]]
    assert abs(sb.cameras_extent(cams) - k["extent"]) < 1e-12
    w = k["wider"]
    cam = sb.PinholeCamera(np.eye(3), np.zeros(3), (100, 100), tuple(w["principal_point"]), *w["size"])
    wider = cam.with_image_size(*w["new_size"])
    assert list(wider.principal_point) == w["new_principal_point"]
    assert wider.focal == cam.focal


def test_camera_uniform_inverts_pose():
    """camera.rs:103-118 through the library's PinholeCamera::uniform."""
    from helpers import moved_camera

    camera = moved_camera()
    u = camera.uniform()
    rows = np.array([[u.world_to_camera_rows[r][c] for c in range(4)] for r in range(3)], np.float64)
    point = np.array([0.5, -1.0, 4.0])
    in_camera = rows[:, :3] @ point + rows[:, 3]
    back = camera.rotation @ in_camera + camera.translation
    assert np.linalg.norm(back - point) < 1e-5
    assert (u.tiles_x, u.tiles_y) == (2, 2)


def _euler(roll, pitch, yaw):
    cr, sr, cp, sp, cy, sy = np.cos(roll), np.sin(roll), np.cos(pitch), np.sin(pitch), np.cos(yaw), np.sin(yaw)
    rx = np.array([[1, 0, 0], [0, cr, -sr], [0, sr, cr]])
    ry = np.array([[cp, 0, sp], [0, 1, 0], [-sp, 0, cp]])
    rz = np.array([[cy, -sy, 0], [sy, cy, 0], [0, 0, 1]])
    return rz @ ry @ rx


def test_pose_gradient_of_a_linear_loss():
    """camera_pose.rs:150-209: the chain rule against finite differences of a loss linear
    in the world-to-camera entries."""
    k = KNOWN["pose"]["linear_loss_gradient"]
    initial = sb.PinholeCamera(_euler(*k["camera_euler"]), np.array(k["camera_translation"]), tuple(k["focal"]),
                               (16.0, 16.0), 32, 32)
    coeff = np.concatenate([np.array(k["world_to_camera_rotation_rows"]).reshape(-1),
                            k["world_to_camera_translation"], k["focal"]]).astype(np.float32)
    gradient = camera_gradient(coeff)
    coeff = coeff.astype(np.float64)

    def loss(correction, focal_log_scale):
        cam = corrected_camera(initial, correction, focal_log_scale)
        w, t = cam.world_to_camera()
        return float(np.sum(coeff[:9] * w.reshape(-1)) + np.sum(coeff[9:12] * t) + coeff[12] * cam.focal[0]
                     + coeff[13] * cam.focal[1])

    correction = PoseCorrection(np.array(k["correction_rotation"]), np.array(k["correction_translation"]))
    fls = k["focal_log_scale"]
    analytic = pose_gradient(initial, correction, fls, gradient)
    eps = 1e-6
    for axis in range(3):
        d = np.zeros(3)
        d[axis] = eps
        num = (loss(PoseCorrection(correction.rotation + d, correction.translation), fls)
               - loss(PoseCorrection(correction.rotation - d, correction.translation), fls)) / (2 * eps)
        assert abs(num - analytic.rotation[axis]) < k["tolerance"]
        num = (loss(PoseCorrection(correction.rotation, correction.translation + d), fls)
               - loss(PoseCorrection(correction.rotation, correction.translation - d), fls)) / (2 * eps)
        assert abs(num - analytic.translation[axis]) < k["tolerance"]
    num = (loss(correction, fls + eps) - loss(correction, fls - eps)) / (2 * eps)
    assert abs(num - analytic.focal_log_scale) < k["tolerance"]


def test_pose_refinement_steps():
    """pose_refinement.rs:166-220."""
    k = KNOWN["pose"]
    cams = [sb.PinholeCamera(np.eye(3), np.array([float(i), 0.0, 0.0]), (100, 100), (10, 10), 20, 20) for i in range(2)]
    refinement = sb.PoseRefinement(cams, sb.LEARNING_RATES_3DGS, k["step_translation"]["extent"])
    g = camera_gradient([0] * 9 + [1, 0, 0] + [0, 0])
    refinement.step(1, g, 1.0)
    moved = refinement.camera(1).translation
    assert abs(moved[0] - k["step_translation"]["expected_x"]) < k["step_translation"]["tolerance"]
    assert np.array_equal(refinement.camera(1).rotation, np.eye(3))
    refinement.step(0, g, 1.0)
    assert np.array_equal(refinement.camera(0).translation, np.zeros(3))
    assert refinement.focal_scale() == 1.0
    rates = sb.LearningRates(camera_focal=k["focal_step"]["rate"])
    refinement = sb.PoseRefinement(cams, rates, 1.0)
    refinement.step(0, camera_gradient([0] * 12 + [-1, -1]), 1.0)
    assert abs(np.log(refinement.focal_scale()) - k["focal_step"]["expected_log_scale"]) < k["focal_step"]["tolerance"]
    assert refinement.camera(1).focal[0] == 100.0 * refinement.focal_scale()
    with pytest.raises(sb.SplatError):
        refinement.step(0, camera_gradient([float("nan")] * 14), 1.0)


def test_packing():
    k = KNOWN["packing"]
    cloud = sb.GaussianCloud(
        positions=np.array(k["positions"]).reshape(2, 3), log_scales=np.array(k["log_scales"]).reshape(2, 3),
        rotations=np.array(k["rotations"]).reshape(2, 4), opacity_logits=np.array(k["opacity_logits"]),
        sh=np.array(k["sh_dc"]).reshape(2, 1, 3),
    )
    packed = cloud.to_packed()
    assert packed.size == 28
    assert np.array_equal(packed[14:17], np.array(k["packed_14_17"], np.float32))
    assert packed[10] == np.float32(k["packed_10"])
    back = sb.GaussianCloud.from_packed(packed)
    assert np.array_equal(back.positions, cloud.positions) and np.array_equal(back.sh, cloud.sh)
    for p in (0.01, 0.1, 0.5, 0.9):
        assert abs(float(sb.sigmoid(sb.logit(p))) - p) < 1e-6
    assert abs(float(sb.gaussians.SH_C0 * sb.rgb_to_sh_dc(0.8) + 0.5) - 0.8) < 1e-6


def test_constants_match_the_headers():
    """shaders.rs:50-63: the constants every kernel relies on."""
    k = KNOWN["constants"]
    text = (Path(__file__).resolve().parents[1] / "include" / "splat_constants.h").read_text()
    for name, header in [("TILE", "SP_TILE"), ("PARAM_STRIDE", "SP_PARAM_STRIDE_SH0"), ("GRAD_STRIDE", "SP_GRAD_STRIDE"),
                         ("CAMERA_GRAD_STRIDE", "SP_CAMERA_GRAD_STRIDE"), ("DEPTH_BITS", "SP_DEPTH_BITS"),
                         ("SSIM_RADIUS", "SP_SSIM_RADIUS"), ("INTERSECTIONS_PER_GAUSSIAN", "SP_INTERSECTIONS_PER_GAUSSIAN")]:
        assert f"#define {header} {k[name]}\n" in text, name
    for name, header in [("SH_C0", "SP_SH_C0"), ("COVARIANCE_BLUR", "SP_COVARIANCE_BLUR"), ("NEAR_Z", "SP_NEAR_Z"),
                         ("VIEW_LIMIT_FACTOR", "SP_VIEW_LIMIT_FACTOR"), ("MAX_ALPHA", "SP_MAX_ALPHA"),
                         ("SSIM_SIGMA", "SP_SSIM_SIGMA"), ("SSIM_C1", "SP_SSIM_C1"), ("SSIM_C2", "SP_SSIM_C2"),
                         ("MIN_TRANSMITTANCE", "SP_MIN_TRANSMITTANCE")]:
        line = next(l for l in text.splitlines() if l.startswith(f"#define {header} "))
        assert np.float32(line.split()[2].rstrip("f")) == np.float32(k[name]), name
    assert ctypes.sizeof(_lib.CameraGradient) == k["CameraGradient_bytes"]
    assert ctypes.sizeof(_lib.Projected) == k["Projected_bytes"]
    assert ctypes.sizeof(_lib.CameraUniform) == k["CameraUniform_bytes"]
    assert ctypes.sizeof(_lib.IntersectionMeta) == k["IntersectionMeta_bytes"]
    assert ctypes.sizeof(_lib.DensifyStats) == k["DensifyStats_bytes"]
