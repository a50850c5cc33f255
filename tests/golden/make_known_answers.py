"""Writes reference_known_answers.json: the known answers the reference's own tests hold
for the splatting path, with their inputs, tolerances and the file:line each comes from.

The reference (instantsplat-rs) is Rust + WGSL on wgpu and cannot run here, and its tests
store no golden vectors (they draw inputs from rand's StdRng at test time), so these
constants — stated in its test sources — are what pins the oracle and the CUDA path. The
expected values are computed here from the tests' own formulas (e.g. 0.8 * exp(-0.5 * 4 /
4.3)) in f32, as the tests compute them.

    python tests/golden/make_known_answers.py
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "reference_known_answers.json"


def f32(x) -> float:
    return float(np.float32(x))


def main() -> None:
    known_gaussian = {
        "source": "instantsplat-rs/src/rasterizer_tests.rs:86-127 (renders_a_known_gaussian)",
        "image": {"width": 32, "height": 32, "focal": 100.0, "principal_point": [16, 16]},
        "gaussian": {"position": [0.0, 0.0, 5.0], "sigma": 0.1, "opacity": 0.8, "rgb": [1.0, 0.0, 0.0]},
        "tolerance": 1e-3,
        "premultiplied": [
            {"pixel": [16, 16], "rgb": [f32(0.8), 0.0, 0.0]},
            {"pixel": [18, 16], "rgb": [f32(0.8 * np.exp(np.float32(-0.5 * 4.0 / 4.3))), 0.0, 0.0]},
            {"pixel": [16, 13], "rgb": [f32(0.8 * np.exp(np.float32(-0.5 * 9.0 / 4.3))), 0.0, 0.0]},
        ],
        "alpha": [{"pixel": [18, 16], "value": f32(0.8 * np.exp(np.float32(-0.5 * 4.0 / 4.3)))}],
        "transmittance": [{"pixel": [16, 16], "value": 0.2}],
        "exact_corners": [{"pixel": [0, 0], "rgb": [0.0, 0.0, 0.0]}, {"pixel": [31, 31], "rgb": [0.0, 0.0, 0.0]}],
        "background": [0.50196, 0.50196, 0.50196],
        "over_background_center": [f32(0.8 + 0.2 * 0.50196), f32(0.2 * 0.50196), f32(0.2 * 0.50196)],
        "rgba8": [{"pixel": [16, 16], "value": [255, 0, 0, 204]}, {"pixel": [0, 0], "value": [0, 0, 0, 0]}],
    }
    culled = {
        "source": "instantsplat-rs/src/rasterizer_tests.rs:129-135 (a_gaussian_behind_the_camera_is_culled)",
        "image": {"width": 32, "height": 32, "focal": 100.0, "principal_point": [16, 16]},
        "gaussian": {"position": [0.0, 0.0, -5.0], "sigma": 0.1, "opacity": 0.8, "rgb": [1.0, 0.0, 0.0]},
        "every_pixel": [0.0, 0.0, 0.0, 1.0],
    }
    ssim_taps = {
        "source": "instantsplat-rs/src/loss.rs:121-129 (ssim_taps_are_the_3dgs_window)",
        "sum": 1.0,
        "sum_tolerance": 1e-6,
        "center": 0.26601,
        "center_tolerance": 1e-5,
        "edge": 0.0010284,
        "edge_tolerance": 1e-6,
        "symmetric_pair": [1, 9],
    }
    loss_terms = {
        "source": "instantsplat-rs/src/loss.rs:131-138 (mean_loss_terms)",
        "pixel_loss": [0.2, 1.0, 0.5, 2.0, 0.4, 0.0, 0.1, 1.0],
        "expected": {"l1": 0.3, "alpha": 0.5, "dssim": 0.3, "total": 1.5},
        "tolerance": 1e-6,
        "weights_source": "instantsplat-rs/src/loss.rs:32-36",
        "weights": {"l1": 0.8, "dssim": 0.2, "alpha": 1.0},
    }
    learning_rates = {
        "source": "instantsplat-rs/src/optimizer.rs:278-290 (slots_get_their_group_rate)",
        "position_scale": 2.0,
        "rates_3dgs": {"position": 1.6e-4, "log_scale": 5e-3, "rotation": 1e-3, "opacity": 5e-2, "sh_dc": 2.5e-3,
                       "camera_rotation": 1e-2, "camera_translation": 1e-2, "camera_focal": 0.0},
        "by_slot_exact": [{"slot": 0, "value": f32(np.float32(1.6e-4) * np.float32(2.0))}, {"slot": 3, "value": f32(5e-3)},
                          {"slot": 6, "value": f32(1e-3)}, {"slot": 10, "value": f32(5e-2)},
                          {"slot": 13, "value": f32(2.5e-3)}],
    }
    position_rate = {
        "source": "instantsplat-rs/src/optimizer.rs:292-298 (position_rate_decays_to_one_percent)",
        "cases": [
            {"step": 0, "steps": 1000, "value": 1.0, "exact": True},
            {"step": 999, "steps": 1000, "value": 0.01, "tolerance": 1e-6},
            {"step": 500, "steps": 1001, "value": 0.1, "tolerance": 1e-6},
            {"step": 0, "steps": 1, "value": 1.0, "exact": True},
        ],
    }
    cap = f32(np.log(np.float32(0.02)))
    clamp = {
        "source": "instantsplat-rs/src/prune.rs:113-141 (clamp_caps_absolute_scale_and_anisotropy)",
        "log_scales": [[-3.0, -3.0, -3.0], [-3.0, -3.0, 0.0], [-5.0, -5.0, -1.0]],
        "cases": [
            {"extent": 1.0, "expected": [[cap, cap, cap], [cap, cap, cap], [-5.0, -5.0, cap]], "exact": True},
            {"extent": 100.0, "expected": [[-3.0, -3.0, -3.0], [-3.0, -3.0, f32(-3.0 + np.log(np.float32(10.0)))],
                                           [-5.0, -5.0, f32(-5.0 + np.log(np.float32(10.0)))]], "tolerance": 1e-6},
        ],
    }
    cameras = {
        "extent_source": "instantsplat-rs/src/camera.rs:284-296 (extent_is_1_1_times_farthest_camera)",
        "centres_x": [-1.0, 1.0, 3.0],
        "extent": 2.2,
        "wider_source": "instantsplat-rs/src/camera.rs:265-282 (a_wider_image_keeps_the_center_and_the_scale)",
        "wider": {"principal_point": [9.5, 14.5], "size": [20, 30], "new_size": [40, 30],
                  "new_principal_point": [19.5, 14.5]},
    }
    pose = {
        "source": "instantsplat-rs/src/pose_refinement.rs:166-220 and camera_pose.rs:114-225",
        # The rates are f32 constants widened to f64 (pose_refinement.rs:421).
        "step_translation": {"rate": 1e-2, "extent": 2.0, "expected_x": 1.0 + float(np.float32(1e-2)) * 2.0,
                             "tolerance": 1e-12},
        "linear_loss_gradient": {
            "world_to_camera_rotation_rows": [[0.3, -1.2, 0.7], [2.0, 0.1, -0.4], [-0.9, 0.5, 1.3]],
            "world_to_camera_translation": [0.8, -0.6, 1.1],
            "focal": [0.02, -0.05],
            "correction_rotation": [0.2, -0.1, 0.3],
            "correction_translation": [-0.3, 0.4, 0.1],
            "focal_log_scale": 0.05,
            "camera_euler": [0.4, -0.7, 1.1],
            "camera_translation": [1.5, -2.0, 0.7],
            "focal": [40.0, 42.0],
            "tolerance": 1e-6,
        },
        "focal_step": {"rate": 1e-3, "expected_log_scale": float(np.float32(1e-3)), "tolerance": 1e-12},
    }
    constants = {
        "source": "instantsplat-rs/src/shaders.rs:50-63 and shaders/common.wgsl:7-36",
        "TILE": 16, "PARAM_STRIDE": 14, "GRAD_STRIDE": 10, "CAMERA_GRAD_STRIDE": 14, "DEPTH_BITS": 20,
        "SSIM_RADIUS": 5, "SSIM_SIGMA": 1.5, "CameraGradient_bytes": 56, "Projected_bytes": 80,
        "CameraUniform_bytes": 80, "IntersectionMeta_bytes": 20, "DensifyStats_bytes": 16,
        "SH_C0": 0.28209479, "COVARIANCE_BLUR": 0.3, "NEAR_Z": 0.01, "VIEW_LIMIT_FACTOR": 1.3,
        "MAX_ALPHA": 0.99, "MIN_TRANSMITTANCE": 1e-4, "SSIM_C1": 0.0001, "SSIM_C2": 0.0009,
        "INTERSECTIONS_PER_GAUSSIAN": 24, "MAX_TILES": 4096,
    }
    packing = {
        "source": "instantsplat-rs/src/gaussians.rs:410-424 (packed_layout_round_trips)",
        "positions": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0],
        "log_scales": [-1.0, -2.0, -3.0, -4.0, -5.0, -6.0],
        "rotations": [1.0, 0.0, 0.0, 0.0, 0.5, 0.5, 0.5, 0.5],
        "opacity_logits": [0.1, 0.2],
        "sh_dc": [7.0, 8.0, 9.0, 10.0, 11.0, 12.0],
        "packed_14_17": [4.0, 5.0, 6.0],
        "packed_10": 0.1,
    }
    data = {
        "note": "Known answers from the reference's tests (instantsplat-rs); written by make_known_answers.py",
        "known_gaussian": known_gaussian,
        "culled": culled,
        "ssim_taps": ssim_taps,
        "loss_terms": loss_terms,
        "learning_rates": learning_rates,
        "position_rate": position_rate,
        "clamp": clamp,
        "cameras": cameras,
        "pose": pose,
        "constants": constants,
        "packing": packing,
    }
    OUT.write_text(json.dumps(data, indent=1) + "\n")
    print(OUT)


if __name__ == "__main__":
    main()
