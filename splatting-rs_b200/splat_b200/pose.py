"""Camera pose refinement (host, f64) — instantsplat-rs/src/camera_pose.rs and
pose_refinement.rs, computed by libsplat_b200's host code."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import CameraGradient, PinholeCameraC, PoseCorrectionC, PoseGradientC
from .camera import PinholeCamera
from .optimizer import LearningRates

FIXED_VIEW = 0


@dataclass
class PoseCorrection:
    """PoseCorrection (camera_pose.rs:14-21)."""

    rotation: np.ndarray = field(default_factory=lambda: np.zeros(3))
    translation: np.ndarray = field(default_factory=lambda: np.zeros(3))

    def to_c(self) -> PoseCorrectionC:
        c = PoseCorrectionC()
        for i in range(3):
            c.rotation[i] = float(self.rotation[i])
            c.translation[i] = float(self.translation[i])
        return c


@dataclass
class PoseGradient:
    """PoseGradient (camera_pose.rs:23-29)."""

    rotation: np.ndarray
    translation: np.ndarray
    focal_log_scale: float

    @staticmethod
    def from_c(c: PoseGradientC) -> "PoseGradient":
        return PoseGradient(np.array(list(c.rotation)), np.array(list(c.translation)), c.focal_log_scale)


def camera_gradient(values) -> CameraGradient:
    """A CameraGradient from 14 floats (rows of dW, dt, dfocal)."""
    v = np.asarray(values, np.float32).reshape(14)
    g = CameraGradient()
    for r in range(3):
        for c in range(3):
            g.world_to_camera_rotation_rows[r][c] = float(v[r * 3 + c])
        g.world_to_camera_translation[r] = float(v[9 + r])
    g.focal[0], g.focal[1] = float(v[12]), float(v[13])
    return g


def corrected_camera(initial: PinholeCamera, correction: PoseCorrection, focal_log_scale: float) -> PinholeCamera:
    """camera_pose.rs:59-68."""
    out = PinholeCameraC()
    _lib.check(
        _lib.load().sp_corrected_camera(
            ctypes.byref(initial.to_c()), ctypes.byref(correction.to_c()), focal_log_scale, ctypes.byref(out)
        ),
        what="corrected_camera",
    )
    return PinholeCamera.from_c(out)


def pose_gradient(
    initial: PinholeCamera, correction: PoseCorrection, focal_log_scale: float, gradient: CameraGradient
) -> PoseGradient:
    """camera_pose.rs:81-99."""
    out = PoseGradientC()
    _lib.check(
        _lib.load().sp_pose_gradient_of(
            ctypes.byref(initial.to_c()),
            ctypes.byref(correction.to_c()),
            focal_log_scale,
            ctypes.byref(gradient),
            ctypes.byref(out),
        ),
        what="pose_gradient",
    )
    return PoseGradient.from_c(out)


class PoseRefinement:
    """PoseRefinement (pose_refinement.rs:50-163)."""

    def __init__(self, initial: list[PinholeCamera], learning_rates: LearningRates, extent: float):
        self.lib = _lib.load()
        arr = (PinholeCameraC * len(initial))(*[c.to_c() for c in initial])
        handle = ctypes.c_void_p()
        rates = learning_rates.to_c()
        _lib.check(
            self.lib.sp_pose_refinement_create(arr, len(initial), ctypes.byref(rates), float(extent), ctypes.byref(handle)),
            what="PoseRefinement::new",
        )
        self.handle = handle.value
        self.view_count = len(initial)

    def camera(self, view: int) -> PinholeCamera:
        out = PinholeCameraC()
        _lib.check(self.lib.sp_pose_refinement_camera(self.handle, view, ctypes.byref(out)), what="camera")
        return PinholeCamera.from_c(out)

    def step(self, view: int, gradient: CameraGradient, rate_factor: float) -> None:
        _lib.check(
            self.lib.sp_pose_refinement_step(self.handle, view, ctypes.byref(gradient), float(rate_factor)),
            what=f"view {view}: pose step",
        )

    def correction(self, view: int) -> PoseCorrection:
        out = PoseCorrectionC()
        _lib.check(self.lib.sp_pose_refinement_correction(self.handle, view, ctypes.byref(out)), what="correction")
        return PoseCorrection(np.array(list(out.rotation)), np.array(list(out.translation)))

    def focal_scale(self) -> float:
        return float(self.lib.sp_pose_refinement_focal_scale(self.handle))

    def last_gradient(self) -> PoseGradient:
        out = PoseGradientC()
        _lib.check(self.lib.sp_pose_refinement_last_gradient(self.handle, ctypes.byref(out)), what="last_gradient")
        return PoseGradient.from_c(out)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_pose_refinement_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class DevicePoses:
    """The pose refinement on the GPU (sp_device_poses): a copy of a host PoseRefinement's
    state bound to a rasterizer. Each training step refines the pose of the view it trained
    from the camera gradient in device memory and sets the camera of the next view, with no
    host synchronisation; download() brings the state back into the host refinement."""

    def __init__(self, rasterizer, refinement: PoseRefinement):
        self.lib = _lib.load()
        self.rasterizer = rasterizer
        self.refinement = refinement
        handle = ctypes.c_void_p()
        _lib.check(self.lib.sp_device_poses_create(rasterizer.handle, refinement.handle, ctypes.byref(handle)),
                   rasterizer.ctx.handle, "DevicePoses")
        self.handle = handle.value

    def set_camera(self, view: int) -> None:
        """The rasterizer's camera := view's corrected camera (enqueued)."""
        _lib.check(self.lib.sp_device_poses_set_camera(self.handle, view), self.rasterizer.ctx.handle, "set_camera")

    def step(self, view: int, next_view: int, rate_factor: float) -> None:
        """The refinement step of `view`, then the camera of `next_view` (enqueued)."""
        _lib.check(self.lib.sp_device_poses_step(self.handle, view, next_view, float(rate_factor)),
                   self.rasterizer.ctx.handle, "pose step")

    def download(self) -> PoseRefinement:
        """Synchronises and copies the device state into the host refinement (returned)."""
        _lib.check(self.lib.sp_device_poses_download(self.handle, self.refinement.handle), self.rasterizer.ctx.handle,
                   "download")
        return self.refinement

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_device_poses_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()
