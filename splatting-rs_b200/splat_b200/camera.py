"""Pinhole cameras in the OpenCV convention (x right, y down, z forward), pixel centres at
integer coordinates — instantsplat-rs/src/camera.rs."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field, replace

import numpy as np

from . import _lib
from ._lib import CameraUniform, PinholeCameraC

TILE = 16


@dataclass
class PinholeCamera:
    """PinholeCamera (camera.rs:8-17): camera-to-world rotation and centre, in f64."""

    rotation: np.ndarray = field(default_factory=lambda: np.eye(3))
    translation: np.ndarray = field(default_factory=lambda: np.zeros(3))
    focal: tuple[float, float] = (1.0, 1.0)
    principal_point: tuple[float, float] = (0.0, 0.0)
    width: int = 1
    height: int = 1

    def __post_init__(self) -> None:
        self.rotation = np.asarray(self.rotation, dtype=np.float64).reshape(3, 3)
        self.translation = np.asarray(self.translation, dtype=np.float64).reshape(3)
        self.focal = (float(self.focal[0]), float(self.focal[1]))
        self.principal_point = (float(self.principal_point[0]), float(self.principal_point[1]))

    def world_to_camera(self) -> tuple[np.ndarray, np.ndarray]:
        """camera.rs:46-49: (R^T, -R^T C)."""
        rotation = self.rotation.T
        return rotation, -(rotation @ self.translation)

    def uniform(self) -> CameraUniform:
        """PinholeCamera::uniform (camera.rs:51-70), computed by the library."""
        out = CameraUniform()
        rot = np.ascontiguousarray(self.rotation, dtype=np.float64).reshape(9)
        t = np.ascontiguousarray(self.translation, dtype=np.float64)
        f = np.array(self.focal, dtype=np.float64)
        pp = np.array(self.principal_point, dtype=np.float64)
        as_ptr = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))  # noqa: E731
        _lib.check(
            _lib.load().sp_camera_uniform_from_pinhole(
                as_ptr(rot), as_ptr(t), as_ptr(f), as_ptr(pp), self.width, self.height, ctypes.byref(out)
            ),
            what="camera uniform",
        )
        return out

    def position(self) -> np.ndarray:
        return self.translation

    def with_image_size(self, width: int, height: int) -> "PinholeCamera":
        """camera.rs:72-87: same pose and focal, the old centre at the new one's."""
        shift = lambda new, old: (new - old) / 2.0  # noqa: E731
        return replace(
            self,
            principal_point=(
                self.principal_point[0] + shift(width, self.width),
                self.principal_point[1] + shift(height, self.height),
            ),
            width=width,
            height=height,
        )

    def to_c(self) -> PinholeCameraC:
        c = PinholeCameraC()
        for i, v in enumerate(self.rotation.reshape(9)):
            c.rotation[i] = float(v)
        for i in range(3):
            c.translation[i] = float(self.translation[i])
        c.focal[0], c.focal[1] = self.focal
        c.principal_point[0], c.principal_point[1] = self.principal_point
        c.width, c.height = self.width, self.height
        return c

    @staticmethod
    def from_c(c: PinholeCameraC) -> "PinholeCamera":
        return PinholeCamera(
            rotation=np.array(list(c.rotation)).reshape(3, 3),
            translation=np.array(list(c.translation)),
            focal=(c.focal[0], c.focal[1]),
            principal_point=(c.principal_point[0], c.principal_point[1]),
            width=c.width,
            height=c.height,
        )


def cameras_extent(cameras: list[PinholeCamera]) -> float:
    """camera.rs:96-101: 1.1 x the radius of the smallest sphere about the mean centre."""
    if not cameras:
        raise ValueError("no cameras")
    centres = np.stack([c.position() for c in cameras])
    centre = centres.mean(axis=0)
    return float(np.max(np.linalg.norm(centres - centre, axis=1)) * 1.1)


def look_at(eye, target, up, focal: float, width: int, height: int) -> PinholeCamera:
    """A camera at `eye` looking at `target`, image y pointing against `up`; principal
    point at (width / 2, height / 2) as the reference's tests place it
    (rasterizer_tests.rs:16-25)."""
    eye = np.asarray(eye, dtype=np.float64)
    forward = np.asarray(target, dtype=np.float64) - eye
    forward /= np.linalg.norm(forward)
    right = np.cross(forward, np.asarray(up, dtype=np.float64))
    if np.linalg.norm(right) < 1e-9:
        right = np.cross(forward, np.array([1.0, 0.0, 0.0]))
    right /= np.linalg.norm(right)
    down = np.cross(forward, right)
    rotation = np.stack([right, down, forward], axis=1)
    return PinholeCamera(
        rotation=rotation,
        translation=eye,
        focal=(focal, focal),
        principal_point=(width // 2, height // 2),
        width=width,
        height=height,
    )


def focal_for_fov(width: int, fov_degrees: float) -> float:
    """Focal length in pixels of a horizontal field of view."""
    return (width / 2.0) / np.tan(np.radians(fov_degrees) / 2.0)
