"""Gaussian parameters in the 3DGS parametrisation and their packed layout —
instantsplat-rs/src/gaussians.rs. Degree 0 packs 14 floats per Gaussian, exactly the
reference's layout; degrees 1-3 append the higher SH coefficients (coefficient k of
channel c at slot 11 + 3k + c), 59 floats at degree 3."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

SH_C0 = np.float32(0.28209479)
SLOT_POSITION = 0
SLOT_LOG_SCALE = 3
SLOT_ROTATION = 6
SLOT_OPACITY = 10
SLOT_SH = 11


def param_stride(sh_degree: int) -> int:
    return 11 + 3 * (sh_degree + 1) ** 2


@dataclass
class GaussianCloud:
    """GaussianCloud (gaussians.rs:14-25), row-major arrays, one Gaussian per row."""

    positions: np.ndarray  # [N, 3]
    log_scales: np.ndarray  # [N, 3]
    rotations: np.ndarray  # [N, 4] (w, x, y, z), not necessarily unit
    opacity_logits: np.ndarray  # [N]
    sh: np.ndarray  # [N, (d + 1)^2, 3]; sh[:, 0] is the reference's sh_dc

    def __post_init__(self) -> None:
        n = len(self.positions)
        self.positions = np.asarray(self.positions, np.float32).reshape(n, 3)
        self.log_scales = np.asarray(self.log_scales, np.float32).reshape(n, 3)
        self.rotations = np.asarray(self.rotations, np.float32).reshape(n, 4)
        self.opacity_logits = np.asarray(self.opacity_logits, np.float32).reshape(n)
        self.sh = np.asarray(self.sh, np.float32).reshape(n, -1, 3)
        k = self.sh.shape[1]
        if k not in (1, 4, 9, 16):
            raise ValueError(f"{k} SH coefficients per channel")

    def __len__(self) -> int:
        return len(self.positions)

    @property
    def sh_degree(self) -> int:
        return int(round(np.sqrt(self.sh.shape[1]))) - 1

    @property
    def sh_dc(self) -> np.ndarray:
        return self.sh[:, 0, :]

    def centroid(self) -> np.ndarray:
        if len(self) == 0:
            raise ValueError("centroid of no Gaussians")
        return self.positions.astype(np.float64).mean(axis=0)

    def to_packed(self) -> np.ndarray:
        """GaussianCloud::to_packed (gaussians.rs:54-65), extended with the SH rest."""
        n = len(self)
        packed = np.empty((n, param_stride(self.sh_degree)), np.float32)
        packed[:, 0:3] = self.positions
        packed[:, 3:6] = self.log_scales
        packed[:, 6:10] = self.rotations
        packed[:, 10] = self.opacity_logits
        packed[:, 11:] = self.sh.reshape(n, -1)
        return packed.reshape(-1)

    @staticmethod
    def from_packed(packed: np.ndarray, sh_degree: int = 0) -> "GaussianCloud":
        """GaussianCloud::from_packed (gaussians.rs:67-84)."""
        stride = param_stride(sh_degree)
        packed = np.asarray(packed, np.float32)
        if packed.size % stride:
            raise ValueError(f"packed length {packed.size}")
        p = packed.reshape(-1, stride)
        return GaussianCloud(
            positions=p[:, 0:3].copy(),
            log_scales=p[:, 3:6].copy(),
            rotations=p[:, 6:10].copy(),
            opacity_logits=p[:, 10].copy(),
            sh=p[:, 11:].reshape(len(p), -1, 3).copy(),
        )


def sigmoid(x):
    return np.float32(1.0) / (np.float32(1.0) + np.exp(-np.float32(x)))


def logit(p: float) -> float:
    """gaussians.rs:88-92."""
    if not 0.0 < p < 1.0:
        raise ValueError(f"logit of {p}")
    return float(np.log(np.float32(p) / (np.float32(1.0) - np.float32(p))))


def rgb_to_sh_dc(rgb):
    """gaussians.rs:94-97."""
    return (np.asarray(rgb, np.float32) - np.float32(0.5)) / SH_C0
