"""Adam over the packed Gaussian parameters with the scale clamp fused in — a mirror of
instantsplat-rs/src/optimizer.rs over libsplat_b200."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import numpy as np

from . import _lib
from ._lib import LearningRatesC
from .rasterizer import Context, DeviceArray, Rasterizer

ADAM_BETA1 = np.float32(0.9)
ADAM_BETA2 = np.float32(0.999)
ADAM_EPSILON = np.float32(1e-15)
POSITION_RATE_FINAL_OVER_INITIAL = np.float32(0.01)


@dataclass(frozen=True)
class LearningRates:
    """LearningRates (optimizer.rs:17-26); `sh_rest` is the rate of the SH coefficients of
    degree 1-3 (3DGS uses the dc rate / 20)."""

    position: float = 1.6e-4
    log_scale: float = 5e-3
    rotation: float = 1e-3
    opacity: float = 5e-2
    sh_dc: float = 2.5e-3
    camera_rotation: float = 1e-2
    camera_translation: float = 1e-2
    camera_focal: float = 0.0
    sh_rest: float = 2.5e-3 / 20.0

    def to_c(self) -> LearningRatesC:
        return LearningRatesC(
            self.position,
            self.log_scale,
            self.rotation,
            self.opacity,
            self.sh_dc,
            self.camera_rotation,
            self.camera_translation,
            self.camera_focal,
            self.sh_rest,
        )

    def by_slot(self, position_scale: float, stride: int = 14) -> np.ndarray:
        """LearningRates::by_slot (optimizer.rs:82-100), f32 arithmetic."""
        out = np.empty(stride, np.float32)
        for slot in range(stride):
            if slot < 3:
                out[slot] = np.float32(self.position) * np.float32(position_scale)
            elif slot < 6:
                out[slot] = self.log_scale
            elif slot < 10:
                out[slot] = self.rotation
            elif slot == 10:
                out[slot] = self.opacity
            elif slot < 14:
                out[slot] = self.sh_dc
            else:
                out[slot] = self.sh_rest
        return out


# optimizer.rs:32-51.
LEARNING_RATES_3DGS = LearningRates()
LEARNING_RATES_SHORT_RUN = replace(LEARNING_RATES_3DGS, camera_rotation=1e-3, camera_translation=1e-3)


def position_rate_factor(step: int, steps: int) -> float:
    """optimizer.rs:59-62 (computed by the library). Raises where the reference asserts."""
    value = _lib.load().sp_position_rate_factor(step, steps)
    if value < 0:
        raise ValueError(f"step {step} of {steps}")
    return float(value)


class Adam:
    """Adam (optimizer.rs:118-276): moments on the device, step counter on the host."""

    def __init__(
        self,
        ctx: Context,
        params,
        gradients,
        gaussian_count: int,
        learning_rates: LearningRates = LEARNING_RATES_3DGS,
        position_scale: float = 1.0,
        sh_degree: int = 0,
        _handle: int | None = None,
    ):
        self.ctx = ctx
        self.lib = ctx.lib
        self.gaussian_count = int(gaussian_count)
        self.sh_degree = sh_degree
        self.learning_rates = learning_rates
        self.position_scale = position_scale
        self._params = params
        self._gradients = gradients
        if _handle is not None:
            self.handle = _handle
            return
        handle = ctypes.c_void_p()
        rates = learning_rates.to_c()
        status = self.lib.sp_adam_create(
            ctx.handle,
            ctypes.c_void_p(Rasterizer._pointer(params)),
            ctypes.c_void_p(self._gradient_pointer(gradients)),
            self.gaussian_count,
            sh_degree,
            ctypes.byref(rates),
            float(position_scale),
            ctypes.byref(handle),
        )
        _lib.check(status, ctx.handle, "Adam::new")
        self.handle = handle.value

    @staticmethod
    def _gradient_pointer(gradients) -> int:
        if isinstance(gradients, Rasterizer):
            return gradients.param_gradients_pointer()
        return Rasterizer._pointer(gradients)

    def resumed(self, params, gradients, gaussian_count: int, first_moment, second_moment) -> "Adam":
        """Adam::resumed (optimizer.rs:164-188)."""
        m = np.ascontiguousarray(first_moment, np.float32)
        v = np.ascontiguousarray(second_moment, np.float32)
        handle = ctypes.c_void_p()
        status = self.lib.sp_adam_resume(
            self.handle,
            ctypes.c_void_p(Rasterizer._pointer(params)),
            ctypes.c_void_p(self._gradient_pointer(gradients)),
            int(gaussian_count),
            m.ctypes.data_as(ctypes.c_void_p),
            v.ctypes.data_as(ctypes.c_void_p),
            ctypes.byref(handle),
        )
        _lib.check(status, self.ctx.handle, "Adam::resumed")
        return Adam(
            self.ctx,
            params,
            gradients,
            gaussian_count,
            self.learning_rates,
            self.position_scale,
            self.sh_degree,
            _handle=handle.value,
        )

    def resumed_device(self, params, gradients, gaussian_count: int, first_moment, second_moment) -> "Adam":
        """Adam::resumed (optimizer.rs:164-188) from moments in device memory (tensors of
        gaussian_count * stride floats, e.g. a densification's), copied."""
        handle = ctypes.c_void_p()
        status = self.lib.sp_adam_resume_device(
            self.handle,
            ctypes.c_void_p(Rasterizer._pointer(params)),
            ctypes.c_void_p(self._gradient_pointer(gradients)),
            int(gaussian_count),
            ctypes.c_void_p(Rasterizer._pointer(first_moment)),
            ctypes.c_void_p(Rasterizer._pointer(second_moment)),
            ctypes.byref(handle),
        )
        _lib.check(status, self.ctx.handle, "Adam::resumed")
        return Adam(
            self.ctx,
            params,
            gradients,
            gaussian_count,
            self.learning_rates,
            self.position_scale,
            self.sh_degree,
            _handle=handle.value,
        )

    def encode_step(self, position_rate_factor: float = 1.0) -> None:
        """Adam::encode_step (optimizer.rs:248-264), the clamp fused."""
        _lib.check(self.lib.sp_adam_step(self.handle, float(position_rate_factor)), self.ctx.handle, "Adam step")

    def advance(self, position_rate_factor: float = 1.0) -> None:
        _lib.check(self.lib.sp_adam_advance(self.handle, float(position_rate_factor)), self.ctx.handle, "advance")

    def step_range(self, first: int, count: int) -> None:
        _lib.check(self.lib.sp_adam_step_range(self.handle, int(first), int(count)), self.ctx.handle, "step_range")

    def steps_taken(self) -> int:
        return int(self.lib.sp_adam_steps_taken(self.handle))

    def read_moments(self) -> tuple[np.ndarray, np.ndarray]:
        stride = 11 + 3 * (self.sh_degree + 1) ** 2
        m = np.empty(self.gaussian_count * stride, np.float32)
        v = np.empty_like(m)
        _lib.check(
            self.lib.sp_adam_read_moments(self.handle, m.ctypes.data_as(ctypes.c_void_p), v.ctypes.data_as(ctypes.c_void_p)),
            self.ctx.handle,
            "read_moments",
        )
        return m, v

    def moment_tensors(self):
        """The first and second moments as CUDA tensor views (N * stride floats each)."""
        import torch

        stride = 11 + 3 * (self.sh_degree + 1) ** 2
        shape = (self.gaussian_count * stride,)
        device = f"cuda:{self.ctx.device}"
        return (torch.as_tensor(DeviceArray(self.lib.sp_adam_first_moment_device(self.handle), shape), device=device),
                torch.as_tensor(DeviceArray(self.lib.sp_adam_second_moment_device(self.handle), shape), device=device))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_adam_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()
