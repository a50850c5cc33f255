"""Adaptive density control — a mirror of instantsplat-rs/src/densify.rs on the device.

The reference reads the parameters, Adam's moments and the densify statistics back, rebuilds
them on the CPU (`densify`, densify.rs:147-257) and uploads new buffers
(`Trainer::densify_async`, training.rs:238-266). Here the same decisions run as kernels
where the buffers are (sp_densify_plan / sp_densify_apply): only the report comes back.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib

# What an opacity reset lowers the opacities to, as 3DGS (densify.rs:47-48).
RESET_OPACITY = 0.01


@dataclass(frozen=True)
class DensifySettings:
    """DensifySettings (densify.rs:19-45)."""

    interval: int
    start: int
    stop_fraction: float
    gradient_threshold: float
    split_scale_fraction: float
    prune_opacity: float
    max_screen_radius: float
    max_growth: float
    opacity_reset_interval: int | None = None

    def to_c(self) -> _lib.DensifySettingsC:
        c = _lib.DensifySettingsC()
        c.interval, c.start = int(self.interval), int(self.start)
        c.stop_fraction = self.stop_fraction
        c.gradient_threshold = self.gradient_threshold
        c.split_scale_fraction = self.split_scale_fraction
        c.prune_opacity = self.prune_opacity
        c.max_screen_radius = self.max_screen_radius
        c.max_growth = self.max_growth
        c.opacity_reset_interval = int(self.opacity_reset_interval or 0)
        if self.opacity_reset_interval is not None and self.opacity_reset_interval <= 0:
            raise ValueError(f"opacity reset interval {self.opacity_reset_interval}")
        return c

    def densifies_after(self, done: int, steps: int) -> bool:
        """Whether the Gaussians are densified after `done` (1-based) of `steps` steps
        (densify.rs:77-83)."""
        value = _lib.load().sp_densify_after(ctypes.byref(self.to_c()), int(done), int(steps))
        if value < 0:
            raise ValueError(f"densify interval {self.interval}, step {done} of {steps}")
        return bool(value)

    def resets_opacity_after(self, done: int) -> bool:
        """Whether the densification after `done` steps also resets the opacities
        (densify.rs:84-94)."""
        value = _lib.load().sp_resets_opacity_after(ctypes.byref(self.to_c()), int(done))
        if value < 0:
            raise ValueError(
                f"opacity reset interval {self.opacity_reset_interval}: a multiple of the densify interval "
                f"{self.interval}"
            )
        return bool(value)

    def max_count(self, initial_count: int) -> int:
        """training.rs:245: `(initial_count as f32 * max_growth) as usize`."""
        value = np.float32(np.float32(initial_count) * np.float32(self.max_growth))
        return int(value) if value > 0 else 0


# DENSIFY_SHORT_RUN (densify.rs:59-69).
DENSIFY_SHORT_RUN = DensifySettings(
    interval=50,
    start=50,
    stop_fraction=0.5,
    gradient_threshold=2e-4,
    split_scale_fraction=0.01,
    prune_opacity=0.005,
    max_screen_radius=100.0,
    max_growth=2.0,
    opacity_reset_interval=None,
)


@dataclass(frozen=True)
class DensifyReport:
    """DensifyReport (densify.rs:97-128)."""

    before: int
    cloned: int
    split: int
    pruned_transparent: int
    pruned_oversized: int
    opacity_reset: bool
    over_budget: int
    after: int

    @staticmethod
    def from_c(c: _lib.DensifyReportC) -> "DensifyReport":
        return DensifyReport(int(c.before), int(c.cloned), int(c.split), int(c.pruned_transparent),
                             int(c.pruned_oversized), bool(c.opacity_reset), int(c.over_budget), int(c.after))

    def __str__(self) -> str:
        text = (f"{self.before} -> {self.after} Gaussians: cloned {self.cloned}, split {self.split}, pruned "
                f"{self.pruned_transparent} transparent and {self.pruned_oversized} oversized")
        if self.over_budget > 0:
            text += f", {self.over_budget} more over the growth cap"
        if self.opacity_reset:
            text += f", opacities reset to {RESET_OPACITY}"
        return text


class DensifyError(ValueError):
    """Every Gaussian would be pruned (densify.rs:255 panics); carries the report."""

    def __init__(self, report: DensifyReport):
        super().__init__(f"densification pruned every Gaussian: {report}")
        self.report = report


@dataclass
class Densified:
    """Densified (densify.rs:130-136): device tensors of after * stride floats each."""

    params: object
    first_moment: object
    second_moment: object
    report: DensifyReport


def densify(rasterizer, adam, extent: float, max_count: int, settings: DensifySettings, reset_opacity: bool,
            seed: int) -> Densified:
    """densify (densify.rs:147-257) of `rasterizer`'s Gaussians (their parameters and the
    statistics its backward passes accumulated) with `adam`'s moments, on the device."""
    import torch

    lib = rasterizer.lib
    if not extent > 0:
        raise ValueError(f"camera extent {extent}")
    plan = ctypes.c_void_p()
    report_c = _lib.DensifyReportC()
    status = lib.sp_densify_plan(rasterizer.handle, adam.handle, float(extent), int(max_count),
                                 ctypes.byref(settings.to_c()), int(bool(reset_opacity)), int(seed),
                                 ctypes.byref(plan), ctypes.byref(report_c))
    report = DensifyReport.from_c(report_c)
    if status != 0 and report.after == 0 and report.before > 0:
        raise DensifyError(report)
    _lib.check(status, rasterizer.ctx.handle, "densify plan")
    try:
        device = f"cuda:{rasterizer.ctx.device}"
        floats = report.after * rasterizer.stride
        params = torch.empty(floats, dtype=torch.float32, device=device)
        first = torch.empty_like(params)
        second = torch.empty_like(params)
        _lib.check(
            lib.sp_densify_apply(plan.value, params.data_ptr(), first.data_ptr(), second.data_ptr(), report.after),
            rasterizer.ctx.handle,
            "densify apply",
        )
    finally:
        lib.sp_densify_destroy(plan.value)
    return Densified(params, first, second, report)
