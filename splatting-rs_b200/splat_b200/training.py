"""The training step loop — a mirror of `Trainer` (instantsplat-rs/src/training.rs:86-443),
the caller that switches its `Rasterizer` / `Adam` for libsplat_b200: one view per step,
views cycled in order, the position rate decayed over the run, the camera gradient read
back for the pose refinement when poses are refined, and with densify settings the
densification due before a step (training.rs:221-266), run on the device (densify.py)."""

from __future__ import annotations

import numpy as np

from .camera import PinholeCamera, cameras_extent
from .densify import DensifyReport, DensifySettings, densify
from .gaussians import GaussianCloud
from .optimizer import Adam, LearningRates, LEARNING_RATES_3DGS, position_rate_factor
from .pose import PoseRefinement
from .rasterizer import Context, LossTerms, Rasterizer, Rendered, default_options


def ground_truth_rgba(rgb: np.ndarray, foreground: np.ndarray) -> np.ndarray:
    """loss::ground_truth_rgba (loss.rs:95-104): rgb times the mask, then the mask."""
    mask = np.asarray(foreground, np.float32).reshape(-1, 1)
    rgb = np.asarray(rgb, np.float32).reshape(-1, 3)
    return np.concatenate([rgb * mask, mask], axis=1).reshape(-1)


class Trainer:
    """Trainer::new / step / train_step / loss / render over one device."""

    def __init__(
        self,
        cloud: GaussianCloud,
        cameras: list[PinholeCamera],
        ground_truth: np.ndarray,
        learning_rates: LearningRates = LEARNING_RATES_3DGS,
        refine_poses: bool = False,
        ctx: Context | None = None,
        backward_mode: int | None = None,
        densify: DensifySettings | None = None,
        capacity: str = "fixed",
    ):
        """`capacity`: "fixed", the reference's 24 (Gaussian, tile) pairs per Gaussian
        (rasterizer.rs:27), or "scan": the intersection lists sized from the scan of every
        view's forward pass, with a quarter of headroom, at construction and after each
        densification (sp_intersections_needed / sp_reserve_intersections). Either way a step
        whose lists overflow raises SplatError(SP_ERR_OVERFLOW) naming the pairs it needed."""
        import torch

        if capacity not in ("fixed", "scan"):
            raise ValueError(f"capacity policy {capacity!r}: 'fixed' or 'scan'")

        if not cameras:
            raise ValueError("no views")
        width, height = cameras[0].width, cameras[0].height
        for c in cameras:
            if (c.width, c.height) != (width, height):
                raise ValueError("every view must have the same size")
        self.ctx = ctx or Context(0)
        device = f"cuda:{self.ctx.device}"
        self.cameras = list(cameras)
        self.sh_degree = cloud.sh_degree
        self.params = torch.from_numpy(cloud.to_packed()).to(device)
        gt = np.ascontiguousarray(ground_truth, np.float32).reshape(-1)
        if gt.size != len(cameras) * width * height * 4:
            raise ValueError("ground truth buffer size")
        self.ground_truth = torch.from_numpy(gt).to(device)
        options = default_options(sh_degree=self.sh_degree)
        if backward_mode is not None:
            options.backward_mode = backward_mode
        if capacity == "scan":
            options.intersections_per_gaussian = 1  # grown from the scan below
        self.options = options
        self.capacity_policy = capacity
        self.width, self.height = width, height
        self.rasterizer = Rasterizer(
            self.ctx, self.params, len(cloud), width, height, self.ground_truth, len(cameras), options
        )
        self.gaussian_count = self.initial_gaussian_count = len(cloud)
        self.densify = densify
        self.densifications: list[DensifyReport] = []
        self.extent = cameras_extent(self.cameras)
        if not self.extent > 0:
            raise ValueError(f"camera extent {self.extent}: the views' cameras are all at the same position")
        self.poses = PoseRefinement(self.cameras, learning_rates, self.extent) if refine_poses else None
        self.adam = Adam(
            self.ctx,
            self.params,
            self.rasterizer,
            len(cloud),
            learning_rates,
            np.float32(self.extent),
            sh_degree=self.sh_degree,
        )
        if capacity == "scan":
            self._size_intersections()

    def _size_intersections(self) -> None:
        """The "scan" capacity policy: every view's forward pass (its lists may overflow the
        current capacity; the scan still counts every pair), then the largest count plus a
        quarter reserved."""
        needed = 0
        for view in range(self.view_count):
            self.rasterizer.set_camera(self.camera(view))
            self.rasterizer.encode_forward()
            needed = max(needed, self.rasterizer.intersections_needed())
        self.rasterizer.reserve_intersections(needed + needed // 4 + 1024)

    @property
    def view_count(self) -> int:
        return len(self.cameras)

    def camera(self, view: int) -> PinholeCamera:
        return self.poses.camera(view) if self.poses else self.cameras[view]

    def step(self, view: int, rate_factor: float) -> None:
        """Trainer::step_async (training.rs:197-209), one library call (sp_train_step);
        with pose refinement its camera gradient comes back in the same call."""
        result = self.rasterizer.train_step(self.adam, self.camera(view), view, rate_factor,
                                            read_back=self.poses is not None)
        if self.poses is not None:
            self.poses.step(view, result[0], rate_factor)

    def train_step(self, step: int, steps: int) -> DensifyReport | None:
        """Trainer::train_step_async (training.rs:221-229): the densification due after the
        previous step if any, then the step. The densification's report when there was one
        (`params` is then a new buffer)."""
        settings = self.densify
        report = None
        if settings is not None and step > 0 and settings.densifies_after(step, steps):
            report = self.densify_now(settings)
        self.step(step % self.view_count, position_rate_factor(step, steps))
        return report

    def densify_now(self, settings: DensifySettings) -> DensifyReport:
        """Trainer::densify_async (training.rs:238-266) on the device: densifies, then
        rebuilds the rasterizer and Adam at the new count (the statistics start over)."""
        max_count = settings.max_count(self.initial_gaussian_count)
        seed = len(self.densifications)
        reset_opacity = settings.resets_opacity_after(self.adam.steps_taken())
        out = densify(self.rasterizer, self.adam, self.extent, max_count, settings, reset_opacity, seed)
        count = out.report.after
        rasterizer = Rasterizer(self.ctx, out.params, count, self.width, self.height, self.ground_truth,
                                self.view_count, self.options)
        adam = self.adam.resumed_device(out.params, rasterizer, count, out.first_moment, out.second_moment)
        self.rasterizer.close()
        self.adam.close()
        self.params, self.rasterizer, self.adam = out.params, rasterizer, adam
        self.gaussian_count = count
        self.densifications.append(out.report)
        if self.capacity_policy == "scan":
            self._size_intersections()
        return out.report

    def loss(self, view: int) -> LossTerms:
        """Trainer::loss_async (training.rs:366-374)."""
        self.rasterizer.set_camera(self.camera(view))
        self.rasterizer.encode_forward()
        self.rasterizer.encode_loss(view)
        return self.rasterizer.read_loss()

    def render(self, view: int) -> Rendered:
        return self.rasterizer.render(self.camera(view))

    def cloud(self) -> GaussianCloud:
        return GaussianCloud.from_packed(self.params.cpu().numpy(), self.sh_degree)
