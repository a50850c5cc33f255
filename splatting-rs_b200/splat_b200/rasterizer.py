"""The differentiable rasterizer — a Python mirror of instantsplat-rs's `Rasterizer`
(rasterizer.rs:134-565) over the C ABI of libsplat_b200.

Device memory the caller owns (the packed parameters, the ground truth) is passed as CUDA
tensors; the library borrows their pointers, as `Rasterizer::new` borrows its
`&wgpu::Buffer`s, and the tensors must outlive the rasterizer. The library owns every
intermediate buffer and the parameter gradients.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import (
    CameraGradient,
    CameraUniform,
    IntersectionMeta,
    LossTermsC,
    Options,
    SP_BWD_ATOMIC,
    SP_BWD_DETERMINISTIC,
    SP_KEYS_FULL32,
    SP_KEYS_REF20,
    SP_TILES_ELLIPSE,
    SP_TILES_RECTANGLE,
)
from .camera import PinholeCamera

# rasterizer.rs:19-22.
BACKGROUND = np.array([0.50196, 0.50196, 0.50196], np.float32)
GROUND_TRUTH_STRIDE = 4


class DeviceArray:
    """A borrowed device buffer as a CUDA array (``__cuda_array_interface__``), so that
    ``torch.as_tensor(..., device="cuda")`` views it without a copy."""

    def __init__(self, pointer: int, shape: tuple[int, ...], typestr: str = "<f4"):
        self.__cuda_array_interface__ = {
            "shape": shape,
            "typestr": typestr,
            "data": (int(pointer), False),
            "version": 3,
            "strides": None,
        }


def _torch():
    import torch

    return torch


# CUDA's handle of the legacy default stream (cudaStreamLegacy). torch reports its default
# stream as handle 0, which the C ABI reads as "give the context a stream of its own".
CUDA_STREAM_LEGACY = 0x1


class Context:
    """One CUDA device and the stream the library enqueues on (Gpu, gpu.rs:13-66). By
    default the current torch stream of the device, so that the library's work orders with
    torch's: tensor copies, CUDA events and NCCL collectives on that stream see it."""

    def __init__(self, device: int = 0, stream: int | None = None):
        self.lib = _lib.load()
        handle = ctypes.c_void_p()
        if stream is None:
            torch = _torch()
            if not torch.cuda.is_available():
                raise _lib.SplatError(_lib.SP_ERR_NO_DEVICE, "no CUDA device")
            stream = torch.cuda.current_stream(device).cuda_stream or CUDA_STREAM_LEGACY
        status = self.lib.sp_context_create_on_stream(device, ctypes.c_void_p(stream), ctypes.byref(handle))
        _lib.check(status, None, "sp_context_create")
        self.handle = handle.value
        self.device = device

    @property
    def stream(self) -> int:
        """The handle of the stream the library enqueues on."""
        return int(self.lib.sp_context_stream(self.handle) or 0)

    def sync(self) -> None:
        _lib.check(self.lib.sp_context_sync(self.handle), self.handle, "sync")

    def profile(self, enable: bool) -> None:
        """Starts or stops CUDA-event timing around every kernel launch."""
        _lib.check(self.lib.sp_profile_enable(self.handle, 1 if enable else 0), self.handle, "profile")

    def read_profile(self) -> dict[str, tuple[float, int]]:
        """{kernel: (device ms, launches)} of the launches recorded since the last read."""
        k = len(_lib.KERNEL_NAMES)
        ms = (ctypes.c_double * k)()
        launches = (ctypes.c_uint64 * k)()
        _lib.check(self.lib.sp_profile_read(self.handle, ms, launches), self.handle, "read_profile")
        return {name: (ms[i], int(launches[i])) for i, name in enumerate(_lib.KERNEL_NAMES)}

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


@dataclass
class Rendered:
    """One rendered view (rasterizer.rs:77-132): premultiplied rgb and transmittance."""

    width: int
    height: int
    rgbt: np.ndarray  # [height * width * 4]

    def pixel(self, x: int, y: int) -> np.ndarray:
        i = (y * self.width + x) * 4
        return self.rgbt[i : i + 4]

    def premultiplied(self, x: int, y: int) -> np.ndarray:
        return self.pixel(x, y)[:3]

    def transmittance(self, x: int, y: int) -> float:
        return float(self.pixel(x, y)[3])

    def alpha(self, x: int, y: int) -> float:
        return 1.0 - self.transmittance(x, y)

    def over_background(self, x: int, y: int) -> np.ndarray:
        return self.premultiplied(x, y) + self.transmittance(x, y) * BACKGROUND

    @staticmethod
    def to_u8(value) -> np.ndarray:
        """(value.clamp(0, 1) * 255).round() as u8 (rasterizer.rs:107-109), halves away from zero."""
        v = np.clip(np.asarray(value, np.float32), 0.0, 1.0) * np.float32(255.0)
        return np.floor(v + np.float32(0.5)).astype(np.uint8)

    def to_rgba8(self) -> np.ndarray:
        """rasterizer.rs:118-131: straight colour with the coverage as alpha."""
        img = self.rgbt.reshape(self.height, self.width, 4)
        alpha = np.float32(1.0) - img[..., 3]
        safe = np.where(alpha > 0, alpha, np.float32(1.0))
        straight = np.where(alpha[..., None] > 0, img[..., :3] / safe[..., None], np.float32(0.0))
        return np.concatenate([self.to_u8(straight), self.to_u8(alpha)[..., None]], axis=-1)

    def to_rgb8(self) -> np.ndarray:
        img = self.rgbt.reshape(self.height, self.width, 4)
        return self.to_u8(img[..., :3] + img[..., 3:4] * BACKGROUND)


@dataclass
class LossTerms:
    """LossTerms (loss.rs:38-64)."""

    l1: float = 0.0
    alpha: float = 0.0
    dssim: float = 0.0
    total: float = 0.0

    @staticmethod
    def from_pixel_loss(pixel_loss: np.ndarray) -> "LossTerms":
        p = np.asarray(pixel_loss, np.float32).reshape(-1, 4).astype(np.float64)
        if len(p) == 0:
            raise ValueError("pixel loss length 0")
        m = p.mean(axis=0)
        return LossTerms(float(np.float32(m[0])), float(np.float32(m[1])), float(np.float32(m[2])), float(np.float32(m[3])))


def default_options(
    sh_degree: int = 0,
    backward_mode: int = SP_BWD_ATOMIC,
    key_mode: int = SP_KEYS_REF20,
    intersections_per_gaussian: int = 24,
    accumulate_gradients: bool = False,
    tile_culling: int = 0,
) -> Options:
    opt = Options()
    _lib.load().sp_options_default(ctypes.byref(opt))
    opt.sh_degree = sh_degree
    opt.backward_mode = backward_mode
    opt.key_mode = key_mode
    opt.intersections_per_gaussian = intersections_per_gaussian
    opt.accumulate_gradients = 1 if accumulate_gradients else 0
    opt.tile_culling = tile_culling
    return opt


class Rasterizer:
    """Rasterizer (rasterizer.rs:134-565) over libsplat_b200."""

    def __init__(
        self,
        ctx: Context,
        params,
        gaussian_count: int,
        width: int,
        height: int,
        ground_truth=None,
        view_count: int = 0,
        options: Options | None = None,
    ):
        self.ctx = ctx
        self.lib = ctx.lib
        self.options = options if options is not None else default_options()
        self.width, self.height = int(width), int(height)
        self.gaussian_count = int(gaussian_count)
        self.view_count = int(view_count)
        self._params = params  # kept alive: the library borrows the pointer
        self._ground_truth = ground_truth
        handle = ctypes.c_void_p()
        status = self.lib.sp_rasterizer_create(
            ctx.handle,
            ctypes.c_void_p(self._pointer(params)),
            self.gaussian_count,
            self.width,
            self.height,
            ctypes.c_void_p(self._pointer(ground_truth) if ground_truth is not None else 0),
            self.view_count,
            ctypes.byref(self.options),
            ctypes.byref(handle),
        )
        _lib.check(status, ctx.handle, "Rasterizer::new")
        self.handle = handle.value
        self.stride = int(self.lib.sp_rasterizer_param_stride(self.handle))
        self.tiles_x = (self.width + 15) // 16
        self.tiles_y = (self.height + 15) // 16

    @staticmethod
    def _pointer(tensor) -> int:
        if hasattr(tensor, "data_ptr"):
            if not tensor.is_cuda or not tensor.is_contiguous():
                raise ValueError("device buffers must be contiguous CUDA tensors")
            return tensor.data_ptr()
        return int(tensor)

    def _check(self, status: int, what: str) -> None:
        _lib.check(status, self.ctx.handle, what)

    @property
    def pixel_count(self) -> int:
        return self.width * self.height

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_rasterizer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    # rasterizer.rs:398-442 ------------------------------------------------------------

    def set_camera(self, camera: PinholeCamera | CameraUniform) -> None:
        uniform = camera.uniform() if isinstance(camera, PinholeCamera) else camera
        self._check(self.lib.sp_set_camera(self.handle, ctypes.byref(uniform)), "set_camera")

    def encode_forward(self) -> None:
        self._check(self.lib.sp_forward(self.handle), "forward")

    def encode_loss(self, view: int) -> None:
        self._check(self.lib.sp_loss(self.handle, view), "loss")

    def encode_backward(self) -> None:
        self._check(self.lib.sp_backward(self.handle), "backward")

    # rasterizer.rs:446-456 ------------------------------------------------------------

    def _write(self, fn, data, what: str) -> None:
        if hasattr(data, "data_ptr"):
            if data.numel() != self.pixel_count * 4:
                raise ValueError(f"{what}: {data.numel()} floats for {self.pixel_count} pixels")
            self._check(fn(self.handle, ctypes.c_void_p(self._pointer(data)), 1), what)
            return
        arr = np.ascontiguousarray(data, np.float32).reshape(-1)
        if arr.size != self.pixel_count * 4:
            raise ValueError(f"{what}: {arr.size} floats for {self.pixel_count} pixels")
        self._check(fn(self.handle, arr.ctypes.data_as(ctypes.c_void_p), 0), what)

    def write_loss_gradient(self, gradient) -> None:
        self._write(self.lib.sp_write_loss_gradient, gradient, "write_loss_gradient")

    def write_image(self, rgbt) -> None:
        self._write(self.lib.sp_write_image, rgbt, "write_image")

    # device views -----------------------------------------------------------------------

    def param_gradients(self):
        """The gradients as a CUDA tensor view (rasterizer.rs:467-469)."""
        torch = _torch()
        ptr = self.lib.sp_param_gradients(self.handle)
        return torch.as_tensor(DeviceArray(ptr, (self.gaussian_count * self.stride,)), device=f"cuda:{self.ctx.device}")

    def param_gradients_pointer(self) -> int:
        return int(self.lib.sp_param_gradients(self.handle))

    def camera_gradient_tensor(self):
        torch = _torch()
        ptr = self.lib.sp_camera_gradient_device(self.handle)
        return torch.as_tensor(DeviceArray(ptr, (14,)), device=f"cuda:{self.ctx.device}")

    def densify_stats_tensor(self):
        """The accumulated densify statistics as an (N, 4) CUDA tensor view."""
        torch = _torch()
        ptr = self.lib.sp_densify_stats_device(self.handle)
        return torch.as_tensor(DeviceArray(ptr, (self.gaussian_count, 4)), device=f"cuda:{self.ctx.device}")

    def zero_param_gradients(self) -> None:
        self._check(self.lib.sp_zero_param_gradients(self.handle), "zero_param_gradients")

    def clear_densify_stats(self) -> None:
        self._check(self.lib.sp_clear_densify_stats(self.handle), "clear_densify_stats")

    # read-backs (rasterizer.rs:458-549) -------------------------------------------------

    def _read(self, fn, shape, dtype, what: str) -> np.ndarray:
        out = np.empty(shape, dtype)
        self._check(fn(self.handle, out.ctypes.data_as(ctypes.c_void_p)), what)
        return out

    def read_loss_gradient(self) -> np.ndarray:
        return self._read(self.lib.sp_read_loss_gradient, self.pixel_count * 4, np.float32, "read_loss_gradient")

    def read_param_gradients(self) -> np.ndarray:
        return self._read(
            self.lib.sp_read_param_gradients, self.gaussian_count * self.stride, np.float32, "read_param_gradients"
        )

    def read_densify_stats(self) -> np.ndarray:
        """[N, 4]: mean_gradient_sum, visible_count, max_radius, 0."""
        return self._read(
            self.lib.sp_read_densify_stats, (self.gaussian_count, 4), np.float32, "read_densify_stats"
        )

    def write_densify_stats(self, stats) -> None:
        """Overwrites the accumulated densify statistics ((N, 4) float32; diagnostics)."""
        host = np.ascontiguousarray(stats, np.float32).reshape(self.gaussian_count, 4)
        self._check(self.lib.sp_write_densify_stats(self.handle, host.ctypes.data_as(ctypes.c_void_p)),
                    "write_densify_stats")

    def read_camera_gradient(self) -> CameraGradient:
        out = CameraGradient()
        self._check(self.lib.sp_read_camera_gradient(self.handle, ctypes.byref(out)), "read_camera_gradient")
        return out

    def read_image(self) -> Rendered:
        rgbt = self._read(self.lib.sp_read_image, self.pixel_count * 4, np.float32, "read_image")
        return Rendered(self.width, self.height, rgbt)

    def read_pixel_loss(self) -> np.ndarray:
        return self._read(self.lib.sp_read_pixel_loss, self.pixel_count * 4, np.float32, "read_pixel_loss")

    def read_loss(self) -> LossTerms:
        out = LossTermsC()
        self._check(self.lib.sp_read_loss(self.handle, ctypes.byref(out)), "read_loss")
        return LossTerms(out.l1, out.alpha, out.dssim, out.total)

    def read_intersections(self) -> IntersectionMeta:
        """Raises SplatError(SP_ERR_OVERFLOW) where the reference panics (rasterizer.rs:536-544)."""
        out = IntersectionMeta()
        self._check(self.lib.sp_read_intersections(self.handle, ctypes.byref(out)), "read_intersections")
        return out

    def read_intersections_unchecked(self) -> IntersectionMeta:
        out = IntersectionMeta()
        status = self.lib.sp_read_intersections(self.handle, ctypes.byref(out))
        if status not in (_lib.SP_OK, _lib.SP_ERR_OVERFLOW):
            self._check(status, "read_intersections")
        return out

    def intersections_needed(self) -> int:
        """The (Gaussian, tile) pairs the last forward pass's scan counted, before truncation at
        the capacity (sp_intersections_needed)."""
        out = ctypes.c_uint64()
        self._check(self.lib.sp_intersections_needed(self.handle, ctypes.byref(out)), "intersections_needed")
        return int(out.value)

    def reserve_intersections(self, capacity: int) -> None:
        """Grows the intersection buffers to `capacity` pairs (sp_reserve_intersections); the
        next backward needs a forward pass first."""
        self._check(self.lib.sp_reserve_intersections(self.handle, int(capacity)), "reserve_intersections")

    def debug_stall_sort_partition(self, partition: int | None) -> None:
        """Error-path test switch (sp_debug_stall_sort_partition): sort partition `partition`
        never posts its look-back record, so the next one's wait runs out (SP_ERR_TIMEOUT);
        None switches it off."""
        value = 0xFFFFFFFF if partition is None else int(partition)
        self._check(self.lib.sp_debug_stall_sort_partition(self.handle, value), "debug_stall_sort_partition")

    def encode_backward_blend(self) -> None:
        """The blend half of encode_backward (sp_backward_blend)."""
        self._check(self.lib.sp_backward_blend(self.handle), "backward_blend")

    def encode_backward_project(self, first: int, count: int) -> None:
        """The projection backward of Gaussians [first, first + count) (sp_backward_project)."""
        self._check(self.lib.sp_backward_project(self.handle, int(first), int(count)), "backward_project")

    def encode_backward_adam(self, adam, rate_factor: float) -> None:
        """encode_backward then adam.encode_step(rate_factor) as one fused pass
        (sp_backward_adam); the parameter gradients are consumed, not written."""
        self._check(self.lib.sp_backward_adam(self.handle, adam.handle, float(rate_factor)), "backward_adam")

    def train_step(self, adam, camera: PinholeCamera | CameraUniform, view: int, rate_factor: float,
                   read_back: bool = True):
        """One whole training step (Trainer::step_async, training.rs:197-209) in one call;
        with `read_back`, returns (camera gradient, loss terms) read back together."""
        uniform = camera.uniform() if isinstance(camera, PinholeCamera) else camera
        if not read_back:
            self._check(self.lib.sp_train_step(self.handle, adam.handle, ctypes.byref(uniform), view,
                                               float(rate_factor), None, None), "train_step")
            return None
        gradient, loss = CameraGradient(), LossTermsC()
        self._check(self.lib.sp_train_step(self.handle, adam.handle, ctypes.byref(uniform), view, float(rate_factor),
                                           ctypes.byref(gradient), ctypes.byref(loss)), "train_step")
        return gradient, LossTerms(loss.l1, loss.alpha, loss.dssim, loss.total)

    def train_step_host_poses(self, adam, poses, view: int, rate_factor: float) -> LossTerms:
        """Trainer::step_async with pose refinement in one call (sp_train_step_host_poses):
        the refinement's camera of `view`, the step, the camera gradient read back, the host
        pose step. Returns the step's loss terms."""
        loss = LossTermsC()
        self._check(self.lib.sp_train_step_host_poses(self.handle, adam.handle, poses.handle, view, float(rate_factor),
                                                       ctypes.byref(loss)), "train_step_host_poses")
        return LossTerms(loss.l1, loss.alpha, loss.dssim, loss.total)

    def train_step_device_poses(self, adam, poses, view: int, next_view: int, rate_factor: float,
                                loss_sums=None) -> None:
        """One training step with the poses refined on the device (sp_train_step_device_poses),
        enqueued without synchronising; `loss_sums`, a pinned float64 tensor of 4, receives the
        loss sums asynchronously."""
        ptr = ctypes.c_void_p(loss_sums.data_ptr() if loss_sums is not None else 0)
        self._check(self.lib.sp_train_step_device_poses(self.handle, adam.handle, poses.handle, view, next_view,
                                                         float(rate_factor), ptr), "train_step_device_poses")

    def render(self, camera: PinholeCamera | CameraUniform) -> Rendered:
        """Rasterizer::render (rasterizer.rs:552-564)."""
        uniform = camera.uniform() if isinstance(camera, PinholeCamera) else camera
        out = np.empty(self.pixel_count * 4, np.float32)
        self._check(
            self.lib.sp_render(self.handle, ctypes.byref(uniform), out.ctypes.data_as(ctypes.c_void_p)), "render"
        )
        return Rendered(self.width, self.height, out)

    # diagnostics -------------------------------------------------------------------------

    def read_projected(self) -> np.ndarray:
        """The 80-B Projected records (rasterizer.rs:46-61) as a structured array."""
        dtype = np.dtype(
            [
                ("mean", "<f4", 2),
                ("_pad0", "<f4", 2),
                ("conic", "<f4", 3),
                ("depth", "<f4"),
                ("color", "<f4", 3),
                ("opacity", "<f4"),
                ("radius", "<u4"),
                ("_pad1", "<u4"),
                ("tile_min", "<u4", 2),
                ("tile_max", "<u4", 2),
                ("_pad2", "<u4", 2),
            ]
        )
        assert dtype.itemsize == 80
        return self._read(self.lib.sp_read_projected, self.gaussian_count, dtype, "read_projected")

    def read_sorted_intersections(self) -> tuple[np.ndarray, np.ndarray]:
        meta = self.read_intersections_unchecked()
        keys = np.empty(max(meta.count, 1), np.uint64)
        gaussians = np.empty(max(meta.count, 1), np.uint32)
        self._check(
            self.lib.sp_read_sorted_intersections(
                self.handle, keys.ctypes.data_as(ctypes.c_void_p), gaussians.ctypes.data_as(ctypes.c_void_p)
            ),
            "read_sorted_intersections",
        )
        return keys[: meta.count], gaussians[: meta.count]

    def read_tile_ranges(self) -> np.ndarray:
        return self._read(self.lib.sp_read_tile_ranges, self.tiles_x * self.tiles_y * 2, np.uint32, "read_tile_ranges")

    def read_contributions(self) -> np.ndarray:
        return self._read(self.lib.sp_read_contributions, self.pixel_count, np.uint32, "read_contributions")

    def read_tile_offsets(self) -> np.ndarray:
        return self._read(self.lib.sp_read_tile_offsets, self.gaussian_count, np.uint32, "read_tile_offsets")

    def count_blend_work(self) -> tuple[int, int, int]:
        """(forward pairs visited, backward pairs replayed, pairs blended) of the last forward
        pass."""
        fwd, bwd, taken = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        self._check(self.lib.sp_count_blend_work(self.handle, ctypes.byref(fwd), ctypes.byref(bwd),
                                                 ctypes.byref(taken)), "count")
        return int(fwd.value), int(bwd.value), int(taken.value)

    def read_gaussian_blend_gradients(self) -> np.ndarray:
        return self._read(
            self.lib.sp_read_gaussian_blend_gradients, (self.gaussian_count, 10), np.float32, "blend gradients"
        )


__all__ = [
    "BACKGROUND",
    "Context",
    "DeviceArray",
    "LossTerms",
    "Rasterizer",
    "Rendered",
    "default_options",
    "SP_BWD_ATOMIC",
    "SP_BWD_DETERMINISTIC",
    "SP_KEYS_FULL32",
    "SP_KEYS_REF20",
]
