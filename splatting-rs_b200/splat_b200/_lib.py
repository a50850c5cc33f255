"""ctypes binding of libsplat_b200.so (include/splat.h).

The library is the product: every call below runs the hand-written sm_100a kernels. There
is no fallback — importing this module without the built library, or calling into it
without a CUDA device, raises.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_float, c_int, c_uint32, c_uint64, c_void_p, c_char_p
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libsplat_b200.so"

# Status codes (sp_status).
SP_OK = 0
SP_ERR_INVALID = 1
SP_ERR_TOO_MANY_TILES = 2
SP_ERR_OVERFLOW = 3
SP_ERR_TIMEOUT = 4
SP_ERR_CUDA = 5
SP_ERR_NCCL = 6
SP_ERR_NONFINITE = 7
SP_ERR_NO_DEVICE = 8
SP_ERR_OUT_OF_MEMORY = 9

SP_KEYS_REF20 = 0
SP_KEYS_FULL32 = 1
SP_BWD_DETERMINISTIC = 0
SP_BWD_ATOMIC = 1
SP_TILES_RECTANGLE = 0
SP_TILES_ELLIPSE = 1

# Kernels of the per-kernel profiler (SP_K_*), in enum order.
KERNEL_NAMES = (
    "project",
    "scan",
    "emit",
    "sort",
    "ranges",
    "blend_forward",
    "ssim",
    "loss",
    "blend_backward",
    "project_backward",
    "adam",
    "tile_order",
    "backward_adam",
    "densify",
    "peer_adam",
)


class CameraUniform(ctypes.Structure):
    """CameraUniform (camera.rs:23-31), 80 bytes."""

    _fields_ = [
        ("world_to_camera_rows", (c_float * 4) * 3),
        ("focal", c_float * 2),
        ("principal_point", c_float * 2),
        ("width", c_uint32),
        ("height", c_uint32),
        ("tiles_x", c_uint32),
        ("tiles_y", c_uint32),
    ]


class CameraGradient(ctypes.Structure):
    """CameraGradient (camera.rs:39-43), 56 bytes."""

    _fields_ = [
        ("world_to_camera_rotation_rows", (c_float * 3) * 3),
        ("world_to_camera_translation", c_float * 3),
        ("focal", c_float * 2),
    ]


class IntersectionMeta(ctypes.Structure):
    """IntersectionMeta (rasterizer.rs:29-37), 20 bytes."""

    _fields_ = [
        ("count", c_uint32),
        ("sort_blocks", c_uint32),
        ("histogram_length", c_uint32),
        ("overflow", c_uint32),
        ("capacity", c_uint32),
    ]


class DensifyStats(ctypes.Structure):
    """DensifyStats (rasterizer.rs:63-75), 16 bytes."""

    _fields_ = [("mean_gradient_sum", c_float), ("visible_count", c_float), ("max_radius", c_float), ("_pad", c_float)]


class Projected(ctypes.Structure):
    """Projected (rasterizer.rs:46-61), 80 bytes."""

    _fields_ = [
        ("mean", c_float * 2),
        ("_pad0", c_float * 2),
        ("conic", c_float * 3),
        ("depth", c_float),
        ("color", c_float * 3),
        ("opacity", c_float),
        ("radius", c_uint32),
        ("_pad1", c_uint32),
        ("tile_min", c_uint32 * 2),
        ("tile_max", c_uint32 * 2),
        ("_pad2", c_uint32 * 2),
    ]


class LossWeights(ctypes.Structure):
    _fields_ = [("l1", c_float), ("dssim", c_float), ("alpha", c_float)]


class LossTermsC(ctypes.Structure):
    _fields_ = [("l1", c_float), ("alpha", c_float), ("dssim", c_float), ("total", c_float)]


class LearningRatesC(ctypes.Structure):
    _fields_ = [
        ("position", c_float),
        ("log_scale", c_float),
        ("rotation", c_float),
        ("opacity", c_float),
        ("sh_dc", c_float),
        ("camera_rotation", c_float),
        ("camera_translation", c_float),
        ("camera_focal", c_float),
        ("sh_rest", c_float),
    ]


class Options(ctypes.Structure):
    _fields_ = [
        ("key_mode", c_uint32),
        ("backward_mode", c_uint32),
        ("sh_degree", c_uint32),
        ("intersections_per_gaussian", c_uint32),
        ("accumulate_gradients", c_uint32),
        ("loss_weights", LossWeights),
        ("tile_culling", c_uint32),
    ]


class DensifySettingsC(ctypes.Structure):
    """sp_densify_settings (DensifySettings, densify.rs:19-45), 40 bytes."""

    _fields_ = [
        ("interval", c_uint32),
        ("start", c_uint32),
        ("stop_fraction", c_float),
        ("gradient_threshold", c_float),
        ("split_scale_fraction", c_float),
        ("prune_opacity", c_float),
        ("max_screen_radius", c_float),
        ("max_growth", c_float),
        ("opacity_reset_interval", c_uint32),
        ("_pad", c_uint32),
    ]


class DensifyReportC(ctypes.Structure):
    """sp_densify_report (DensifyReport, densify.rs:97-111), 64 bytes."""

    _fields_ = [
        ("before", c_uint64),
        ("cloned", c_uint64),
        ("split", c_uint64),
        ("pruned_transparent", c_uint64),
        ("pruned_oversized", c_uint64),
        ("over_budget", c_uint64),
        ("after", c_uint64),
        ("opacity_reset", c_uint32),
        ("_pad", c_uint32),
    ]


class PeerHandleC(ctypes.Structure):
    """sp_peer_handle: a rank's parameter and gradient buffers as CUDA IPC handles."""

    _fields_ = [
        ("params", ctypes.c_uint8 * 64),
        ("gradients", ctypes.c_uint8 * 64),
        ("params_offset", c_uint64),
        ("gradients_offset", c_uint64),
        ("gaussian_count", c_uint64),
        ("stride", c_uint32),
        ("device", ctypes.c_int32),
    ]


class PinholeCameraC(ctypes.Structure):
    _fields_ = [
        ("rotation", c_double * 9),
        ("translation", c_double * 3),
        ("focal", c_double * 2),
        ("principal_point", c_double * 2),
        ("width", c_uint32),
        ("height", c_uint32),
    ]


class PoseCorrectionC(ctypes.Structure):
    _fields_ = [("rotation", c_double * 3), ("translation", c_double * 3)]


class PoseGradientC(ctypes.Structure):
    _fields_ = [("rotation", c_double * 3), ("translation", c_double * 3), ("focal_log_scale", c_double)]


# Every exported symbol with its (restype, argtypes).
_P = c_void_p
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "sp_version": (c_char_p, []),
    "sp_status_string": (c_char_p, [c_int]),
    "sp_context_create": (c_int, [c_int, POINTER(_P)]),
    "sp_context_create_on_stream": (c_int, [c_int, _P, POINTER(_P)]),
    "sp_context_destroy": (None, [_P]),
    "sp_context_sync": (c_int, [_P]),
    "sp_context_stream": (_P, [_P]),
    "sp_last_error": (c_char_p, [_P]),
    "sp_camera_uniform_from_pinhole": (
        c_int,
        [POINTER(c_double), POINTER(c_double), POINTER(c_double), POINTER(c_double), c_uint32, c_uint32,
         POINTER(CameraUniform)],
    ),
    "sp_options_default": (None, [POINTER(Options)]),
    "sp_rasterizer_create": (
        c_int, [_P, _P, c_uint64, c_uint32, c_uint32, _P, c_uint32, POINTER(Options), POINTER(_P)]
    ),
    "sp_rasterizer_destroy": (None, [_P]),
    "sp_rasterizer_param_stride": (c_uint32, [_P]),
    "sp_set_camera": (c_int, [_P, POINTER(CameraUniform)]),
    "sp_forward": (c_int, [_P]),
    "sp_loss": (c_int, [_P, c_uint32]),
    "sp_backward": (c_int, [_P]),
    "sp_backward_blend": (c_int, [_P]),
    "sp_backward_project": (c_int, [_P, c_uint64, c_uint64]),
    "sp_write_loss_gradient": (c_int, [_P, _P, c_int]),
    "sp_write_image": (c_int, [_P, _P, c_int]),
    "sp_param_gradients": (_P, [_P]),
    "sp_zero_param_gradients": (c_int, [_P]),
    "sp_camera_gradient_device": (_P, [_P]),
    "sp_densify_stats_device": (_P, [_P]),
    "sp_read_loss_gradient": (c_int, [_P, _P]),
    "sp_read_param_gradients": (c_int, [_P, _P]),
    "sp_read_densify_stats": (c_int, [_P, _P]),
    "sp_write_densify_stats": (c_int, [_P, _P]),
    "sp_read_camera_gradient": (c_int, [_P, POINTER(CameraGradient)]),
    "sp_read_image": (c_int, [_P, _P]),
    "sp_read_pixel_loss": (c_int, [_P, _P]),
    "sp_read_loss": (c_int, [_P, POINTER(LossTermsC)]),
    "sp_loss_sums_noalloc": (c_int, [c_int, _P, c_uint64, _P, _P]),
    "sp_read_intersections": (c_int, [_P, POINTER(IntersectionMeta)]),
    "sp_render": (c_int, [_P, POINTER(CameraUniform), _P]),
    "sp_backward_adam": (c_int, [_P, _P, c_float]),
    "sp_train_step": (
        c_int, [_P, _P, POINTER(CameraUniform), c_uint32, c_float, POINTER(CameraGradient), POINTER(LossTermsC)]
    ),
    "sp_read_projected": (c_int, [_P, _P]),
    "sp_read_sorted_intersections": (c_int, [_P, _P, _P]),
    "sp_read_tile_ranges": (c_int, [_P, _P]),
    "sp_read_contributions": (c_int, [_P, _P]),
    "sp_read_tile_offsets": (c_int, [_P, _P]),
    "sp_read_gaussian_blend_gradients": (c_int, [_P, _P]),
    "sp_clear_densify_stats": (c_int, [_P]),
    "sp_count_blend_work": (c_int, [_P, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)]),
    "sp_debug_stall_sort_partition": (c_int, [_P, c_uint32]),
    "sp_intersections_needed": (c_int, [_P, POINTER(c_uint64)]),
    "sp_reserve_intersections": (c_int, [_P, c_uint64]),
    "sp_debug_falloff_powers": (c_int, [c_void_p, c_uint64, c_void_p, c_void_p]),
    "sp_debug_adam_quotients": (c_int, [c_void_p, c_void_p, c_uint64, c_void_p, c_void_p]),
    "sp_profile_enable": (c_int, [_P, c_int]),
    "sp_profile_read": (c_int, [_P, POINTER(c_double), POINTER(c_uint64)]),
    "sp_adam_create": (c_int, [_P, _P, _P, c_uint64, c_uint32, POINTER(LearningRatesC), c_float, POINTER(_P)]),
    "sp_adam_resume": (c_int, [_P, _P, _P, c_uint64, _P, _P, POINTER(_P)]),
    "sp_adam_destroy": (None, [_P]),
    "sp_adam_step": (c_int, [_P, c_float]),
    "sp_adam_advance": (c_int, [_P, c_float]),
    "sp_adam_step_range": (c_int, [_P, c_uint64, c_uint64]),
    "sp_adam_steps_taken": (c_uint32, [_P]),
    "sp_adam_read_moments": (c_int, [_P, _P, _P]),
    "sp_adam_first_moment_device": (_P, [_P]),
    "sp_peer_export": (c_int, [_P, POINTER(PeerHandleC)]),
    "sp_peer_exchange_create": (c_int, [_P, c_uint32, c_uint32, POINTER(PeerHandleC), POINTER(_P)]),
    "sp_peer_exchange_step": (c_int, [_P, c_float]),
    "sp_peer_exchange_destroy": (None, [_P]),
    "sp_comm_unique_id": (c_int, [_P]),
    "sp_comm_nccl_version": (c_int, []),
    "sp_comm_init": (c_int, [_P, _P, c_uint32, c_uint32, c_uint32, POINTER(_P)]),
    "sp_comm_destroy": (None, [_P]),
    "sp_comm_rank": (c_uint32, [_P]),
    "sp_comm_world": (c_uint32, [_P]),
    "sp_comm_barrier": (c_int, [_P]),
    "sp_comm_wait": (c_int, [_P]),
    "sp_allreduce_grads": (c_int, [_P, _P]),
    "sp_adam_step_sharded": (c_int, [_P, _P, c_float]),
    "sp_exchange_create": (c_int, [_P, _P, c_uint32, POINTER(_P)]),
    "sp_exchange_mode": (c_uint32, [_P]),
    "sp_exchange_probe_link": (c_int, [_P, c_uint32, c_uint64, POINTER(c_float)]),
    "sp_exchange_step": (c_int, [_P, c_float]),
    "sp_exchange_gather_moments": (c_int, [_P]),
    "sp_exchange_destroy": (None, [_P]),
    "sp_comm_merge_densify_stats": (c_int, [_P, _P]),
    "sp_adam_second_moment_device": (_P, [_P]),
    "sp_position_rate_factor": (c_float, [c_uint64, c_uint64]),
    "sp_adam_resume_device": (c_int, [_P, _P, _P, c_uint64, _P, _P, POINTER(_P)]),
    "sp_densify_after": (c_int, [POINTER(DensifySettingsC), c_uint64, c_uint64]),
    "sp_resets_opacity_after": (c_int, [POINTER(DensifySettingsC), c_uint64]),
    "sp_densify_plan": (
        c_int,
        [_P, _P, c_float, c_uint64, POINTER(DensifySettingsC), c_int, c_uint64, POINTER(_P),
         POINTER(DensifyReportC)],
    ),
    "sp_densify_apply": (c_int, [_P, _P, _P, _P, c_uint64]),
    "sp_densify_destroy": (None, [_P]),
    "sp_corrected_camera": (
        c_int, [POINTER(PinholeCameraC), POINTER(PoseCorrectionC), c_double, POINTER(PinholeCameraC)]
    ),
    "sp_pose_gradient_of": (
        c_int,
        [POINTER(PinholeCameraC), POINTER(PoseCorrectionC), c_double, POINTER(CameraGradient),
         POINTER(PoseGradientC)],
    ),
    "sp_pose_refinement_create": (
        c_int, [POINTER(PinholeCameraC), c_uint32, POINTER(LearningRatesC), c_float, POINTER(_P)]
    ),
    "sp_pose_refinement_destroy": (None, [_P]),
    "sp_pose_refinement_camera": (c_int, [_P, c_uint32, POINTER(PinholeCameraC)]),
    "sp_pose_refinement_step": (c_int, [_P, c_uint32, POINTER(CameraGradient), c_float]),
    "sp_pose_refinement_correction": (c_int, [_P, c_uint32, POINTER(PoseCorrectionC)]),
    "sp_pose_refinement_focal_scale": (c_double, [_P]),
    "sp_pose_refinement_last_gradient": (c_int, [_P, POINTER(PoseGradientC)]),
    "sp_train_step_host_poses": (c_int, [_P, _P, _P, c_uint32, c_float, POINTER(LossTermsC)]),
    "sp_device_poses_create": (c_int, [_P, _P, POINTER(_P)]),
    "sp_device_poses_destroy": (None, [_P]),
    "sp_device_poses_set_camera": (c_int, [_P, c_uint32]),
    "sp_device_poses_step": (c_int, [_P, c_uint32, c_uint32, c_float]),
    "sp_device_poses_download": (c_int, [_P, _P]),
    "sp_train_step_device_poses": (c_int, [_P, _P, _P, c_uint32, c_uint32, c_float, _P]),
    "sp_ply_write": (c_int, [c_char_p, _P, c_uint64, c_uint32, c_int]),
    "sp_ply_read_header": (c_int, [c_char_p, POINTER(c_uint64), POINTER(c_uint32)]),
    "sp_ply_read": (c_int, [c_char_p, _P, c_uint64, c_uint32, c_int]),
    "sp_ply_error": (c_char_p, []),
}


class SplatError(RuntimeError):
    """An sp_status other than SP_OK, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} ({_STATUS_NAMES.get(status, status)})")
        self.status = status


_STATUS_NAMES = {
    SP_ERR_INVALID: "SP_ERR_INVALID",
    SP_ERR_TOO_MANY_TILES: "SP_ERR_TOO_MANY_TILES",
    SP_ERR_OVERFLOW: "SP_ERR_OVERFLOW",
    SP_ERR_TIMEOUT: "SP_ERR_TIMEOUT",
    SP_ERR_CUDA: "SP_ERR_CUDA",
    SP_ERR_NCCL: "SP_ERR_NCCL",
    SP_ERR_NONFINITE: "SP_ERR_NONFINITE",
    SP_ERR_NO_DEVICE: "SP_ERR_NO_DEVICE",
    SP_ERR_OUT_OF_MEMORY: "SP_ERR_OUT_OF_MEMORY",
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library with its prototypes set. Raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise ImportError(
                f"{LIBRARY_PATH} is missing: build it with `python splatting-rs_b200/build.py` "
                "(or __graft_entry__.build()); there is no fallback implementation"
            )
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def check(status: int, ctx: int | None = None, what: str = "") -> None:
    if status == SP_OK:
        return
    lib = load()
    message = lib.sp_last_error(ctx).decode() if ctx else lib.sp_status_string(status).decode()
    raise SplatError(status, f"{what}: {message}" if what else message)
