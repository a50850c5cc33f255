"""Splat files around the training path: the binary PLY of the 3DGS reference implementation
(instantsplat-rs/src/splat_ply.rs, native in libsplat_b200: sp_ply_*) and the cameras.json
of the 3DGS reference with the principal point added (instantsplat-rs/src/cameras_json.rs).

PLY files are read and written as the reference does at SH degree 0; at degrees 1-3 the
3DGS f_rest_* properties carry the higher coefficients (channel-major), which the
reference's writer lacks and its reader skips. Device tensors are written and filled
directly (one transfer each way).
"""

from __future__ import annotations

import ctypes
import json
import math
from decimal import Decimal
from pathlib import Path

import numpy as np

from . import _lib
from .camera import PinholeCamera
from .gaussians import GaussianCloud, param_stride


class SplatFileError(ValueError):
    """A file the reference's reader refuses (its anyhow messages)."""


def _check(status: int, what: str) -> None:
    if status != 0:
        message = (_lib.load().sp_ply_error() or b"").decode(errors="replace")
        if status == 1:
            raise SplatFileError(message or what)
        raise _lib.SplatError(status, f"{what}: {message}")


def _path(path) -> bytes:
    return str(Path(path)).encode()


def write_splat_ply(path, cloud: GaussianCloud) -> None:
    """write_splat_ply (splat_ply.rs:18-46), at the cloud's SH degree."""
    packed = np.ascontiguousarray(cloud.to_packed(), np.float32)
    _check(_lib.load().sp_ply_write(_path(path), packed.ctypes.data_as(ctypes.c_void_p), len(cloud),
                                    cloud.sh_degree, 0), "write_splat_ply")


def write_splat_ply_device(path, params, count: int, sh_degree: int = 0) -> None:
    """write_splat_ply of `count` Gaussians packed in a CUDA tensor (e.g. a trainer's params)."""
    from .rasterizer import Rasterizer

    _check(_lib.load().sp_ply_write(_path(path), ctypes.c_void_p(Rasterizer._pointer(params)), int(count),
                                    int(sh_degree), 1), "write_splat_ply")


def read_splat_ply_header(path) -> tuple[int, int]:
    """(vertex count, SH degree of the f_rest_* properties)."""
    count, degree = ctypes.c_uint64(), ctypes.c_uint32()
    _check(_lib.load().sp_ply_read_header(_path(path), ctypes.byref(count), ctypes.byref(degree)), "read header")
    return int(count.value), int(degree.value)


def read_splat_ply(path, sh_degree: int | None = None) -> GaussianCloud:
    """read_splat_ply (splat_ply.rs:48-112). `sh_degree` None takes the file's; 0 is the
    reference's reader (f_rest_* skipped)."""
    count, file_degree = read_splat_ply_header(path)
    degree = file_degree if sh_degree is None else int(sh_degree)
    packed = np.empty(count * param_stride(degree), np.float32)
    _check(_lib.load().sp_ply_read(_path(path), packed.ctypes.data_as(ctypes.c_void_p), count, degree, 0),
           "read_splat_ply")
    return GaussianCloud.from_packed(packed, degree)


def read_splat_ply_device(path, sh_degree: int | None = None, device: int = 0):
    """The file's Gaussians packed into a new CUDA tensor; returns (tensor, count, degree)."""
    import torch

    count, file_degree = read_splat_ply_header(path)
    degree = file_degree if sh_degree is None else int(sh_degree)
    params = torch.empty(count * param_stride(degree), dtype=torch.float32, device=f"cuda:{device}")
    torch.cuda.synchronize(device)
    _check(_lib.load().sp_ply_read(_path(path), ctypes.c_void_p(params.data_ptr()), count, degree, 1),
           "read_splat_ply")
    return params, count, degree


# ---- cameras.json (cameras_json.rs)


def rust_display(value: float) -> str:
    """Rust's `{}` of an f64: the shortest digits that read back to the same value (as
    Python's repr), never in exponent form, integers without a fraction."""
    value = float(value)
    if math.isnan(value):
        return "NaN"
    if math.isinf(value):
        return "inf" if value > 0 else "-inf"
    text = repr(value)
    if "e" in text or "E" in text:
        text = format(Decimal(text), "f")
    if text.endswith(".0"):
        text = text[:-2]
    return text


def write_cameras_json(path, cameras: list[tuple[str, PinholeCamera]]) -> None:
    """write_cameras_json (cameras_json.rs:17-51): one line per view, as the reference
    formats it."""
    Path(path).write_text(cameras_json_text(cameras))


def cameras_json_text(cameras: list[tuple[str, PinholeCamera]]) -> str:
    lines = ["["]
    for index, (name, camera) in enumerate(cameras):
        r = np.asarray(camera.rotation, np.float64).reshape(3, 3)
        t = np.asarray(camera.translation, np.float64).reshape(3)
        rows = ", ".join("[" + ", ".join(rust_display(r[i, j]) for j in range(3)) + "]" for i in range(3))
        d = rust_display
        lines.append(
            f'  {{"id": {index}, "img_name": "{name}", "width": {camera.width}, "height": {camera.height}, '
            f'"position": [{d(t[0])}, {d(t[1])}, {d(t[2])}], "rotation": [{rows}], '
            f'"fx": {d(camera.focal[0])}, "fy": {d(camera.focal[1])}, '
            f'"cx": {d(camera.principal_point[0])}, "cy": {d(camera.principal_point[1])}}}'
            + ("," if index + 1 < len(cameras) else "")
        )
    lines.append("]")
    return "\n".join(lines) + "\n"


def read_cameras_json(path) -> list[tuple[str, PinholeCamera]]:
    """read_cameras_json (cameras_json.rs:53-112). Cameras without cx / cy are refused."""
    return parse_cameras_json(Path(path).read_text(), str(path))


def parse_cameras_json(text: str, label: str) -> list[tuple[str, PinholeCamera]]:
    try:
        entries = json.loads(text)
    except json.JSONDecodeError as e:
        raise SplatFileError(f"parsing {label}: {e}") from e
    if not isinstance(entries, list):
        raise SplatFileError(f"{label}: not a JSON array")

    def number_of(value, key):
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise SplatFileError(f'{label}: "{key}" is not a number')
        return float(value)

    def numbers(value, count):
        if not isinstance(value, list) or any(isinstance(v, bool) or not isinstance(v, (int, float)) for v in value):
            raise SplatFileError(f"{label}: expected an array of numbers")
        if len(value) != count:
            raise SplatFileError(f"{label}: expected {count} numbers")
        return [float(v) for v in value]

    out = []
    for entry in entries:
        def field(key):
            if not isinstance(entry, dict) or key not in entry:
                raise SplatFileError(f'{label}: a camera has no "{key}" (written by an older version?)')
            return entry[key]

        name = field("img_name")
        if not isinstance(name, str):
            raise SplatFileError(f'{label}: "img_name" is not a string')
        position = numbers(field("position"), 3)
        rows = field("rotation")
        if not isinstance(rows, list):
            raise SplatFileError(f'{label}: "rotation" is not an array')
        rows = [numbers(row, 3) for row in rows]
        if len(rows) != 3:
            raise SplatFileError(f'{label}: "rotation" needs 3 rows')
        focal = (number_of(field("fx"), "fx"), number_of(field("fy"), "fy"))
        principal = (number_of(field("cx"), "cx"), number_of(field("cy"), "cy"))
        # `as u32`: truncation, saturating at 0 and u32::MAX.
        width = int(min(max(number_of(field("width"), "width"), 0.0), 4294967295.0))
        height = int(min(max(number_of(field("height"), "height"), 0.0), 4294967295.0))
        out.append((name, PinholeCamera(np.array(rows, np.float64), np.array(position, np.float64), focal, principal,
                                        width, height)))
    return out


# ------------------------------------------------------------------ training views (PNG)

# training_frames.rs:16-20: what transparent pixels are blended onto, and the alpha from
# which a pixel is foreground.
BACKGROUND_RGB8 = (128, 128, 128)
FOREGROUND_MIN_ALPHA = 128


def training_view_from_rgba8(rgba: np.ndarray, camera: PinholeCamera) -> tuple[np.ndarray, np.ndarray]:
    """training_view_from_image (training_frames.rs:71-115) at the camera's own size: the
    colour composited on BACKGROUND_RGB8 by alpha in integer arithmetic
    (composite_on_background, training_frames.rs:37-46), rgb = channel / 255 as float32, and
    foreground = alpha >= 128. `rgba` is height x width x 4 uint8. Returns (rgb of P x 3,
    foreground of P booleans). Views at another size than the camera's are refused (the
    reference resizes them; the training path here takes views at the camera's size)."""
    rgba = np.asarray(rgba)
    if rgba.dtype != np.uint8 or rgba.ndim != 3 or rgba.shape[2] != 4:
        raise SplatFileError("a training view is an RGBA image of 8-bit channels")
    height, width = rgba.shape[:2]
    if (width, height) != (camera.width, camera.height):
        raise SplatFileError(f"the image is {width}x{height}, its camera is {camera.width}x{camera.height}")
    alpha = rgba[:, :, 3:4].astype(np.uint32)
    background = np.array(BACKGROUND_RGB8, np.uint32)
    composited = (rgba[:, :, :3].astype(np.uint32) * alpha + background * (255 - alpha)) // 255
    foreground = (rgba[:, :, 3] >= FOREGROUND_MIN_ALPHA).reshape(-1)
    if not foreground.any():
        raise SplatFileError("the view has no foreground pixel")
    rgb = composited.astype(np.float32).reshape(-1, 3) / np.float32(255.0)
    return rgb, foreground


def read_training_view(path, camera: PinholeCamera) -> tuple[np.ndarray, np.ndarray]:
    """load_training_view (training_frames.rs:60-66) of a PNG at the camera's size."""
    from PIL import Image

    with Image.open(path) as image:
        rgba = np.asarray(image.convert("RGBA"))
    return training_view_from_rgba8(rgba, camera)


def read_fit_run(directory) -> tuple[GaussianCloud, list[PinholeCamera], np.ndarray]:
    """A fit run's splat.ply, cameras.json and input_view{i}.png, as the reference's step
    timing loads them (examples/step_timing.rs:31-40): the cloud, the cameras in file order and
    the ground truth of every view (loss::ground_truth_rgba, loss.rs:95-104), views x P x 4."""
    directory = Path(directory)
    cloud = read_splat_ply(directory / "splat.ply")
    cameras = [camera for _, camera in read_cameras_json(directory / "cameras.json")]
    views = []
    for i, camera in enumerate(cameras):
        rgb, foreground = read_training_view(directory / f"input_view{i}.png", camera)
        mask = foreground.astype(np.float32)[:, None]
        views.append(np.concatenate([rgb * mask, mask], axis=1))
    return cloud, cameras, np.stack(views)
