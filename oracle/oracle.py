"""numpy/ctypes front end of the CPU oracle (liboracle_splat.so) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use this module, as
the checker or as the timed CPU baseline. Nothing in the product (splatting-rs_b200/) imports
it. See splat_oracle.h for what it restates and how it is pinned.
"""

from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY_PATH = HERE / "liboracle_splat.so"

PROJECTED_DTYPE = np.dtype(
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
META_DTYPE = np.dtype([(k, "<u4") for k in ("count", "sort_blocks", "histogram_length", "overflow", "capacity")])
CAMERA_DTYPE = np.dtype(
    [
        ("rows", "<f4", (3, 4)),
        ("focal", "<f4", 2),
        ("principal_point", "<f4", 2),
        ("width", "<u4"),
        ("height", "<u4"),
        ("tiles_x", "<u4"),
        ("tiles_y", "<u4"),
    ]
)
assert PROJECTED_DTYPE.itemsize == 80 and CAMERA_DTYPE.itemsize == 80 and META_DTYPE.itemsize == 20


def build() -> Path:
    """Builds liboracle_splat.so with oracle/Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIBRARY_PATH))
        _lib.or_scan.restype = c_uint64
        _lib.or_bin.restype = c_uint64
        _lib.or_bias_correction.restype = c_float
        _lib.or_bias_correction.argtypes = [c_float, c_uint32]
        _lib.or_libm_expf.restype = c_float
        _lib.or_libm_expf.argtypes = [c_float]
        _lib.or_sp_expf.restype = c_float
        _lib.or_sp_expf.argtypes = [c_float]
        _lib.or_sp_expf_exact.restype = c_float
        _lib.or_sp_expf_exact.argtypes = [c_float]
        _lib.or_train_step.restype = c_double
        _lib.or_get_threads.restype = c_int
        _lib.or_splitmix64.restype = c_uint64
        _lib.or_total_order_key.restype = c_uint32
        _lib.or_densify.restype = c_int
    return _lib


def _p(a: np.ndarray) -> c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(c_void_p)


def camera_array(uniform) -> np.ndarray:
    """An 80-byte camera record from a ctypes CameraUniform (or anything with its fields)."""
    cam = np.zeros(1, CAMERA_DTYPE)
    cam["rows"][0] = np.array([[uniform.world_to_camera_rows[r][c] for c in range(4)] for r in range(3)], np.float32)
    cam["focal"][0] = [uniform.focal[0], uniform.focal[1]]
    cam["principal_point"][0] = [uniform.principal_point[0], uniform.principal_point[1]]
    cam["width"], cam["height"] = uniform.width, uniform.height
    cam["tiles_x"], cam["tiles_y"] = uniform.tiles_x, uniform.tiles_y
    return cam


def camera_from_pinhole(rotation, translation, focal, principal_point, width: int, height: int) -> np.ndarray:
    """PinholeCamera::uniform (camera.rs:46-70) in numpy: world-to-camera rows (R^T, -R^T c)
    formed in f64 and rounded once to f32, focal and principal point to f32, tiles of 16
    pixels rounded up. The 80-byte camera record the oracle's functions take."""
    r = np.asarray(rotation, np.float64).reshape(3, 3)
    c = [float(v) for v in np.asarray(translation, np.float64).reshape(3)]
    w = r.T
    cam = np.zeros(1, CAMERA_DTYPE)
    for row in range(3):
        # -(w[row, 0] c0 + w[row, 1] c1 + w[row, 2] c2), summed left to right as the reference.
        t = -((float(w[row, 0]) * c[0] + float(w[row, 1]) * c[1]) + float(w[row, 2]) * c[2])
        cam["rows"][0, row, :3] = w[row].astype(np.float32)
        cam["rows"][0, row, 3] = np.float32(t)
    cam["focal"][0] = np.array([focal[0], focal[1]], np.float64).astype(np.float32)
    cam["principal_point"][0] = np.array([principal_point[0], principal_point[1]], np.float64).astype(np.float32)
    cam["width"], cam["height"] = width, height
    cam["tiles_x"], cam["tiles_y"] = (width + 15) // 16, (height + 15) // 16
    return cam


def camera_of(camera) -> np.ndarray:
    """camera_from_pinhole of an object with the PinholeCamera fields (rotation, translation,
    focal, principal_point, width, height)."""
    return camera_from_pinhole(camera.rotation, camera.translation, camera.focal, camera.principal_point,
                               camera.width, camera.height)


def set_threads(threads: int) -> None:
    lib().or_set_threads(int(threads))


def threads() -> int:
    return int(lib().or_get_threads())


def sp_expf(x: float) -> float:
    return float(lib().or_sp_expf(float(x)))


def sp_expf_exact(x: float) -> float:
    return float(lib().or_sp_expf_exact(float(x)))


def libm_expf(x: float) -> float:
    return float(lib().or_libm_expf(float(x)))


def project(params: np.ndarray, sh_degree: int, cam: np.ndarray):
    stride = 11 + 3 * (sh_degree + 1) ** 2
    params = np.ascontiguousarray(params, np.float32)
    n = params.size // stride
    proj = np.zeros(n, PROJECTED_DTYPE)
    counts = np.zeros(n, np.uint32)
    lib().or_project(_p(params), c_uint64(n), c_uint32(sh_degree), _p(cam), _p(proj), _p(counts))
    return proj, counts


def scan(counts: np.ndarray, capacity: int):
    offsets = np.zeros(len(counts), np.uint32)
    meta = np.zeros(1, META_DTYPE)
    total = lib().or_scan(_p(np.ascontiguousarray(counts, np.uint32)), c_uint64(len(counts)), c_uint64(capacity),
                          _p(offsets), _p(meta))
    return offsets, meta[0], int(total)


def bin_intersections(proj: np.ndarray, offsets: np.ndarray, cam: np.ndarray, capacity: int, key_mode: int = 0):
    n = len(proj)
    span = (proj["tile_max"].astype(np.int64) - proj["tile_min"].astype(np.int64))
    total = int(np.sum((span[:, 0] * span[:, 1])[proj["radius"] != 0])) if n else 0
    count = min(total, capacity)
    keys = np.zeros(max(count, 1), np.uint64)
    gauss = np.zeros(max(count, 1), np.uint32)
    slots = np.zeros(max(count, 1), np.uint32)
    tiles = int(cam["tiles_x"][0]) * int(cam["tiles_y"][0])
    ranges = np.zeros(2 * tiles, np.uint32)
    got = lib().or_bin(_p(proj), _p(offsets), c_uint64(n), _p(cam), c_uint64(capacity), c_int(key_mode), _p(keys),
                       _p(gauss), _p(slots), _p(ranges))
    assert got == count
    return keys[:count], gauss[:count], slots[:count], ranges


def blend_forward(proj, gauss, ranges, cam):
    w, h = int(cam["width"][0]), int(cam["height"][0])
    image = np.zeros(w * h * 4, np.float32)
    contrib = np.zeros(w * h, np.uint32)
    g = np.ascontiguousarray(gauss if len(gauss) else np.zeros(1, np.uint32), np.uint32)
    lib().or_blend_forward(_p(proj), _p(g), _p(ranges), _p(cam), _p(image), _p(contrib))
    return image, contrib


def ssim(image, gt_view, width, height):
    partials = np.zeros(width * height * 12, np.float32)
    lib().or_ssim(_p(np.ascontiguousarray(image, np.float32)), _p(np.ascontiguousarray(gt_view, np.float32)),
                  c_uint32(width), c_uint32(height), _p(partials))
    return partials


class _Weights(ctypes.Structure):
    _fields_ = [("l1", c_float), ("dssim", c_float), ("alpha", c_float)]


def loss(image, gt_view, partials, width, height, weights=(0.8, 0.2, 1.0)):
    grad = np.zeros(width * height * 4, np.float32)
    pixel_loss = np.zeros(width * height * 4, np.float32)
    w = _Weights(*weights)
    lib().or_loss(_p(np.ascontiguousarray(image, np.float32)), _p(np.ascontiguousarray(gt_view, np.float32)),
                  _p(partials), c_uint32(width), c_uint32(height), ctypes.byref(w), _p(grad), _p(pixel_loss))
    return grad, pixel_loss


def blend_backward(proj, gauss, slots, ranges, cam, image, contrib, loss_gradient, capacity):
    out = np.zeros(max(capacity, 1) * 10, np.float32)
    g = np.ascontiguousarray(gauss if len(gauss) else np.zeros(1, np.uint32), np.uint32)
    s = np.ascontiguousarray(slots if len(slots) else np.zeros(1, np.uint32), np.uint32)
    lib().or_blend_backward(_p(proj), _p(g), _p(s), _p(ranges), _p(cam), _p(image), _p(contrib),
                            _p(np.ascontiguousarray(loss_gradient, np.float32)), _p(out))
    return out


def blend_backward_magnitudes(proj, gauss, slots, ranges, cam, image, contrib, loss_gradient, capacity):
    """blend_backward, and per slot the sums of the absolute values of its per-pixel terms
    (float64, capacity x 10)."""
    out = np.zeros(max(capacity, 1) * 10, np.float32)
    mags = np.zeros(max(capacity, 1) * 10, np.float64)
    g = np.ascontiguousarray(gauss if len(gauss) else np.zeros(1, np.uint32), np.uint32)
    s = np.ascontiguousarray(slots if len(slots) else np.zeros(1, np.uint32), np.uint32)
    lib().or_blend_backward_magnitudes(_p(proj), _p(g), _p(s), _p(ranges), _p(cam), _p(image), _p(contrib),
                                       _p(np.ascontiguousarray(loss_gradient, np.float32)), _p(out), _p(mags))
    return out, mags.reshape(-1, 10)


def gaussian_sums_of_slots(fwd, slot_values: np.ndarray) -> np.ndarray:
    """Per Gaussian, the float64 sum of its rectangle's slots (offsets[g] .. + tile count) of
    `slot_values` (slots x k), as project_backward.wgsl:38-55 gathers them."""
    proj = fwd["proj"]
    count = ((proj["tile_max"][:, 0].astype(np.int64) - proj["tile_min"][:, 0]) *
             (proj["tile_max"][:, 1].astype(np.int64) - proj["tile_min"][:, 1]))
    count[proj["radius"] == 0] = 0
    first = fwd["offsets"].astype(np.int64)
    values = np.asarray(slot_values, np.float64)
    csum = np.concatenate([np.zeros((1, values.shape[1])), np.cumsum(values, axis=0)])
    last = np.minimum(first + count, len(values))
    return csum[last] - csum[np.minimum(first, last)]


def gradient_error_scale(params, sh_degree, cam, fwd, slot_magnitudes) -> np.ndarray:
    """Per parameter gradient (n x stride, float64): sum over the 9 blend sums k of
    |d gradient / d blend sum k| x (the sum of |terms| that blend sum k gathers). A rounding
    of the blend's per-pixel terms by a relative e, in any order of summation, moves a
    parameter gradient by at most about e x this scale: the tests' element-wise floor. The
    projection backward is linear in the blend sums, so its Jacobian's columns come from
    nine passes with a unit blend sum per Gaussian."""
    params = np.ascontiguousarray(params, np.float32)
    stride = 11 + 3 * (sh_degree + 1) ** 2
    n = params.size // stride
    count = int(fwd["meta"]["count"])
    magnitude = gaussian_sums_of_slots(fwd, np.asarray(slot_magnitudes)[:, :9])
    scale = np.zeros((n, stride), np.float64)
    first = fwd["offsets"].astype(np.int64)
    visible = np.nonzero(fwd["proj"]["radius"])[0]
    visible = visible[first[visible] < count]
    for k in range(9):
        unit = np.zeros((max(count, 1), 10), np.float32)
        unit[first[visible], k] = 1.0
        column, _, _ = project_backward(params, sh_degree, cam, fwd["proj"], fwd["offsets"], unit.reshape(-1),
                                        count)
        scale += np.abs(column.reshape(n, stride).astype(np.float64)) * magnitude[:, k:k + 1]
    return scale


def project_backward(params, sh_degree, cam, proj, offsets, slot_gradients, capacity, stats=None):
    stride = 11 + 3 * (sh_degree + 1) ** 2
    params = np.ascontiguousarray(params, np.float32)
    n = params.size // stride
    grads = np.zeros(n * stride, np.float32)
    camera = np.zeros(14, np.float32)
    stats = np.zeros((n, 4), np.float32) if stats is None else stats
    lib().or_project_backward(_p(params), c_uint64(n), c_uint32(sh_degree), _p(cam), _p(proj), _p(offsets),
                              _p(slot_gradients), c_uint64(capacity), _p(grads), _p(camera), _p(stats))
    return grads, camera, stats


def learning_rates_by_slot(rates: ctypes.Structure, position_scale: float, stride: int) -> np.ndarray:
    out = np.zeros(stride, np.float32)
    lib().or_learning_rates_by_slot(ctypes.byref(rates), c_float(position_scale), c_uint32(stride), _p(out))
    return out


def bias_correction(beta: float, step: int) -> float:
    return float(lib().or_bias_correction(beta, step))


def adam_step(params, grads, m, v, stride, lr_by_slot, step, max_log_scale, max_log_anisotropy):
    """In place on params, m, v (float32 arrays)."""
    n = params.size // stride
    lib().or_adam_step(_p(params), _p(np.ascontiguousarray(grads, np.float32)), _p(m), _p(v), c_uint64(n),
                       c_uint32(stride), _p(np.ascontiguousarray(lr_by_slot, np.float32)),
                       c_float(bias_correction(0.9, step)), c_float(bias_correction(0.999, step)),
                       c_float(max_log_scale), c_float(max_log_anisotropy))


def render(params, sh_degree, cam, capacity=None, key_mode=0):
    """project -> scan -> bin -> blend: everything of one forward pass, as a dict."""
    proj, counts = project(params, sh_degree, cam)
    capacity = capacity if capacity is not None else 24 * len(proj)
    offsets, meta, total = scan(counts, capacity)
    keys, gauss, slots, ranges = bin_intersections(proj, offsets, cam, capacity, key_mode)
    image, contrib = blend_forward(proj, gauss, ranges, cam)
    return dict(proj=proj, counts=counts, offsets=offsets, meta=meta, total=total, keys=keys, gauss=gauss,
                slots=slots, ranges=ranges, image=image, contrib=contrib, capacity=capacity)


def backward(params, sh_degree, cam, fwd, loss_gradient, stats=None):
    """blend backward -> projection backward for a forward pass from `render`."""
    slot_grads = blend_backward(fwd["proj"], fwd["gauss"], fwd["slots"], fwd["ranges"], cam, fwd["image"],
                                fwd["contrib"], loss_gradient, fwd["capacity"])
    count = int(fwd["meta"]["count"])
    grads, camera, stats = project_backward(params, sh_degree, cam, fwd["proj"], fwd["offsets"], slot_grads,
                                            count, stats)
    return dict(slot_gradients=slot_grads, param_gradients=grads, camera_gradient=camera, stats=stats)


def train_step(params, sh_degree, cam, gt_view, m, v, lr_by_slot, step, max_log_scale, max_log_anisotropy):
    """One full CPU training step, in place on params, m, v. Returns (mean loss, intersections)."""
    n = params.size // (11 + 3 * (sh_degree + 1) ** 2)
    count = c_uint64(0)
    loss_value = lib().or_train_step(_p(params), c_uint64(n), c_uint32(sh_degree), _p(cam),
                                     _p(np.ascontiguousarray(gt_view, np.float32)), _p(m), _p(v),
                                     _p(np.ascontiguousarray(lr_by_slot, np.float32)), c_uint32(step),
                                     c_float(max_log_scale), c_float(max_log_anisotropy), ctypes.byref(count))
    return float(loss_value), int(count.value)


class DensifyReportC(ctypes.Structure):
    """sp_densify_report (64 bytes)."""

    _fields_ = [(k, c_uint64) for k in ("before", "cloned", "split", "pruned_transparent", "pruned_oversized",
                                         "over_budget", "after")] + [("opacity_reset", c_uint32), ("_pad", c_uint32)]


REPORT_FIELDS = ("before", "cloned", "split", "pruned_transparent", "pruned_oversized", "over_budget", "after",
                 "opacity_reset")


def densify(params, first, second, stats, stride, extent, max_count, settings, reset_opacity, seed):
    """densify (densify.rs:147-257). `settings` is an sp_densify_settings ctypes structure,
    `stats` an (n, 4) float32 array of sp_densify_stats. Returns (params, first, second,
    report dict); raises ValueError when every Gaussian was pruned."""
    params = np.ascontiguousarray(params, np.float32).reshape(-1)
    first = np.ascontiguousarray(first, np.float32).reshape(-1)
    second = np.ascontiguousarray(second, np.float32).reshape(-1)
    stats = np.ascontiguousarray(stats, np.float32).reshape(-1, 4)
    n = params.size // stride
    assert stats.shape[0] == n and first.size == second.size == params.size
    report = DensifyReportC()
    # The first call sizes the outputs (status 2 when they do not fit).
    status = lib().or_densify(_p(params), _p(first), _p(second), _p(stats), c_uint64(n), c_uint32(stride),
                              c_float(extent), c_uint64(max_count), ctypes.byref(settings), c_int(reset_opacity),
                              c_uint64(seed), None, None, None, c_uint64(0), ctypes.byref(report))
    out = {k: int(getattr(report, k)) for k in REPORT_FIELDS}
    if status == 1:
        raise ValueError(f"densification pruned every Gaussian: {out}")
    after = out["after"]
    p, m, v = (np.empty(after * stride, np.float32) for _ in range(3))
    status = lib().or_densify(_p(params), _p(first), _p(second), _p(stats), c_uint64(n), c_uint32(stride),
                              c_float(extent), c_uint64(max_count), ctypes.byref(settings), c_int(reset_opacity),
                              c_uint64(seed), _p(p), _p(m), _p(v), c_uint64(after), ctypes.byref(report))
    assert status == 0, status
    return p, m, v, out


def splitmix64(seed: int, index: int) -> int:
    return int(lib().or_splitmix64(c_uint64(seed), c_uint64(index)))


def total_order_key(value: float) -> int:
    return int(lib().or_total_order_key(c_float(value)))
