"""The C ABI without a GPU: the library loads, exports every function include/splat.h
declares, its structs have the reference's #[repr(C)] layouts, and its host-only calls and
argument checks behave as documented."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import splat_b200 as sb
from splat_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    """Functions include/*.h declares for the library to export: the prototypes of the
    headers with an extern "C" block (splat_math.h only holds inline helpers compiled into
    their callers)."""
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        if 'extern "C"' not in header.read_text():
            continue
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"#define[^\n]*", "", text)
        for match in re.finditer(r"\b(sp_[a-z0-9_]+)\s*\(([^;{]*)\)\s*([;{])", text):
            if match.group(3) == ";":
                names.add(match.group(1))
    return names


def test_library_exports_every_declared_function():
    lib = _lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIBRARY_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (sp_[a-z0-9_]+)", out))
    declared = declared_functions()
    assert len(declared) > 50
    assert declared <= exported, f"declared but not exported: {sorted(declared - exported)}"
    assert declared <= set(_lib.SIGNATURES), f"not bound in _lib: {sorted(declared - set(_lib.SIGNATURES))}"
    for name in declared:
        assert getattr(lib, name) is not None


def test_struct_layouts_match_the_reference():
    """CameraUniform (camera.rs:23-31), CameraGradient (camera.rs:39-43), IntersectionMeta
    and Projected and DensifyStats (rasterizer.rs:29-75)."""
    c = _lib.CameraUniform
    assert ctypes.sizeof(c) == 80
    assert (c.focal.offset, c.principal_point.offset, c.width.offset, c.tiles_y.offset) == (48, 56, 64, 76)
    g = _lib.CameraGradient
    assert ctypes.sizeof(g) == 56 and g.world_to_camera_translation.offset == 36 and g.focal.offset == 48
    p = _lib.Projected
    assert ctypes.sizeof(p) == 80
    assert (p.conic.offset, p.depth.offset, p.color.offset, p.opacity.offset, p.radius.offset) == (16, 28, 32, 44, 48)
    assert (p.tile_min.offset, p.tile_max.offset) == (56, 64)
    assert ctypes.sizeof(_lib.IntersectionMeta) == 20 and ctypes.sizeof(_lib.DensifyStats) == 16
    assert ctypes.sizeof(_lib.Options) == 36 and _lib.Options.tile_culling.offset == 32
    assert ctypes.sizeof(_lib.DensifySettingsC) == 40 and ctypes.sizeof(_lib.DensifyReportC) == 64
    assert ctypes.sizeof(_lib.PeerHandleC) == 160


def test_default_options_are_the_reference_behaviour():
    opt = sb.default_options()
    assert opt.key_mode == sb.SP_KEYS_REF20 and opt.sh_degree == 0
    assert opt.intersections_per_gaussian == 24 and opt.accumulate_gradients == 0
    w = opt.loss_weights
    assert (np.float32(w.l1), np.float32(w.dssim), np.float32(w.alpha)) == (np.float32(0.8), np.float32(0.2), 1.0)


def test_camera_uniform_matches_numpy():
    rng = np.random.default_rng(4)
    q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
    if np.linalg.det(q) < 0:
        q[:, 0] *= -1
    cam = sb.PinholeCamera(q, rng.normal(size=3), (123.4, 130.5), (60.5, 40.25), 121, 80)
    u = cam.uniform()
    w, t = cam.world_to_camera()
    rows = np.array([[u.world_to_camera_rows[r][c] for c in range(4)] for r in range(3)])
    assert np.array_equal(rows[:, :3], w.astype(np.float32)) and np.array_equal(rows[:, 3], t.astype(np.float32))
    assert (u.tiles_x, u.tiles_y) == (8, 5)
    assert tuple(u.focal) == (np.float32(123.4), np.float32(130.5))


def test_host_side_argument_checks():
    lib = _lib.load()
    handle = ctypes.c_void_p()
    assert lib.sp_rasterizer_create(None, None, 0, 0, 0, None, 0, None, ctypes.byref(handle)) == _lib.SP_ERR_INVALID
    assert lib.sp_adam_create(None, None, None, 0, 0, None, 1.0, ctypes.byref(handle)) == _lib.SP_ERR_INVALID
    assert lib.sp_forward(None) == _lib.SP_ERR_INVALID
    assert lib.sp_position_rate_factor(10, 10) < 0
    assert lib.sp_status_string(3) == b"SP_ERR_OVERFLOW"
    assert lib.sp_loss_sums_noalloc(0, None, 1, None, None) == _lib.SP_ERR_INVALID


def test_no_device_is_reported_without_a_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    lib = _lib.load()
    handle = ctypes.c_void_p()
    assert lib.sp_context_create(0, ctypes.byref(handle)) == _lib.SP_ERR_NO_DEVICE
    with pytest.raises(sb.SplatError):
        sb.Context(0, stream=0)


def test_python_mirror_refuses_host_tensors():
    import torch

    with pytest.raises(ValueError):
        sb.Rasterizer._pointer(torch.zeros(4))


def test_profiler_kernel_names_follow_the_header_enum():
    """KERNEL_NAMES indexes sp_profile_read's arrays: one name per SP_K_* value, in order."""
    text = (ROOT / "include" / "splat.h").read_text()
    values = {m.group(1).lower(): int(m.group(2)) for m in re.finditer(r"SP_K_(\w+) = (\d+)", text)}
    count = values.pop("count")
    assert count == len(_lib.KERNEL_NAMES)
    assert [name for name, _ in sorted(values.items(), key=lambda kv: kv[1])] == list(_lib.KERNEL_NAMES)


def test_a_c_caller_links_and_runs(tmp_path):
    """tests/c_abi/abi_test.c, compiled with gcc against include/ and linked to the library:
    the headers compile as C and the host-only entry points behave as declared."""
    exe = tmp_path / "abi_test"
    lib_dir = _lib.LIBRARY_PATH.parent
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(ROOT / "tests" / "c_abi" / "abi_test.c"),
                    f"-L{lib_dir}", f"-Wl,-rpath,{lib_dir}", "-lsplat_b200", "-lm", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe), str(tmp_path / "abi.ply")], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "ok"
