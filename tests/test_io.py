"""Splat files (CPU): the PLY writer and reader (native, sp_ply_*) and cameras.json, against
the reference's own tests (splat_ply.rs:114-142, cameras_json.rs:114-140), its reader's
refusals (splat_ply.rs:54-112), an independent numpy parser of the 3DGS layout, and — where
the reference tree is present — the example files the reference ships."""

from __future__ import annotations

import math
import re
from pathlib import Path

import numpy as np
import pytest

import splat_b200 as sb
from splat_b200 import io

# The reference's example scene (instantsplat-rs/web/example), copied out of the reference tree
# by tests/golden/fetch_web_example.py (which __graft_entry__.build() runs where the tree is).
REFERENCE_EXAMPLE = Path(__file__).resolve().parent / "golden" / "web_example"

PROPERTIES_SH0 = ["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2", "opacity", "scale_0", "scale_1",
                  "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]


def two_gaussians() -> sb.GaussianCloud:
    """splat_ply.rs:120-126."""
    return sb.GaussianCloud(
        positions=np.array([[1.0, 2.0, 3.0], [-4.0, 5.5, 6.25]], np.float32),
        log_scales=np.array([[-1.0, -2.0, -3.0], [-4.0, -5.0, -6.0]], np.float32),
        rotations=np.array([[1.0, 0.0, 0.0, 0.0], [0.5, -0.5, 0.5, 0.5]], np.float32),
        opacity_logits=np.array([0.1, -2.2], np.float32),
        sh=np.array([[0.7, 0.8, 0.9], [-1.0, 1.1, 1.2]], np.float32).reshape(2, 1, 3),
    )


def parse_ply(data: bytes):
    """An independent reader of the 3DGS binary PLY: (property names, float32 records)."""
    end = data.index(b"end_header\n") + len(b"end_header\n")
    names = [line.split()[2] for line in data[:end].decode().splitlines() if line.startswith("property float")]
    return names, np.frombuffer(data[end:], "<f4").reshape(-1, len(names))


def clouds_equal(a: sb.GaussianCloud, b: sb.GaussianCloud) -> bool:
    return all(np.array_equal(getattr(a, f), getattr(b, f))
               for f in ("positions", "log_scales", "rotations", "opacity_logits", "sh"))


def test_ply_round_trips(tmp_path):
    """splat_ply.rs:114-142: the file's length, the property order, and the cloud back."""
    cloud = two_gaussians()
    path = tmp_path / "round_trip.ply"
    io.write_splat_ply(path, cloud)
    data = path.read_bytes()
    header_end = data.index(b"end_header\n") + 11
    assert len(data) == header_end + 2 * len(PROPERTIES_SH0) * 4
    assert ("property float f_dc_0\nproperty float f_dc_1\nproperty float f_dc_2\nproperty float opacity\n"
            "property float scale_0\n") in data[:header_end].decode()
    assert clouds_equal(io.read_splat_ply(path), cloud)


def test_ply_layout_is_the_3dgs_one(tmp_path):
    """The header and records byte for byte as splat_ply.rs:22-46 writes them."""
    cloud = two_gaussians()
    path = tmp_path / "a.ply"
    io.write_splat_ply(path, cloud)
    data = path.read_bytes()
    header = ("ply\nformat binary_little_endian 1.0\ncomment Exported from instantsplat-rs\nelement vertex 2\n"
              + "".join(f"property float {p}\n" for p in PROPERTIES_SH0) + "end_header\n")
    assert data.startswith(header.encode())
    names, records = parse_ply(data)
    assert names == PROPERTIES_SH0
    expected = np.concatenate([cloud.positions, np.zeros((2, 3), np.float32), cloud.sh_dc,
                               cloud.opacity_logits[:, None], cloud.log_scales, cloud.rotations], axis=1)
    assert np.array_equal(records, expected)


@pytest.mark.parametrize("degree", [1, 2, 3])
def test_higher_sh_degrees_use_the_3dgs_f_rest_layout(tmp_path, degree):
    """f_rest_{c (K-1) + k - 1} is coefficient k of channel c; reading at the file's degree
    gives the cloud back, at degree 0 the reference's reader (SH rest dropped), above the
    file's degree zeros."""
    rng = np.random.default_rng(degree)
    k = (degree + 1) ** 2
    n = 37
    cloud = sb.GaussianCloud(rng.normal(size=(n, 3)), rng.normal(size=(n, 3)), rng.normal(size=(n, 4)),
                             rng.normal(size=n), rng.normal(size=(n, k, 3)))
    path = tmp_path / "sh.ply"
    io.write_splat_ply(path, cloud)
    names, records = parse_ply(path.read_bytes())
    rest = [f"f_rest_{j}" for j in range(3 * (k - 1))]
    assert names == PROPERTIES_SH0[:9] + rest + PROPERTIES_SH0[9:]
    for c in range(3):
        for j in range(1, k):
            assert np.array_equal(records[:, 9 + c * (k - 1) + (j - 1)], cloud.sh[:, j, c])
    assert io.read_splat_ply_header(path) == (n, degree)
    assert clouds_equal(io.read_splat_ply(path), cloud)
    dc_only = io.read_splat_ply(path, sh_degree=0)
    assert dc_only.sh_degree == 0 and np.array_equal(dc_only.sh[:, 0], cloud.sh[:, 0])
    if degree < 3:
        above = io.read_splat_ply(path, sh_degree=3)
        assert np.array_equal(above.sh[:, :k], cloud.sh) and not above.sh[:, k:].any()


def test_reader_takes_properties_in_any_order_and_skips_extras(tmp_path):
    cloud = two_gaussians()
    names = ["extra", "rot_3", "rot_2", "rot_1", "rot_0", "scale_2", "scale_1", "scale_0", "opacity", "f_dc_2",
             "f_dc_1", "f_dc_0", "z", "y", "x", "red"]
    columns = {"x": cloud.positions[:, 0], "y": cloud.positions[:, 1], "z": cloud.positions[:, 2],
               "f_dc_0": cloud.sh_dc[:, 0], "f_dc_1": cloud.sh_dc[:, 1], "f_dc_2": cloud.sh_dc[:, 2],
               "opacity": cloud.opacity_logits, "extra": np.full(2, 7.0), "red": np.full(2, 9.0)}
    for a in range(3):
        columns[f"scale_{a}"] = cloud.log_scales[:, a]
    for a in range(4):
        columns[f"rot_{a}"] = cloud.rotations[:, a]
    body = np.stack([columns[n] for n in names], axis=1).astype("<f4").tobytes()
    header = ("ply\ncomment other tool\nformat binary_little_endian 1.0\nelement vertex 2\n"
              + "".join(f"property float {n}\n" for n in names) + "end_header\n")
    path = tmp_path / "other.ply"
    path.write_bytes(header.encode() + body)
    assert clouds_equal(io.read_splat_ply(path), cloud)


@pytest.mark.parametrize(
    "text,message",
    [
        ("plx\nend_header\n", "not a PLY file"),
        ("ply\nformat binary_little_endian 1.0\nelement vertex 1\n", "header never ends"),
        ("ply\nelement face 3\nend_header\n", "unsupported element face"),
        ("ply\nelement vertex 1\nproperty uchar red\nend_header\n", "property red is uchar, not float"),
        ("ply\nformat ascii 1.0\nend_header\n", 'unexpected header line "format ascii 1.0\\n"'),
        ("ply\nproperty float x\nend_header\n", "no vertex element"),
        ("ply\nelement vertex 1\nproperty float x\nend_header\n", "no property y"),
    ],
)
def test_reader_refuses_what_the_reference_refuses(tmp_path, text, message):
    path = tmp_path / "bad.ply"
    path.write_bytes(text.encode())
    with pytest.raises(io.SplatFileError, match=re.escape(message)):
        io.read_splat_ply(path, sh_degree=0)


def test_short_file_is_refused(tmp_path):
    cloud = two_gaussians()
    path = tmp_path / "short.ply"
    io.write_splat_ply(path, cloud)
    path.write_bytes(path.read_bytes()[:-4])
    with pytest.raises(io.SplatFileError, match="failed to fill whole buffer"):
        io.read_splat_ply(path)


def _euler(roll, pitch, yaw):
    """nalgebra Rotation3::from_euler_angles(roll, pitch, yaw) = Rz(yaw) Ry(pitch) Rx(roll)."""
    cr, sr, cp, sp, cy, sy = (math.cos(roll), math.sin(roll), math.cos(pitch), math.sin(pitch), math.cos(yaw),
                              math.sin(yaw))
    return np.array([[cy * cp, cy * sp * sr - sy * cr, cy * sp * cr + sy * sr],
                     [sy * cp, sy * sp * sr + cy * cr, sy * sp * cr - cy * sr],
                     [-sp, cp * sr, cp * cr]])


def test_cameras_json_round_trips(tmp_path):
    """cameras_json.rs:114-140."""
    camera = sb.PinholeCamera(_euler(0.1, 0.2, 0.3), np.array([1.5, -2.0, 3.25]), (400.0, 410.0), (146.5, 258.5),
                              294, 518)
    path = tmp_path / "cameras.json"
    io.write_cameras_json(path, [("frame_0001.png", camera)])
    back = io.read_cameras_json(path)
    assert len(back) == 1 and back[0][0] == "frame_0001.png"
    got = back[0][1]
    assert np.array_equal(got.rotation, camera.rotation) and np.array_equal(got.translation, camera.translation)
    assert tuple(got.focal) == (400.0, 410.0) and tuple(got.principal_point) == (146.5, 258.5)
    assert (got.width, got.height) == (294, 518)
    text = path.read_text()
    assert text.startswith('[\n  {"id": 0, "img_name": "frame_0001.png", "width": 294, "height": 518, '
                           '"position": [1.5, -2, 3.25], "rotation": [[')
    assert text.endswith('"fx": 400, "fy": 410, "cx": 146.5, "cy": 258.5}\n]\n')


def test_rust_float_display():
    assert [io.rust_display(v) for v in (400.0, -2.0, 0.1, 1e-7, 1e21, -0.0, 0.30000000000000004)] == [
        "400", "-2", "0.1", "0.0000001", "1000000000000000000000", "-0", "0.30000000000000004"]


@pytest.mark.parametrize(
    "text,message",
    [
        ("{}", "not a JSON array"),
        ('[{"img_name": "a"}]', 'has no "position"'),
        ('[{"img_name": 3}]', '"img_name" is not a string'),
        ('[{"img_name": "a", "position": [1, 2], "rotation": []}]', "expected 3 numbers"),
        ('[{"img_name": "a", "position": [1, 2, 3], "rotation": [[1, 0, 0]]}]', '"rotation" needs 3 rows'),
        ('[{"img_name": "a", "position": [1, 2, 3], "rotation": [[1,0,0],[0,1,0],[0,0,1]], "fx": 1, "fy": 1}]',
         'has no "cx"'),
    ],
)
def test_cameras_json_refusals(text, message):
    with pytest.raises(io.SplatFileError, match=message):
        io.parse_cameras_json(text, "cameras.json")


@pytest.mark.skipif(not (REFERENCE_EXAMPLE / "splat.ply").exists(), reason="the example scene was not fetched")
def test_reads_the_reference_example_files():
    """The example splat and cameras the reference ships (web/example)."""
    count, degree = io.read_splat_ply_header(REFERENCE_EXAMPLE / "splat.ply")
    cloud = io.read_splat_ply(REFERENCE_EXAMPLE / "splat.ply")
    assert len(cloud) == count > 0 and cloud.sh_degree == degree
    names, records = parse_ply((REFERENCE_EXAMPLE / "splat.ply").read_bytes())
    assert np.array_equal(cloud.positions[:, 0], records[:, names.index("x")])
    assert np.array_equal(cloud.rotations[:, 3], records[:, names.index("rot_3")])
    cameras = io.read_cameras_json(REFERENCE_EXAMPLE / "cameras.json")
    assert len(cameras) > 0
    for _, camera in cameras:
        assert camera.width > 0 and camera.height > 0
        assert np.allclose(camera.rotation @ camera.rotation.T, np.eye(3), atol=1e-5)


def test_training_view_composites_and_masks():
    """training_view_from_image (training_frames.rs:71-115) at the camera's size: colours
    blended onto the 128-grey background by alpha in integer arithmetic, foreground where
    alpha >= 128 (the reference's composites_shrinks_and_masks test without its resize)."""
    rgba = np.zeros((2, 3, 4), np.uint8)
    rgba[0, 0] = [255, 0, 0, 255]    # opaque red
    rgba[0, 1] = [0, 0, 255, 0]      # transparent: the hidden blue does not show
    rgba[0, 2] = [200, 100, 50, 128]  # half: (c 128 + 128 127) / 255, foreground
    rgba[1, :] = [10, 20, 30, 127]   # just below the foreground alpha
    camera = sb.PinholeCamera(np.eye(3), np.zeros(3), (10.0, 10.0), (1.0, 0.5), 3, 2)
    rgb, foreground = io.training_view_from_rgba8(rgba, camera)
    assert foreground.tolist() == [True, False, True, False, False, False]
    expect = lambda c, a: ((c * a + 128 * (255 - a)) // 255) / np.float32(255.0)  # noqa: E731
    assert np.array_equal(rgb[0], np.array([1.0, expect(0, 255), expect(0, 255)], np.float32))
    assert np.array_equal(rgb[1], np.full(3, np.float32(128) / np.float32(255), np.float32))
    assert np.array_equal(rgb[2], np.array([expect(200, 128), expect(100, 128), expect(50, 128)], np.float32))
    with pytest.raises(io.SplatFileError):
        io.training_view_from_rgba8(rgba, camera.with_image_size(4, 2))
    with pytest.raises(io.SplatFileError, match="no foreground"):
        io.training_view_from_rgba8(np.zeros((2, 3, 4), np.uint8), camera)


@pytest.mark.skipif(not (REFERENCE_EXAMPLE / "splat.ply").exists(), reason="the example scene was not fetched")
def test_reads_the_reference_example_run():
    """The example run as the reference's step timing loads it (examples/step_timing.rs:31-40)."""
    cloud, cameras, gt = io.read_fit_run(REFERENCE_EXAMPLE)
    assert len(cloud) == 222909 and cloud.sh_degree == 0 and len(cameras) == 6
    assert gt.shape == (6, 392 * 518, 4)
    assert np.all((gt[..., 3] == 0.0) | (gt[..., 3] == 1.0))
    assert np.all(gt[..., :3] <= gt[..., 3:4])
