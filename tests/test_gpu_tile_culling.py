"""Tile culling by the ellipse (SP_TILES_ELLIPSE) against the reference's rectangles
(SP_TILES_RECTANGLE) on the CUDA path, the same seeded scenes through the C ABI.

Bars:
  - every culled list is its rectangle list with entries removed, in the same order, and
    every removed (tile, Gaussian) pair has alpha below 1/255 at every pixel centre of the
    tile (checked in f64 from the projected records, with a 0.1 % margin);
  - images and per-pixel losses bit for bit; parameter gradients element-wise within twice
    the gradients' parity bar against the oracle (1e-4 relative + 4 float32 roundings of the
    gradient's rounding scale, 1e-2 of it in the covariance-chain slots, as
    tests/test_gpu_parity_full.py): both sides sum the same terms by float atomics in
    different orders; densify statistics within 1e-4 of their largest or 4 times the spread
    of two runs;
  - 20 training steps: every step's loss within 1e-5 relative.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import splat_b200 as sb
from helpers import camera_at_origin, make_rasterizer, random_cloud
from splat_b200 import scenes

pytestmark = pytest.mark.gpu

# The gradients' parity bar (tests/test_gpu_parity_full.py): 1e-4 relative plus 4 float32
# roundings of the rounding scale, whose covariance-chain slots (3-9) take 1e-2 of it.
RTOL = 1e-4
ROUNDINGS = 4.0 * 2.0 ** -24
CHAIN_SLOTS = slice(3, 10)
CHAIN_FLOOR = 1e-2


def cases():
    out = {
        "random600_80x48": (random_cloud(600, np.random.default_rng(7)), camera_at_origin(80, 48, 60.0)),
        "random3000_sh3_256x192": (random_cloud(3000, np.random.default_rng(9), sh_degree=3),
                                   camera_at_origin(256, 192, 180.0)),
        "random500_sh2_37x29": (random_cloud(500, np.random.default_rng(13), sh_degree=2),
                                camera_at_origin(37, 29, 30.0)),
    }
    s = scenes.config(2, scale=0.01)
    out["config2_5k_sh3_1024x768"] = (s.cloud, s.cameras[3])
    s = scenes.config(3, scale=0.002)
    base = s.cameras[0]
    out["config3_6k_sh3_2560x1440"] = (s.cloud, sb.PinholeCamera(
        base.rotation, base.translation, (base.focal[0] * 2560 / base.width, base.focal[1] * 2560 / base.width),
        (1280.0, 720.0), 2560, 1440))
    return out


CASES = cases()


def run(ctx, cloud, camera, culling, weights):
    rast, _, _ = make_rasterizer(ctx, cloud, camera, backward_mode=sb.SP_BWD_ATOMIC, tile_culling=culling)
    rast.encode_forward()
    meta = rast.read_intersections()
    _, gauss = rast.read_sorted_intersections()
    out = dict(count=int(meta.count), gauss=gauss, ranges=rast.read_tile_ranges().reshape(-1, 2),
               image=rast.read_image().rgbt,
               projected=rast.read_projected())
    rast.write_loss_gradient(weights)
    rast.encode_backward()
    out["gradients"] = rast.read_param_gradients()
    out["stats"] = rast.read_densify_stats()
    rast.close()
    return out


def max_alpha(projected, g: int, tile: int, camera) -> float:
    """The largest alpha of Gaussian g over the pixel centres of `tile` inside the image,
    in f64 (rasterize_forward.wgsl:52-62 without the 0.99 cap)."""
    tiles_x = (camera.width + 15) // 16
    tx, ty = tile % tiles_x, tile // tiles_x
    xs = np.arange(16 * tx, min(16 * tx + 16, camera.width), dtype=np.float64)
    ys = np.arange(16 * ty, min(16 * ty + 16, camera.height), dtype=np.float64)
    p = projected[g]
    dx = xs[None, :] - float(p["mean"][0])
    dy = ys[:, None] - float(p["mean"][1])
    a, b, c = (float(v) for v in p["conic"])
    power = -0.5 * (a * dx * dx + c * dy * dy) - b * dx * dy
    power = np.where(power > 0.0, -np.inf, power)  # the blend skips power > 0
    return float(np.max(float(p["opacity"]) * np.exp(power)))


@pytest.mark.parametrize("name", list(CASES))
def test_culled_lists_drop_only_pairs_that_never_blend(ctx, name):
    cloud, camera = CASES[name]
    weights = np.zeros(camera.width * camera.height * 4, np.float32)
    full = run(ctx, cloud, camera, sb.SP_TILES_RECTANGLE, weights)
    culled = run(ctx, cloud, camera, sb.SP_TILES_ELLIPSE, weights)
    assert 0 < culled["count"] < full["count"]
    dropped = 0
    for tile, ((s0, e0), (s1, e1)) in enumerate(zip(full["ranges"], culled["ranges"])):
        whole = full["gauss"][s0:e0]
        kept = culled["gauss"][s1:e1]
        keep = np.isin(whole, kept)
        assert np.array_equal(whole[keep], kept), f"{name}: tile {tile} is not a sub-list in order"
        for g in whole[~keep]:
            alpha = max_alpha(full["projected"], int(g), tile, camera)
            assert alpha < (1.0 / 255.0) * 0.999, f"{name}: tile {tile} dropped Gaussian {g} (alpha {alpha})"
            dropped += 1
    assert dropped == full["count"] - culled["count"]
    print(f"{name}: {full['count']} -> {culled['count']} intersections")


@pytest.mark.parametrize("name", list(CASES))
def test_culling_changes_no_result(ctx, name):
    cloud, camera = CASES[name]
    weights = np.random.default_rng(4).uniform(-1.0, 1.0, camera.width * camera.height * 4).astype(np.float32)
    full = run(ctx, cloud, camera, sb.SP_TILES_RECTANGLE, weights)
    again = run(ctx, cloud, camera, sb.SP_TILES_RECTANGLE, weights)
    culled = run(ctx, cloud, camera, sb.SP_TILES_ELLIPSE, weights)
    assert np.array_equal(culled["image"].view(np.uint32), full["image"].view(np.uint32)), f"{name}: image"
    stride = sb.param_stride(cloud.sh_degree)
    g_full = full["gradients"].reshape(-1, stride)
    g_culled = culled["gradients"].reshape(-1, stride)
    # Float atomics in another order on both sides: each within the parity bar of the oracle's
    # gradients, so the two within twice it, element by element. (A bar from the spread of
    # two runs is one sample of the atomics' order and does not bound the next.)
    packed = cloud.to_packed()
    cam = oracle.camera_of(camera)
    fwd = oracle.render(packed, cloud.sh_degree, cam)
    _, magnitudes = oracle.blend_backward_magnitudes(fwd["proj"], fwd["gauss"], fwd["slots"], fwd["ranges"], cam,
                                                     fwd["image"], fwd["contrib"], weights, fwd["capacity"])
    scale = oracle.gradient_error_scale(packed, cloud.sh_degree, cam, fwd, magnitudes).reshape(-1, stride)
    allowed = ROUNDINGS * scale
    allowed[:, CHAIN_SLOTS] = np.maximum(allowed[:, CHAIN_SLOTS], CHAIN_FLOOR * scale[:, CHAIN_SLOTS])
    bar = 2.0 * (RTOL * np.abs(g_full).astype(np.float64) + allowed)
    excess = np.abs(g_culled.astype(np.float64) - g_full) - bar
    assert np.all(excess <= 0.0), (name, np.argwhere(excess > 0.0)[:10].tolist())
    # Every gradient the rectangles' run gives is also the second run's within the same bar.
    assert np.all(np.abs(again["gradients"].reshape(-1, stride).astype(np.float64) - g_full) <= bar), name
    assert np.array_equal(culled["stats"][:, 1:3], full["stats"][:, 1:3])
    # The mean-gradient sums are norms of atomically summed gradients: the same bar.
    stat_spread = np.abs(again["stats"][:, 0] - full["stats"][:, 0]).max()
    stat_error = np.abs(culled["stats"][:, 0] - full["stats"][:, 0]).max()
    assert stat_error <= 4.0 * stat_spread + 1e-4 * np.abs(full["stats"][:, 0]).max() + 1e-9, name


def test_culling_rejects_the_deterministic_backward(ctx):
    cloud, camera = CASES["random600_80x48"]
    with pytest.raises(sb.SplatError):
        make_rasterizer(ctx, cloud, camera, backward_mode=sb.SP_BWD_DETERMINISTIC, tile_culling=sb.SP_TILES_ELLIPSE)


def test_training_losses_agree(ctx):
    """20 steps of config 0 (3 views), Adam fused: the same losses with either tile mode."""
    import torch

    s = scenes.config(0, scale=0.25)
    cams = s.cameras
    rng = np.random.default_rng(2)
    gt = rng.uniform(0.0, 1.0, (len(cams), cams[0].width * cams[0].height * 4)).astype(np.float32)
    gt[:, 3::4] = (gt[:, 3::4] > 0.5).astype(np.float32)
    losses = {}
    for culling in (sb.SP_TILES_RECTANGLE, sb.SP_TILES_ELLIPSE):
        params = torch.from_numpy(s.cloud.to_packed()).cuda()
        gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
        rast = sb.Rasterizer(ctx, params, len(s.cloud), cams[0].width, cams[0].height, gt_dev, len(cams),
                             sb.default_options(tile_culling=culling))
        adam = sb.Adam(ctx, params, rast, len(s.cloud), sb.LEARNING_RATES_3DGS, np.float32(sb.cameras_extent(cams)))
        losses[culling] = [rast.train_step(adam, cams[i % len(cams)], i % len(cams), sb.position_rate_factor(i, 20))[1]
                           .total for i in range(20)]
    a, b = np.array(losses[sb.SP_TILES_RECTANGLE]), np.array(losses[sb.SP_TILES_ELLIPSE])
    assert np.all(np.abs(a - b) <= 1e-5 * np.abs(a)), (a, b)
