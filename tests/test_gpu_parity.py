"""Parity of the CUDA path (through the C ABI) with the CPU oracle on seeded inputs.

Bars (the north star's):
  - projection depth, radius and tile rectangle, tile lists, sort order and tile ranges:
    bit-exact (the projection and the oracle share operation order and exp);
  - images: within 1e-4 absolute (premultiplied colours and transmittance lie in [0, 1]),
    with per-pixel contributor counts equal except at alpha/termination thresholds the
    hardware exp lands on the other side of (< 0.5 % of pixels);
  - gradients: |cuda - oracle| <= 1e-4 * max|oracle| + 1e-6 per parameter slot, over all
    Gaussians (fp32 sums in a different order);
  - Adam + clamp: bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import splat_b200 as sb
from helpers import camera_at_origin, make_rasterizer, random_cloud
from splat_b200 import scenes

pytestmark = pytest.mark.gpu

IMAGE_TOL = 1e-4
GRAD_REL_TOL = 1e-4


def scene_cases():
    rng = np.random.default_rng(7)
    cases = {
        "random600_80x48": (random_cloud(600, rng), camera_at_origin(80, 48, 60.0)),
        "random3000_sh3_256x192": (random_cloud(3000, np.random.default_rng(9), sh_degree=3),
                                   camera_at_origin(256, 192, 180.0)),
        # Ragged image sizes (partial tiles and partial 8 x 8 warp blocks) and SH 1, 2.
        "random800_sh1_100x70": (random_cloud(800, np.random.default_rng(12), sh_degree=1),
                                 camera_at_origin(100, 70, 70.0)),
        "random500_sh2_37x29": (random_cloud(500, np.random.default_rng(13), sh_degree=2),
                                camera_at_origin(37, 29, 30.0)),
    }
    s = scenes.config(0, scale=0.25)
    cases["config0_5k_256"] = (s.cloud, s.cameras[1])
    s = scenes.config(2, scale=0.01)
    cases["config2_5k_sh3_1024x768"] = (s.cloud, s.cameras[3])
    return cases


CASES = scene_cases()


def oracle_forward(cloud, camera, **kw):
    return oracle.render(cloud.to_packed(), cloud.sh_degree, oracle.camera_array(camera.uniform()), **kw)


@pytest.mark.parametrize("name", list(CASES))
def test_projection_bit_exact(ctx, name):
    cloud, camera = CASES[name]
    rast, _, _ = make_rasterizer(ctx, cloud, camera)
    rast.encode_forward()
    got = rast.read_projected()
    want = oracle_forward(cloud, camera)["proj"]
    for field in ("radius", "tile_min", "tile_max", "depth", "mean", "conic", "opacity", "color"):
        assert np.array_equal(got[field], want[field]), f"{name}: {field} differs"
    fwd = oracle_forward(cloud, camera)
    assert np.array_equal(rast.read_tile_offsets(), fwd["offsets"]), f"{name}: tile offsets differ"


@pytest.mark.parametrize("name", list(CASES))
def test_tile_lists_bit_exact(ctx, name):
    cloud, camera = CASES[name]
    rast, _, _ = make_rasterizer(ctx, cloud, camera)
    rast.encode_forward()
    meta = rast.read_intersections()
    keys, gauss = rast.read_sorted_intersections()
    want = oracle_forward(cloud, camera)
    assert meta.count == len(want["keys"]) and meta.overflow == 0
    assert np.array_equal(keys, want["keys"]), f"{name}: sorted keys differ"
    assert np.array_equal(gauss, want["gauss"]), f"{name}: sort order differs"
    assert np.array_equal(rast.read_tile_ranges(), want["ranges"]), f"{name}: tile ranges differ"


@pytest.mark.parametrize("key_mode,width,height", [(sb.SP_KEYS_REF20, 1920, 1080), (sb.SP_KEYS_FULL32, 1920, 1080),
                                                    (sb.SP_KEYS_REF20, 2560, 1440)])
def test_tile_lists_over_4096_tiles(ctx, key_mode, width, height):
    """1920 x 1080 has 8160 tiles, which the reference's 32-bit keys refuse
    (rasterizer.rs:188-192): REF20 order in compressed 32-bit keys (the frame's depth-key
    range), FULL32 in 64-bit keys; 2560 x 1440 (14400 tiles) in the reference's layout in 64
    bits. The same order as the oracle's either way, read back in the reference's layout."""
    s = scenes.config(3, scale=0.002)
    cloud = s.cloud
    base = s.cameras[0]
    camera = sb.PinholeCamera(base.rotation, base.translation,
                              (base.focal[0] * width / base.width, base.focal[1] * width / base.width),
                              (width / 2.0, height / 2.0), width, height)
    rast, _, _ = make_rasterizer(ctx, cloud, camera, key_mode=key_mode)
    rast.encode_forward()
    keys, gauss = rast.read_sorted_intersections()
    want = oracle_forward(cloud, camera, key_mode=key_mode)
    assert len(keys) > 1000
    assert np.array_equal(keys, want["keys"]) and np.array_equal(gauss, want["gauss"])
    assert np.array_equal(rast.read_tile_ranges(), want["ranges"])


@pytest.mark.parametrize("name", list(CASES))
def test_image_matches(ctx, name):
    cloud, camera = CASES[name]
    rast, _, _ = make_rasterizer(ctx, cloud, camera)
    rast.encode_forward()
    image = rast.read_image().rgbt
    contrib = rast.read_contributions()
    want = oracle_forward(cloud, camera)
    worst = float(np.max(np.abs(image - want["image"])))
    assert worst < IMAGE_TOL, f"{name}: largest pixel difference {worst}"
    mismatched = float(np.mean(contrib != want["contrib"]))
    assert mismatched < 5e-3, f"{name}: {mismatched:.4%} of contributor counts differ"


def _falloff_items(rng, count):
    """Blend records (words [0], [1]) and pixels: conics from round to needle-thin (the
    off-diagonal up to 0.999 of its bound, where the three terms of the power cancel), pixels
    from the centre out to powers of about -100, integer pixel coordinates as the kernels use."""
    a = np.exp(rng.uniform(np.log(1e-4), np.log(20.0), count)).astype(np.float32)
    c = np.exp(rng.uniform(np.log(1e-4), np.log(20.0), count)).astype(np.float32)
    b = (rng.uniform(-0.999, 0.999, count) * np.sqrt(a * c)).astype(np.float32)
    mean = rng.uniform(0.0, 2048.0, (count, 2)).astype(np.float32)
    level = np.where(rng.random(count) < 0.5, 20.0, 200.0)  # |power| up to about level / 2
    px = np.floor(mean[:, 0] + rng.uniform(-1, 1, count) * np.minimum(np.sqrt(level / a), 3000)).astype(np.float32)
    py0 = np.floor(mean[:, 1] + rng.uniform(-1, 1, count) * np.minimum(np.sqrt(level / c), 3000)).astype(np.float32)
    items = np.zeros((count, 12), np.float32)
    items[:, 0:2] = mean
    items[:, 2] = a
    items[:, 3] = b
    items[:, 4] = c
    items[:, 5] = 0.5  # opacity (not read)
    items[:, 8] = px
    items[:, 9] = py0
    items[:, 10] = py0 + 4.0  # the lane's second pixel, four rows below
    return items


def _oracle_powers(items):
    """The power in the oracle's (and rasterize_forward.wgsl:60-63's) operation order, one
    float32 rounding per operation: -0.5 (a d0 d0 + c d1 d1) - b d0 d1, d = mean - pixel."""
    f = np.float32
    out = np.empty((len(items), 2), np.float32)
    d0 = items[:, 0] - items[:, 8]
    for k, row in enumerate((9, 10)):
        d1 = items[:, 1] - items[:, row]
        quad = (items[:, 2] * d0) * d0 + (items[:, 4] * d1) * d1
        out[:, k] = f(-0.5) * quad - (items[:, 3] * d0) * d1
    return out


def test_blend_falloff_power_bit_exact(ctx):
    """The blend kernels' falloff power equals the oracle's bit for bit, cancelling cases
    included: the take (alpha >= 1/255) and clamp (0.99) decisions rest on it. (Packed f32x2
    forms of the same operations fail this test: the compiler fuses them into FFMA2.)"""
    import ctypes

    import torch
    from splat_b200 import _lib

    items = _falloff_items(np.random.default_rng(61), 1 << 20)
    want = _oracle_powers(items)
    d_items = torch.from_numpy(items).cuda()
    d_powers = torch.empty((len(items), 2), dtype=torch.float32, device="cuda")
    lib = _lib.load()
    status = lib.sp_debug_falloff_powers(ctypes.c_void_p(d_items.data_ptr()), len(items),
                                         ctypes.c_void_p(d_powers.data_ptr()),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == _lib.SP_OK
    got = d_powers.cpu().numpy()
    assert np.all(np.isfinite(want)) and 0.2 < np.mean((want > -10.0) & (want <= 0.0)) < 0.9
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), int(np.sum(got != want))


def test_divisions_are_ieee_quotients(ctx):
    """The kernels' divisions without the IEEE division instruction sequence
    (csrc/exact_div.cuh) equal IEEE float32 division bit for bit (NaN for NaN): Adam's by
    the bias corrections through a double-precision reciprocal and by sqrt(v_hat) + epsilon
    through a double-precision Newton-Raphson reciprocal, and the projection's div_rn for
    any divisor. Random dividends over every exponent; the bias corrections of the first
    20,000 steps; divisors from 1e-15 to 1e19, powers of two, infinity; and for div_rn
    random divisors over every bit pattern (both signs, zeros, subnormals, above 2^126,
    infinities, NaN)."""
    import ctypes

    import torch
    from splat_b200 import _lib

    rng = np.random.default_rng(67)
    n = 1 << 23
    x = rng.integers(0, 1 << 32, size=n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    t = np.arange(1, 20_001, dtype=np.float32)
    corrections = np.concatenate([np.float32(1) - np.power(np.float32(0.9), t),
                                  np.float32(1) - np.power(np.float32(0.999), t)]).astype(np.float32)
    y = np.empty(n, np.float32)
    half, quarter = n // 2, n // 4
    y[:half] = rng.choice(corrections, half)
    y[half:] = np.exp(rng.uniform(np.log(1e-15), np.log(1e19), n - half)).astype(np.float32)
    y[half:half + 64] = np.float32(2.0) ** np.arange(-48, 16, dtype=np.float32)
    # A quarter of the divisors over every bit pattern, then the edges by name.
    y[half + quarter:] = rng.integers(0, 1 << 32, size=n - half - quarter, dtype=np.uint64).astype(np.uint32).view(
        np.float32)
    edges = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1.1754942e-38, 1.1754944e-38,
                      -1.1754944e-38, 8.507059e37, 8.5070597e37, -8.5070597e37, 3.4028235e38, -3.4028235e38,
                      -1.0, -0.5, -3.0], np.float32)
    y[-64:-64 + len(edges)] = edges
    y[-16:] = np.inf
    d_x, d_y = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    out = torch.empty((n, 3), dtype=torch.float32, device="cuda")
    lib = _lib.load()
    status = lib.sp_debug_adam_quotients(ctypes.c_void_p(d_x.data_ptr()), ctypes.c_void_p(d_y.data_ptr()), n,
                                         ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == _lib.SP_OK
    got = out.cpu().numpy()
    with np.errstate(all="ignore"):
        want = x / y
    bias = (y > 0) & (y <= 1)
    update = ((y >= np.float32(2.0) ** -126) & (y <= np.float32(2.0) ** 126)) | (y == np.inf)

    def same(a, b):
        nan = np.isnan(b)
        return np.array_equal(np.isnan(a), nan) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))

    def differ(a, b):
        return int(np.sum(a.view(np.uint32) != b.view(np.uint32)))

    assert bias.sum() > half and update.sum() > half
    assert same(got[bias, 0], want[bias]), differ(got[bias, 0], want[bias])
    assert same(got[update, 1], want[update]), differ(got[update, 1], want[update])
    assert (~update).sum() > n // 16  # div_rn's fallback is exercised
    assert same(got[:, 2], want), differ(got[:, 2], want)


def test_blend_work_counts(ctx):
    """sp_count_blend_work (roofline accounting): the pairs blended, replayed and visited nest,
    and the pairs replayed are the sum of the contributor counts the forward wrote."""
    cloud, camera = CASES["config2_5k_sh3_1024x768"]
    rast, _, _ = make_rasterizer(ctx, cloud, camera)
    rast.encode_forward()
    visited, replayed, taken = rast.count_blend_work()
    assert 0 < taken <= replayed <= visited
    assert replayed == int(rast.read_contributions().astype(np.int64).sum())


def test_loss_matches(ctx):
    rng = np.random.default_rng(5)
    width, height = 40, 24
    pixels = width * height
    mask = (rng.random(pixels) < 0.6).astype(np.float32)
    gt = np.concatenate([rng.random((pixels, 3)).astype(np.float32) * mask[:, None], mask[:, None]], axis=1).reshape(-1)
    rgbt = np.concatenate([rng.random((pixels, 3)), rng.uniform(0.1, 0.9, (pixels, 1))], axis=1).astype(np.float32).reshape(-1)
    cloud = random_cloud(4, rng)
    rast, _, _ = make_rasterizer(ctx, cloud, camera_at_origin(width, height, 40.0), ground_truth=gt)
    rast.write_image(rgbt)
    rast.encode_loss(0)
    got_grad, got_loss = rast.read_loss_gradient(), rast.read_pixel_loss()
    partials = oracle.ssim(rgbt, gt, width, height)
    want_grad, want_loss = oracle.loss(rgbt, gt, partials, width, height)
    assert np.max(np.abs(got_loss - want_loss)) < 1e-5
    scale = np.max(np.abs(want_grad))
    assert np.max(np.abs(got_grad - want_grad)) <= 1e-4 * scale
    terms = rast.read_loss()
    ref = sb.LossTerms.from_pixel_loss(want_loss)
    assert abs(terms.total - ref.total) < 1e-6 and abs(terms.dssim - ref.dssim) < 1e-6


# The rotation slots (6-9) go through d_q = (d_unit - q <q, d_unit>) / |q| over differences
# of near-equal products (project_backward.wgsl:182-188), which amplifies the last-bit
# differences of the fp32 blend sums (summed in another order) by up to ~100x on a few
# Gaussians; their bar is 1e-3 of the slot's largest gradient. Both halves of the chain
# are pinned tighter on their own: the per-Gaussian blend sums within 1e-4
# (test_blend_sums_match) and the projection backward bit-exact given the same blend sums
# (test_projection_backward_bit_exact).
ROTATION_REL_TOL = 1e-3


def _check_gradients(name, got, want, stride):
    got = got.reshape(-1, stride)
    want = want.reshape(-1, stride)
    for slot in range(stride):
        tol = ROTATION_REL_TOL if 6 <= slot < 10 else GRAD_REL_TOL
        scale = float(np.max(np.abs(want[:, slot])))
        err = float(np.max(np.abs(got[:, slot] - want[:, slot])))
        assert err <= tol * scale + 1e-6, f"{name}: slot {slot} error {err:.3e} vs scale {scale:.3e}"


def _oracle_blend_sums(cloud, fwd, slot_gradients):
    """Per Gaussian, the sum of its slots in slot order (project_backward.wgsl:38-55)."""
    slots = slot_gradients.reshape(-1, 10)
    out = np.zeros((len(cloud), 10), np.float32)
    proj = fwd["proj"]
    for g in np.nonzero(proj["radius"])[0]:
        span = proj["tile_max"][g].astype(np.int64) - proj["tile_min"][g].astype(np.int64)
        o = int(fwd["offsets"][g])
        for row in slots[o : o + int(span[0] * span[1])]:
            out[g] += row
    return out


@pytest.mark.parametrize("mode", [sb.SP_BWD_DETERMINISTIC, sb.SP_BWD_ATOMIC])
@pytest.mark.parametrize("name", ["random600_80x48", "config2_5k_sh3_1024x768"])
def test_blend_sums_match(ctx, name, mode):
    cloud, camera = CASES[name]
    weights = np.random.default_rng(11).uniform(-1.0, 1.0, camera.width * camera.height * 4).astype(np.float32)
    rast, _, _ = make_rasterizer(ctx, cloud, camera, backward_mode=mode)
    rast.encode_forward()
    rast.write_loss_gradient(weights)
    rast.encode_backward()
    got = rast.read_gaussian_blend_gradients()
    cam = oracle.camera_array(camera.uniform())
    packed = cloud.to_packed()
    fwd = oracle.render(packed, cloud.sh_degree, cam)
    want = _oracle_blend_sums(cloud, fwd, oracle.backward(packed, cloud.sh_degree, cam, fwd, weights)["slot_gradients"])
    for c in range(9):
        scale = float(np.max(np.abs(want[:, c])))
        err = float(np.max(np.abs(got[:, c] - want[:, c])))
        assert err <= GRAD_REL_TOL * scale + 1e-7, f"{name}: blend sum {c} error {err:.3e} vs scale {scale:.3e}"


@pytest.mark.parametrize("name", list(CASES))
def test_projection_backward_bit_exact(ctx, name):
    """Given the same per-Gaussian blend sums, the CUDA projection backward (compiled
    without FMA contraction) reproduces the oracle's parameter gradients bit for bit."""
    cloud, camera = CASES[name]
    weights = np.random.default_rng(13).uniform(-1.0, 1.0, camera.width * camera.height * 4).astype(np.float32)
    rast, _, _ = make_rasterizer(ctx, cloud, camera, backward_mode=sb.SP_BWD_ATOMIC)
    rast.encode_forward()
    rast.write_loss_gradient(weights)
    rast.encode_backward()
    got = rast.read_param_gradients()
    sums = rast.read_gaussian_blend_gradients()
    cam = oracle.camera_array(camera.uniform())
    packed = cloud.to_packed()
    fwd = oracle.render(packed, cloud.sh_degree, cam)
    count = int(fwd["meta"]["count"])
    slots = np.zeros((max(count, 1), 10), np.float32)
    for g in np.nonzero(fwd["proj"]["radius"])[0]:
        slots[int(fwd["offsets"][g])] = sums[g]  # the whole sum in the Gaussian's first slot
    want, _, _ = oracle.project_backward(packed, cloud.sh_degree, cam, fwd["proj"], fwd["offsets"], slots.reshape(-1),
                                         count)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("mode", [sb.SP_BWD_DETERMINISTIC, sb.SP_BWD_ATOMIC])
@pytest.mark.parametrize("name", list(CASES))
def test_backward_matches(ctx, name, mode):
    cloud, camera = CASES[name]
    rng = np.random.default_rng(11)
    weights = rng.uniform(-1.0, 1.0, camera.width * camera.height * 4).astype(np.float32)
    rast, _, _ = make_rasterizer(ctx, cloud, camera, backward_mode=mode)
    rast.encode_forward()
    rast.write_loss_gradient(weights)
    rast.encode_backward()
    got = rast.read_param_gradients()
    got_camera = np.ctypeslib.as_array(rast.read_camera_gradient().world_to_camera_rotation_rows).reshape(-1)
    cam = oracle.camera_array(camera.uniform())
    packed = cloud.to_packed()
    fwd = oracle.render(packed, cloud.sh_degree, cam)
    bwd = oracle.backward(packed, cloud.sh_degree, cam, fwd, weights)
    _check_gradients(name, got, bwd["param_gradients"], sb.param_stride(cloud.sh_degree))
    cg = rast.read_camera_gradient()
    got_cam = np.array(
        [cg.world_to_camera_rotation_rows[r][c] for r in range(3) for c in range(3)]
        + list(cg.world_to_camera_translation) + list(cg.focal), np.float32)
    want_cam = bwd["camera_gradient"]
    assert np.max(np.abs(got_cam - want_cam)) <= 1e-3 * np.max(np.abs(want_cam)) + 1e-6, (got_cam, want_cam)
    stats = rast.read_densify_stats()
    assert np.array_equal(stats[:, 1], bwd["stats"][:, 1]) and np.array_equal(stats[:, 2], bwd["stats"][:, 2])
    assert np.max(np.abs(stats[:, 0] - bwd["stats"][:, 0])) <= 1e-3 * np.max(bwd["stats"][:, 0]) + 1e-6
    del got_camera


def test_deterministic_backward_is_bit_stable(ctx):
    cloud, camera = CASES["config0_5k_256"]
    weights = np.random.default_rng(3).uniform(-1, 1, camera.width * camera.height * 4).astype(np.float32)
    rast, _, _ = make_rasterizer(ctx, cloud, camera, backward_mode=sb.SP_BWD_DETERMINISTIC)
    runs = []
    for _ in range(2):
        rast.encode_forward()
        rast.write_loss_gradient(weights)
        rast.encode_backward()
        runs.append(rast.read_param_gradients())
    assert np.array_equal(runs[0], runs[1])


@pytest.mark.parametrize("sh_degree", [0, 3])
def test_adam_bit_exact(ctx, sh_degree):
    import torch

    rng = np.random.default_rng(21)
    n = 1037
    stride = sb.param_stride(sh_degree)
    params = rng.normal(0, 1, n * stride).astype(np.float32)
    params.reshape(n, stride)[:, 3:6] = rng.normal(-4, 1.5, (n, 3))
    grads = rng.normal(0, 1e-3, n * stride).astype(np.float32)
    p_dev = torch.from_numpy(params.copy()).cuda()
    g_dev = torch.from_numpy(grads).cuda()
    rates = sb.LEARNING_RATES_3DGS
    extent = 3.3
    adam = sb.Adam(ctx, p_dev, g_dev, n, rates, extent, sh_degree=sh_degree)
    p_ref, m_ref, v_ref = params.copy(), np.zeros_like(params), np.zeros_like(params)
    for step in range(1, 4):
        factor = sb.position_rate_factor(step - 1, 10)
        adam.encode_step(factor)
        lr = oracle.learning_rates_by_slot(rates.to_c(), np.float32(extent) * np.float32(factor), stride)
        oracle.adam_step(p_ref, grads, m_ref, v_ref, stride, lr, step, float(np.log(np.float32(0.02 * np.float32(extent)))),
                         float(np.log(np.float32(10.0))))
    ctx.sync()
    m, v = adam.read_moments()
    assert np.array_equal(m, m_ref) and np.array_equal(v, v_ref)
    assert np.array_equal(p_dev.cpu().numpy(), p_ref)


def test_overflow_is_reported(ctx):
    """rasterizer.rs:536-544 panics; the C ABI returns SP_ERR_OVERFLOW."""
    cloud, camera = CASES["config0_5k_256"]
    rast, _, _ = make_rasterizer(ctx, cloud, camera, intersections_per_gaussian=1)
    rast.encode_forward()
    with pytest.raises(sb.SplatError) as err:
        rast.read_intersections()
    assert err.value.status == 3
    meta = rast.read_intersections_unchecked()
    assert meta.overflow == 1 and meta.count == meta.capacity == len(cloud)
    # The capped list is still the oracle's prefix order.
    keys, gauss = rast.read_sorted_intersections()
    want = oracle_forward(cloud, camera, capacity=len(cloud))
    assert np.array_equal(keys, want["keys"]) and np.array_equal(gauss, want["gauss"])


def test_everything_culled(ctx):
    cloud = random_cloud(50, np.random.default_rng(1))
    cloud.positions[:, 2] *= -1.0  # behind the camera
    camera = camera_at_origin(40, 30, 30.0)
    rast, _, _ = make_rasterizer(ctx, cloud, camera)
    rast.encode_forward()
    assert rast.read_intersections().count == 0
    img = rast.read_image().rgbt.reshape(-1, 4)
    assert np.all(img[:, :3] == 0.0) and np.all(img[:, 3] == 1.0)
    rast.write_loss_gradient(np.ones(40 * 30 * 4, np.float32))
    rast.encode_backward()
    assert np.all(rast.read_param_gradients() == 0.0)


@pytest.mark.parametrize("sh_degree", [0, 3])
def test_fused_backward_adam_equals_backward_then_adam(ctx, sh_degree):
    """sp_backward_adam against sp_backward then sp_adam_step (deterministic backward, 3
    steps): parameters, both moments, camera gradient and densify statistics bit for bit."""
    import torch

    rng = np.random.default_rng(5 + sh_degree)
    cloud = random_cloud(3000, rng, sh_degree=sh_degree)
    camera = camera_at_origin(160, 120, 120.0)
    gt = np.random.default_rng(2).uniform(0, 1, 160 * 120 * 4).astype(np.float32)
    runs = []
    for fused in (False, True):
        rast, params, _ = make_rasterizer(ctx, cloud, camera, ground_truth=gt,
                                          backward_mode=sb.SP_BWD_DETERMINISTIC)
        adam = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, 2.5, sh_degree=sh_degree)
        cams = []
        for step in range(3):
            factor = sb.position_rate_factor(step, 10)
            rast.encode_forward()
            rast.encode_loss(0)
            if fused:
                rast.encode_backward_adam(adam, factor)
            else:
                rast.encode_backward()
                adam.encode_step(factor)
            cams.append(bytes(rast.read_camera_gradient()))
        m, v = adam.read_moments()
        runs.append((params.cpu().numpy().copy(), m, v, cams, rast.read_densify_stats().copy()))
        assert adam.steps_taken() == 3
        del adam, rast
    for a, b in zip(runs[0], runs[1]):
        if isinstance(a, list):
            assert a == b
        else:
            assert np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def test_fused_backward_adam_rejects_foreign_state(ctx):
    import torch

    cloud = random_cloud(200, np.random.default_rng(3))
    camera = camera_at_origin(64, 48, 50.0)
    rast, params, _ = make_rasterizer(ctx, cloud, camera)
    other = torch.zeros_like(params)
    adam = sb.Adam(ctx, other, rast, len(cloud), sb.LEARNING_RATES_3DGS, 2.5)
    rast.encode_forward()
    rast.encode_loss(0)
    with pytest.raises(sb.SplatError) as err:
        rast.encode_backward_adam(adam, 1.0)
    assert err.value.status == sb._lib.SP_ERR_INVALID


def test_context_enqueues_on_the_current_torch_stream():
    """The library's work orders with torch's: on torch's default stream (handle 0) the
    context enqueues on the legacy default stream, on any other stream on that stream, so
    CUDA events, tensor copies and NCCL collectives on it see the library's work."""
    import torch

    assert torch.cuda.current_stream(0).cuda_stream == 0
    ctx = sb.Context(0)
    assert ctx.stream == sb.rasterizer.CUDA_STREAM_LEGACY
    side = torch.cuda.Stream(0)
    with torch.cuda.stream(side):
        other = sb.Context(0)
        assert other.stream == side.cuda_stream
    # A torch event pair brackets the library's work: a forward of config 0 takes time.
    cloud, camera = CASES["config0_5k_256"]
    rast, _, _ = make_rasterizer(ctx, cloud, camera)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(20):
        rast.encode_forward()
    stop.record()
    stop.synchronize()
    # Without the ordering the pair would close before the forwards ran.
    assert ctx.lib.sp_context_sync(ctx.handle) == 0
    image = rast.read_image().rgbt
    assert np.isfinite(image).all()
    assert start.elapsed_time(stop) > 0.01
