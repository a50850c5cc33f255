"""Parity at the benchmark's full sizes, on the path the benchmark times.

Cases:
  - config 2 (500k Gaussians, SH degree 3, 1024 x 768), one view: the rectangle lists
    (projection, tile offsets, keys, sort order, ranges) bit-exact; then the benchmark's own
    options (tile culling by the ellipse, atomic backward) against the oracle: image, loss,
    parameter and camera gradients, densify statistics;
  - config 3 (3M Gaussians, SH degree 3, 1920 x 1080, 8160 tiles: beyond the reference's
    4096), one camera: keys, order and ranges bit-exact, image;
  - the reference's own example scene (instantsplat-rs/web/example: 222,909 SH-degree-0
    Gaussians, 392 x 518, its PNG targets), one training step with the benchmark's options.

The chain is checked stage by stage, each stage against the oracle on the same inputs:
  1. forward (projection, binning, sort, blend) against the oracle's own forward;
  2. loss (SSIM, L1, alpha): the oracle's loss of the image the GPU rendered;
  3. backward (blend backward, projection backward): the oracle's backward from the GPU's
     image, contributor counts and loss gradient;
and end to end by the example scene's training step.

Bars:
  - tile lists, sort order, tile ranges, projected fields: bit-exact;
  - image, per channel: |cuda - oracle| <= 1e-4 |oracle| + 1e-6 on every pixel whose
    contributor count agrees with the oracle's. The decisions that depend on alpha (the 1/255
    take test, the 0.99 clamp) are made on the exact falloff power against per-Gaussian
    thresholds and agree everywhere; the termination test (transmittance below 1e-4) reads the
    blended transmittance, which the hardware exp2 leaves a few roundings from the oracle's,
    so on a few pixels (at most 1e-4 of them) one more or one fewer Gaussian is blended: there
    the difference is that Gaussian's share, below 1e-4 x (1 + largest colour);
  - loss gradient: 1e-4 relative + 1e-3 of its largest; loss terms: 1e-4 relative (the GPU
    sums the SSIM window separably, the oracle tap by tap: the window variances, E[x^2] - mu^2,
    cancel, and the SSIM gradient divides by them);
  - parameter gradients, element-wise: |cuda - oracle| <= 1e-4 |oracle| + 4 x 2^-24 x S,
    where S is the gradient's rounding scale (oracle.gradient_error_scale: the sum over the
    nine blend sums of |d gradient / d blend sum| times that blend sum's magnitude, the sum
    over its pixels of the magnitude of everything its term is computed from, times the
    pixel's contributor count; or_blend_backward_magnitudes). The GPU sums each Gaussian's
    per-pixel terms in another order than the oracle (warp trees and atomics against the
    reference's slot order), rounds its exp differently and recovers the transmittance by
    a reciprocal; each moves a term by a few float32 roundings of that scale. Where terms
    cancel (|gradient| << S) a relative bar alone cannot hold for any reordering of float32
    sums. The log-scale and rotation slots (3-9) add a floor of 1e-2 x S: they come out of
    dL/dSigma through the covariance and quaternion chain, whose own terms cancel (a
    near-isotropic Gaussian's rotation gradient is zero up to rounding);
  - camera gradient (14 floats): element-wise 1e-4 relative;
  - densify statistics: visible counts and radii bit-exact;
  - one training step (example scene): parameters equal to the oracle's step within what
    Adam's first update makes of the two end-to-end gradients (it moves a parameter by its
    rate times g / (|g| + 1e-15): a sign, except for gradients near 1e-15) plus the update's
    rounding (4 ulp of the parameter + 1e-6 of the rate), and within twice the rate where the
    oracle's gradient is within its rounding bar of zero (its sign is rounding); opposite signs
    elsewhere on at most 1e-3 of the parameters.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import splat_b200 as sb
from helpers import make_rasterizer
from splat_b200 import io as splat_io
from splat_b200 import scenes

pytestmark = pytest.mark.gpu

RTOL = 1e-4
EPS = 2.0 ** -24
ROUNDINGS = 4.0  # measured at most 0.04 (config 2: 0.01; the example scene: 0.034)
# Log-scale and rotation slots: their gradients come out of dL/dSigma through the covariance
# and quaternion chain, whose own terms cancel (for a near-isotropic Gaussian the rotation
# gradient is zero up to rounding): a floor of 1e-2 of the scale (measured at most 3.3e-3).
CHAIN_SLOTS = range(3, 10)
CHAIN_FLOOR = 1e-2
IMAGE_FLOOR = 1e-6
LOSS_GRADIENT_FLOOR = 1e-3  # of the largest loss gradient (measured at most 2.6e-4)
LOSS_TERMS_RTOL = 1e-4
THRESHOLD_PIXELS = 1e-4  # largest fraction of pixels blended past the other side's termination
BENCH_OPTIONS = dict(backward_mode=sb.SP_BWD_ATOMIC, tile_culling=sb.SP_TILES_ELLIPSE)


def _masked_target(image: np.ndarray) -> np.ndarray:
    """The benchmark's target from a render: rgb x mask, mask = coverage > 0.5."""
    rgbt = image.reshape(-1, 4)
    mask = ((1.0 - rgbt[:, 3]) > 0.5).astype(np.float32)
    return np.concatenate([rgbt[:, :3] * mask[:, None], mask[:, None]], axis=1).reshape(-1).astype(np.float32)


class Reference:
    """The oracle's forward of one view, its loss and backward on given inputs."""

    def __init__(self, cloud, camera, gt: np.ndarray):
        self.cloud, self.camera, self.gt = cloud, camera, gt
        self.packed = cloud.to_packed()
        self.cam = oracle.camera_of(camera)
        self.fwd = oracle.render(self.packed, cloud.sh_degree, self.cam)

    def loss(self, image):
        partials = oracle.ssim(image, self.gt, self.camera.width, self.camera.height)
        return oracle.loss(image, self.gt, partials, self.camera.width, self.camera.height)

    def backward(self, image, contributions, loss_gradient):
        """Parameter and camera gradients, densify statistics and the gradients' rounding scale."""
        f = self.fwd
        slots, magnitudes = oracle.blend_backward_magnitudes(f["proj"], f["gauss"], f["slots"], f["ranges"], self.cam,
                                                             image, contributions, loss_gradient, f["capacity"])
        count = int(f["meta"]["count"])
        gradients, camera, stats = oracle.project_backward(self.packed, self.cloud.sh_degree, self.cam, f["proj"],
                                                           f["offsets"], slots, count)
        scale = oracle.gradient_error_scale(self.packed, self.cloud.sh_degree, self.cam, f, magnitudes)
        return gradients, camera, stats, scale


def check_image(name, image, contributions, ref: Reference):
    want = ref.fwd["image"].reshape(-1, 4)
    got = image.reshape(-1, 4)
    agree = contributions == ref.fwd["contrib"]
    diff = np.abs(got - want)
    bar = RTOL * np.abs(want) + IMAGE_FLOOR
    worst = float(np.max(diff[agree] - bar[agree])) if agree.any() else 0.0
    assert worst <= 0.0, f"{name}: pixel error above 1e-4 relative + 1e-6 by {worst:.3e}"
    others = ~agree
    assert others.mean() <= THRESHOLD_PIXELS, f"{name}: {others.mean():.2e} of contributor counts differ"
    if others.any():
        colour = float(np.max(ref.fwd["proj"]["color"]))
        assert float(diff[others].max()) <= 1e-4 * (1.0 + colour), f"{name}: threshold pixel error"
    return {"max_relative": float(np.max(diff[agree] / (np.abs(want[agree]) + IMAGE_FLOOR))),
            "threshold_pixels": int(others.sum())}


def check_gradients(name, got, want, scale, stride, failures):
    got = got.reshape(-1, stride).astype(np.float64)
    want = want.reshape(-1, stride).astype(np.float64)
    excess = np.abs(got - want) - RTOL * np.abs(want)
    allowed = ROUNDINGS * EPS * scale
    allowed[:, CHAIN_SLOTS.start:CHAIN_SLOTS.stop] = np.maximum(allowed[:, CHAIN_SLOTS.start:CHAIN_SLOTS.stop],
                                                                CHAIN_FLOOR * scale[:, CHAIN_SLOTS.start:CHAIN_SLOTS.stop])
    bad = excess > allowed
    others = np.ones(stride, bool)
    others[CHAIN_SLOTS.start:CHAIN_SLOTS.stop] = False
    ratio = float(np.max(excess[:, others] / np.maximum(EPS * scale[:, others], 1e-300)))
    chain = float(np.max(excess[:, ~others] / np.maximum(scale[:, ~others], 1e-300)))
    if bad.any():
        detail = [(int(g), int(k), float(got[g, k]), float(want[g, k]), float(scale[g, k]))
                  for g, k in np.argwhere(bad)[:30]]
        failures.append(f"{name}: {int(bad.sum())} gradients outside 1e-4 relative + {ROUNDINGS:g} roundings (worst "
                        f"{ratio:.1f} roundings; (Gaussian, slot, cuda, oracle, scale): {detail})")
    return {"worst_roundings": ratio, "worst_chain_fraction_of_scale": chain,
            "within_1e-4_relative": float(np.mean(excess <= 0.0)), "elements": int(got.size)}


def check_camera_gradient(name, rast, want, failures):
    cg = rast.read_camera_gradient()
    got = np.array([cg.world_to_camera_rotation_rows[r][c] for r in range(3) for c in range(3)]
                   + list(cg.world_to_camera_translation) + list(cg.focal), np.float64)
    want = want.astype(np.float64)
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
    if not np.all(rel <= RTOL):
        failures.append(f"{name}: camera gradient relative errors {rel}")
    return float(rel.max())


def run_bench_path(ctx, name, ref: Reference):
    """The benchmark's options through the C ABI, stage by stage against the oracle (module
    docstring). Every stage is checked; the failures are reported together with the
    per-stage statistics."""
    failures = []
    camera = ref.camera
    rast, params, gt = make_rasterizer(ctx, ref.cloud, camera, ground_truth=ref.gt, **BENCH_OPTIONS)
    rast.encode_forward()
    image = rast.read_image().rgbt
    # Contributor counts are list indices, which the culled lists shorten: they are compared on
    # the reference's rectangle lists, whose image must be the culled one bit for bit.
    rect, _, _ = make_rasterizer(ctx, ref.cloud, camera, ground_truth=ref.gt, backward_mode=sb.SP_BWD_ATOMIC)
    rect.encode_forward()
    assert np.array_equal(rect.read_image().rgbt, image), f"{name}: the culled image differs from the rectangles'"
    contributions = rect.read_contributions()
    stats = {"image": check_image(name, image, contributions, ref)}
    rect.close()

    rast.encode_loss(0)
    lg = rast.read_loss_gradient()
    want_lg, want_pixel_loss = ref.loss(image)
    largest = float(np.abs(want_lg).max())
    err = np.abs(lg - want_lg)
    outside = err > RTOL * np.abs(want_lg) + LOSS_GRADIENT_FLOOR * largest
    stats["loss_gradient"] = {"max_error_of_largest": float(err.max() / largest),
                              "within_1e-4_relative": float(np.mean(err <= RTOL * np.abs(want_lg)))}
    if outside.any():
        failures.append(f"{name}: loss gradient: {int(outside.sum())} elements outside, largest error "
                        f"{err.max() / largest:.3e} of the largest")
    terms = rast.read_loss()
    want = sb.LossTerms.from_pixel_loss(want_pixel_loss)
    for a, b in ((terms.l1, want.l1), (terms.dssim, want.dssim), (terms.alpha, want.alpha), (terms.total, want.total)):
        if abs(a - b) > LOSS_TERMS_RTOL * abs(b) + 1e-9:
            failures.append(f"{name}: loss terms {terms} vs {want}")
            break

    rast.encode_backward()
    want_grads, want_camera, want_stats, scale = ref.backward(image, contributions, lg)
    stride = sb.param_stride(ref.cloud.sh_degree)
    stats["gradients"] = check_gradients(name, rast.read_param_gradients(), want_grads, scale, stride, failures)
    stats["camera_max_relative"] = check_camera_gradient(name, rast, want_camera, failures)
    st = rast.read_densify_stats()
    if not (np.array_equal(st[:, 1], want_stats[:, 1]) and np.array_equal(st[:, 2], want_stats[:, 2])):
        failures.append(f"{name}: densify statistics (visible counts, radii) differ")
    rast.close()
    assert not failures, f"{failures}; statistics: {stats}"
    return stats


# ---------------------------------------------------------------------------- config 2


@pytest.fixture(scope="module")
def config2():
    scene = scenes.config(2)
    camera = scene.cameras[3]
    truth = oracle.render(scene.truth.to_packed(), scene.truth.sh_degree, oracle.camera_of(camera))["image"]
    return Reference(scene.cloud, camera, _masked_target(truth))


def test_config2_full_rectangle_lists_bit_exact(ctx, config2):
    ref = config2
    rast, _, _ = make_rasterizer(ctx, ref.cloud, ref.camera)
    rast.encode_forward()
    meta = rast.read_intersections()
    assert meta.count == len(ref.fwd["keys"]) > 1_000_000 and meta.overflow == 0
    got = rast.read_projected()
    for field in ("radius", "tile_min", "tile_max", "depth", "mean", "conic", "opacity", "color"):
        assert np.array_equal(got[field], ref.fwd["proj"][field]), f"projected {field} differs"
    assert np.array_equal(rast.read_tile_offsets(), ref.fwd["offsets"])
    keys, gaussians = rast.read_sorted_intersections()
    assert np.array_equal(keys, ref.fwd["keys"]) and np.array_equal(gaussians, ref.fwd["gauss"])
    assert np.array_equal(rast.read_tile_ranges(), ref.fwd["ranges"])


def test_config2_full_benchmark_path(ctx, config2):
    stats = run_bench_path(ctx, "config 2", config2)
    print(f"config 2 full size: {stats}")


# ---------------------------------------------------------------------------- config 3


def test_config3_full_camera_keys_bit_exact(ctx):
    scene = scenes.config(3)
    camera = scene.cameras[0]
    rast, _, _ = make_rasterizer(ctx, scene.cloud, camera)
    rast.encode_forward()
    keys, gaussians = rast.read_sorted_intersections()
    want = oracle.render(scene.cloud.to_packed(), scene.cloud.sh_degree, oracle.camera_of(camera))
    assert len(keys) == len(want["keys"]) > 10_000_000
    assert np.array_equal(keys, want["keys"]) and np.array_equal(gaussians, want["gauss"])
    assert np.array_equal(rast.read_tile_ranges(), want["ranges"])
    image = rast.read_image().rgbt
    diff = np.abs(image - want["image"]).reshape(-1, 4)
    agree = rast.read_contributions() == want["contrib"]
    assert np.all(diff[agree] <= RTOL * np.abs(want["image"].reshape(-1, 4)[agree]) + IMAGE_FLOOR)
    assert (~agree).mean() <= THRESHOLD_PIXELS


# ------------------------------------------------------------------- web/example scene


def test_web_example_training_step(ctx):
    """One training step of the reference's timing scene (examples/step_timing.rs) with the
    benchmark's options: forward, loss and backward stage by stage against the oracle, then the
    one-call step (sp_train_step: backward and Adam fused) against the oracle's whole step."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import fetch_web_example

    if not fetch_web_example.available():
        pytest.skip("the example scene was not fetched (tests/golden/fetch_web_example.py)")
    cloud, cameras, gt = splat_io.read_fit_run(fetch_web_example.TARGET)
    view = 1
    camera = cameras[view]
    ref = Reference(cloud, camera, gt[view].reshape(-1))
    stats = run_bench_path(ctx, "web/example", ref)
    print(f"web/example: {stats}")

    rates = sb.LEARNING_RATES_SHORT_RUN
    extent = np.float32(sb.cameras_extent(cameras))
    rast, params, _ = make_rasterizer(ctx, cloud, camera, ground_truth=ref.gt, **BENCH_OPTIONS)
    rast.encode_forward()
    rast.encode_loss(0)
    rast.encode_backward()
    gpu_gradients = rast.read_param_gradients().astype(np.float64)
    adam = sb.Adam(ctx, params, rast, len(cloud), rates, float(extent))
    _, loss = rast.train_step(adam, camera, 0, 1.0)
    stride = sb.param_stride(0)
    want = ref.packed.copy()
    m, v = np.zeros_like(want), np.zeros_like(want)
    lr = oracle.learning_rates_by_slot(rates.to_c(), extent, stride)
    want_loss, _ = oracle.train_step(want, 0, ref.cam, ref.gt, m, v, lr, 1, float(np.log(np.float32(0.02) * extent)),
                                     float(np.log(np.float32(10.0))))
    assert abs(loss.total - want_loss) <= 1e-5 * abs(want_loss)
    # The oracle's own end-to-end gradient (its forward, loss and backward) and its rounding scale.
    f = ref.fwd
    lg, _ = ref.loss(f["image"])
    oracle_gradients, _, _, scale = ref.backward(f["image"], f["contrib"], lg)
    oracle_gradients = oracle_gradients.astype(np.float64)
    got = params.cpu().numpy()
    rate = np.tile(lr, len(cloud)).astype(np.float64)
    spacing = np.abs(np.spacing(want.astype(np.float32))).astype(np.float64)
    # Adam's first update (optimizer.rs:64-66, adam.wgsl:20-37) is rate * g / (|g| + 1e-15): the
    # two steps can differ by the rate times the difference of that map at the two gradients
    # (a sign, except where |g| is near 1e-15), plus the roundings of the update.
    update = lambda g: g / (np.abs(g) + 1e-15)  # noqa: E731
    allowed = 2.0 * rate * np.abs(update(gpu_gradients) - update(oracle_gradients)) + 4.0 * spacing + 1e-6 * rate
    # A gradient within its rounding bar of zero has no sign to agree on (e.g. a near-isotropic
    # Gaussian's rotation gradient): its step is the rate either way.
    bar = (RTOL * np.abs(oracle_gradients).reshape(len(cloud), stride) + ROUNDINGS * EPS * scale)
    bar[:, CHAIN_SLOTS.start:CHAIN_SLOTS.stop] += CHAIN_FLOOR * scale[:, CHAIN_SLOTS.start:CHAIN_SLOTS.stop]
    noise = np.abs(oracle_gradients) <= bar.reshape(-1)
    allowed[noise] += 2.0 * rate[noise]
    # The scale clamp (clamp_scales.wgsl:15-29) ties a Gaussian's three log-scales to the largest
    # of them: each may move as far as any of the three.
    scales = allowed.reshape(len(cloud), stride)[:, 3:6]
    scales[:] = scales.max(axis=1, keepdims=True)
    differ = np.abs(got.astype(np.float64) - want) > allowed
    detail = [(int(i) // stride, int(i) % stride, float(got[i]), float(want[i]), float(gpu_gradients[i]),
               float(oracle_gradients[i])) for i in np.nonzero(differ)[0][:8]]
    assert not np.any(differ), (f"{int(np.sum(differ))} parameters differ after the step beyond Adam's map: "
                                f"(Gaussian, slot, cuda, oracle, cuda gradient, oracle gradient) {detail}")
    flipped = (np.sign(gpu_gradients) != np.sign(oracle_gradients)) & ~noise
    assert np.mean(flipped) <= 1e-3, f"{np.mean(flipped):.2e} of the gradients have the other sign"
