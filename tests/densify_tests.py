"""The reference's densification tests (instantsplat-rs/src/densify.rs:299-448), written
against a `densify` function so that each runs on the CPU oracle and on the device path:

    densify(params, first, second, stats, sh_degree, extent, max_count, settings,
            reset_opacity, seed) -> (params, first, second, report dict)

raising ValueError where the reference panics. The split test drives `split_child` through
a densification that splits every Gaussian: the children come out in the order the
reference's single SplitMix64 stream draws them."""

from __future__ import annotations

import math

import numpy as np
import pytest

import splat_b200 as sb

STRIDE = 14  # PARAM_STRIDE of the reference (SH degree 0)


def logit(p: float) -> float:
    """gaussians.rs:92-95 in f32."""
    p = np.float32(p)
    return float(np.float32(np.log(np.float32(p / (np.float32(1.0) - p)))))


def sigmoid(x: float) -> float:
    return float(np.float32(1.0) / (np.float32(1.0) + np.exp(np.float32(-x))))


def six_gaussians():
    """densify.rs:304-335: extent 10 splits above ln(0.1). Gaussian 0 is small with a high
    gradient, 1 large with a high gradient, 2 transparent, 3 oversized on screen, 4 small
    with a low gradient, 5 never visible."""
    log_scales = [-4.0, -1.0, -4.0, -4.0, -4.0, -4.0]
    opacities = [0.5, 0.5, 0.001, 0.5, 0.5, 0.5]
    params = []
    for g in range(6):
        params += [float(g), 0.0, 5.0]
        params += [log_scales[g], log_scales[g] - 1.0, log_scales[g] - 2.0]
        params += [1.0, 0.0, 0.0, 0.0, logit(opacities[g])]
        params += [0.1 * g, 0.2, 0.3]
    params = np.array(params, np.float32)
    first = np.arange(params.size, dtype=np.float32) + 1.0
    second = first * np.float32(10.0)
    stats = np.array([[3e-3, 4.0, 5.0, 0.0], [2e-3, 4.0, 30.0, 0.0], [1.0, 4.0, 5.0, 0.0], [1.0, 4.0, 200.0, 0.0],
                      [1e-4, 4.0, 5.0, 0.0], [0.0, 0.0, 0.0, 0.0]], np.float32)
    return params, first, second, stats


def clones_small_splits_large_and_prunes(densify):
    """densify.rs:336-383."""
    params, first, second, stats = six_gaussians()
    p, m, v, report = densify(params, first, second, stats, 0, 10.0, 100, sb.DENSIFY_SHORT_RUN, False, 1)
    assert report == dict(before=6, cloned=1, split=1, pruned_transparent=1, pruned_oversized=1, over_budget=0,
                          opacity_reset=0, after=6)

    def gaussian(g):
        return p[g * STRIDE:(g + 1) * STRIDE]

    # Kept in order: 0, 4, 5 with their moments; then the clone of 0 and the two children
    # of 1, with zero moments.
    assert np.array_equal(gaussian(0), params[:STRIDE])
    assert gaussian(1)[0] == 4.0
    assert gaussian(2)[0] == 5.0
    assert np.array_equal(m[STRIDE:2 * STRIDE], first[4 * STRIDE:5 * STRIDE])
    assert np.array_equal(v[:STRIDE], second[:STRIDE])
    assert np.array_equal(gaussian(3), params[:STRIDE])
    assert np.all(m[3 * STRIDE:] == 0.0) and np.all(v[3 * STRIDE:] == 0.0)
    original = params[STRIDE:2 * STRIDE]
    for child in (gaussian(4), gaussian(5)):
        for k in range(3, 6):
            assert abs(child[k] - (original[k] - np.log(np.float32(1.6)))) < 1e-6, f"child log scale {child[k]}"
        assert np.array_equal(child[6:], original[6:])
        # Within 4 sigma (e^-1 along x) of the original center.
        offset = float(np.sqrt(np.sum((child[:3] - original[:3]) ** 2)))
        assert 0.0 < offset < 4.0 * math.exp(-1.0), f"child offset {offset}"
    assert not np.array_equal(gaussian(4)[:3], gaussian(5)[:3])


def the_growth_cap_densifies_the_highest_gradients_first(densify):
    """densify.rs:384-393: 4 kept after pruning; one more allowed: Gaussian 0 (3e-3 / 4)
    beats 1 (2e-3 / 4)."""
    params, first, second, stats = six_gaussians()
    _, _, _, report = densify(params, first, second, stats, 0, 10.0, 5, sb.DENSIFY_SHORT_RUN, False, 1)
    assert (report["cloned"], report["split"], report["over_budget"], report["after"]) == (1, 0, 1, 5)


def split_samples_spread_like_the_gaussian(densify):
    """densify.rs:395-409: sigma (0.1, 0.01, 0.01) turned 90 degrees about z (long axis y);
    4000 children drawn from SplitMix64(9): their deviation along each axis."""
    half = np.float32(math.sqrt(0.5))
    gaussian = np.zeros(STRIDE, np.float32)
    gaussian[3:6] = np.log(np.array([0.1, 0.01, 0.01], np.float32))
    gaussian[6:10] = [half, 0.0, 0.0, half]
    count = 2000  # two children each
    params = np.tile(gaussian, count)
    zeros = np.zeros_like(params)
    stats = np.tile(np.array([1.0, 1.0, 0.0, 0.0], np.float32), (count, 1))
    p, _, _, report = densify(params, zeros, zeros, stats, 0, 1.0, 10 * count, sb.DENSIFY_SHORT_RUN, False, 9)
    assert report["split"] == count and report["after"] == 2 * count
    samples = p.reshape(-1, STRIDE)

    def deviation(k):
        return float(np.sqrt(np.mean(samples[:, k].astype(np.float64) ** 2)))

    assert abs(deviation(1) - 0.1) < 0.005, f"y deviation {deviation(1)}"
    assert abs(deviation(0) - 0.01) < 0.0005, f"x deviation {deviation(0)}"
    assert abs(deviation(2) - 0.01) < 0.0005, f"z deviation {deviation(2)}"


def an_opacity_reset_lowers_every_opacity_and_its_moments(densify):
    """densify.rs:410-431."""
    params, first, second, stats = six_gaussians()
    p, m, v, report = densify(params, first, second, stats, 0, 10.0, 100, sb.DENSIFY_SHORT_RUN, True, 1)
    assert report["opacity_reset"] == 1
    for g in range(report["after"]):
        slot = g * STRIDE + 10
        assert abs(sigmoid(p[slot]) - sb.RESET_OPACITY) < 1e-6, f"opacity {sigmoid(p[slot])}"
        assert (m[slot], v[slot]) == (0.0, 0.0)
    # Other moments are kept.
    assert m[0] == first[0]
    resets = sb.DensifySettings(**{**sb.DENSIFY_SHORT_RUN.__dict__, "opacity_reset_interval": 100})
    assert (resets.resets_opacity_after(50), resets.resets_opacity_after(100)) == (False, True)


def pruning_everything_is_refused(densify):
    """densify.rs:439-447 (should_panic "densification pruned every Gaussian")."""
    params, first, second, stats = six_gaussians()
    for g in range(6):
        params[g * STRIDE + 10] = logit(0.001)
    with pytest.raises(ValueError, match="densification pruned every Gaussian"):
        densify(params, first, second, stats, 0, 10.0, 100, sb.DENSIFY_SHORT_RUN, False, 1)


ALL = (
    clones_small_splits_large_and_prunes,
    the_growth_cap_densifies_the_highest_gradients_first,
    split_samples_spread_like_the_gaussian,
    an_opacity_reset_lowers_every_opacity_and_its_moments,
    pruning_everything_is_refused,
)


# ---- the two implementations


def oracle_densify(params, first, second, stats, sh_degree, extent, max_count, settings, reset_opacity, seed):
    import oracle

    return oracle.densify(params, first, second, stats, sb.param_stride(sh_degree), extent, max_count,
                          settings.to_c(), int(bool(reset_opacity)), seed)


def cuda_densify(params, first, second, stats, sh_degree, extent, max_count, settings, reset_opacity, seed,
                 ctx=None):
    """Through the C ABI: a rasterizer over the parameters, an optimiser resumed from the
    moments, the statistics written, then sp_densify_plan / sp_densify_apply."""
    import torch

    ctx = ctx or sb.Context(0)
    stride = sb.param_stride(sh_degree)
    n = params.size // stride
    device = f"cuda:{ctx.device}"
    p = torch.from_numpy(np.ascontiguousarray(params, np.float32)).to(device)
    gt = torch.zeros(16 * 16 * 4, dtype=torch.float32, device=device)
    rast = sb.Rasterizer(ctx, p, n, 16, 16, gt, 1, sb.default_options(sh_degree=sh_degree))
    fresh = sb.Adam(ctx, p, rast, n, sb.LEARNING_RATES_3DGS, 1.0, sh_degree=sh_degree)
    adam = fresh.resumed(p, rast, n, first, second)
    rast.write_densify_stats(stats)
    try:
        out = sb.densify(rast, adam, extent, max_count, settings, reset_opacity, seed)
    finally:
        ctx.sync()
    r = out.report
    report = dict(before=r.before, cloned=r.cloned, split=r.split, pruned_transparent=r.pruned_transparent,
                  pruned_oversized=r.pruned_oversized, over_budget=r.over_budget, opacity_reset=int(r.opacity_reset),
                  after=r.after)
    return out.params.cpu().numpy(), out.first_moment.cpu().numpy(), out.second_moment.cpu().numpy(), report
