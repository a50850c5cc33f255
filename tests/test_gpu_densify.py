"""Device densification (sp_densify_plan / sp_densify_apply) against the CPU oracle's
restatement of densify (instantsplat-rs/src/densify.rs:147-257) on the same seeded inputs.

Bar: the report, every kept Gaussian and every moment bit for bit; the new Gaussians bit for
bit except the split children's centres, which go through exp, ln and cos (the oracle uses
the host libm in single precision, as the reference; the device the f64 functions rounded
once): within 1e-5 relative + 1e-6 absolute, and at least 99% of those floats bit for bit.
Then the trainer: a densification on the device followed by a step equals the reference's
flow (read back, densify on the host, resume Adam from host moments) followed by the same
step."""

from __future__ import annotations

import numpy as np
import pytest

import densify_tests as dt
import oracle
import splat_b200 as sb
from splat_b200 import scenes

pytestmark = pytest.mark.gpu


def random_inputs(n: int, sh_degree: int, seed: int, tie_levels: int | None = None):
    """Parameters around the prune and split thresholds, random moments, and statistics with
    some Gaussians never visible, some oversized on screen and, with `tie_levels`, mean
    gradients on a few levels (many equal keys: the selection's index-order ties)."""
    rng = np.random.default_rng(seed)
    stride = sb.param_stride(sh_degree)
    params = rng.normal(0.0, 1.0, (n, stride)).astype(np.float32)
    params[:, 3:6] = rng.uniform(-7.0, -1.0, (n, 3))
    params[:, 6:10] = rng.normal(0.0, 1.0, (n, 4))
    params[:, 10] = rng.uniform(-7.0, 3.0, n)  # logit(0.005) = -5.29
    first = rng.normal(0.0, 1e-3, (n, stride)).astype(np.float32)
    second = rng.uniform(0.0, 1e-5, (n, stride)).astype(np.float32)
    stats = np.zeros((n, 4), np.float32)
    visible = rng.choice(np.array([0.0, 1.0, 2.0, 4.0], np.float32), n, p=[0.1, 0.3, 0.3, 0.3])
    if tie_levels:
        mean = (rng.integers(1, tie_levels + 1, n) * np.float32(1e-4)).astype(np.float32)
        stats[:, 0] = mean * visible  # visible is a power of two: sum / visible is `mean` again
    else:
        stats[:, 0] = rng.uniform(0.0, 6e-4, n).astype(np.float32) * visible
    stats[:, 1] = visible
    stats[:, 2] = rng.uniform(0.0, 120.0, n)
    return params.reshape(-1), first.reshape(-1), second.reshape(-1), stats


def compare(device, reference, stride):
    p, m, v, report = device
    rp, rm, rv, rreport = reference
    assert report == rreport
    after = report["after"]
    copies = after - report["cloned"] - 2 * report["split"]
    assert p.size == rp.size == after * stride
    assert np.array_equal(m.view(np.uint32), rm.view(np.uint32)), "first moments"
    assert np.array_equal(v.view(np.uint32), rv.view(np.uint32)), "second moments"
    p, rp = p.reshape(after, stride), rp.reshape(after, stride)
    assert np.array_equal(p[:copies].view(np.uint32), rp[:copies].view(np.uint32)), "kept Gaussians"
    assert np.array_equal(p[copies:, 3:].view(np.uint32), rp[copies:, 3:].view(np.uint32)), "new Gaussians"
    centres, rcentres = p[copies:, :3], rp[copies:, :3]
    np.testing.assert_allclose(centres, rcentres, rtol=1e-5, atol=1e-6)
    if centres.size:
        exact = float(np.mean(centres.view(np.uint32) == rcentres.view(np.uint32)))
        assert exact >= 0.99, f"only {exact:.4f} of the new centres bit for bit"


CASES = [
    # n, SH degree, max_count (None: room for every candidate), reset, tie levels
    (7, 0, None, False, None),
    (5_000, 0, None, False, None),
    (50_003, 1, "cap", False, 64),
    (50_003, 3, "cap", True, None),
    (20_000, 2, "none", False, None),
    (1_500_000, 0, "cap", False, 16),
]


@pytest.mark.parametrize("n,sh_degree,cap,reset,ties", CASES,
                         ids=[f"{c[0]}_sh{c[1]}_{c[2]}_{'reset' if c[3] else 'keep'}_{c[4]}" for c in CASES])
def test_densify_matches_the_oracle(ctx, n, sh_degree, cap, reset, ties):
    params, first, second, stats = random_inputs(n, sh_degree, seed=n + sh_degree, tie_levels=ties)
    stride = sb.param_stride(sh_degree)
    settings = sb.DENSIFY_SHORT_RUN
    probe = oracle.densify(params, first, second, stats, stride, 2.0, 10 * n, settings.to_c(), 0, 0)[3]
    kept = probe["after"] - probe["cloned"] - probe["split"]  # every candidate taken
    candidates = probe["cloned"] + probe["split"]
    if cap is None:
        max_count = 10 * n
    elif cap == "none":
        max_count = kept
    else:
        max_count = kept + candidates // 3
    seed = 5
    reference = oracle.densify(params, first, second, stats, stride, 2.0, max_count, settings.to_c(), int(reset), seed)
    device = dt.cuda_densify(params, first, second, stats, sh_degree, 2.0, max_count, settings, reset, seed, ctx=ctx)
    if cap == "cap":
        assert reference[3]["over_budget"] > 0
    compare(device, reference, stride)


def test_every_gaussian_pruned_is_refused_with_the_report(ctx):
    params, first, second, stats = dt.six_gaussians()
    params = params.copy()
    params[10::dt.STRIDE] = dt.logit(0.001)
    with pytest.raises(sb.DensifyError) as info:
        dt.cuda_densify(params, first, second, stats, 0, 10.0, 100, sb.DENSIFY_SHORT_RUN, False, 1, ctx=ctx)
    assert info.value.report.before == 6 and info.value.report.pruned_transparent == 6


def _trainer(ctx, densify=None):
    scene = scenes.config(0)
    gts = []
    for cam in scene.cameras:
        rgbt = oracle.render(scene.truth.to_packed(), 0, oracle.camera_array(cam.uniform()))["image"].reshape(-1, 4)
        mask = ((1.0 - rgbt[:, 3]) > 0.5).astype(np.float32)
        gts.append(np.concatenate([rgbt[:, :3] * mask[:, None], mask[:, None]], axis=1))
    gt = np.stack(gts).astype(np.float32)
    return sb.Trainer(scene.cloud, scene.cameras, gt, ctx=ctx, backward_mode=sb.SP_BWD_DETERMINISTIC,
                      densify=densify)


def test_trainer_densification_equals_the_host_rebuild(ctx):
    """training.rs:238-266 on the device (Trainer.densify_now) from the state after 30 steps:
    its Gaussians and moments against the oracle's densify of the read-back state; then one
    more step of the trainer against the same step after the reference's rebuild (a new
    rasterizer, Adam::resumed from host moments): bit for bit."""
    import torch

    settings = sb.DensifySettings(**{**sb.DENSIFY_SHORT_RUN.__dict__, "interval": 30, "start": 30})
    steps = 100
    run = _trainer(ctx, settings)
    for step in range(30):
        run.train_step(step, steps)
    params = run.params.cpu().numpy()
    first, second = run.adam.read_moments()
    stats = run.rasterizer.read_densify_stats()
    stride = run.rasterizer.stride
    max_count = settings.max_count(run.initial_gaussian_count)
    reference = oracle.densify(params, first, second, stats, stride, run.extent, max_count, settings.to_c(), 0, 0)
    report = run.densify_now(settings)  # seed 0: the first densification
    assert report.after != report.before and run.gaussian_count == report.after
    m, v = run.adam.read_moments()
    densified = run.params.cpu().numpy()
    compare((densified, m, v, dict(before=report.before, cloned=report.cloned, split=report.split,
                                   pruned_transparent=report.pruned_transparent,
                                   pruned_oversized=report.pruned_oversized, over_budget=report.over_budget,
                                   opacity_reset=int(report.opacity_reset), after=report.after)),
            reference, stride)

    # The reference's rebuild of the densified state, then step 30 on both.
    host_params = torch.from_numpy(densified.copy()).cuda()
    rast = sb.Rasterizer(ctx, host_params, report.after, run.width, run.height, run.ground_truth, run.view_count,
                         run.options)
    adam = run.adam.resumed(host_params, rast, report.after, reference[1], reference[2])
    assert adam.steps_taken() == run.adam.steps_taken() == 30
    view = 30 % run.view_count
    rast.train_step(adam, run.camera(view), view, sb.position_rate_factor(30, steps))
    run.step(view, sb.position_rate_factor(30, steps))
    ctx.sync()
    assert np.array_equal(run.params.cpu().numpy().view(np.uint32), host_params.cpu().numpy().view(np.uint32))


def test_training_with_densification_runs_and_lowers_the_loss(ctx):
    """DENSIFY_SHORT_RUN's schedule on a 150-step run: densified after steps 50 and 75 (interval
    25 here), the count changes, the loss falls."""
    settings = sb.DensifySettings(**{**sb.DENSIFY_SHORT_RUN.__dict__, "interval": 25, "start": 50})
    steps = 150
    trainer = _trainer(ctx, settings)
    first = trainer.loss(0).total
    reports = [r for r in (trainer.train_step(step, steps) for step in range(steps)) if r is not None]
    assert [r.before for r in reports][0] == trainer.initial_gaussian_count
    assert len(reports) == 2 and trainer.gaussian_count == reports[-1].after
    assert trainer.gaussian_count <= settings.max_count(trainer.initial_gaussian_count)
    last = trainer.loss(0).total
    assert last < first, (first, last)


def test_trainer_writes_and_reads_its_splat_on_the_device(ctx, tmp_path):
    """The trainer's Gaussians written to a PLY straight from device memory (sp_ply_write) and
    read back into a device tensor (sp_ply_read): the same floats; the host reader agrees."""
    from splat_b200 import io

    trainer = _trainer(ctx)
    for step in range(5):
        trainer.train_step(step, 10)
    ctx.sync()
    path = tmp_path / "splat.ply"
    io.write_splat_ply_device(path, trainer.params, trainer.gaussian_count, trainer.sh_degree)
    back, count, degree = io.read_splat_ply_device(path, device=ctx.device)
    assert (count, degree) == (trainer.gaussian_count, trainer.sh_degree)
    assert np.array_equal(back.cpu().numpy(), trainer.params.cpu().numpy())
    host = io.read_splat_ply(path)
    assert np.array_equal(host.to_packed().reshape(-1), trainer.params.cpu().numpy())
