"""The reference's own GPU tests, run on the CPU oracle (the checker must pass them)."""

from __future__ import annotations

import pytest

import reference_tests as rt
from backends import OracleBackend


def make(n, camera, sh_degree=0, ground_truth=None):
    return OracleBackend(n, camera, sh_degree, ground_truth)


def test_forward_matches_the_cpu_reference():
    rt.forward_matches_the_cpu_reference(make)


@pytest.mark.parametrize("moved", [False, True])
def test_backward_matches_finite_differences(moved):
    rt.gradient_check(make, rt.moved_camera() if moved else rt.camera_at_origin(32, 32, 40.0))


@pytest.mark.parametrize("sh_degree", [1, 3])
def test_sh_backward_matches_finite_differences(sh_degree):
    """The SH degree 1-3 extension (no reference counterpart): the same check."""
    rt.gradient_check(make, rt.moved_camera(), sh_degree=sh_degree)


def test_identical_images_have_zero_loss():
    rt.identical_images_have_zero_loss(make)


def test_loss_terms_match_the_cpu_reference():
    rt.loss_terms_match_the_cpu_reference(make)


def test_loss_gradient_matches_finite_differences():
    rt.loss_gradient_matches_finite_differences(make)


def test_densify_stats_match_the_cpu_mean_gradient():
    rt.densify_stats_match_the_cpu_mean_gradient(make)


def test_pose_gradient_matches_finite_differences():
    rt.pose_gradient_matches_finite_differences(make)


# ---- densify.rs:299-448 on the oracle

import densify_tests as dt  # noqa: E402


@pytest.mark.parametrize("case", dt.ALL, ids=[c.__name__ for c in dt.ALL])
def test_densify(case):
    case(dt.oracle_densify)


def test_densifies_every_interval_over_the_first_half():
    """densify.rs:433-437 (the host logic through the C ABI)."""
    import splat_b200 as sb

    after = [done for done in range(1, 301) if sb.DENSIFY_SHORT_RUN.densifies_after(done, 300)]
    assert after == [50, 100, 150]


def test_densify_settings_refuse_what_the_reference_asserts():
    """densify.rs:78-93: interval 0, a step outside 1..=steps, and an opacity reset interval
    that is not a multiple of the densify interval."""
    import splat_b200 as sb

    base = sb.DENSIFY_SHORT_RUN.__dict__
    with pytest.raises(ValueError):
        sb.DensifySettings(**{**base, "interval": 0}).densifies_after(1, 10)
    with pytest.raises(ValueError):
        sb.DENSIFY_SHORT_RUN.densifies_after(0, 10)
    with pytest.raises(ValueError):
        sb.DENSIFY_SHORT_RUN.densifies_after(11, 10)
    with pytest.raises(ValueError):
        sb.DensifySettings(**{**base, "opacity_reset_interval": 75}).resets_opacity_after(150)
    assert not sb.DENSIFY_SHORT_RUN.resets_opacity_after(100)
    assert sb.DENSIFY_SHORT_RUN.max_count(265_000) == 530_000


def test_splitmix64_known_answer():
    """SplitMix64 (densify.rs:275-297) seeded with 0: its published first output."""
    import oracle

    assert oracle.splitmix64(0, 0) == 0xE220A8397B1DCDAF


def test_densify_report_display():
    """DensifyReport's Display (densify.rs:113-128)."""
    import splat_b200 as sb

    report = sb.DensifyReport(6, 1, 1, 1, 1, True, 2, 6)
    assert str(report) == ("6 -> 6 Gaussians: cloned 1, split 1, pruned 1 transparent and 1 oversized, "
                           "2 more over the growth cap, opacities reset to 0.01")
