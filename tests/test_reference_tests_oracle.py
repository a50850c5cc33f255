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
