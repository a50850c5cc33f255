"""The reference's own GPU tests (rasterizer_tests.rs, loss_tests.rs, densify_tests.rs,
pose_tests.rs), run on the CUDA path through the C ABI with the reference's tolerances."""

from __future__ import annotations

import pytest

import reference_tests as rt
import splat_b200 as sb

pytestmark = pytest.mark.gpu


def make(n, camera, sh_degree=0, ground_truth=None):
    from backends import CudaBackend

    return CudaBackend(n, camera, sh_degree, ground_truth)


def make_atomic(n, camera, sh_degree=0, ground_truth=None):
    from backends import CudaBackend

    return CudaBackend(n, camera, sh_degree, ground_truth, backward_mode=sb.SP_BWD_ATOMIC)


def test_forward_matches_the_cpu_reference():
    rt.forward_matches_the_cpu_reference(make)


@pytest.mark.parametrize("factory", [make, make_atomic], ids=["deterministic", "atomic"])
@pytest.mark.parametrize("moved", [False, True])
def test_backward_matches_finite_differences(moved, factory):
    rt.gradient_check(factory, rt.moved_camera() if moved else rt.camera_at_origin(32, 32, 40.0))


@pytest.mark.parametrize("sh_degree", [1, 3])
def test_sh_backward_matches_finite_differences(sh_degree):
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


# ---- densify.rs:299-448 on the device path

import densify_tests as dt  # noqa: E402


@pytest.mark.parametrize("case", dt.ALL, ids=[c.__name__ for c in dt.ALL])
def test_densify(case, ctx):
    case(lambda *args: dt.cuda_densify(*args, ctx=ctx))
