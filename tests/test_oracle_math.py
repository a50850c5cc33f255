"""Accuracy of sp_expf (include/splat_math.h), the exp that the projection kernels and the CPU
oracle share so that radii and tile rectangles come out bit-identical on both sides.

It decides the Gaussians' scales (exp of the log-scales), the opacity sigmoid and the SSIM
window, so it is measured over the whole float range it accepts and, densely, over the
arguments those uses meet (log-scales and negated opacity logits within [-16, 16], window
exponents within [-6, 0]):
  - against the correctly rounded exp (float64 exp rounded once to float32): equal on more
    than 99.99 % of the arguments and never more than 1 ulp apart (an exhaustive run over
    every float in [-105, 88.72] against the long-double exp found no difference at all);
  - monotone non-decreasing over the sampled arguments in increasing order (the blend kernels
    rely on it; the exhaustive run over every float in [-105, 1] found no decrease);
  - against the host libm's expf (glibc, the oracle's and the reference's host exp): at most
    1 ulp apart;
  - against CUDA's expf (torch.exp on a float32 CUDA tensor; CUDA documents a 2-ulp bound for
    expf): at most 2 ulp apart (GPU test).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle

FLT_MIN = np.float32(1.17549435e-38)


def _arguments() -> np.ndarray:
    rng = np.random.default_rng(2024)
    return np.concatenate(
        [
            rng.uniform(-104.0, 88.72, 100_000),
            rng.uniform(-16.0, 16.0, 200_000),
            rng.uniform(-6.0, 0.0, 50_000),
            np.linspace(-1.0, 1.0, 20_001),
            [0.0, -0.0, 88.7228, -87.33, -103.9, 1e-8, -1e-8],
        ]
    ).astype(np.float32)


def _ulp(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in units in the last place of two arrays of positive float32."""
    return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))


def _sp_expf(xs: np.ndarray) -> np.ndarray:
    return np.array([oracle.sp_expf(float(x)) for x in xs], np.float32)


@pytest.fixture(scope="module")
def table():
    xs = _arguments()
    return xs, _sp_expf(xs), np.exp(xs.astype(np.float64)).astype(np.float32)


def test_sp_expf_within_one_ulp_of_the_correctly_rounded_exp(table):
    xs, got, want = table
    normal = want >= FLT_MIN
    assert _ulp(got[normal], want[normal]).max() <= 1
    subnormal = (want > 0) & ~normal
    if subnormal.any():
        assert _ulp(got[subnormal], want[subnormal]).max() <= 1
    # The results are the correctly rounded ones.
    assert np.mean(got[normal] == want[normal]) > 0.9999


def test_sp_expf_is_monotone(table):
    xs, got, _ = table
    order = np.argsort(xs, kind="stable")
    assert np.all(np.diff(got[order].astype(np.float64)) >= 0.0)


def test_sp_expf_within_one_ulp_of_libm(table):
    xs, got, _ = table
    sample = xs[::7]
    libm = np.array([oracle.libm_expf(float(x)) for x in sample], np.float32)
    mine = got[::7]
    positive = libm > 0
    assert _ulp(mine[positive], libm[positive]).max() <= 1


def test_sp_expf_special_values():
    assert np.isnan(oracle.sp_expf(float("nan")))
    assert oracle.sp_expf(89.0) == float("inf")
    assert oracle.sp_expf(float("inf")) == float("inf")
    assert oracle.sp_expf(-105.0) == 0.0
    assert oracle.sp_expf(float("-inf")) == 0.0
    assert oracle.sp_expf(0.0) == 1.0


@pytest.mark.gpu
def test_sp_expf_within_two_ulp_of_cuda_expf(table):
    import torch

    xs, got, _ = table
    cuda = torch.exp(torch.from_numpy(xs).cuda()).cpu().numpy()
    positive = (cuda > 0) & (got > 0) & np.isfinite(cuda)
    assert _ulp(got[positive], cuda[positive]).max() <= 2
