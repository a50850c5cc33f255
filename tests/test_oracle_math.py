"""Accuracy of the exps the CUDA kernels and the CPU oracle share (include/splat_math.h), so
that radii, tile rectangles and the blend's alpha decisions come out bit-identical on both sides.

sp_expf (single precision) gives the Gaussians' scales (exp of the log-scales), the opacity
sigmoid and the SSIM window; sp_expf_exact (double precision, rounded once) gives the blend's
alpha in the oracle and the per-Gaussian power thresholds of the CUDA blend kernels. Both are
measured over the whole float range they accept and, densely, over the arguments those uses meet
(log-scales, negated opacity logits and falloff powers within [-16, 16], window exponents within
[-6, 0]):
  - sp_expf against the correctly rounded exp (float64 exp rounded once to float32): at most
    1 ulp apart, equal on more than 90 % of the arguments;
  - sp_expf_exact against the correctly rounded exp: equal on more than 99.99 % of the
    arguments and never more than 1 ulp apart (an exhaustive run over every float in
    [-105, 88.72] against the long-double exp found no difference at all), and monotone
    non-decreasing over the sampled arguments in increasing order (the blend kernels' thresholds
    rely on it; the exhaustive run over every float in [-105, 1] found no decrease);
  - both against the host libm's expf (glibc, the oracle's and the reference's host exp): at
    most 1 ulp apart;
  - both against CUDA's expf (torch.exp on a float32 CUDA tensor; CUDA documents a 2-ulp bound
    for expf): at most 2 ulp apart (GPU test).
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


EXPS = {"sp_expf": oracle.sp_expf, "sp_expf_exact": oracle.sp_expf_exact}
# Least share of the arguments where each is the correctly rounded result.
CORRECTLY_ROUNDED = {"sp_expf": 0.9, "sp_expf_exact": 0.9999}


@pytest.fixture(scope="module")
def table():
    xs = _arguments()
    values = {name: np.array([fn(float(x)) for x in xs], np.float32) for name, fn in EXPS.items()}
    return xs, values, np.exp(xs.astype(np.float64)).astype(np.float32)


@pytest.mark.parametrize("name", list(EXPS))
def test_within_one_ulp_of_the_correctly_rounded_exp(table, name):
    xs, values, want = table
    got = values[name]
    normal = want >= FLT_MIN
    assert _ulp(got[normal], want[normal]).max() <= 1
    subnormal = (want > 0) & ~normal
    if subnormal.any():
        assert _ulp(got[subnormal], want[subnormal]).max() <= 1
    assert np.mean(got[normal] == want[normal]) > CORRECTLY_ROUNDED[name]


def test_sp_expf_exact_is_monotone(table):
    xs, values, _ = table
    order = np.argsort(xs, kind="stable")
    assert np.all(np.diff(values["sp_expf_exact"][order].astype(np.float64)) >= 0.0)


@pytest.mark.parametrize("name", list(EXPS))
def test_within_one_ulp_of_libm(table, name):
    xs, values, _ = table
    sample = xs[::7]
    libm = np.array([oracle.libm_expf(float(x)) for x in sample], np.float32)
    mine = values[name][::7]
    positive = libm > 0
    assert _ulp(mine[positive], libm[positive]).max() <= 1


@pytest.mark.parametrize("name", list(EXPS))
def test_special_values(name):
    fn = EXPS[name]
    assert np.isnan(fn(float("nan")))
    assert fn(89.0) == float("inf")
    assert fn(float("inf")) == float("inf")
    assert fn(-105.0) == 0.0
    assert fn(float("-inf")) == 0.0
    assert fn(0.0) == 1.0


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(EXPS))
def test_within_two_ulp_of_cuda_expf(table, name):
    import torch

    xs, values, _ = table
    got = values[name]
    cuda = torch.exp(torch.from_numpy(xs).cuda()).cpu().numpy()
    positive = (cuda > 0) & (got > 0) & np.isfinite(cuda)
    assert _ulp(got[positive], cuda[positive]).max() <= 2


# Adam's bias-corrected moments (adam.wgsl:30-31: m / (1 - beta1^t), v / (1 - beta2^t)) are IEEE
# float divisions in the reference and the oracle; the CUDA kernels form them as the float
# rounding of x * RN64(1 / b) (div_by_bias in csrc/exact_div.cuh, with a proof that the two are
# equal for every float x and every float b in [2^-126, 1]). Checked here with numpy's IEEE
# float32 division and float64 product.


def _bias_corrections(beta: float, steps: int) -> np.ndarray:
    t = np.arange(1, steps + 1, dtype=np.float32)
    return (np.float32(1.0) - np.power(np.float32(beta), t)).astype(np.float32)


def _div_by_bias(x: np.ndarray, b: np.float32) -> np.ndarray:
    return (x.astype(np.float64) * (1.0 / np.float64(b))).astype(np.float32)


def _same_floats(got: np.ndarray, want: np.ndarray) -> bool:
    nan = np.isnan(want)
    return bool(np.array_equal(np.isnan(got), nan) and np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32)))


def test_division_by_the_bias_corrections_is_the_ieee_quotient():
    biases = np.unique(np.concatenate([_bias_corrections(0.9, 20_000), _bias_corrections(0.999, 20_000)]))
    assert biases.min() > 0 and biases.max() == 1.0 and len(biases) > 10_000
    # Every significand (x in [1, 2)) for a sample of the corrections, the first steps' included:
    # for quotients in the normal range the rounding depends on the significands only.
    significands = (np.arange(1 << 23, dtype=np.uint32) | np.uint32(0x3F800000)).view(np.float32)
    sample = np.unique(np.concatenate([_bias_corrections(0.9, 4), _bias_corrections(0.999, 4),
                                       biases[np.linspace(0, len(biases) - 1, 24).astype(int)]]))
    for b in sample:
        assert _same_floats(_div_by_bias(significands, b), significands / b), b
    # Random bit patterns (every exponent: zeros, subnormals, infinities, NaN) for every correction.
    rng = np.random.default_rng(5)
    x = rng.integers(0, 1 << 32, size=2048, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = np.concatenate([x, np.array([0.0, -0.0, np.inf, -np.inf, 1e-45, -1e-45, 3.4028235e38], np.float32)])
    for chunk in np.array_split(biases, 16):
        b = chunk[:, None]
        with np.errstate(over="ignore", invalid="ignore"):
            want = x[None, :] / b
            got = (x[None, :].astype(np.float64) * (1.0 / b.astype(np.float64))).astype(np.float32)
        assert _same_floats(got.ravel(), want.ravel())
