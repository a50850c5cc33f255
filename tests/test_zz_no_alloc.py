"""sp_loss_sums_noalloc, the entry point for callers that cannot allocate device memory
(their device memory belongs to their own allocator, or a cudaMalloc's device-wide
synchronisation would stall them): it must give the loss that sp_read_loss gives, call
after call, using only the buffers the caller passes and the library's fixed scratch.

Collected last (file name), so that a run stopping at the first failure has run every
other test first; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import splat_b200 as sb
from helpers import make_rasterizer, random_cloud
from splat_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_PIXELS = 4194304  # SP_NOALLOC_MAX_PIXELS in include/splat.h


def _noalloc_sums(lib, device, pixel_loss, pixels, sums, stream) -> int:
    return lib.sp_loss_sums_noalloc(
        device, ctypes.c_void_p(pixel_loss.data_ptr()), pixels, ctypes.c_void_p(sums.data_ptr()), ctypes.c_void_p(stream)
    )


def test_noalloc_loss_sums_match_read_loss(ctx):
    import torch

    rng = np.random.default_rng(31)
    width, height = 96, 64
    pixels = width * height
    cloud = random_cloud(300, rng)
    camera = sb.PinholeCamera(np.eye(3), np.zeros(3), (70.0, 70.0), (48, 32), width, height)
    mask = (rng.random(pixels) < 0.5).astype(np.float32)
    gt = np.concatenate([rng.random((pixels, 3)).astype(np.float32) * mask[:, None], mask[:, None]], axis=1)
    rast, _, _ = make_rasterizer(ctx, cloud, camera, ground_truth=gt.reshape(-1))
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        # A different render each call: the scratch keeps the previous call's contents.
        camera.translation[0] = 0.05 * call
        rast.set_camera(camera)
        rast.encode_forward()
        rast.encode_loss(0)
        want = rast.read_loss()
        pixel_loss = torch.from_numpy(rast.read_pixel_loss()).cuda()
        sums = torch.zeros(4, dtype=torch.float64, device="cuda")
        assert _noalloc_sums(lib, 0, pixel_loss, pixels, sums, stream) == _lib.SP_OK
        torch.cuda.synchronize()
        got = (sums.cpu().numpy() / pixels).astype(np.float32)
        for value, expected in zip(got, (want.l1, want.alpha, want.dssim, want.total)):
            assert abs(float(value) - expected) < 1e-6, (call, got, want)


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    import torch

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    sums = torch.zeros(4, dtype=torch.float64, device="cuda")
    pixel_loss = torch.zeros(16, dtype=torch.float32, device="cuda")
    assert _noalloc_sums(lib, 0, pixel_loss, MAX_PIXELS + 1, sums, stream) == _lib.SP_ERR_INVALID
    assert _noalloc_sums(lib, 0, pixel_loss, 0, sums, stream) == _lib.SP_ERR_INVALID
