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


def test_noalloc_at_exactly_the_largest_size(ctx):
    """A 2048 x 2048 frame is exactly SP_NOALLOC_MAX_PIXELS pixels: the entry point takes it
    (every one of its 1024 scratch blocks in use) and gives the loss of sp_read_loss."""
    import torch

    rng = np.random.default_rng(47)
    width = height = 2048
    pixels = width * height
    assert pixels == MAX_PIXELS
    cloud = random_cloud(2000, rng)
    camera = sb.PinholeCamera(np.eye(3), np.zeros(3), (1400.0, 1400.0), (1024, 1024), width, height)
    mask = (rng.random(pixels) < 0.5).astype(np.float32)
    gt = np.concatenate([rng.random((pixels, 3)).astype(np.float32) * mask[:, None], mask[:, None]], axis=1)
    # Enough list capacity for the frame's 192k (Gaussian, tile) pairs: the loss of a truncated
    # frame is reported as an overflow.
    rast, _, _ = make_rasterizer(ctx, cloud, camera, ground_truth=gt.reshape(-1), intersections_per_gaussian=128)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    rast.encode_forward()
    rast.encode_loss(0)
    want = rast.read_loss()
    pixel_loss = torch.from_numpy(rast.read_pixel_loss()).cuda()
    sums = torch.zeros(4, dtype=torch.float64, device="cuda")
    for _ in range(2):
        sums.fill_(-1.0)
        assert _noalloc_sums(lib, 0, pixel_loss, pixels, sums, stream) == _lib.SP_OK
        torch.cuda.synchronize()
        got = (sums.cpu().numpy() / pixels).astype(np.float32)
        for value, expected in zip(got, (want.l1, want.alpha, want.dssim, want.total)):
            assert abs(float(value) - expected) < 1e-6, (got, want)
    rast.close()


def test_noalloc_allocates_no_device_memory(ctx):
    """After a first call on the device (which may load the library's kernels and its scratch
    array), further calls leave the device's free memory unchanged (cudaMemGetInfo)."""
    import torch

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    pixels = 1 << 20
    pixel_loss = torch.rand(pixels * 4, dtype=torch.float32, device="cuda")
    sums = torch.zeros(4, dtype=torch.float64, device="cuda")
    assert _noalloc_sums(lib, 0, pixel_loss, pixels, sums, stream) == _lib.SP_OK
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(0)
    for _ in range(3):
        assert _noalloc_sums(lib, 0, pixel_loss, pixels, sums, stream) == _lib.SP_OK
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(0)
    assert free_after == free_before
    want = pixel_loss.view(-1, 4).double().sum(dim=0).cpu().numpy()
    assert np.allclose(sums.cpu().numpy(), want, rtol=1e-12, atol=0.0)


def test_noalloc_rejects_misaligned_buffers(ctx):
    """The kernel reads float4 pixels and writes double sums: sub-views that are not aligned
    for them are refused on the host, before anything is enqueued."""
    import torch

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    pixel_loss = torch.zeros(64, dtype=torch.float32, device="cuda")
    sums = torch.zeros(8, dtype=torch.float64, device="cuda")
    misaligned_pixels = ctypes.c_void_p(pixel_loss.data_ptr() + 4)
    misaligned_sums = ctypes.c_void_p(sums.data_ptr() + 4)
    good_pixels = ctypes.c_void_p(pixel_loss.data_ptr())
    good_sums = ctypes.c_void_p(sums.data_ptr())
    s = ctypes.c_void_p(stream)
    assert lib.sp_loss_sums_noalloc(0, misaligned_pixels, 8, good_sums, s) == _lib.SP_ERR_INVALID
    assert lib.sp_loss_sums_noalloc(0, good_pixels, 8, misaligned_sums, s) == _lib.SP_ERR_INVALID
    assert lib.sp_loss_sums_noalloc(0, good_pixels, 8, good_sums, s) == _lib.SP_OK
    torch.cuda.synchronize()
