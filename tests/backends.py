"""Two implementations of the same small interface, so that the reference's tests can be
run both on the CPU oracle (the checker) and on the CUDA path through the C ABI:

    render(packed) -> rgbt            forward pass of `packed` at the backend's camera
    backward(packed, weights) -> (param gradients, camera gradient[14], densify stats)
    loss(rgbt, ground_truth) -> (pixel_loss, loss_gradient)
    set_camera(camera)
"""

from __future__ import annotations

import numpy as np

import oracle
import splat_b200 as sb


class OracleBackend:
    name = "oracle"

    def __init__(self, n: int, camera: sb.PinholeCamera, sh_degree: int = 0, ground_truth=None):
        self.n = n
        self.sh_degree = sh_degree
        self.ground_truth = ground_truth
        self.stats = np.zeros((n, 4), np.float32)
        self.set_camera(camera)

    def set_camera(self, camera: sb.PinholeCamera) -> None:
        self.camera = camera
        self.cam = oracle.camera_array(camera.uniform())

    def render(self, packed: np.ndarray) -> np.ndarray:
        return oracle.render(np.ascontiguousarray(packed, np.float32), self.sh_degree, self.cam)["image"]

    def backward(self, packed: np.ndarray, weights: np.ndarray):
        packed = np.ascontiguousarray(packed, np.float32)
        fwd = oracle.render(packed, self.sh_degree, self.cam)
        out = oracle.backward(packed, self.sh_degree, self.cam, fwd, np.ascontiguousarray(weights, np.float32),
                              self.stats)
        return out["param_gradients"], out["camera_gradient"], self.stats.copy()

    def loss(self, rgbt: np.ndarray):
        w, h = self.camera.width, self.camera.height
        partials = oracle.ssim(rgbt, self.ground_truth, w, h)
        grad, pixel_loss = oracle.loss(rgbt, self.ground_truth, partials, w, h)
        return pixel_loss, grad


class CudaBackend:
    name = "cuda"

    def __init__(self, n: int, camera: sb.PinholeCamera, sh_degree: int = 0, ground_truth=None,
                 backward_mode: int = sb.SP_BWD_DETERMINISTIC):
        import torch

        self.torch = torch
        self.ctx = sb.Context(0)
        self.n = n
        self.sh_degree = sh_degree
        stride = sb.param_stride(sh_degree)
        self.params = torch.zeros(n * stride, dtype=torch.float32, device="cuda")
        gt = ground_truth if ground_truth is not None else np.zeros(camera.width * camera.height * 4, np.float32)
        self.gt = torch.from_numpy(np.ascontiguousarray(gt, np.float32)).cuda()
        opts = sb.default_options(sh_degree=sh_degree, backward_mode=backward_mode)
        self.rast = sb.Rasterizer(self.ctx, self.params, n, camera.width, camera.height, self.gt, 1, opts)
        self.set_camera(camera)

    def set_camera(self, camera: sb.PinholeCamera) -> None:
        self.camera = camera
        self.rast.set_camera(camera)

    def _upload(self, packed) -> None:
        self.params.copy_(self.torch.from_numpy(np.ascontiguousarray(packed, np.float32)))

    def render(self, packed: np.ndarray) -> np.ndarray:
        self._upload(packed)
        return self.rast.render(self.camera).rgbt

    def backward(self, packed: np.ndarray, weights: np.ndarray):
        self._upload(packed)
        self.rast.set_camera(self.camera)
        self.rast.encode_forward()
        self.rast.write_loss_gradient(np.ascontiguousarray(weights, np.float32))
        self.rast.encode_backward()
        g = self.rast.read_camera_gradient()
        camera = np.array([g.world_to_camera_rotation_rows[r][c] for r in range(3) for c in range(3)]
                          + list(g.world_to_camera_translation) + list(g.focal), np.float32)
        return self.rast.read_param_gradients(), camera, self.rast.read_densify_stats()

    def loss(self, rgbt: np.ndarray):
        self.rast.write_image(np.ascontiguousarray(rgbt, np.float32))
        self.rast.encode_loss(0)
        return self.rast.read_pixel_loss(), self.rast.read_loss_gradient()
