"""The view-sharded multi-rank path on CPU: 2 gloo ranks, the gradients of each rank's view
from the oracle, summed by all_reduce, then Adam — must equal one process summing the same
views' gradients and stepping once. Also the shard arithmetic. No GPU involved."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

from splat_b200.sharding import shard_range, view_of

ROOT = Path(__file__).resolve().parents[1]


def test_view_assignment_covers_every_view_once_per_cycle():
    views, world = 24, 4
    for step in range(0, 12):
        got = [view_of(step, r, world, views) for r in range(world)]
        assert got == [(step * world + r) % views for r in range(world)]
    seen = [view_of(s, r, world, views) for s in range(views // world) for r in range(world)]
    assert sorted(seen) == list(range(views))
    assert [view_of(s, 0, 1, 3) for s in range(5)] == [0, 1, 2, 0, 1]  # one rank: training.rs:227


@pytest.mark.parametrize("count,world", [(1000, 2), (1037, 4), (5, 8), (0, 2)])
def test_shards_partition_the_range(count, world):
    shards = [shard_range(count, r, world) for r in range(world)]
    covered = []
    for first, n in shards:
        assert first % 4 == 0 or n == 0
        covered.extend(range(first, first + n))
    assert covered == list(range(count))


def _scene():
    sys.path.insert(0, str(ROOT / "tests"))
    import splat_b200 as sb
    from helpers import random_cloud

    rng = np.random.default_rng(2)
    cloud = random_cloud(300, rng)
    cams = [sb.PinholeCamera(np.eye(3), np.array([0.1 * v, 0.0, 0.0]), (60.0, 60.0), (32, 24), 64, 48)
            for v in range(4)]
    gt = rng.uniform(0.0, 1.0, (len(cams), 64 * 48 * 4)).astype(np.float32)
    gt[:, 3::4] = (gt[:, 3::4] > 0.5).astype(np.float32)
    return cloud, cams, gt


def _gradient(oracle, cloud, camera, gt_view, packed):
    cam = oracle.camera_array(camera.uniform())
    fwd = oracle.render(packed, 0, cam)
    partials = oracle.ssim(fwd["image"], gt_view, camera.width, camera.height)
    loss_gradient, _ = oracle.loss(fwd["image"], gt_view, partials, camera.width, camera.height)
    return oracle.backward(packed, 0, cam, fwd, loss_gradient)["param_gradients"]


class _OracleAdam:
    """The CPU oracle's Adam behind the interface GradientExchange drives (encode_step,
    advance + step_range), over numpy views of the exchange's tensors."""

    def __init__(self, oracle, params, gradients, lr):
        self.oracle, self.params, self.gradients, self.lr = oracle, params, gradients, lr
        self.m, self.v = np.zeros_like(params), np.zeros_like(params)
        self.step = 0

    def _apply(self, first: int, count: int) -> None:
        lo, hi = first * 14, (first + count) * 14
        self.oracle.adam_step(self.params[lo:hi], self.gradients[lo:hi], self.m[lo:hi], self.v[lo:hi], 14, self.lr,
                              self.step, float(np.log(np.float32(0.02))), float(np.log(np.float32(10.0))))

    def encode_step(self, rate_factor: float) -> None:
        self.advance(rate_factor)
        self._apply(0, len(self.params) // 14)

    def advance(self, rate_factor: float) -> None:
        self.step += 1

    def step_range(self, first: int, count: int) -> None:
        self._apply(first, count)


def _rank_main(rank: int, world: int, port: int, out_dir: str, mode: str, chunks: int) -> None:
    import torch
    import torch.distributed as dist

    sys.path[:0] = [str(ROOT / "splatting-rs_b200"), str(ROOT / "oracle")]
    import oracle
    import splat_b200 as sb
    from splat_b200.sharding import GradientExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cloud, cams, gt = _scene()
    params = torch.from_numpy(cloud.to_packed().copy())
    gradients = torch.zeros_like(params)
    lr = sb.LEARNING_RATES_3DGS.by_slot(np.float32(1.0), 14)
    adam = _OracleAdam(oracle, params.numpy(), gradients.numpy(), lr)
    exchange = GradientExchange(adam, params, gradients, len(cloud), 14, rank, world, mode, chunks=chunks)
    for step in range(2):
        view = view_of(step, rank, world, len(cams))
        gradients.copy_(torch.from_numpy(_gradient(oracle, cloud, cams[view], gt[view], params.numpy())))
        exchange(1.0)
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), params.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode,chunks", [("allreduce", 1), ("sharded", 1), ("sharded", 4)])
def test_two_gloo_ranks_equal_one_process_summing_their_views(tmp_path, mode, chunks):
    """Two ranks, each the gradient of its own view, exchanged by an all-reduce or by a
    reduce-scatter + Adam on each rank's half + all-gather (in place, as on the GPUs; whole,
    or range by range with asynchronous collectives): the same parameters on both ranks,
    equal to one process summing both views' gradients."""
    import torch.multiprocessing as mp

    import oracle
    import splat_b200 as sb

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), mode, chunks), nprocs=world,
                       join=True, start_method="spawn")
    ranks = [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]
    assert np.array_equal(ranks[0], ranks[1]), "ranks diverged"
    # One process: the same two steps, each summing the gradients of views
    # step*world .. step*world + world - 1 in rank order.
    cloud, cams, gt = _scene()
    packed = cloud.to_packed().copy()
    m, v = np.zeros_like(packed), np.zeros_like(packed)
    lr = sb.LEARNING_RATES_3DGS.by_slot(np.float32(1.0), 14)
    for step in range(2):
        grads = [_gradient(oracle, cloud, cams[view_of(step, r, world, len(cams))], gt[view_of(step, r, world, len(cams))],
                           packed) for r in range(world)]
        total = grads[0] + grads[1]
        oracle.adam_step(packed, total, m, v, 14, lr, step + 1, float(np.log(np.float32(0.02))),
                         float(np.log(np.float32(10.0))))
    assert np.array_equal(ranks[0], packed)
