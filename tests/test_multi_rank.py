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


def _stats_and_gradient(oracle, camera, gt_view, packed, stats):
    cam = oracle.camera_array(camera.uniform())
    fwd = oracle.render(packed, 0, cam)
    partials = oracle.ssim(fwd["image"], gt_view, camera.width, camera.height)
    loss_gradient, _ = oracle.loss(fwd["image"], gt_view, partials, camera.width, camera.height)
    return oracle.backward(packed, 0, cam, fwd, loss_gradient, stats)["param_gradients"]


_DENSIFY_ARGS = dict(extent=0.15, seed=3)


def _densify_packed(cloud):
    """The scene's Gaussians with every other one three e-folds smaller, so that the
    densification both splits (large) and clones (small) after Adam's scale clamp."""
    packed = cloud.to_packed().copy()
    packed.reshape(-1, 14)[::2, 3:6] -= 3.0
    return packed


def _settings():
    import splat_b200 as sb

    # A low threshold, and splits above ln(0.1 * 0.15) = -4.2 (the clamp caps the log scales
    # at ln(0.02) = -3.9).
    return sb.DensifySettings(**{**sb.DENSIFY_SHORT_RUN.__dict__, "gradient_threshold": 1e-6,
                                 "split_scale_fraction": 0.1})


def _densify_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch
    import torch.distributed as dist

    sys.path[:0] = [str(ROOT / "splatting-rs_b200"), str(ROOT / "oracle")]
    import oracle
    import splat_b200 as sb
    from splat_b200.sharding import GradientExchange, merge_densify_stats

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cloud, cams, gt = _scene()
    params = torch.from_numpy(_densify_packed(cloud))
    gradients = torch.zeros_like(params)
    lr = sb.LEARNING_RATES_3DGS.by_slot(np.float32(1.0), 14)
    adam = _OracleAdam(oracle, params.numpy(), gradients.numpy(), lr)
    exchange = GradientExchange(adam, params, gradients, len(cloud), 14, rank, world, "sharded")
    stats = torch.zeros((len(cloud), 4), dtype=torch.float32)
    for step in range(2):
        view = view_of(step, rank, world, len(cams))
        gradients.copy_(torch.from_numpy(_stats_and_gradient(oracle, cams[view], gt[view], params.numpy(),
                                                             stats.numpy())))
        exchange(1.0)
    merge_densify_stats(stats)
    first, second = torch.from_numpy(adam.m), torch.from_numpy(adam.v)
    exchange.gather_moments(first, second)
    p, m, v, report = oracle.densify(params.numpy(), first.numpy(), second.numpy(), stats.numpy(), 14,
                                     _DENSIFY_ARGS["extent"], 10 * len(cloud), _settings().to_c(), 0,
                                     _DENSIFY_ARGS["seed"])
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), p=p, m=m, v=v, stats=stats.numpy(),
             split=report["split"], cloned=report["cloned"])
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_densify_as_one_process():
    """Densification after two view-sharded steps on two ranks: the ranks' statistics merged
    (sums, largest radius) and the sharded moments gathered, then the same densify on each
    rank: both ranks equal, and equal to one process that summed both views' gradients and
    merged the two ranks' statistics the same way."""
    import tempfile

    import torch.multiprocessing as mp

    import oracle
    import splat_b200 as sb

    world = 2
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_densify_rank_main, args=(world, _free_port(), out), nprocs=world, join=True,
                           start_method="spawn")
        ranks = [dict(np.load(os.path.join(out, f"rank{r}.npz"))) for r in range(world)]
    for key in ("p", "m", "v", "stats"):
        assert np.array_equal(ranks[0][key], ranks[1][key]), key
    assert ranks[0]["split"] > 0 and ranks[0]["cloned"] > 0

    cloud, cams, gt = _scene()
    packed = _densify_packed(cloud)
    m, v = np.zeros_like(packed), np.zeros_like(packed)
    lr = sb.LEARNING_RATES_3DGS.by_slot(np.float32(1.0), 14)
    per_rank = [np.zeros((len(cloud), 4), np.float32) for _ in range(world)]
    for step in range(2):
        grads = []
        for r in range(world):
            view = view_of(step, r, world, len(cams))
            grads.append(_stats_and_gradient(oracle, cams[view], gt[view], packed, per_rank[r]))
        oracle.adam_step(packed, grads[0] + grads[1], m, v, 14, lr, step + 1, float(np.log(np.float32(0.02))),
                         float(np.log(np.float32(10.0))))
    merged = per_rank[0] + per_rank[1]
    merged[:, 2] = np.maximum(per_rank[0][:, 2], per_rank[1][:, 2])
    merged[:, 3] = 0.0
    assert np.array_equal(ranks[0]["stats"], merged)
    p, mm, vv, _ = oracle.densify(packed, m, v, merged, 14, _DENSIFY_ARGS["extent"], 10 * len(cloud),
                                  _settings().to_c(), 0, _DENSIFY_ARGS["seed"])
    assert np.array_equal(ranks[0]["p"], p) and np.array_equal(ranks[0]["m"], mm) and np.array_equal(ranks[0]["v"], vv)


class _FakeRasterizer:
    gaussian_count = 1000
    stride = 14

    def param_gradients(self):
        import torch

        return torch.zeros(self.gaussian_count * self.stride)


def test_the_exchange_choice(monkeypatch):
    """make_exchange: the peer exchange by default where the Gaussians split evenly, the NCCL
    sharded one when the ranks cannot map each other's buffers (every rank learns it in the
    set-up's collectives), the all-reduce when they do not split evenly."""
    import torch

    from splat_b200 import sharding

    calls = []

    class Failing:
        def __init__(self, *args, **kwargs):
            calls.append(args)
            raise RuntimeError("a rank could not export its buffers for the peer exchange")

    monkeypatch.setattr(sharding, "_PeerExchange", Failing)
    params = torch.zeros(1000 * 14)
    chosen = sharding.make_exchange(None, params, _FakeRasterizer(), 0, 2)
    assert chosen.mode == "sharded" and len(calls) == 1
    uneven = _FakeRasterizer()
    uneven.gaussian_count = 1001
    assert sharding.make_exchange(None, torch.zeros(1001 * 14), uneven, 0, 2).mode == "allreduce"
    assert sharding.make_exchange(None, params, _FakeRasterizer(), 0, 1).mode == "allreduce"
    with pytest.raises(RuntimeError):
        sharding.make_exchange(None, params, _FakeRasterizer(), 0, 2, mode="peer")
