"""Two GPUs against one GPU with the same batch (the multi-GPU check of the view-sharded
step): each of two NCCL ranks renders its own view, the gradients are reduce-scattered,
Adam runs on each rank's half of the Gaussians and the parameters are all-gathered. One GPU
accumulates the same two views' gradients (in rank order) and takes one full Adam step. In
the deterministic backward the parameters agree bit for bit, with the NCCL exchange
("sharded") and with the peer-memory one ("peer": one kernel per rank sums the ranks'
gradients over NVLink, steps Adam on its share and stores the parameters into both ranks'
buffers). Needs two GPUs; skipped on one."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu

STEPS = 3


def _scene():
    sys.path[:0] = [str(ROOT / "splatting-rs_b200"), str(ROOT / "tests")]
    import splat_b200 as sb
    from helpers import random_cloud

    rng = np.random.default_rng(11)
    cloud = random_cloud(4000, rng, sh_degree=1)
    cams = [sb.PinholeCamera(np.eye(3), np.array([0.15 * v, 0.05 * v, 0.0]), (150.0, 150.0), (80, 60), 160, 120)
            for v in range(4)]
    gt = rng.uniform(0.0, 1.0, (len(cams), 160 * 120 * 4)).astype(np.float32)
    gt[:, 3::4] = (gt[:, 3::4] > 0.5).astype(np.float32)
    return cloud, cams, gt


def _rank_main(rank: int, world: int, port: int, out_dir: str, mode: str) -> None:
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    sys.path[:0] = [str(ROOT / "splatting-rs_b200")]
    import splat_b200 as sb
    from splat_b200.sharding import ViewShardedStep

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cloud, cams, gt = _scene()
    ctx = sb.Context(rank)
    params = torch.from_numpy(cloud.to_packed()).cuda()
    gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
    opts = sb.default_options(sh_degree=1, backward_mode=sb.SP_BWD_DETERMINISTIC)
    rast = sb.Rasterizer(ctx, params, len(cloud), 160, 120, gt_dev, len(cams), opts)
    adam = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, 2.0, sh_degree=1)
    step = ViewShardedStep(rast, adam, params, [c.uniform() for c in cams], rank, world, mode=mode)
    assert step.exchange.mode == mode
    for s in range(STEPS):
        step(s, sb.position_rate_factor(s, 10))
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), params.cpu().numpy())
    dist.barrier()
    step.exchange.close()
    dist.barrier()
    dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["sharded", "peer"])
def test_two_gpus_equal_one_gpu_with_the_same_batch(ctx, tmp_path, mode):
    import torch
    import torch.multiprocessing as mp

    import splat_b200 as sb
    from splat_b200.sharding import view_of

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), mode), nprocs=world, join=True,
                       start_method="spawn")
    ranks = [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]
    assert np.array_equal(ranks[0], ranks[1]), "the ranks' parameters diverged"

    cloud, cams, gt = _scene()
    params = torch.from_numpy(cloud.to_packed()).cuda()
    gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
    opts = sb.default_options(sh_degree=1, backward_mode=sb.SP_BWD_DETERMINISTIC, accumulate_gradients=True)
    rast = sb.Rasterizer(ctx, params, len(cloud), 160, 120, gt_dev, len(cams), opts)
    adam = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, 2.0, sh_degree=1)
    for s in range(STEPS):
        rast.zero_param_gradients()
        for r in range(world):
            v = view_of(s, r, world, len(cams))
            rast.set_camera(cams[v])
            rast.encode_forward()
            rast.encode_loss(v)
            rast.encode_backward()
        adam.encode_step(sb.position_rate_factor(s, 10))
    ctx.sync()
    assert np.array_equal(params.cpu().numpy().view(np.uint32), ranks[0].view(np.uint32))


def _densify_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    sys.path[:0] = [str(ROOT / "splatting-rs_b200")]
    import splat_b200 as sb
    from splat_b200.sharding import ViewShardedStep

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cloud, cams, gt = _scene()
    ctx = sb.Context(rank)
    params = torch.from_numpy(cloud.to_packed()).cuda()
    gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
    opts = sb.default_options(sh_degree=1, backward_mode=sb.SP_BWD_DETERMINISTIC)
    rast = sb.Rasterizer(ctx, params, len(cloud), 160, 120, gt_dev, len(cams), opts)
    adam = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, 2.0, sh_degree=1)
    step = ViewShardedStep(rast, adam, params, [c.uniform() for c in cams], rank, world)
    assert step.exchange.mode == "peer"
    settings = sb.DensifySettings(**{**sb.DENSIFY_SHORT_RUN.__dict__, "gradient_threshold": 1e-5})
    for s in range(STEPS):
        step(s, sb.position_rate_factor(s, 10))
    report = step.densify(settings, 2.0, settings.max_count(len(cloud)), False, 0)
    for s in range(STEPS, STEPS + 2):
        step(s, sb.position_rate_factor(s, 10))
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"densified{rank}.npy"), step.params.cpu().numpy())
    np.save(os.path.join(out_dir, f"report{rank}.npy"), np.array([report.before, report.after, report.split]))
    dist.barrier()
    step.exchange.close()
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpus_densify_identically(tmp_path):
    """Three view-sharded steps on two GPUs, a densification (statistics merged, moment shards
    gathered, then the same densify on each rank), two more steps: both ranks hold the same
    Gaussians, at a count the densification changed."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.start_processes(_densify_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    reports = [np.load(tmp_path / f"report{r}.npy") for r in range(world)]
    assert np.array_equal(reports[0], reports[1]) and reports[0][1] != reports[0][0]
    ranks = [np.load(tmp_path / f"densified{r}.npy") for r in range(world)]
    assert np.array_equal(ranks[0].view(np.uint32), ranks[1].view(np.uint32))
