"""The multi-GPU step through the library alone (sp_comm_*, sp_exchange_*): no
torch.distributed anywhere in these processes; torch only provides device memory. The
communicator's 128-byte id travels from rank 0 to the others over a multiprocessing queue, as a
Rust caller would pass it over any host channel.

- Two GPUs, each rank accumulating a block of two views per step (the batch semantic: every
  rank's views, then one Adam step), through each exchange mode: the parameters equal, bit for
  bit in the deterministic backward, one GPU accumulating the same blocks, summing the blocks'
  gradients in rank order and taking one Adam step. Then the densify statistics merged through
  the communicator equal on both ranks and sum the visible counts.
- One GPU: a communicator of two ranks whose second rank never joins gives up after its time
  limit with SP_ERR_TIMEOUT (host-side wait; no GPU wait is involved).
"""

from __future__ import annotations

import os
import sys
import time
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu

STEPS = 3
VIEWS_PER_RANK = 2
WORLD = 2


def _scene():
    sys.path[:0] = [str(ROOT / "splatting-rs_b200"), str(ROOT / "tests")]
    import splat_b200 as sb
    from helpers import random_cloud

    rng = np.random.default_rng(23)
    cloud = random_cloud(4000, rng, sh_degree=1)
    cams = [sb.PinholeCamera(np.eye(3), np.array([0.12 * v, 0.04 * v, 0.0]), (150.0, 150.0), (80, 60), 160, 120)
            for v in range(WORLD * VIEWS_PER_RANK)]
    gt = rng.uniform(0.0, 1.0, (len(cams), 160 * 120 * 4)).astype(np.float32)
    gt[:, 3::4] = (gt[:, 3::4] > 0.5).astype(np.float32)
    return cloud, cams, gt


def _rank_main(rank: int, queues, out_dir: str, modes) -> None:
    import torch

    sys.path[:0] = [str(ROOT / "splatting-rs_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import splat_b200 as sb
    from splat_b200.comm import Communicator
    from splat_b200.sharding import ViewShardedStep

    torch.cuda.set_device(rank)
    ctx = sb.Context(rank)
    if rank == 0:
        uid = Communicator.unique_id()
        for q in queues[1:]:
            q.put(uid)
    else:
        uid = queues[rank].get(timeout=60)
    comm = Communicator(ctx, uid, WORLD, rank, timeout_ms=60_000)
    cloud, cams, gt = _scene()
    gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
    opts = sb.default_options(sh_degree=1, backward_mode=sb.SP_BWD_DETERMINISTIC, accumulate_gradients=True)
    for mode in modes:
        params = torch.from_numpy(cloud.to_packed()).cuda()
        rast = sb.Rasterizer(ctx, params, len(cloud), 160, 120, gt_dev, len(cams), opts)
        adam = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, 2.0, sh_degree=1)
        rast.clear_densify_stats()
        step = ViewShardedStep(rast, adam, params, [c.uniform() for c in cams], rank, WORLD, mode=mode, comm=comm,
                               views_per_rank=VIEWS_PER_RANK)
        assert step.exchange.mode == mode, (step.exchange.mode, mode)
        for s in range(STEPS):
            step(s, sb.position_rate_factor(s, 10))
        comm.wait()
        np.save(os.path.join(out_dir, f"{mode}{rank}.npy"), params.cpu().numpy())
        if mode == modes[-1]:
            comm.merge_densify_stats(rast)
            np.save(os.path.join(out_dir, f"stats{rank}.npy"), rast.read_densify_stats())
        step.exchange.close()
        comm.barrier()
        comm.wait()
        rast.close()
        adam.close()
    comm.close()


def test_two_gpus_through_the_library_alone(ctx, tmp_path):
    import torch
    import torch.multiprocessing as mp

    import splat_b200 as sb
    from splat_b200.sharding import views_of

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    modes = ["peer", "sharded", "allreduce"]
    spawn = mp.get_context("spawn")
    queues = [spawn.Queue() for _ in range(WORLD)]
    procs = [spawn.Process(target=_rank_main, args=(r, queues, str(tmp_path), modes)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    # One GPU: each step, every rank's block accumulated on its own, the blocks summed in rank
    # order, one Adam step.
    cloud, cams, gt = _scene()
    params = torch.from_numpy(cloud.to_packed()).cuda()
    gt_dev = torch.from_numpy(gt.reshape(-1)).cuda()
    opts = sb.default_options(sh_degree=1, backward_mode=sb.SP_BWD_DETERMINISTIC, accumulate_gradients=True)
    rast = sb.Rasterizer(ctx, params, len(cloud), 160, 120, gt_dev, len(cams), opts)
    adam = sb.Adam(ctx, params, rast, len(cloud), sb.LEARNING_RATES_3DGS, 2.0, sh_degree=1)
    gradients = rast.param_gradients()
    for s in range(STEPS):
        total = None
        for r in range(WORLD):
            rast.zero_param_gradients()
            for v in views_of(s, r, WORLD, len(cams), VIEWS_PER_RANK):
                rast.set_camera(cams[v])
                rast.encode_forward()
                rast.encode_loss(v)
                rast.encode_backward()
            block = rast.read_param_gradients()
            total = block if total is None else total + block
        gradients.copy_(torch.from_numpy(total).cuda())
        adam.encode_step(sb.position_rate_factor(s, 10))
    ctx.sync()
    want = params.cpu().numpy().view(np.uint32)
    for mode in modes:
        for r in range(WORLD):
            got = np.load(tmp_path / f"{mode}{r}.npy").view(np.uint32)
            assert np.array_equal(got, want), f"{mode}, rank {r}: parameters differ from one GPU's"
    stats = [np.load(tmp_path / f"stats{r}.npy") for r in range(WORLD)]
    assert np.array_equal(stats[0], stats[1])
    # Each rank saw each Gaussian at most once per view: the merged visible counts reach the
    # views of both ranks.
    assert stats[0][:, 1].max() > STEPS * VIEWS_PER_RANK


def _lonely_rank(out: str) -> None:
    sys.path[:0] = [str(ROOT / "splatting-rs_b200")]
    import splat_b200 as sb
    from splat_b200.comm import Communicator

    ctx = sb.Context(0)
    uid = Communicator.unique_id()
    start = time.monotonic()
    try:
        Communicator(ctx, uid, 2, 0, timeout_ms=2000)
        status = 0
    except sb.SplatError as e:
        status = e.status
    Path(out).write_text(f"{status} {time.monotonic() - start:.3f}")


def test_comm_init_gives_up_when_a_rank_never_joins(tmp_path):
    import torch.multiprocessing as mp

    from splat_b200 import _lib

    out = tmp_path / "lonely.txt"
    spawn = mp.get_context("spawn")
    p = spawn.Process(target=_lonely_rank, args=(str(out),))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 0
    status, seconds = out.read_text().split()
    assert int(status) == _lib.SP_ERR_TIMEOUT
    assert 1.5 <= float(seconds) < 60.0
