"""The intersection capacity sized from the scan (the survey's capacity policy; the reference
fixes it at 24 N, rasterizer.rs:27, and panics on overflow, rasterizer.rs:536-544): after an
overflow, sp_intersections_needed gives the scan's uncapped pair count and
sp_reserve_intersections grows the lists, after which the forward pass gives the full lists
bit for bit (the oracle's), and the backward the gradients of a rasterizer created large
enough. The Trainer's "scan" policy trains as the fixed one."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import splat_b200 as sb
from helpers import make_rasterizer
from splat_b200 import scenes

pytestmark = pytest.mark.gpu


def _scene():
    s = scenes.config(0, scale=0.25)
    return s.cloud, s.cameras[1]


@pytest.mark.parametrize("mode", [sb.SP_BWD_ATOMIC, sb.SP_BWD_DETERMINISTIC])
def test_reserve_after_overflow_gives_the_full_lists(ctx, mode):
    cloud, camera = _scene()
    rast, _, _ = make_rasterizer(ctx, cloud, camera, intersections_per_gaussian=1, backward_mode=mode)
    rast.encode_forward()
    with pytest.raises(sb.SplatError) as err:
        rast.read_intersections()
    assert err.value.status == 3
    needed = rast.intersections_needed()
    want = oracle.render(cloud.to_packed(), cloud.sh_degree, oracle.camera_array(camera.uniform()))
    assert needed == len(want["keys"]) > len(cloud)
    assert str(needed) in str(err.value)  # the error names the pairs the frame needs
    rast.encode_loss(0)  # the loss of a truncated frame comes with the overflow error too
    with pytest.raises(sb.SplatError) as err:
        rast.read_loss()
    assert err.value.status == 3

    rast.reserve_intersections(needed)
    rast.reserve_intersections(needed // 2)  # never shrinks
    rast.encode_forward()
    meta = rast.read_intersections()
    assert meta.overflow == 0 and meta.count == needed and meta.capacity == needed
    keys, gauss = rast.read_sorted_intersections()
    assert np.array_equal(keys, want["keys"]) and np.array_equal(gauss, want["gauss"])

    # The backward over the grown lists equals a rasterizer created with the fixed 24 N.
    big, _, _ = make_rasterizer(ctx, cloud, camera, backward_mode=mode)
    grads = []
    for r in (rast, big):
        r.encode_forward()
        r.encode_loss(0)
        r.encode_backward()
        grads.append(r.read_param_gradients())
    if mode == sb.SP_BWD_DETERMINISTIC:
        assert np.array_equal(grads[0], grads[1])
    else:
        scale = np.max(np.abs(grads[1])) + 1e-12
        assert np.max(np.abs(grads[0] - grads[1])) <= 1e-5 * scale  # float atomics' order only
    rast.close()
    big.close()


def test_reserve_rejects_capacities_of_2_to_the_32(ctx):
    cloud, camera = _scene()
    rast, _, _ = make_rasterizer(ctx, cloud, camera)
    with pytest.raises(sb.SplatError) as err:
        rast.reserve_intersections(1 << 32)
    assert err.value.status == 1
    rast.close()


def test_trainer_scan_capacity_trains_as_the_fixed_one(ctx):
    s = scenes.config(0, scale=0.1)
    cams = s.cameras
    gt = np.zeros((len(cams), cams[0].height * cams[0].width, 4), np.float32)
    gt[..., 3] = 1.0
    losses = {}
    for policy in ("fixed", "scan"):
        trainer = sb.Trainer(s.cloud, cams, gt, ctx=ctx, backward_mode=sb.SP_BWD_DETERMINISTIC, capacity=policy)
        for step in range(6):
            trainer.train_step(step, 6)
        losses[policy] = [trainer.loss(v).total for v in range(len(cams))]
        # The last loss's forward pass: its lists fit the capacity the policy chose.
        assert trainer.rasterizer.read_intersections().overflow == 0
    assert losses["fixed"] == losses["scan"]
