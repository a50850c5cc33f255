"""Error paths of the device side that no normal frame reaches.

- The sort's decoupled look-back is the one place a kernel waits on another block. Its wait
  is bounded: after its iteration limit it raises SP_ERR_TIMEOUT in the frame's status word
  and returns. sp_debug_stall_sort_partition makes one partition never post, so that the
  next one's wait runs out (with a short limit): the error must come back through
  sp_read_intersections and sp_train_step, the context must stay usable, and the next
  frame with the switch off must equal a frame that never timed out.
- Overflow of the intersection list: the reference's read_step_async -> read_intersections
  panics (training.rs:271, rasterizer.rs:536-544); sp_train_step returns SP_ERR_OVERFLOW.

No GPU fault is provoked: the stalled wait ends on its own limit and every access stays in
bounds (the timed-out frame's tile ranges are left empty).
"""

from __future__ import annotations

import numpy as np
import pytest

import splat_b200 as sb
from helpers import make_rasterizer
from splat_b200 import _lib, scenes

pytestmark = pytest.mark.gpu

SORT_PARTITION = 6144  # kSortPartition: keys per onesweep partition


def _status(excinfo) -> int:
    return excinfo.value.status


def test_lookback_wait_runs_out_and_the_context_recovers(ctx):
    scene = scenes.config(0, scale=0.5)
    cam = scene.cameras[0]
    rast, params, _ = make_rasterizer(ctx, scene.cloud, cam, backward_mode=sb.SP_BWD_DETERMINISTIC)
    rast.encode_forward()
    meta = rast.read_intersections()
    assert meta.count > 3 * SORT_PARTITION, "the case needs several sort partitions"
    keys, gaussians = rast.read_sorted_intersections()
    image = rast.read_image().rgbt

    # Partition 0 never posts: partition 1's wait runs out.
    rast.debug_stall_sort_partition(0)
    rast.encode_forward()
    with pytest.raises(sb.SplatError) as e:
        rast.read_intersections()
    assert _status(e) == _lib.SP_ERR_TIMEOUT
    # The status was reported once and cleared; the frame rendered nothing (empty ranges).
    assert np.all(rast.read_tile_ranges() == 0)

    rast.debug_stall_sort_partition(None)
    rast.encode_forward()
    rast.read_intersections()
    k2, g2 = rast.read_sorted_intersections()
    assert np.array_equal(k2, keys) and np.array_equal(g2, gaussians)
    assert np.array_equal(rast.read_image().rgbt, image)

    # The one-call training step reports the timeout too, and the next step succeeds.
    adam = sb.Adam(ctx, params, rast, len(scene.cloud), sb.LEARNING_RATES_3DGS, 3.3)
    rast.debug_stall_sort_partition(1)
    with pytest.raises(sb.SplatError) as e:
        rast.train_step(adam, cam, 0, 1.0)
    assert _status(e) == _lib.SP_ERR_TIMEOUT
    rast.debug_stall_sort_partition(None)
    gradient, loss = rast.train_step(adam, cam, 0, 1.0)
    assert np.isfinite(loss.total)
    rast.read_intersections()


def test_stalling_a_partition_past_the_last_changes_nothing(ctx):
    scene = scenes.config(0, scale=0.25)
    cam = scene.cameras[1]
    rast, _, _ = make_rasterizer(ctx, scene.cloud, cam)
    rast.encode_forward()
    keys, _ = rast.read_sorted_intersections()
    rast.debug_stall_sort_partition(1 << 20)
    rast.encode_forward()
    rast.read_intersections()
    k2, _ = rast.read_sorted_intersections()
    assert np.array_equal(k2, keys)


def test_train_step_reports_overflow(ctx):
    """One intersection per Gaussian cannot hold Gaussians that cover several tiles: the step
    runs on the truncated list and sp_train_step returns SP_ERR_OVERFLOW."""
    scene = scenes.config(0, scale=0.1)
    cam = scene.cameras[0]
    rast, params, _ = make_rasterizer(ctx, scene.cloud, cam, intersections_per_gaussian=1)
    adam = sb.Adam(ctx, params, rast, len(scene.cloud), sb.LEARNING_RATES_3DGS, 3.3)
    with pytest.raises(sb.SplatError) as e:
        rast.train_step(adam, cam, 0, 1.0)
    assert _status(e) == _lib.SP_ERR_OVERFLOW
    with pytest.raises(sb.SplatError) as e:
        rast.read_intersections()
    assert _status(e) == _lib.SP_ERR_OVERFLOW
    # With room for the list the same step succeeds.
    ok, ok_params, _ = make_rasterizer(ctx, scene.cloud, cam)
    ok_adam = sb.Adam(ctx, ok_params, ok, len(scene.cloud), sb.LEARNING_RATES_3DGS, 3.3)
    ok.train_step(ok_adam, cam, 0, 1.0)
