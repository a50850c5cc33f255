"""View-sharded data parallelism over one node: each rank renders its own views with the
parameters replicated, the parameter gradients are summed across ranks, then every rank
takes the same Adam step. The reference trains one view per step on one device
(instantsplat-rs/src/training.rs:197-229); with one rank this is exactly that step.

The exchange is one all-reduce (sum) of the N * stride fp32 gradients per step, issued
through torch.distributed (NCCL over NVLink on GPUs, gloo on CPU) on the gradient buffer the
library owns, viewed as a tensor without a copy.
"""

from __future__ import annotations


def view_of(step: int, rank: int, world: int, views: int) -> int:
    """The view rank `rank` trains at `step`: ranks take consecutive views, so that one
    step of `world` ranks covers views step*world .. step*world + world - 1 (mod views)."""
    return (step * world + rank) % views


def shard_range(count: int, rank: int, world: int, align: int = 4) -> tuple[int, int]:
    """Contiguous [first, first + n) share of `count` items for `rank`, boundaries on
    multiples of `align` (so that Adam's float4 path stays aligned)."""
    per = -(-count // world)
    per = -(-per // align) * align
    first = min(rank * per, count)
    return first, max(0, min(count, first + per) - first)


class ViewShardedStep:
    """One training step on this rank: set the camera of its view, forward, loss,
    backward, sum the gradients over the ranks, Adam (the scale clamp fused)."""

    def __init__(self, rasterizer, adam, uniforms, rank: int, world: int, group=None):
        self.rasterizer = rasterizer
        self.adam = adam
        self.uniforms = uniforms
        self.rank = rank
        self.world = world
        self.group = group
        self.gradients = rasterizer.param_gradients() if world > 1 else None

    def __call__(self, step: int, rate_factor: float) -> int:
        view = view_of(step, self.rank, self.world, len(self.uniforms))
        r = self.rasterizer
        r.set_camera(self.uniforms[view])
        r.encode_forward()
        r.encode_loss(view)
        r.encode_backward()
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(self.gradients, group=self.group)
        self.adam.encode_step(rate_factor)
        return view
