"""View-sharded data parallelism over one node: each rank renders its own views with the
parameters replicated, the parameter gradients are summed across ranks, then the parameters
take one Adam step identical on every rank. The reference trains one view per step on one
device (instantsplat-rs/src/training.rs:197-229); with one rank this is exactly that step.

Two exchanges, through torch.distributed (NCCL over NVLink on GPUs, gloo on CPU) on the
buffers the library and the caller own, viewed as tensors without a copy:

- "sharded" (when the Gaussians split evenly over the ranks): a reduce-scatter of the
  gradients, so that each rank holds the summed gradients of its own contiguous share of
  the Gaussians; Adam (and the scale clamp) on that share only (sp_adam_step_range); an
  all-gather of the updated parameters. The same bytes cross NVLink as with an all-reduce,
  and each rank does 1/world of the Adam work.
- "allreduce": one all-reduce (sum) of the gradients, then the full Adam step on every rank.
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


def even_shards(gaussians: int, world: int) -> bool:
    """Whether the sharded exchange applies: equal whole-Gaussian shares for every rank."""
    return world > 1 and gaussians % world == 0


class GradientExchange:
    """The step's exchange and Adam update for one rank (see the module docstring).

    `params` and `gradients` are flat tensors of gaussians * stride floats (the caller's
    parameter buffer and the rasterizer's gradient buffer); `adam` steps `params` from
    `gradients`."""

    def __init__(self, adam, params, gradients, gaussians: int, stride: int, rank: int, world: int,
                 mode: str | None = None, group=None):
        if mode is None:
            mode = "sharded" if even_shards(gaussians, world) else "allreduce"
        if mode == "sharded" and not even_shards(gaussians, world):
            raise ValueError(f"{gaussians} Gaussians do not split evenly over {world} ranks")
        if mode not in ("sharded", "allreduce"):
            raise ValueError(f"unknown exchange {mode!r}")
        self.adam, self.params, self.gradients = adam, params, gradients
        self.rank, self.world, self.mode, self.group = rank, world, mode, group
        self.share = gaussians // world
        self.first = rank * self.share
        lo, hi = self.first * stride, (self.first + self.share) * stride
        self.gradient_shard = gradients[lo:hi]
        self.param_shard = params[lo:hi]

    def __call__(self, rate_factor: float) -> None:
        import torch.distributed as dist

        if self.world == 1:
            self.adam.encode_step(rate_factor)
        elif self.mode == "sharded":
            # In place: each rank's share of the gradient buffer receives the sum over ranks.
            dist.reduce_scatter_tensor(self.gradient_shard, self.gradients, group=self.group)
            self.adam.advance(rate_factor)
            self.adam.step_range(self.first, self.share)
            dist.all_gather_into_tensor(self.params, self.param_shard, group=self.group)
        else:
            dist.all_reduce(self.gradients, group=self.group)
            self.adam.encode_step(rate_factor)


class ViewShardedStep:
    """One training step on this rank: set the camera of its view, forward, loss,
    backward, the gradient exchange and Adam (the scale clamp fused)."""

    def __init__(self, rasterizer, adam, params, uniforms, rank: int, world: int, mode: str | None = None,
                 group=None):
        self.rasterizer = rasterizer
        self.adam = adam
        self.uniforms = uniforms
        self.rank = rank
        self.world = world
        self.exchange = GradientExchange(adam, params, rasterizer.param_gradients(), rasterizer.gaussian_count,
                                         rasterizer.stride, rank, world, mode, group)

    def __call__(self, step: int, rate_factor: float) -> int:
        view = view_of(step, self.rank, self.world, len(self.uniforms))
        r = self.rasterizer
        r.set_camera(self.uniforms[view])
        r.encode_forward()
        r.encode_loss(view)
        if self.world == 1:
            # Backward with the Adam step fused into the projection backward.
            r.encode_backward_adam(self.adam, rate_factor)
        else:
            r.encode_backward()
            self.exchange(rate_factor)
        return view
