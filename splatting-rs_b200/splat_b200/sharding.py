"""View-sharded data parallelism over one node: each rank renders its own views with the
parameters replicated, the parameter gradients are summed across ranks, then the parameters
take one Adam step identical on every rank. The reference trains one view per step on one
device (instantsplat-rs/src/training.rs:197-229); with one rank this is exactly that step.

With a comm.Communicator (the library's own NCCL communicator, sp_comm_*) every exchange
below runs inside libsplat_b200 (sp_exchange_*), with no torch.distributed call: the form a
caller without PyTorch uses, and the benchmark's. Without one, the same three exchanges run
through torch.distributed (NCCL over NVLink on GPUs, gloo on CPU) on the buffers the library and
the caller own, viewed as tensors without a copy:

- "sharded" (when the Gaussians split evenly over the ranks): a reduce-scatter of the
  gradients, so that each rank holds the summed gradients of its own share of the
  Gaussians; Adam (and the scale clamp) on that share only (sp_adam_step_range); an
  all-gather of the updated parameters. The same bytes cross NVLink as with an all-reduce,
  and each rank does 1/world of the Adam work. With `chunks` > 1 the Gaussians are cut
  into ranges: the projection backward runs range by range, each range's reduce-scatter is
  issued as soon as its gradients are written and runs beside the backward of the next
  ones, and each range's all-gather beside the Adam steps of the next ones; a rank's share is
  then its 1/world of every range. Measured on two B200s with 4 ranges this was slower than
  one (the ranges' backward launches end in partial waves, and the concurrent NCCL kernels
  slow the Adam steps), so one range is the default.
- "allreduce": one all-reduce (sum) of the gradients, then the full Adam step on every rank.
- "peer" (the default where it applies): no library collective for the data. One kernel per
  rank (sp_peer_exchange_step) reads its share of every rank's gradients over peer memory
  (NVLink loads from buffers mapped with CUDA IPC), sums them in rank order, steps Adam on the
  share and stores the parameters into every rank's buffer (NVLink stores); two one-element
  NCCL all-reduces on the stream order it after every rank's backward and before every rank's
  next forward. The transfer and the Adam step run in the same kernel, tile by tile.

Densification (densify.rs:147-257) with several ranks: each rank's backward passes
accumulated the densify statistics of its own views, so they are merged first (sums of the
mean-gradient sums and visible counts, the largest screen radius: what one device would
have accumulated over all the views, up to the order of the sums), and in the sharded and
peer exchanges each rank's moments are current only on its own share, so the shares are
all-gathered. Every rank then runs the same densification on the same inputs and gets the
same Gaussians (the kernels are deterministic).
"""

from __future__ import annotations

import math


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


def chunk_ranges(gaussians: int, chunks: int, world: int, align: int = 256) -> list[tuple[int, int]]:
    """`chunks` consecutive ranges covering the Gaussians, each starting on a multiple of
    `align` (the projection backward's block) with a length divisible by `world`."""
    step = align * world // math.gcd(align, world)
    size = -(-gaussians // chunks)
    size = -(-size // step) * step
    out, first = [], 0
    while first < gaussians:
        count = min(size, gaussians - first)
        out.append((first, count))
        first += count
    return out


def merge_densify_stats(stats, group=None) -> None:
    """In place on `stats` ((N, 4) float32: mean-gradient sum, visible count, max radius, pad),
    every rank's statistics merged: the first two summed, the radius the largest."""
    import torch.distributed as dist

    summed = stats.clone()
    dist.all_reduce(summed, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(stats, op=dist.ReduceOp.MAX, group=group)
    stats[:, :2] = summed[:, :2]


class GradientExchange:
    """The step's exchange and Adam update for one rank (see the module docstring).

    `params` and `gradients` are flat tensors of gaussians * stride floats (the caller's
    parameter buffer and the rasterizer's gradient buffer); `adam` steps `params` from
    `gradients`."""

    def __init__(self, adam, params, gradients, gaussians: int, stride: int, rank: int, world: int,
                 mode: str | None = None, group=None, chunks: int = 1):
        if mode is None:
            mode = "sharded" if even_shards(gaussians, world) else "allreduce"
        if mode in ("sharded", "peer") and not even_shards(gaussians, world):
            raise ValueError(f"{gaussians} Gaussians do not split evenly over {world} ranks")
        if mode not in ("sharded", "allreduce", "peer"):
            raise ValueError(f"unknown exchange {mode!r}")
        self.adam, self.params, self.gradients = adam, params, gradients
        self.rank, self.world, self.mode, self.group = rank, world, mode, group
        self.stride = stride
        self.ranges = chunk_ranges(gaussians, chunks, world) if mode == "sharded" else [(0, gaussians)]
        if mode == "sharded" and any(count % world for _, count in self.ranges):
            raise ValueError("every range must split evenly over the ranks")
        self._peer = None
        if mode == "peer":
            self._peer = _PeerExchange(adam, rank, world, group)

    def _share(self, first: int, count: int) -> tuple[int, int]:
        """This rank's part [first, first + n) of the range."""
        part = count // self.world
        return first + self.rank * part, part

    def _views(self, tensor, first: int, count: int):
        """The range and this rank's part of it, as views of a flat parameter-like tensor."""
        s = self.stride
        own, part = self._share(first, count)
        return tensor[first * s:(first + count) * s], tensor[own * s:(own + part) * s]

    def backward_step(self, project, rate_factor: float) -> None:
        """The projection backward (`project(first, count)`, e.g. the rasterizer's
        encode_backward_project), the exchange and the Adam step, the collectives of each
        range overlapping the work on the next ones."""
        import torch.distributed as dist

        if self._peer is not None:
            project(0, self.ranges[0][1])
            self._peer.step(rate_factor)
            return
        if self.world == 1 or self.mode != "sharded":
            for first, count in self.ranges:
                project(first, count)
            self(rate_factor)
            return
        scatters = []
        for first, count in self.ranges:
            project(first, count)
            whole, own = self._views(self.gradients, first, count)
            # In place: this rank's part of the range receives the sum over the ranks.
            scatters.append(dist.reduce_scatter_tensor(own, whole, group=self.group, async_op=True))
        self.adam.advance(rate_factor)
        gathers = []
        for (first, count), scatter in zip(self.ranges, scatters):
            scatter.wait()
            self.adam.step_range(*self._share(first, count))
            whole, own = self._views(self.params, first, count)
            gathers.append(dist.all_gather_into_tensor(whole, own, group=self.group, async_op=True))
        for gather in gathers:
            gather.wait()

    def __call__(self, rate_factor: float) -> None:
        """The exchange and the Adam step after a whole backward (gradients all written)."""
        if self._peer is not None:
            self._peer.step(rate_factor)
        elif self.mode == "sharded" and self.world > 1:
            self.backward_step(lambda first, count: None, rate_factor)
        else:
            self._replicated(rate_factor)

    def gather_moments(self, first, second) -> None:
        """Makes Adam's moments (flat tensors like the parameters) whole on every rank: in
        the sharded exchange each rank updated only its share of every range."""
        import torch.distributed as dist

        if self.world == 1 or self.mode not in ("sharded", "peer"):
            return
        for moment in (first, second):
            for first_gaussian, count in self.ranges:
                whole, own = self._views(moment, first_gaussian, count)
                dist.all_gather_into_tensor(whole, own, group=self.group)

    def close(self) -> None:
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def _replicated(self, rate_factor: float) -> None:
        import torch.distributed as dist

        if self.world > 1:
            dist.all_reduce(self.gradients, group=self.group)
        self.adam.encode_step(rate_factor)


def make_exchange(adam, params, rasterizer, rank: int, world: int, mode: str | None = None,
                  group=None, comm=None):
    """The exchange of `mode` for a library optimiser and rasterizer; by default the peer
    exchange when the Gaussians split evenly over several ranks (the sharded NCCL one when the
    ranks cannot map each other's buffers), else the all-reduce. With `comm` (a
    comm.Communicator) the library's own exchange (sp_exchange_*) is used, with no
    torch.distributed call; otherwise the torch.distributed forms of this module."""
    if comm is not None:
        from .comm import Exchange

        return Exchange(comm, adam, mode or "auto")
    count = rasterizer.gaussian_count
    if mode in ("sharded", "peer") and not even_shards(count, world):
        mode = None
    if mode is None and world > 1 and even_shards(count, world):
        from ._lib import SplatError

        try:
            return GradientExchange(adam, params, rasterizer.param_gradients(), count, rasterizer.stride, rank,
                                    world, "peer", group)
        except (RuntimeError, SplatError):
            mode = "sharded"
    return GradientExchange(adam, params, rasterizer.param_gradients(), count, rasterizer.stride, rank, world,
                            mode, group)


class _PeerExchange:
    """The "peer" exchange: sp_peer_exchange_* (one kernel sums the ranks' gradients of this
    rank's share over peer memory, steps Adam on it and stores the parameters into every rank's
    buffer), between two one-element NCCL all-reduces on the stream that order it after every
    rank's backward and before every rank's next forward."""

    def __init__(self, adam, rank: int, world: int, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib

        self.lib = adam.lib
        self.group = group
        own = _lib.PeerHandleC()
        exported = self.lib.sp_peer_export(adam.handle, ctypes.byref(own))
        # Every rank joins the gather, an empty blob for a rank that could not export.
        blobs = [None] * world
        dist.all_gather_object(blobs, bytes(own) if exported == 0 else b"", group=group)
        if any(not blob for blob in blobs):
            raise RuntimeError("a rank could not export its buffers for the peer exchange")
        handles = (_lib.PeerHandleC * world)()
        for r, blob in enumerate(blobs):
            ctypes.memmove(ctypes.byref(handles[r]), blob, ctypes.sizeof(_lib.PeerHandleC))
        out = ctypes.c_void_p()
        status = self.lib.sp_peer_exchange_create(adam.handle, rank, world, handles, ctypes.byref(out))
        # Every rank learns whether every rank could map its peers before any uses the exchange.
        ok = torch.tensor([1 if status == 0 else 0], dtype=torch.int32, device=f"cuda:{adam.ctx.device}")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if status == 0 and int(ok.item()) == 0:
            self.lib.sp_peer_exchange_destroy(out.value)
            raise RuntimeError("a peer rank could not map the exchange buffers")
        _lib.check(status, adam.ctx.handle, "sp_peer_exchange_create")
        self.handle = out.value
        self.ctx = adam.ctx
        self.token = torch.zeros(1, dtype=torch.float32, device=f"cuda:{adam.ctx.device}")

    def _barrier(self) -> None:
        import torch.distributed as dist

        dist.all_reduce(self.token, group=self.group)

    def step(self, rate_factor: float) -> None:
        from . import _lib

        self._barrier()  # every rank's gradients are written
        _lib.check(self.lib.sp_peer_exchange_step(self.handle, float(rate_factor)), self.ctx.handle,
                   "sp_peer_exchange_step")
        self._barrier()  # every rank's parameters are written

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_peer_exchange_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


def views_of(step: int, rank: int, world: int, views: int, views_per_rank: int = 1) -> list[int]:
    """The views rank `rank` trains at `step` with `views_per_rank` views per rank and step: the
    ranks take consecutive blocks, so that one step covers views
    step * world * b .. (step + 1) * world * b - 1 (mod views), in view order across the ranks."""
    first = (step * world + rank) * views_per_rank
    return [(first + k) % views for k in range(views_per_rank)]


class ViewShardedStep:
    """One training step on this rank: for each of its views (`views_per_rank`, one by
    default) set the camera, forward, loss and backward, the gradients summed over its views
    in view order; then the gradient exchange and Adam (the scale clamp fused). With one view
    per rank and step the rank's backward feeds the exchange directly (one GPU: the backward
    with the Adam step fused); with several, the rasterizer must accumulate gradients
    (accumulate_gradients) and they are cleared at the start of each step. The batch of a
    step is then every rank's views, then one Adam step. `loss_index(view)` gives the view's
    index in the rasterizer's ground truth (by default the view itself). With `comm` (a
    comm.Communicator) the exchange is the library's own (sp_exchange_*)."""

    def __init__(self, rasterizer, adam, params, uniforms, rank: int, world: int, mode: str | None = None,
                 group=None, comm=None, views_per_rank: int = 1, loss_index=None):
        self.rasterizer = rasterizer
        self.adam = adam
        self.params = params
        self.uniforms = uniforms
        self.rank = rank
        self.world = world
        self.mode = mode
        self.group = group
        self.comm = comm
        self.views_per_rank = int(views_per_rank)
        self.loss_index = loss_index or (lambda view: view)
        if self.views_per_rank > 1 and not rasterizer.options.accumulate_gradients:
            raise ValueError("several views per step need a rasterizer that accumulates gradients")
        self.exchange = self._exchange(adam, params, rasterizer)

    def _exchange(self, adam, params, rasterizer):
        return make_exchange(adam, params, rasterizer, self.rank, self.world, self.mode, self.group, self.comm)

    def densify(self, settings, extent: float, max_count: int, reset_opacity: bool, seed: int):
        """Trainer::densify_async (training.rs:238-266) on every rank: the statistics merged and
        the moments gathered (module docstring), densify on the device, then this step's
        rasterizer, optimiser and exchange rebuilt at the new count (the statistics start
        over; the exchange is sharded, or peer, again only when the new count splits evenly).
        Every rank must call it at the same step. Returns the DensifyReport."""
        from .densify import densify
        from .rasterizer import Rasterizer

        r = self.rasterizer
        if self.world > 1 and self.comm is not None:
            self.comm.merge_densify_stats(r)
            self.exchange.gather_moments()
        elif self.world > 1:
            merge_densify_stats(r.densify_stats_tensor(), self.group)
            self.exchange.gather_moments(*self.adam.moment_tensors())
        out = densify(r, self.adam, extent, max_count, settings, reset_opacity, seed)
        count = out.report.after
        rasterizer = Rasterizer(r.ctx, out.params, count, r.width, r.height, r._ground_truth, r.view_count,
                                r.options)
        adam = self.adam.resumed_device(out.params, rasterizer, count, out.first_moment, out.second_moment)
        self.exchange.close()
        r.close()
        self.adam.close()
        self.rasterizer, self.adam, self.params = rasterizer, adam, out.params
        self.exchange = self._exchange(adam, out.params, rasterizer)
        return out.report

    def __call__(self, step: int, rate_factor: float) -> int:
        """The step; returns this rank's last view."""
        views = views_of(step, self.rank, self.world, len(self.uniforms), self.views_per_rank)
        r = self.rasterizer
        if self.views_per_rank > 1:
            r.zero_param_gradients()
            for view in views:
                r.set_camera(self.uniforms[view])
                r.encode_forward()
                r.encode_loss(self.loss_index(view))
                r.encode_backward()
            self.exchange(rate_factor)
            return views[-1]
        view = views[0]
        r.set_camera(self.uniforms[view])
        r.encode_forward()
        r.encode_loss(self.loss_index(view))
        if self.world == 1 and not r.options.accumulate_gradients:
            # Backward with the Adam step fused into the projection backward.
            r.encode_backward_adam(self.adam, rate_factor)
        else:
            r.encode_backward_blend()
            self.exchange.backward_step(r.encode_backward_project, rate_factor)
        return view
