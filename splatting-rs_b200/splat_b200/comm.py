"""The multi-GPU view-sharded step through the library's own communicator (sp_comm_*,
sp_exchange_*: NCCL loaded by libsplat_b200 itself), for callers without another collective
library. One process per GPU; every rank makes the same collective calls in the same order.

    uid = Communicator.unique_id()            # on one rank; pass the 128 bytes to the others
    comm = Communicator(ctx, uid, world, rank)
    exchange = Exchange(comm, adam)            # peer memory where it can, else NCCL collectives
    ... each step: backward passes (accumulated over this rank's views), then exchange.step(factor)

The reference trains one view per step on one device (instantsplat-rs/src/training.rs:197-229);
with one rank this is that step.
"""

from __future__ import annotations

import ctypes

from . import _lib

SP_COMM_ID_BYTES = 128
EXCHANGE_MODES = {"auto": 0, "peer": 1, "sharded": 2, "allreduce": 3}
MODE_NAMES = {v: k for k, v in EXCHANGE_MODES.items()}


def nccl_version() -> int:
    """The NCCL version the library loads (e.g. 22703), 0 when it cannot load one."""
    return int(_lib.load().sp_comm_nccl_version())


class Communicator:
    """sp_comm: a communicator of `world` ranks on the context's device; every host wait on the
    other ranks is bounded by `timeout_ms` (the communicator is aborted past it and the call
    raises SplatError(SP_ERR_TIMEOUT))."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * SP_COMM_ID_BYTES)()
        _lib.check(_lib.load().sp_comm_unique_id(buf), what="sp_comm_unique_id")
        return bytes(buf)

    def __init__(self, ctx, unique_id: bytes, world: int, rank: int, timeout_ms: int = 60_000):
        if len(unique_id) != SP_COMM_ID_BYTES:
            raise ValueError("a communicator id has 128 bytes")
        self.lib = _lib.load()
        self.ctx = ctx
        self.world, self.rank = int(world), int(rank)
        buf = (ctypes.c_uint8 * SP_COMM_ID_BYTES).from_buffer_copy(unique_id)
        out = ctypes.c_void_p()
        _lib.check(self.lib.sp_comm_init(ctx.handle, buf, self.world, self.rank, int(timeout_ms), ctypes.byref(out)),
                   ctx.handle, "sp_comm_init")
        self.handle = out.value

    def barrier(self) -> None:
        _lib.check(self.lib.sp_comm_barrier(self.handle), self.ctx.handle, "sp_comm_barrier")

    def wait(self) -> None:
        _lib.check(self.lib.sp_comm_wait(self.handle), self.ctx.handle, "sp_comm_wait")

    def allreduce_gradients(self, rasterizer) -> None:
        _lib.check(self.lib.sp_allreduce_grads(self.handle, rasterizer.handle), self.ctx.handle, "sp_allreduce_grads")

    def adam_step_sharded(self, adam, rate_factor: float) -> None:
        _lib.check(self.lib.sp_adam_step_sharded(self.handle, adam.handle, float(rate_factor)), self.ctx.handle,
                   "sp_adam_step_sharded")

    def merge_densify_stats(self, rasterizer) -> None:
        _lib.check(self.lib.sp_comm_merge_densify_stats(self.handle, rasterizer.handle), self.ctx.handle,
                   "sp_comm_merge_densify_stats")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class Exchange:
    """sp_exchange: the gradient exchange and Adam step of one rank, with the interface of
    sharding.GradientExchange (`mode`, `__call__`, `backward_step`, `gather_moments`, `close`)."""

    def __init__(self, comm: Communicator, adam, mode: str = "auto"):
        self.lib = comm.lib
        self.comm = comm
        self.adam = adam
        out = ctypes.c_void_p()
        _lib.check(self.lib.sp_exchange_create(comm.handle, adam.handle, EXCHANGE_MODES[mode], ctypes.byref(out)),
                   comm.ctx.handle, "sp_exchange_create")
        self.handle = out.value
        self.mode = MODE_NAMES[int(self.lib.sp_exchange_mode(self.handle))]

    def __call__(self, rate_factor: float) -> None:
        """The exchange and the Adam step after this rank's backward passes."""
        _lib.check(self.lib.sp_exchange_step(self.handle, float(rate_factor)), self.comm.ctx.handle,
                   "sp_exchange_step")

    def backward_step(self, project, rate_factor: float) -> None:
        """The projection backward over all Gaussians (`project(first, count)`), then the exchange."""
        project(0, self.adam.gaussian_count)
        self(rate_factor)

    def probe_link(self, peer: int, bytes_: int) -> float:
        """GB/s of one read of `bytes_` of rank `peer`'s gradient buffer over NVLink by this
        GPU (sp_exchange_probe_link; peer-memory exchanges only, between steps)."""
        ms = ctypes.c_float()
        _lib.check(self.lib.sp_exchange_probe_link(self.handle, int(peer), int(bytes_), ctypes.byref(ms)),
                   self.comm.ctx.handle, "sp_exchange_probe_link")
        return bytes_ / (ms.value / 1000.0) / 1e9

    def gather_moments(self, first=None, second=None) -> None:
        _lib.check(self.lib.sp_exchange_gather_moments(self.handle), self.comm.ctx.handle,
                   "sp_exchange_gather_moments")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.sp_exchange_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()
