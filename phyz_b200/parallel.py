"""Multi-GPU plumbing of the batched stepper: one process per GPU, worlds
sharded contiguously, one NCCL all-reduce of the objective per rollout.

Worlds never interact (phyz-gpu steps each world with its own thread and
state: crates/phyz-gpu/src/cuda/mod.rs:879-945), so sharding needs no
per-step communication. Rank g owns a contiguous block of worlds; the model
table is replicated. The only collective is the sum of the per-world
objective over all shards at the end of a rollout, run by the C ABI's
phyzb_reduce_objective (NCCL, loaded by the library) on the simulator's
stream. The communicator id travels from rank 0 to the others over any host
channel; here torch.distributed's object broadcast (gloo or NCCL group).
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, Optional

from . import _lib
from ._lib import check


def shard_bounds(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous split of `total` worlds: rank g gets [g*N/G, (g+1)*N/G)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    return rank * total // world, (rank + 1) * total // world


def weak_block(per_rank: int, rank: int) -> tuple[int, int]:
    """Weak scaling: every rank owns `per_rank` worlds, rank g the g-th block."""
    return rank * per_rank, (rank + 1) * per_rank


def share_bytes(payload: Optional[bytes], rank: int, group=None) -> bytes:
    """Broadcast rank 0's bytes to every rank of the torch.distributed group."""
    import torch.distributed as dist

    obj = [payload if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    if not isinstance(obj[0], (bytes, bytearray)):
        raise RuntimeError("rank 0 did not provide the communicator id")
    return bytes(obj[0])


def new_unique_id() -> bytes:
    lib = _lib.load()
    buf = (C.c_uint8 * _lib.COMM_ID_BYTES)()
    check(lib.phyzb_comm_unique_id(buf))
    return bytes(buf)


class Comm:
    """NCCL communicator of the stepper (phyzb_comm). Every rank constructs
    it collectively; `id_channel(payload, rank)` moves rank 0's id to all
    ranks (default: torch.distributed broadcast)."""

    def __init__(self, rank: int, world: int, device: int, timeout: float = 60.0,
                 id_channel: Optional[Callable[[Optional[bytes], int], bytes]] = None):
        self._lib = _lib.load()
        self.rank, self.world, self.device, self.timeout = rank, world, device, float(timeout)
        channel = id_channel or (lambda payload, r: share_bytes(payload, r))
        uid = channel(new_unique_id() if rank == 0 else None, rank)
        buf = (C.c_uint8 * _lib.COMM_ID_BYTES).from_buffer_copy(uid)
        h = _lib._P()
        check(self._lib.phyzb_comm_init(buf, world, rank, device, self.timeout, C.byref(h)))
        self._h = h

    def reduce_objective(self, sim, kind: int = 0, timeout: Optional[float] = None) -> float:
        """Sum over every rank's worlds of sim's per-world objective."""
        out = C.c_double()
        check(self._lib.phyzb_reduce_objective(sim._h, self._h, int(kind),
                                               float(timeout or self.timeout), C.byref(out)))
        return out.value

    def reduce_objective_device(self, sim, out_ptr: int, kind: int = 0) -> None:
        """Enqueue the reduction into a device scalar without waiting (read it
        after sync)."""
        check(self._lib.phyzb_reduce_objective_device(sim._h, self._h, int(kind), C.c_void_p(int(out_ptr))))

    def sync(self, sim, timeout: Optional[float] = None) -> None:
        """Bounded wait for everything enqueued on sim's stream."""
        check(self._lib.phyzb_comm_sync(self._h, sim._h, float(timeout or self.timeout)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.phyzb_comm_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
