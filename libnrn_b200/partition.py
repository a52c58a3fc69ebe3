"""Partition of a network over GPUs by neuron index, one process per GPU.

Every population of N neurons is split into `world` contiguous slices;
rank r holds neurons [N*r // world, N*(r+1) // world).  Each rank builds the
same network through the same calls on its slices (engine.Network with
``partition=``): the synapses onto its neurons (sources anywhere), its
neurons' state and drive (keyed by global neuron id, so results do not
depend on the split), and the spike exchange -- one NCCL all-gather of the
window's spike ids per window of min(smallest delay, 32) steps, run by the
engine library on its own communicator.  This module holds the host-side
pieces: slice ranges, the launcher environment, and the distribution of the
NCCL unique id over an initialised torch.distributed group.
"""
from __future__ import annotations

import ctypes as C
import os

from . import _native as N


def partition_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """(first index, count) of rank's slice of a population of n neurons."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    lo = n * rank // world
    hi = n * (rank + 1) // world
    return lo, hi - lo


def dist_env() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def comm_unique_id() -> bytes:
    """A new NCCL unique id (128 bytes), made by the engine library."""
    buf = (C.c_uint8 * 128)()
    N.check(N.lib().nrn_comm_unique_id(C.byref(buf)), "nrn_comm_unique_id")
    return bytes(buf)


def share_unique_id(make=comm_unique_id) -> bytes:
    """Rank 0 makes the id, every rank of the default torch.distributed group
    receives it."""
    import torch.distributed as dist

    obj = [make() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("NCCL unique id: expected 128 bytes")
    return bytes(uid)


class StepAgreement:
    """Host-side check, before each run of a partitioned network, that every
    rank is still there and runs the same steps: each rank posts (run index,
    first step, step count) to the torch.distributed store and waits, with a
    time limit, for the others' posts.  A rank that stopped between runs is
    then found on the host before any GPU work of the next run is launched
    (the engine's own bounded waits cover a rank that stops inside a run).
    Raises RuntimeError naming the missing or disagreeing rank."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 60.0, prefix: str = "nrn/run"):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.timeout_s = float(timeout_s)
        self.prefix = prefix
        self.k = 0

    def check(self, first_step: int, steps: int) -> None:
        import datetime

        key = f"{self.prefix}/{self.k}"
        mine = f"{int(first_step)}:{int(steps)}"
        self.store.set(f"{key}/{self.rank}", mine)
        others = [f"{key}/{r}" for r in range(self.world) if r != self.rank]
        try:
            self.store.wait(others, datetime.timedelta(seconds=self.timeout_s))
        except Exception as ex:
            missing = [r for r in range(self.world) if r != self.rank and not self.store.check([f"{key}/{r}"])]
            raise RuntimeError(f"partitioned run {self.k}: rank(s) {missing} did not reach it within "
                               f"{self.timeout_s:g} s") from ex
        for r in range(self.world):
            got = self.store.get(f"{key}/{r}").decode()
            if got != mine:
                raise RuntimeError(f"partitioned run {self.k}: rank {r} runs steps {got}, rank {self.rank} {mine}")
        self.k += 1
