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
