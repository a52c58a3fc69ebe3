"""Host side of the multi-GPU partition, on CPU with world-size-2 gloo
groups: slice ranges, distribution of the NCCL unique id made by the engine
library, and the window exchange protocol (per-rank send blocks of
[window counts][total][ids], one all-gather, unpack into the step slots of the
spike history) checked against the unpartitioned spike list."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from libnrn_b200.partition import partition_range


def test_partition_ranges_cover_population():
    for n in (1, 7, 1000, 838_860 * 8 + 3):
        for world in (1, 2, 3, 8):
            lo_prev, total = 0, 0
            sizes = []
            for r in range(world):
                lo, k = partition_range(n, r, world)
                assert lo == lo_prev
                lo_prev = lo + k
                total += k
                sizes.append(k)
            assert total == n and max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        partition_range(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _pack(local_ids_per_step, win, cap):
    """Send block of one rank for one window: [win counts][total][ids], the
    ids of window step u after those of steps 0..u-1 (the layout the neuron
    update writes); ids past the capacity are dropped and reported."""
    blk = np.zeros(win + 1 + cap, np.int32)
    pos, overflow = 0, False
    for u, ids in enumerate(local_ids_per_step):
        blk[u] = len(ids)
        for x in ids:
            if pos < cap:
                blk[win + 1 + pos] = x
            else:
                overflow = True
            pos += 1
    blk[win] = pos
    return blk, overflow


def _unpack(gathered, win, cap):
    """Ids of every window step over all ranks, lower ranks first (the
    history slot layout)."""
    out = []
    for u in range(win):
        step_ids = []
        for blk in gathered:
            before = int(blk[:u].sum())
            n = int(blk[u])
            step_ids.extend(blk[win + 1 + before:win + 1 + before + n].tolist())
        out.append(step_ids)
    return out


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from libnrn_b200.partition import comm_unique_id, share_unique_id

        uid = share_unique_id(comm_unique_id)
        ids = [None] * world
        dist.all_gather_object(ids, uid)
        # a population of 1000 neurons, spikes drawn from one seed for all;
        # every rank's block has the same size, from the largest slice
        # (uneven splits give ranks different slice sizes)
        n, win, steps = 1000, 15, 90
        cap = min(-(-n // world) * win, 400)
        rng = np.random.default_rng(5)
        spikes = [np.flatnonzero(rng.random(n) < 0.02) for _ in range(steps)]
        lo, k = partition_range(n, rank, world)
        got = []
        for w0 in range(0, steps, win):
            mine = [s[(s >= lo) & (s < lo + k)] for s in spikes[w0:w0 + win]]
            blk, overflow = _pack(mine, win, cap)
            assert not overflow
            t = torch.from_numpy(blk)
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            got.extend(_unpack([p.numpy() for p in parts], win, cap))
        ok = all(np.array_equal(np.sort(g), s) for g, s in zip(got, spikes))
        # rank order within a step: rank r's ids follow those of ranks < r
        ordered = all(np.array_equal(np.asarray(g), s) for g, s in zip(got, spikes))
        q.put((rank, len(uid), all(x == uid for x in ids), ok, ordered))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_window_exchange(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, n_uid, same_uid, ok, ordered in res:
        assert n_uid == 128 and same_uid
        assert ok and ordered


def test_pack_reports_overflow():
    blk, overflow = _pack([np.arange(10), np.arange(10)], 2, 15)
    assert overflow and blk[0] == 10 and blk[1] == 10 and blk[2] == 20
