"""Kernel-level equivalences on the GPU: the LIF update with four neurons a
thread (16-byte-aligned arrays, n a multiple of 4) against the one-neuron
kernel (arrays offset by one float), and the drive drawn ahead
(nrn_cuda_drive_fill) against the drive drawn inside the update."""
import ctypes as C

import numpy as np
import pytest
import torch

from libnrn_b200 import _native as N
from libnrn_b200 import workloads as W

pytestmark = pytest.mark.gpu


def lif_args(n, bufs, step, drive=True, drive_values=None):
    a = N.PopStep()
    a.model = N.MODEL["lif"]
    a.n = n
    a.gid_offset = 7
    a.dt = 1e-4
    a.v, a.refractory, a.spike, a.i_syn = (t.data_ptr() for t in (bufs["v"], bufs["ref"], bufs["spike"], bufs["i"]))
    for k, x in enumerate(W.LIF_BRUNEL):
        a.uniform[k] = float(x)
    if drive:
        a.drive.kind = N.DRIVE["poisson"]
        a.drive.p0 = 2.0
        a.drive.p1 = 0.1e-3 * 250e-12 / 1e-4    # one 0.1 mV PSP as a one-step current
        a.drive.seed = 11
    a.step = step
    a.spike_ids = bufs["ids"].data_ptr()
    a.spike_count = bufs["cnt"].data_ptr()
    if drive_values is not None:
        a.drive_values = drive_values.data_ptr()
    return a


def make_bufs(n, offset, seed):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    def arr(init):
        base = torch.zeros(n + 8, device=dev)
        t = base[offset:offset + n]
        t.copy_(init)
        return t
    v0 = torch.rand(n, device=dev, generator=g) * 0.02
    b = {"v": arr(v0), "ref": arr(torch.zeros(n, device=dev)), "spike": arr(torch.zeros(n, device=dev)),
         "i": arr(torch.rand(n, device=dev, generator=g) * 5e-10),
         "ids": torch.zeros(n, dtype=torch.int32, device=dev), "cnt": torch.zeros(1, dtype=torch.int32, device=dev)}
    return b


def test_lif_four_per_thread_equals_one_per_thread():
    n = 4096 * 3
    aligned, shifted = make_bufs(n, 0, 1), make_bufs(n, 1, 1)
    assert shifted["v"].data_ptr() % 16 != 0 and aligned["v"].data_ptr() % 16 == 0
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for step in range(40):
        got = []
        for b in (aligned, shifted):
            b["cnt"].zero_()
            N.check(N.lib().nrn_cuda_pop_step(C.byref(lif_args(n, b, step)), stream), "pop_step")
            torch.cuda.synchronize()
            c = int(b["cnt"].item())
            got.append((b["v"].cpu().numpy().copy(), b["ref"].cpu().numpy().copy(), b["spike"].cpu().numpy().copy(),
                        np.sort(b["ids"][:c].cpu().numpy())))
        for x, y in zip(*got):
            assert np.array_equal(x, y)
    assert got[0][3].size > 0


def test_drive_drawn_ahead_equals_drawn_in_update():
    n = 4096
    inside, ahead = make_bufs(n, 0, 2), make_bufs(n, 0, 2)
    drv = torch.zeros(n, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for step in range(20):
        N.check(N.lib().nrn_cuda_pop_step(C.byref(lif_args(n, inside, step)), stream), "pop_step")
        a = lif_args(n, ahead, step, drive_values=drv)
        N.check(N.lib().nrn_cuda_drive_fill(C.byref(a), C.c_void_p(drv.data_ptr()), stream), "drive_fill")
        N.check(N.lib().nrn_cuda_pop_step(C.byref(a), stream), "pop_step")
    torch.cuda.synchronize()
    assert torch.equal(inside["v"], ahead["v"]) and torch.equal(inside["ref"], ahead["ref"])
    assert int(inside["cnt"].item()) == int(ahead["cnt"].item()) > 0
