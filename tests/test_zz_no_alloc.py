"""nrn_engine_raster_noalloc: reading the spike raster without allocating.

Callers that cannot call cudaMalloc -- for instance a loop that drains spikes
while the simulation keeps running in real time, where an allocation or free
could stall the device -- read the raster through this entry point.  It must
return exactly what nrn_engine_raster returns.  Two identical engines run
the same network (dyadic weights, so their float reductions agree bit for
bit); one is drained with each entry point, twice in a row.
This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

import fixtures as F
from libnrn_b200 import _native as N
from libnrn_b200.engine import Network

pytestmark = pytest.mark.gpu


def read_noalloc(nw, cap=1 << 17):
    n = C.c_int64()
    st = np.empty(cap, np.int32)
    gd = np.empty(cap, np.int32)
    status = N.lib().nrn_engine_raster_noalloc(nw.h, st.ctypes.data, gd.ctypes.data, cap, C.byref(n))
    return status, st[:n.value], gd[:n.value]


def test_noalloc_raster_equals_allocating_raster_twice():
    net, _ = F.load_net("net_izh")
    a = Network.from_net(net)
    b = Network.from_net(net)
    total = 0
    for _ in range(2):
        a.run(100)
        b.run(100)
        sa, ga = a.raster()                       # allocating entry point
        status, sb, gb = read_noalloc(b)
        assert status == 0, N.lib().nrn_last_error()
        assert len(ga) > 0
        assert np.array_equal(sa, sb) and np.array_equal(ga, gb)
        total += len(gb)
    assert b.counters()[0] == total
    a.close()
    b.close()


def test_noalloc_raster_rejects_more_than_its_limit():
    # every neuron of a large population spikes in the first step
    nw = Network(1e-4)
    nw.add_population("lif", 140_000, [0.0, 0.020, 0.010, 0.020, 0.002, 250e-12, 0.0],
                      drive=("poisson", 40.0, 1e-8), seed=3)
    nw.finalize()
    nw.run(1)
    status, _, _ = read_noalloc(nw)
    assert status == 4                            # NRN_ERR_CAPACITY, raster kept
    assert b"131072" in N.lib().nrn_last_error()
    st, gid = nw.raster()                         # still readable the allocating way
    assert len(gid) == 140_000
    nw.close()
