"""Spike statistics kept on the device (per-neuron count and inter-spike
interval sums, updated by the neuron updates at each spike) equal the
records rebuilt from the spike raster, exactly, before and after a reset."""
import numpy as np
import pytest

import specs as S
from libnrn_b200 import workloads as W
from libnrn_b200.engine import Network
from libnrn_b200.stats import records_from_raster

pytestmark = pytest.mark.gpu


def check(nw, net, st, gid):
    off = 0
    for q, p in enumerate(net["pops"]):
        m = (gid >= off) & (gid < off + p["n"])
        want = records_from_raster(st[m], gid[m] - off, p["n"])
        got = nw.spike_stats(q)
        for f in ("last", "count", "isi_sum", "isi_sum2"):
            assert np.array_equal(got[f], want[f]), (q, f)
        off += p["n"]


@pytest.mark.parametrize("stdp", [False, True])
def test_device_spike_stats_equal_raster(stdp):
    # LIF four neurons per thread (E: 3000, I: 752) and the STDP walk path
    net = S.realize(W.brunel(3000, 752, 200, 50, stdp=stdp, seed=5, steps=800))
    nw = Network.from_net(net, spike_stats=True)
    nw.run(500)
    st, gid = nw.raster()
    assert len(gid) > 1000
    check(nw, net, st, gid)
    s = nw.population_stats(0)
    assert s["n_cv"] > 100 and 0.0 < s["cv_mean"] < 3.0
    assert abs(s["rate_mean_hz"] * 500 * net["dt"] * 3000 - np.count_nonzero(gid < 3000)) < 1e-6
    nw.reset_spike_stats()
    nw.run(300)
    st, gid = nw.raster()
    check(nw, net, st, gid)
    nw.close()


def test_scalar_update_spike_stats_equal_raster():
    # AdEx (one neuron per thread) with conductances
    net = S.realize(S.small_adex(steps=300))
    nw = Network.from_net(net, spike_stats=True)
    nw.run(300)
    st, gid = nw.raster()
    assert len(gid) > 100
    check(nw, net, st, gid)
    nw.close()
