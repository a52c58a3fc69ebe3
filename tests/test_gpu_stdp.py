"""STDP applied by segment walks: parity with the oracle's per-step update
in the cases the walks have to get right -- sources that spike several
times within one delay, several delays per projection, runs longer than the
sweep's staleness limit -- and independence from how a run is split into
calls, CUDA graphs or eager launches, and weight reads in between."""
import os

import numpy as np
import pytest

import specs as S
from libnrn_b200 import workloads as W
from libnrn_b200.engine import Network
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def burst_spec(steps):
    """Brunel network with a 0.2 ms refractory period and reset 2 mV below
    threshold (about 175 Hz; over 1,200 steps some 1,400 inter-spike
    intervals of E sources are shorter than the longest delay, while no
    target spikes more than about 40 times between two walks of a segment,
    inside the 64-step history), and delays 4..12 steps on the plastic E->E
    projection."""
    spec = W.brunel(800, 200, 80, 20, delay=8, stdp=True, seed=21, steps=steps)
    for p in spec["pops"]:
        p["params"][4] = 2e-4
        p["params"][2] = 0.018
    g = spec["projs"][0]["gen"]
    g["dmin"], g["dmax"] = 4, 12
    return spec


def run(net, splits=None, weights_between=False):
    nw = Network.from_net(net)
    total = net["steps"]
    for k in (splits or [total]):
        nw.run(k)
        if weights_between:
            nw.weights(0)
    st, gid = nw.raster()
    w = [nw.weights(q) for q in range(len(net["projs"]))]
    v = nw.state("v")
    nw.close()
    return st, gid, w, v


def test_bursting_sources_match_oracle():
    net = S.realize(burst_spec(1200))
    ref = O.run_oracle(net)
    st, gid, w, v = run(net)
    # the network does burst: some source fires twice within the longest delay
    order = np.lexsort((st, gid))
    g, s = gid[order], st[order]
    isi = np.diff(s)[np.diff(g) == 0]
    assert (isi < 12).any()
    assert np.array_equal(st, ref["spike_step"])
    assert np.array_equal(gid, ref["spike_id"])
    for a, b in zip(w, ref["w_out"]):
        assert np.array_equal(a, b)
    # float atomics sum the inputs in another order than the oracle
    assert float(np.abs(v - ref["final_v"]).max()) <= 1e-5 * float(np.abs(ref["final_v"]).max())


def test_long_run_with_sweep_matches_oracle():
    # longer than the sweep's staleness limit, so swept segments are walked
    net = S.realize(S.small_brunel(stdp=True, steps=2500, seed=7))
    ref = O.run_oracle(net)
    st, gid, w, _ = run(net)
    assert np.array_equal(st, ref["spike_step"])
    assert np.array_equal(gid, ref["spike_id"])
    for a, b in zip(w, ref["w_out"]):
        assert np.array_equal(a, b)


def test_split_runs_and_weight_reads_change_nothing():
    net = S.realize(burst_spec(400))
    whole = run(net)
    split = run(net, splits=[7, 13, 1, 44, 200, 135], weights_between=True)
    for a, b in zip(whole[:2], split[:2]):
        assert np.array_equal(a, b)
    for a, b in zip(whole[2], split[2]):
        assert np.array_equal(a, b)


def test_eager_launches_equal_graphs():
    net = S.realize(burst_spec(300))
    whole = run(net)
    os.environ["NRN_NO_GRAPHS"] = "1"
    try:
        eager = run(net, splits=[100, 200])
    finally:
        del os.environ["NRN_NO_GRAPHS"]
    for a, b in zip(whole[:2], eager[:2]):
        assert np.array_equal(a, b)
    for a, b in zip(whole[2], eager[2]):
        assert np.array_equal(a, b)


def sparse_burst_spec(steps):
    """burst_spec with in-degree 1 E + 1 I: a neuron receives at most two
    synaptic events in a step, and a float sum of two terms does not
    depend on the order in which the reductions land, so runs with
    non-dyadic weights are deterministic."""
    spec = W.brunel(800, 200, 1, 1, delay=8, stdp=True, seed=21, steps=steps)
    for p in spec["pops"]:
        p["params"][4] = 2e-4
        p["params"][2] = 0.018
    g = spec["projs"][0]["gen"]
    g["dmin"], g["dmax"] = 4, 12
    return spec


def test_modulatory_gains_walk_equals_per_step_kernels():
    # gains on the plastic projection: the walks against the per-step STDP
    # kernels (the oracle has no gains), same spikes and weights.  Gains make
    # the delivered values non-dyadic, so the network has at most two inputs
    # per neuron and step (order-independent sums).
    net = S.realize(sparse_burst_spec(300))
    rng = np.random.default_rng(3)
    q = net["projs"][0]
    q["mod"] = rng.uniform(0.5, 1.5, len(q["w"])).astype(np.float32)
    walk = run(net)
    os.environ["NRN_STDP_EAGER"] = "1"
    try:
        eager = run(net)
    finally:
        del os.environ["NRN_STDP_EAGER"]
    for a, b in zip(walk[:2], eager[:2]):
        assert np.array_equal(a, b)
    for a, b in zip(walk[2], eager[2]):
        assert np.array_equal(a, b)


def test_engine_info_reports_window_and_raster_bound():
    net = S.realize(burst_spec(10))
    nw = Network.from_net(net)
    try:
        info = nw.info()
    finally:
        nw.close()
    assert info["window"] == 4                  # the smallest delay of the STDP projection
    assert info["raster_capacity"] >= 1 << 22
    assert info["recorded_neurons"] == sum(p["n"] for p in net["pops"])
