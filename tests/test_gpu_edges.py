"""Edge cases of the engine against the oracle: population sizes that are
not multiples of four (the generic per-neuron update path instead of the
four-per-thread one), a projection without synapses, a network that never
spikes, and runs split into single steps.  Deterministic delivery, so
potentials and weights compare bit for bit."""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))

import specs as S
from libnrn_b200 import workloads as W
from libnrn_b200.engine import Network
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def run(net, splits=None):
    nw = Network.from_net(net, deterministic=True)
    try:
        for k in (splits or [net["steps"]]):
            nw.run(k)
        st, gid = nw.raster()
        w = [nw.weights(q) for q in range(len(net["projs"]))]
        v = nw.state("v")
    finally:
        nw.close()
    return st, gid, w, v


def check(net, splits=None):
    ref = O.run_oracle(net)
    st, gid, w, v = run(net, splits)
    assert np.array_equal(st, ref["spike_step"]) and np.array_equal(gid, ref["spike_id"])
    for a, b in zip(w, ref["w_out"]):
        assert np.array_equal(a, b)
    assert np.array_equal(v, ref["final_v"])
    return st


def test_ragged_population_sizes_with_stdp():
    # 1,001 E + 251 I: neither is a multiple of four
    net = S.realize(W.brunel(1001, 251, 80, 20, stdp=True, steps=300, seed=5))
    st = check(net)
    assert len(st) > 100


def test_projection_without_synapses():
    spec = W.brunel(800, 200, 80, 20, stdp=True, steps=200, seed=6)
    spec["projs"][1]["gen"]["degree"] = 0     # E -> I: no synapses at all
    net = S.realize(spec)
    assert len(net["projs"][1]["w"]) == 0
    check(net)


def test_silent_network():
    # no drive, all potentials at rest: nothing spikes, weights stay clamped
    spec = W.brunel(800, 200, 80, 20, stdp=True, steps=100, seed=7, v0_uniform=False)
    for p in spec["pops"]:
        p["drive"] = None
    net = S.realize(spec)
    st = check(net)
    assert len(st) == 0


def test_single_step_runs_equal_one_run():
    net = S.realize(W.brunel(800, 200, 80, 20, stdp=True, steps=60, seed=8))
    whole = run(net)
    split = run(net, splits=[1] * 60)
    for a, b in zip(whole[:2], split[:2]):
        assert np.array_equal(a, b)
    for a, b in zip(whole[2], split[2]):
        assert np.array_equal(a, b)
    assert np.array_equal(whole[3], split[3])


def test_prepared_graphs_change_nothing():
    # capturing a run's graphs ahead (nrn_engine_prepare) runs no step
    net = S.realize(W.brunel(800, 200, 80, 20, stdp=True, steps=75, seed=9))
    whole = run(net)
    nw = Network.from_net(net, deterministic=True)
    try:
        step0 = nw.step
        nw.prepare(step0, 75)
        nw.prepare(step0 + 7, 33)
        assert nw.step == step0
        assert len(nw.raster()[0]) == 0
        nw.run(75)
        st, gid = nw.raster()
        w = [nw.weights(q) for q in range(len(net["projs"]))]
    finally:
        nw.close()
    assert np.array_equal(st, whole[0]) and np.array_equal(gid, whole[1])
    for a, b in zip(w, whole[2]):
        assert np.array_equal(a, b)
