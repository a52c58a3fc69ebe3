"""Synapse channels (the reference's declared exponential, double-exponential
and AMPA synapse models, include/nrn/synapse/exponential.h:16-21,
double_exponential.h:17-25, ampa.h:17-29, whose forward is a stub in the
reference) fused into the neuron update: the CUDA path against the oracle's
restatement of the same equations on the same network.  Parity is unpinned
by the reference (it has no implementation); weights are dyadic, so every
channel input sums exactly and the comparison is bit for bit."""
import numpy as np
import pytest

import specs as S
from libnrn_b200.engine import Network
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def run_engine(net):
    nw = Network.from_net(net)
    nw.run(net["steps"])
    st, gid = nw.raster()
    v = nw.state("v")
    nw.close()
    return st, gid, v


def test_synapse_channels_match_oracle():
    net = S.synapse_channel_net(steps=600)
    want = O.run_oracle(net)
    st, gid, v = run_engine(net)
    assert len(gid) > 500                      # E and I both active
    assert np.array_equal(st, want["spike_step"])
    assert np.array_equal(gid, want["spike_id"])
    assert np.array_equal(v, want["final_v"])


def test_synapse_channels_change_dynamics():
    """The channels act: the same network with static current synapses
    (every receptor the input current) spikes differently."""
    net = S.synapse_channel_net(steps=300)
    for q in net["projs"]:
        q["receptor"] = "current"
    for p in net["pops"]:
        p["syn"] = None
    a = O.run_oracle(net)
    st, gid, _ = run_engine(net)
    assert np.array_equal(gid, a["spike_id"])
    b = O.run_oracle(S.synapse_channel_net(steps=300))
    assert not (len(b["spike_id"]) == len(a["spike_id"]) and np.array_equal(b["spike_id"], a["spike_id"]))


def test_channel_receptor_needs_channel():
    net = S.synapse_channel_net(steps=10)
    net["pops"][1]["syn"] = None               # E -> I names chan0 of I, now absent
    with pytest.raises(Exception, match="synapse channel"):
        Network.from_net(net)
