"""Checkpoint and restore of the engine's device state: a run continued
from a checkpoint -- in the same engine, or in a new engine built from the
same network -- gives the uninterrupted run bit for bit (spikes, weights and
membrane potentials, with deterministic delivery, whose input sums do not
depend on thread timing); a restored engine's own checkpoint equals the one
it was restored from, with the fast delivery too; checkpoints of another
network are refused."""
import numpy as np
import pytest

import specs as S
from libnrn_b200 import _native as N
from libnrn_b200 import workloads as W
from libnrn_b200.engine import Network

pytestmark = pytest.mark.gpu


def net_stdp(steps):
    # the small Brunel + STDP network (E->E walks, a sweep within 900 steps)
    return S.realize(W.brunel(3000, 750, 200, 50, stdp=True, seed=3, steps=steps))


def test_continue_from_checkpoint_equals_uninterrupted_run():
    net = net_stdp(900)
    a = Network.from_net(net, deterministic=True)
    a.run(300)
    ckpt = a.checkpoint()
    a.run(600)
    st_a, gid_a = a.raster()
    w_a = [a.weights(q) for q in range(len(net["projs"]))]
    v_a = a.state("v")
    # the same engine, rewound
    a.restore(ckpt)
    assert a.step == 300
    a.run(600)
    st_b, gid_b = a.raster()
    w_b = [a.weights(q) for q in range(len(net["projs"]))]
    a.close()
    # a new engine from the same network
    c = Network.from_net(net, deterministic=True)
    c.restore(ckpt)
    c.run(600)
    st_c, gid_c = c.raster()
    w_c = [c.weights(q) for q in range(len(net["projs"]))]
    v_c = c.state("v")
    c.close()
    assert len(gid_a) > 1000
    for st, gid, w in ((st_b, gid_b, w_b), (st_c, gid_c, w_c)):
        # the unread raster of the first 300 steps travels with the checkpoint
        assert np.array_equal(st, st_a) and np.array_equal(gid, gid_a)
        for x, y in zip(w, w_a):
            assert np.array_equal(x, y)
    assert np.array_equal(v_c, v_a)


def test_restore_round_trip_fast_delivery():
    net = net_stdp(300)
    a = Network.from_net(net)
    a.run(300)
    ckpt = a.checkpoint()
    a.close()
    c = Network.from_net(net)
    c.restore(ckpt)
    assert c.step == 300
    assert c.checkpoint() == ckpt
    c.run(30)
    c.close()


def test_checkpoint_of_another_network_is_refused():
    a = Network.from_net(net_stdp(30))
    a.run(30)
    ckpt = a.checkpoint()
    a.close()
    b = Network.from_net(S.realize(W.brunel(3000, 750, 200, 50, stdp=False, seed=3, steps=30)))
    with pytest.raises(N.NrnError):
        b.restore(ckpt)
    with pytest.raises(N.NrnError):
        b.restore(b"not a checkpoint" * 8)
    b.close()
