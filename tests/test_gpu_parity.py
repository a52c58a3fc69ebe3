"""Parity of the CUDA path (through the C ABI) with the reference's outputs
(golden fixtures) and with the oracle (C restatement) on the same inputs."""
import ctypes as C

import numpy as np
import pytest
import torch

import fixtures as F
from libnrn_b200 import _native as N
from libnrn_b200.engine import Network
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_STATE = 1e-5        # one step, per-step state, fp32 relative (AdEx: exp)
TOL_TRAJ = 1e-4         # along chaotic trajectories (summation order, exp)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(1e-30, float(np.abs(b).max())) if b.size else 1.0
    return float(np.abs(a - b).max()) / scale if b.size else 0.0


def run_neuron_gpu(pop, steps, dt, I):
    dev = torch.device("cuda", 0)
    n = pop["n"]
    model = pop["model"]
    v = torch.as_tensor(pop["init_v"] if pop.get("init_v") is not None else
                        np.full(n, -65.0 if model == "izh" else pop["params"][0], np.float32)).to(dev)
    if model == "izh":
        aux0 = pop.get("init_aux")
        aux = torch.as_tensor(aux0 if aux0 is not None else
                              np.full(n, np.float32(pop["params"][1] * -65.0))).to(dev)
    elif model == "adex":
        aux = torch.zeros(n, device=dev)
    else:
        aux = None
    ref = torch.zeros(n, device=dev) if model != "izh" else None
    spike = torch.zeros(n, device=dev)
    isyn = torch.zeros(n, device=dev)
    hp = None
    a = N.PopStep()
    a.model = N.MODEL[model]
    a.n = n
    a.dt = dt
    a.v = v.data_ptr()
    a.aux = aux.data_ptr() if aux is not None else None
    a.refractory = ref.data_ptr() if ref is not None else None
    a.spike = spike.data_ptr()
    a.i_syn = isyn.data_ptr()
    for k, x in enumerate(pop["params"]):
        a.uniform[k] = float(x)
    if pop.get("hp") is not None:
        hp = torch.as_tensor(pop["hp"]).to(dev).contiguous()
        for k in range(hp.shape[0]):
            a.param[k] = hp[k].data_ptr()
    It = torch.as_tensor(np.asarray(I, np.float32)).to(dev)
    out = {k: np.zeros((steps, n), np.float32) for k in ("v", "aux", "ref")}
    out["spike"] = np.zeros((steps, n), np.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    for t in range(steps):
        isyn.copy_(It[t])
        N.check(N.lib().nrn_cuda_pop_step(C.byref(a), C.c_void_p(stream)), "pop_step")
        out["v"][t] = v.cpu().numpy()
        if aux is not None:
            out["aux"][t] = aux.cpu().numpy()
        if ref is not None:
            out["ref"][t] = ref.cpu().numpy()
        out["spike"][t] = (spike.cpu().numpy() != 0)
    return out


@pytest.mark.parametrize("name", ["neuron_lif", "neuron_adex", "neuron_izh"])
def test_neuron_step_matches_reference(name):
    pop, steps, dt, I, ref = F.load_neuron(name)
    got = run_neuron_gpu(pop, steps, dt, I)
    assert np.array_equal(got["spike"], ref["spike"])
    if pop["model"] == "adex":
        for k in ("v", "aux", "ref"):
            assert rel_err(got[k], ref[k]) <= TOL_STATE, k
    else:
        keys = ("v", "aux", "ref") if pop["model"] == "lif" else ("v", "aux")
        for k in keys:
            assert np.array_equal(got[k], ref[k]), k


def engine_run(net):
    nw = Network.from_net(net)
    nw.run(net["steps"])
    st, gid = nw.raster()
    res = {"spike_step": st, "spike_id": gid, "final_v": nw.state("v"), "final_aux": nw.state("aux"),
           "w_out": [nw.weights(q) for q in range(len(net["projs"]))]}
    res["counters"] = nw.counters()
    nw.close()
    return res


@pytest.mark.parametrize("name", ["net_brunel_stdp", "net_brunel_slow", "net_adex", "net_izh"])
def test_network_matches_reference(name):
    net, ref = F.load_net(name)
    got = engine_run(net)
    assert np.array_equal(got["spike_step"], ref["spike_step"])
    assert np.array_equal(got["spike_id"], ref["spike_id"])
    tol = TOL_TRAJ if name in ("net_adex", "net_izh") else TOL_STATE
    assert rel_err(got["final_v"], ref["final_v"]) <= tol
    for a, b in zip(got["w_out"], ref["w_out"]):
        assert rel_err(a, b) <= TOL_STATE
    spikes, events = got["counters"]
    assert spikes == len(ref["spike_id"])
    assert events > 0


def test_generated_connectivity_matches_oracle_generator():
    import specs as S
    from libnrn_b200 import workloads as W
    for spec in (W.brunel(300, 75, 30, 8, steps=1), W.izhikevich(400, 20, steps=1, w_scale=10.0),
                 W.adex_cond(300, 20, steps=1)):
        nw = Network.from_spec(spec, record=False)
        for qi, q in enumerate(spec["projs"]):
            args, kw = S.gen_args(spec, q)
            s, t, w, d = O.gen_fixed_degree(*args, **kw)
            # engine order: by (source, delay), ties in generation order
            order = np.lexsort((d, s))
            got_w = nw.weights(qi)
            assert len(got_w) == len(w)
            assert np.array_equal(got_w, w[order])
        nw.close()


def test_long_run_statistics_match_oracle():
    """Chaotic regime: long runs compared by population rate and CV of the
    inter-spike intervals (within 2%)."""
    import specs as S
    spec = S.small_brunel(stdp=False, steps=3000, seed=5)
    net = S.realize(spec)
    a = O.run_oracle(net)
    b = engine_run(net)

    def stats(step, gid, n, steps, dt):
        rate = len(gid) / n / (steps * dt)
        cvs = []
        order = np.lexsort((step, gid))
        g, s = gid[order], step[order]
        for k in np.unique(g):
            isi = np.diff(s[g == k]) * dt
            if len(isi) > 2:
                cvs.append(isi.std() / isi.mean())
        return rate, float(np.mean(cvs))

    ra, ca = stats(a["spike_step"], a["spike_id"], spec["n_total"], 3000, spec["dt"])
    rb, cb = stats(b["spike_step"], b["spike_id"], spec["n_total"], 3000, spec["dt"])
    assert abs(rb - ra) <= 0.02 * ra
    assert abs(cb - ca) <= 0.02 * ca


@pytest.mark.parametrize("rule", ["er", "distance"])
def test_random_connectivity_matches_oracle_generator(rule):
    """Erdos-Renyi and distance-dependent connectivity drawn on the device
    equals the oracle generator's synapse for synapse (engine order: by
    source and delay, ties in generation order)."""
    import specs as S
    from libnrn_b200 import workloads as W
    spec = W.random_network(3_000, 750, rule=rule, p=0.02, sigma=20e-6, max_distance=1e-3, steps=1)
    for q in spec["projs"]:
        q["gen"]["dmin"], q["gen"]["dmax"], q["gen"]["w_span"] = 10, 20, abs(q["gen"]["w_lo"])
    nw = Network.from_spec(spec, record=False)
    for qi, q in enumerate(spec["projs"]):
        s, t, w, d = S.gen_lists(spec, q)
        order = np.lexsort((d, s))
        got = nw.weights(qi)
        assert len(got) == len(w) > 1000
        assert np.array_equal(got, w[order])
    nw.close()


def test_random_network_runs_like_oracle():
    """A network on device-drawn ER connectivity: the engine's spike trains
    equal the oracle's on the same lists (deterministic delivery)."""
    import specs as S
    from libnrn_b200 import workloads as W
    spec = W.random_network(2_000, 500, rule="er", p=0.04, steps=300)
    net = S.realize(spec)
    want = O.run_oracle(net)
    nw = Network.from_spec(spec, record=True)
    nw.close()
    nw = Network.from_net(net, deterministic=True)
    nw.run(300)
    st, gid = nw.raster()
    nw.close()
    assert len(gid) > 500
    assert np.array_equal(st, want["spike_step"]) and np.array_equal(gid, want["spike_id"])
