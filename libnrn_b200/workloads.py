"""The benchmark networks, as plain data.

Each function returns a network *spec*: populations (model, size, uniform
parameters, per-neuron parameter rule, drive, initial-condition rule) and
projections (a connectivity *generator* rule rather than synapse lists, so a
1e9-synapse network can be generated on the device).  ``engine.Network``
builds a spec on the GPU; the test suite realises the same spec on the host
for the oracle with the same Philox counters.

Units are SI (V, s, F, S, A) for LIF and AdEx, dimensionless for
Izhikevich, as in the reference's option structs (include/nrn/neuron/options.h).

Generator rule ``gen`` of a projection:
  mode    "in"  : every target draws ``degree`` sources (fixed in-degree)
          "out" : every source draws ``degree`` targets (fixed out-degree)
          "er"  : every pair with probability ``p``
          "distance": every pair with probability max(exp(-d^2/(2 sigma^2)),
                  min_probability), d the distance of 1D positions
                  i * max_distance / n
  cols    global id range (offset, n) the draws pick from; defaults to the
          source population ("in") or the target population ("out").
          Draws outside the target population are discarded ("out" mode over
          a range spanning several populations).
  dmin, dmax   delay range in steps (uniform integer)
  w_lo, w_span weight = w_lo + w_span * u01
  id      generator id (Philox counter word c2)
Autapses are excluded.
"""
from __future__ import annotations

import copy

LIF_BRUNEL = [0.0, 0.020, 0.010, 0.020, 0.002, 250e-12, 0.0]
ADEX_BG = [-0.0706, -0.0504, -0.0706, 0.0, 9.37e-3, 0.144, 0.002, 281e-12, 30e-9, 4e-9,
           80.5e-12, 0.002, 0.0]
IZH_RS = [0.02, 0.2, -65.0, 8.0, 30.0]


def _offsets(spec):
    off = 0
    for p in spec["pops"]:
        p["offset"] = off
        off += p["n"]
    spec["n_total"] = off
    return spec


def brunel(n_exc: int = 10_000, n_inh: int = 2_500, c_exc: int = 1_000, c_inh: int = 250, *,
           delay: int = 15, dt: float = 1e-4, steps: int = 10_000, g: float = 5.0,
           j_psp: float = 0.1e-3, stdp: bool = False, seed: int = 1, slow_ratio: int = 1,
           v0_uniform: bool = True) -> dict:
    """Brunel (2000) balanced LIF network, model A.

    Rest 0, threshold 20 mV, reset 10 mV, tau_m 20 ms, t_ref 2 ms, c_m 250 pF.
    A PSP of J = j_psp volts is one step of current w = J*c_m/dt; inhibitory
    weights are -g*w.  External drive: nu_ext = 2*nu_thr through C_E
    sources, i.e. Poisson(2) events of w per step.  With stdp=True, pair
    STDP on E->E (A+ 0.01, A- 0.0105, tau 20 ms, weights clipped to [0, 2w],
    learning rate w so that A+/A- are relative to w).  Initial potentials
    V0 ~ U(0, threshold) when v0_uniform (else all at rest)."""
    c_m = LIF_BRUNEL[5]
    w = j_psp * c_m / dt
    lam = 2.0 * LIF_BRUNEL[1] * dt / (j_psp * LIF_BRUNEL[3])
    spec = {
        "name": "brunel", "dt": dt, "steps": steps, "seed": seed, "slow_ratio": slow_ratio,
        "pops": [
            {"name": "E", "model": "lif", "n": n_exc, "params": list(LIF_BRUNEL),
             "drive": ("poisson", lam, w)},
            {"name": "I", "model": "lif", "n": n_inh, "params": list(LIF_BRUNEL),
             "drive": ("poisson", lam, w)},
        ],
        "projs": [],
    }
    if v0_uniform:
        for p in spec["pops"]:
            p["init"] = {"v": ("uniform", 0.0, LIF_BRUNEL[1], 0)}
    stdp_p = [0.020, 0.020, 0.01, -0.0105, 0.0, 2.0 * w, w]
    for gid, (s, t, deg, wt) in enumerate([(0, 0, c_exc, w), (0, 1, c_exc, w),
                                          (1, 0, c_inh, -g * w), (1, 1, c_inh, -g * w)]):
        spec["projs"].append({
            "src": s, "tgt": t, "receptor": "current",
            "gen": {"mode": "in", "degree": deg, "dmin": delay, "dmax": delay,
                    "w_lo": wt, "w_span": 0.0, "id": gid},
            "plastic": bool(stdp and gid == 0), "stdp": stdp_p,
        })
    return _offsets(spec)


def brunel_stdp_per_gpu(n_gpus: int = 1, steps: int = 10_000, **kw) -> dict:
    """The multi-GPU Brunel + STDP network: 1,048,576 neurons per GPU
    (838,860 E + 209,716 I), in-degree 1,000 E + 250 I, delay 15 steps."""
    return brunel(838_860 * n_gpus, 209_716 * n_gpus, 1_000, 250, steps=steps, stdp=True, **kw)


def adex_cond(n: int = 1_048_576, k_in: int = 1_000, *, dt: float = 1e-4, steps: int = 1_000,
              seed: int = 2, w_exc: float = 0.5e-9, w_inh: float = 2.5e-9,
              rate_ext: float = 5_000.0, dmax: int = 20) -> dict:
    """AdEx (Brette-Gerstner 2005) network with conductance synapses.

    80% excitatory / 20% inhibitory; every neuron receives 0.8*k_in
    excitatory and 0.2*k_in inhibitory synapses (fixed in-degree), delays
    uniform 1..dmax steps.  Excitatory spikes add w_exc to g_exc, inhibitory
    spikes add w_inh to g_inh; conductances decay with tau_syn = 5 ms toward
    reversal potentials 0 mV / -80 mV.  External Poisson input at rate_ext
    per neuron adds w_exc to g_exc per event.  V0 ~ U(-70, -50) mV, w0 = 0."""
    n_e = int(round(0.8 * n))
    n_i = n - n_e
    cond = [5e-3, 5e-3, 0.0, -0.080]
    drive = ("poisson_gexc", rate_ext * dt, w_exc)
    init = {"v": ("uniform", -0.070, 0.020, 0)}
    spec = {
        "name": "adex", "dt": dt, "steps": steps, "seed": seed, "slow_ratio": 1,
        "pops": [
            {"name": "E", "model": "adex", "n": n_e, "params": list(ADEX_BG), "cond": cond,
             "drive": drive, "init": init},
            {"name": "I", "model": "adex", "n": n_i, "params": list(ADEX_BG), "cond": cond,
             "drive": drive, "init": init},
        ],
        "projs": [],
    }
    k_e = int(round(0.8 * k_in))
    k_i = k_in - k_e
    for gid, (s, t, deg, wt, rc) in enumerate([(0, 0, k_e, w_exc, "gexc"), (0, 1, k_e, w_exc, "gexc"),
                                              (1, 0, k_i, w_inh, "ginh"), (1, 1, k_i, w_inh, "ginh")]):
        spec["projs"].append({
            "src": s, "tgt": t, "receptor": rc,
            "gen": {"mode": "in", "degree": deg, "dmin": 1, "dmax": dmax, "w_lo": wt,
                    "w_span": 0.0, "id": gid},
            "plastic": False,
        })
    return _offsets(spec)


def izhikevich(n: int = 1_000_000, k_out: int = 1_000, *, dt: float = 1e-3, steps: int = 1_000,
               seed: int = 3, w_scale: float = 1.0) -> dict:
    """Izhikevich (2003) 80/20 cortical network.

    Excitatory: a=0.02, b=0.2, c=-65+15r^2, d=8-6r^2; inhibitory:
    a=0.02+0.08r, b=0.25-0.05r, c=-65, d=2, with r~U(0,1) per neuron
    (Philox INIT stream, counter word c1 = 1).  Every neuron draws k_out
    postsynaptic targets over the whole network; weights 0.5*U(0,1)
    (excitatory) and -U(0,1) (inhibitory), times w_scale; delays uniform
    1..20 ms (excitatory) and 1 ms (inhibitory).  Thalamic input N(0,1)
    times 5 (excitatory) or 2 (inhibitory).  dt = 1 ms, v0 = -65, u0 = b*v0."""
    n_e = int(round(0.8 * n))
    n_i = n - n_e
    spec = {
        "name": "izhikevich", "dt": dt, "steps": steps, "seed": seed, "slow_ratio": 1,
        "pops": [
            {"name": "E", "model": "izh", "n": n_e, "params": list(IZH_RS), "hetero": "izh_exc",
             "drive": ("gauss", 0.0, 5.0)},
            {"name": "I", "model": "izh", "n": n_i, "params": [0.1, 0.2, -65.0, 2.0, 30.0],
             "hetero": "izh_inh", "drive": ("gauss", 0.0, 2.0)},
        ],
        "projs": [],
    }
    dsteps = max(1, int(round(20e-3 / dt)))
    d1 = max(1, int(round(1e-3 / dt)))
    gid = 0
    for s, wl, ws, dmin, dmax in ((0, 0.0, 0.5 * w_scale, 1, dsteps), (1, -1.0 * w_scale, 1.0 * w_scale, d1, d1)):
        for t in (0, 1):
            spec["projs"].append({
                "src": s, "tgt": t, "receptor": "current",
                "gen": {"mode": "out", "degree": k_out, "dmin": dmin, "dmax": dmax, "w_lo": wl,
                        "w_span": ws, "id": s, "cols": "all"},
                "plastic": False,
            })
            gid += 1
    return _offsets(spec)


def random_network(n_exc: int = 4_000, n_inh: int = 1_000, *, rule: str = "er", p: float = 0.02,
                   sigma: float = 50e-6, max_distance: float = 1e-3, min_probability: float = 0.0,
                   delay: int = 15, dt: float = 1e-4, steps: int = 1_000, g: float = 5.0,
                   j_psp: float = 0.1e-3, seed: int = 5) -> dict:
    """The Brunel LIF populations connected by the reference's other
    topologies, generated on the device: Erdos-Renyi with probability p
    (rule "er", src/connectivity/topology/random.cpp) or the 1D Gaussian
    distance rule (rule "distance", positions i * max_distance / n,
    src/connectivity/topology/distance_dependent.cpp).  Weights and drive
    as in brunel()."""
    spec = brunel(n_exc, n_inh, 1, 1, delay=delay, dt=dt, steps=steps, g=g, j_psp=j_psp, seed=seed)
    for q in spec["projs"]:
        gen = q["gen"]
        gen["mode"] = rule
        gen.pop("degree", None)
        if rule == "er":
            gen["p"] = p
        else:
            gen.update(sigma=sigma, max_distance=max_distance, min_probability=min_probability)
    return spec


def scaled(spec: dict, **over) -> dict:
    """Copy of a spec with fields overridden (steps, seed ...)."""
    s = copy.deepcopy(spec)
    s.update(over)
    return s


def population_arrays(spec: dict, pop: dict) -> dict:
    """Per-neuron arrays of a population: heterogeneous parameters ``hp``
    ([n_params, n] float32 or None) and initial values ``init_v`` /
    ``init_aux`` (float32 [n] or None for the model default).  Drawn from the
    Philox INIT stream keyed by global neuron id, in float32 arithmetic."""
    import numpy as np

    from . import rng

    n, off, seed = pop["n"], pop["offset"], spec["seed"]
    out = {"hp": None, "init_v": None, "init_aux": None}
    h = pop.get("hetero")
    f = np.float32
    if h in ("izh_exc", "izh_inh"):
        r = rng.init_uniform(seed, 1, off, n, 0.0, 1.0)
        hp = np.empty((5, n), np.float32)
        if h == "izh_exc":
            r2 = r * r
            hp[0] = f(0.02)
            hp[1] = f(0.2)
            hp[2] = f(15.0) * r2 + f(-65.0)
            hp[3] = f(8.0) - f(6.0) * r2
        else:
            hp[0] = f(0.02) + f(0.08) * r
            hp[1] = f(0.25) - f(0.05) * r
            hp[2] = f(-65.0)
            hp[3] = f(2.0)
        hp[4] = f(pop["params"][4])
        out["hp"] = hp
        out["init_v"] = np.full(n, -65.0, np.float32)
        out["init_aux"] = (hp[1] * f(-65.0)).astype(np.float32)
    init = pop.get("init") or {}
    if "v" in init:
        kind, lo, span, which = init["v"]
        assert kind == "uniform"
        out["init_v"] = rng.init_uniform(seed, which, off, n, lo, span)
    return out
