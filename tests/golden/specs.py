"""Realises a workload spec (libnrn_b200.workloads) as an oracle network:
host-generated synapse lists (oracle generator, same Philox counters as the
device generator) and per-neuron arrays."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from libnrn_b200 import workloads as W  # noqa: E402
from oracle import oracle as O  # noqa: E402


def gen_args(spec: dict, q: dict):
    """Arguments of the fixed-degree generator for projection q."""
    ps, pt = spec["pops"][q["src"]], spec["pops"][q["tgt"]]
    g = q["gen"]
    assert g["mode"] in ("in", "out"), "random rules: gen_lists"
    out = g["mode"] == "out"
    if out:
        if g.get("cols") == "all":
            col_off, col_n = 0, spec["n_total"]
        else:
            col_off, col_n = pt["offset"], pt["n"]
        args = (spec["seed"], g["id"], ps["n"], ps["offset"], col_n, col_off, g["degree"])
    else:
        args = (spec["seed"], g["id"], ps["n"], ps["offset"], pt["n"], pt["offset"], g["degree"])
    kw = dict(out_degree=out, no_autapses=True, dmin=g["dmin"], dmax=g["dmax"],
              w_lo=g["w_lo"], w_span=g["w_span"], keep=(pt["offset"], pt["offset"] + pt["n"]))
    return args, kw


def gen_lists(spec: dict, q: dict):
    """The synapse list of projection q drawn by the oracle's generator of
    its rule (fixed degree, Erdos-Renyi or distance-dependent)."""
    g = q["gen"]
    if g["mode"] in ("er", "distance"):
        ps, pt = spec["pops"][q["src"]], spec["pops"][q["tgt"]]
        return O.gen_random(g["mode"], spec["seed"], g["id"], ps["n"], pt["n"], pt["offset"],
                            same_pop=q["src"] == q["tgt"], p=g.get("p", 0.0), sigma=g.get("sigma", 0.0),
                            max_distance=g.get("max_distance", 0.0), min_probability=g.get("min_probability", 0.0),
                            dmin=g["dmin"], dmax=g["dmax"], w_lo=g["w_lo"], w_span=g["w_span"])
    args, kw = gen_args(spec, q)
    return O.gen_fixed_degree(*args, **kw)


def realize(spec: dict, *, steps=None, trace_ids=None, dyadic_bits=None) -> dict:
    """dyadic_bits=k rounds every weight to a multiple of 2^-k, so that sums
    of a few weights are exact in fp32 and independent of summation order."""
    net = {"steps": steps if steps is not None else spec["steps"], "dt": spec["dt"],
           "seed": spec["seed"], "slow_ratio": spec.get("slow_ratio", 1), "pops": [], "projs": []}
    for p in spec["pops"]:
        arr = W.population_arrays(spec, p)
        net["pops"].append({"model": p["model"], "n": p["n"], "params": p["params"],
                            "drive": p.get("drive"), "cond": p.get("cond"),
                            "init_v": arr["init_v"], "init_aux": arr["init_aux"], "hp": arr["hp"]})
    for q in spec["projs"]:
        s, t, w, d = gen_lists(spec, q)
        if dyadic_bits is not None:
            w = (np.round(w.astype(np.float64) * 2.0 ** dyadic_bits) / 2.0 ** dyadic_bits).astype(np.float32)
        net["projs"].append({"src": q["src"], "tgt": q["tgt"], "receptor": q["receptor"],
                             "src_idx": s, "tgt_idx": t, "w": w, "delay": d,
                             "plastic": q.get("plastic", False),
                             "stdp": q.get("stdp", [0.02, 0.02, 0.01, -0.012, 0.0, 1.0, 1.0])})
    if trace_ids is not None:
        net["trace_ids"] = list(trace_ids)
    return net


def small_brunel(stdp=True, steps=400, slow_ratio=1, seed=11):
    return W.brunel(800, 200, 80, 20, steps=steps, stdp=stdp, seed=seed, slow_ratio=slow_ratio)


def small_adex(steps=300, seed=12):
    # in-degree scaled 1000 -> 50; weights scaled to keep k*w
    return W.adex_cond(500, 50, steps=steps, seed=seed, w_exc=0.5e-9 * 6, w_inh=2.5e-9 * 6)


def small_izh(steps=300, seed=13):
    return W.izhikevich(500, 50, steps=steps, seed=seed, w_scale=20.0)


def synapse_channel_net(steps=600, seed=21, scale=(0.1, 0.2, 0.3)):
    """The small Brunel network with the reference's declared synapse models
    as synapse channels (parity unpinned: the reference's forwards are
    stubs): E->E through an exponential current channel (tau 5 ms), E->I
    through a double-exponential channel (0.5 / 5 ms), I->E through an
    AMPA-form conductance channel (0.5 / 5 ms) with reversal -10 mV, I->I
    static.  Weights are dyadic, so the channel inputs sum exactly in any
    order."""
    spec = small_brunel(stdp=False, steps=steps, seed=seed)
    net = realize(spec, dyadic_bits=44)
    net["pops"][0]["syn"] = [("exp", 0.5e-3, 5e-3, 0.0), ("ampa", 0.5e-3, 5e-3, -0.010)]
    net["pops"][1]["syn"] = [("dexp", 0.5e-3, 5e-3, 0.0)]
    q = net["projs"]
    q[0]["receptor"] = "chan0"     # E -> E, exponential
    q[1]["receptor"] = "chan0"     # E -> I, double exponential
    q[2]["receptor"] = "chan1"     # I -> E, AMPA form
    q[0]["w"] = _dyadic(q[0]["w"] * np.float32(scale[0]), 44)
    q[1]["w"] = _dyadic(q[1]["w"] * np.float32(scale[1]), 44)
    # conductance weights: |w| / 25 mV
    q[2]["w"] = _dyadic(np.abs(q[2]["w"]) / np.float32(0.025) * np.float32(scale[2]), 44)
    return net


def _dyadic(w, bits):
    return (np.round(np.asarray(w, np.float64) * 2.0 ** bits) / 2.0 ** bits).astype(np.float32)
