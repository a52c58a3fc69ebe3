"""Loads the golden fixtures written by make_golden.py."""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load(name: str) -> dict:
    return dict(np.load(os.path.join(HERE, name + ".npz")))


def desc(arrs: dict) -> dict:
    return json.loads(bytes(arrs["desc"]).decode())


def load_net(name: str):
    """Returns (net, ref): the network description (oracle form, with synapse
    lists) and the reference's recorded outputs."""
    a = load(name)
    d = desc(a)
    net = {"steps": d["steps"], "dt": d["dt"], "seed": d["seed"], "slow_ratio": d["slow_ratio"],
           "pops": [], "projs": [], "trace_ids": a["trace_ids"]}
    for i, p in enumerate(d["pops"]):
        q = dict(p)
        for k in ("init_v", "init_aux", "hp"):
            q[k] = a.get(f"pop{i}_{k}")
        if q.get("drive") is not None:
            q["drive"] = tuple(q["drive"])
        net["pops"].append(q)
    for i, p in enumerate(d["projs"]):
        q = dict(p)
        q["src_idx"] = a[f"proj{i}_src"]
        q["tgt_idx"] = a[f"proj{i}_tgt"]
        q["w"] = a[f"proj{i}_w"]
        q["delay"] = a[f"proj{i}_delay"]
        net["projs"].append(q)
    ref = {k[4:]: a[k] for k in a if k.startswith("ref_") and not k.startswith("ref_w")}
    ref["w_out"] = [a[f"ref_w{i}"] for i in range(len(d["projs"]))]
    return net, ref


def load_neuron(name: str):
    a = load(name)
    d = desc(a)
    pop = {"model": d["model"], "n": d["n"], "params": d["params"], "hp": a.get("hp"),
           "init_v": a.get("init_v"), "init_aux": a.get("init_aux")}
    ref = {k[4:]: a[k] for k in a if k.startswith("ref_")}
    return pop, d["steps"], d["dt"], a["I"], ref


def spikes_by_step(step, ids, steps):
    """List of sorted id arrays per step."""
    order = np.lexsort((ids, step))
    step, ids = step[order], ids[order]
    out = []
    bounds = np.searchsorted(step, np.arange(steps + 1))
    for t in range(steps):
        out.append(ids[bounds[t]:bounds[t + 1]])
    return out
