"""Generates the golden fixtures under tests/golden/ from the reference
implementation itself (oracle/_ref, compiled from the reference's sources by
oracle/Makefile; needs the reference tree, so it runs in the build
container, not on a GPU box).

Each fixture holds the inputs (network description, synapse lists, input
currents) and the reference's outputs.  The script also runs the C
restatement (oracle/nrn_oracle.c) and refuses to write a fixture it does not
reproduce: identical spike trains, state within 1e-5 relative.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import specs as S  # noqa: E402
from oracle import oracle as O  # noqa: E402

# Philox4x32-10 known-answer vectors published with Random123 (kat_vectors):
# (counter words, key words, output words).
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def save_net(name: str, net: dict, ref: dict, meta: dict) -> None:
    arrs = {}
    for i, p in enumerate(net["pops"]):
        for k in ("init_v", "init_aux", "hp"):
            if p.get(k) is not None:
                arrs[f"pop{i}_{k}"] = np.asarray(p[k], np.float32)
    for i, q in enumerate(net["projs"]):
        arrs[f"proj{i}_src"] = q["src_idx"]
        arrs[f"proj{i}_tgt"] = q["tgt_idx"]
        arrs[f"proj{i}_w"] = q["w"]
        arrs[f"proj{i}_delay"] = q["delay"]
        arrs[f"ref_w{i}"] = ref["w_out"][i]
    for k in ("spike_step", "spike_id", "final_v", "final_aux", "final_ref", "trace_v"):
        arrs[f"ref_{k}"] = ref[k]
    arrs["trace_ids"] = np.asarray(net.get("trace_ids", []), np.int32)
    desc = {
        "steps": net["steps"], "dt": net["dt"], "seed": net["seed"], "slow_ratio": net["slow_ratio"],
        "pops": [{k: p[k] for k in ("model", "n", "params", "drive", "cond")} for p in net["pops"]],
        "projs": [{k: q[k] for k in ("src", "tgt", "receptor", "plastic", "stdp")} for q in net["projs"]],
        "meta": meta,
    }
    arrs["desc"] = np.frombuffer(json.dumps(desc).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrs)


def check(a: dict, b: dict, what: str) -> dict:
    same = np.array_equal(a["spike_step"], b["spike_step"]) and np.array_equal(a["spike_id"], b["spike_id"])
    scale = max(1e-30, float(np.abs(b["trace_v"]).max()) if b["trace_v"].size else 1.0)
    rel = float(np.abs(a["trace_v"] - b["trace_v"]).max()) / scale if b["trace_v"].size else 0.0
    wrel = 0.0
    for x, y in zip(a["w_out"], b["w_out"]):
        if y.size:
            wrel = max(wrel, float(np.abs(x - y).max() / max(1e-30, np.abs(y).max())))
    assert same, f"{what}: C restatement spike trains differ from the reference"
    assert rel <= 1e-5 and wrel <= 1e-5, f"{what}: state differs (v {rel}, w {wrel})"
    return {"spikes": int(len(b["spike_id"])), "v_rel": rel, "w_rel": wrel}


def net_case(name: str, spec: dict, dyadic_bits=None) -> None:
    n = spec["n_total"]
    net = S.realize(spec, trace_ids=range(0, n, max(1, n // 64)), dyadic_bits=dyadic_bits)
    ref = O.run_reference(net)
    orc = O.run_oracle(net)
    meta = check(orc, ref, name)
    meta["rate_hz"] = meta["spikes"] / n / (net["steps"] * net["dt"])
    save_net(name, net, ref, meta)
    print(name, meta)


def neuron_case(name: str, model: str, params, n: int, steps: int, dt: float, I, hp=None,
                init_v=None, init_aux=None) -> None:
    pop = {"model": model, "n": n, "params": params, "hp": hp, "init_v": init_v, "init_aux": init_aux}
    ref = O.neuron_reference(pop, steps, dt, I)
    orc = O.neuron_oracle(pop, steps, dt, I)
    # AdEx calls exp: torch's vectorised float exp and libm's expf may differ
    # in the last bit, so AdEx state is held to 1e-5 relative, spikes exactly.
    exact = model != "adex"
    for k in ("v", "aux", "ref", "spike"):
        if exact or k == "spike":
            assert np.array_equal(ref[k], orc[k]), f"{name}: {k} differs"
        else:
            err = np.abs(ref[k].astype(np.float64) - orc[k]) / np.maximum(np.abs(ref[k]), 1e-30)
            err[np.abs(ref[k]) < 1e-30] = 0.0
            assert float(err.max()) <= 1e-5, f"{name}: {k} differs by {float(err.max())}"
    arrs = {f"ref_{k}": ref[k] for k in ("v", "aux", "ref", "spike")}
    arrs["I"] = np.asarray(I, np.float32)
    for k, a in (("hp", hp), ("init_v", init_v), ("init_aux", init_aux)):
        if a is not None:
            arrs[k] = np.asarray(a, np.float32)
    desc = {"model": model, "n": n, "params": list(params), "steps": steps, "dt": dt}
    arrs["desc"] = np.frombuffer(json.dumps(desc).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrs)
    print(name, "spikes", int(ref["spike"].sum()))


def main() -> None:
    if not O.reference_available():
        O.build(reference=True)
    rs = np.random.RandomState(1234)

    # --- neuron-only traces (the reference's *_forward, fixed input currents)
    n = 16
    I = np.empty((1500, n), np.float32)
    I[:] = np.linspace(0.0, 800e-12, n, dtype=np.float32)   # 0..800 pA ramp across neurons
    I[:, 8:] += (rs.rand(1500, 8).astype(np.float32) * 300e-12)  # noisy half
    neuron_case("neuron_lif", "lif", O.LIF_DEFAULT, n, 1500, 1e-4, I,
                init_v=np.linspace(-0.070, -0.049, n, dtype=np.float32))
    I = np.empty((2000, n), np.float32)
    I[:] = np.linspace(0.0, 1.5e-9, n, dtype=np.float32)
    I[:, 8:] += (rs.rand(2000, 8).astype(np.float32) * 0.5e-9)
    neuron_case("neuron_adex", "adex", O.ADEX_DEFAULT, n, 2000, 1e-4, I)
    r = rs.rand(n).astype(np.float32)
    hp = np.stack([np.full(n, 0.02, np.float32), np.full(n, 0.2, np.float32),
                   np.float32(15.0) * r * r + np.float32(-65.0), np.float32(8.0) - np.float32(6.0) * r * r,
                   np.full(n, 30.0, np.float32)]).astype(np.float32)
    I = (rs.randn(1000, n) * 5.0).astype(np.float32) + np.linspace(0, 12, n, dtype=np.float32)
    neuron_case("neuron_izh", "izh", O.IZH_DEFAULT, n, 1000, 1e-3, I, hp=hp,
                init_v=np.full(n, -65.0, np.float32), init_aux=(hp[1] * np.float32(-65.0)))

    # --- networks
    net_case("net_brunel_stdp", S.small_brunel(stdp=True, steps=400))
    net_case("net_brunel_slow", S.small_brunel(stdp=True, steps=300, slow_ratio=10, seed=21))
    # AdEx: libm expf vs torch exp differ in the last bit now and then; in this
    # chaotic network the first spike flips after ~230 steps, so the exact
    # window is 200 steps (longer runs are compared by rate statistics).
    net_case("net_adex", S.small_adex(steps=200))
    # Izhikevich weights are U(0,1) draws; rounded to multiples of 2^-10 here
    # so that every summation order gives the same fp32 input (bit-exact
    # comparisons; the undithered network is compared by rate statistics).
    net_case("net_izh", S.small_izh(steps=300), dyadic_bits=10)

    # --- the reference's Erdos-Renyi connect() (seeded), for connect() parity
    rp, ci, W, M = O.reference_er_connect(100, 100, 16, 0.1, False, 500e-12, 42, True)
    np.savez_compressed(os.path.join(HERE, "er_connect.npz"), row_ptr=rp, col_idx=ci, weights=W, mask=M,
                        desc=np.frombuffer(json.dumps({"n": 100, "block": 16, "p": 0.1, "autapses": False,
                                                       "weight_scale": 500e-12, "seed": 42}).encode(),
                                           np.uint8))

    # --- a user program of the nrn:: API, built against the reference
    #     (oracle/Makefile) and run on its CPU path
    exe = os.path.join(os.path.dirname(O.HERE), "oracle", "_ref", "dropin_brunel_ref")
    import subprocess
    import tempfile
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "ref.bin")
        subprocess.run([exe, out, "cpu", "300"], check=True, stdout=subprocess.DEVNULL)
        raw = open(out, "rb").read()
    hdr = np.frombuffer(raw[:12], np.int32)
    body = np.frombuffer(raw[12:], np.float32)
    ne, ni, nw = (int(x) for x in hdr)
    np.savez_compressed(os.path.join(HERE, "dropin_brunel.npz"), exc=body[:2 * ne].reshape(-1, 2),
                        inh=body[2 * ne:2 * (ne + ni)].reshape(-1, 2), w_ee=body[2 * (ne + ni):])
    print("dropin_brunel", ne, ni)

    # --- Philox known answers
    np.savez_compressed(os.path.join(HERE, "philox_kat.npz"),
                        kat=np.array([list(c) + list(k) + list(o) for c, k, o in PHILOX_KAT], np.uint64))
    print("done")


if __name__ == "__main__":
    main()
