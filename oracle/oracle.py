"""Python binding of the CPU oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by bench.py's CPU-baseline leg, as the checker.  The product package
(``libnrn_b200``) never imports this module.

Two CPU implementations share one network description:

* ``run_oracle``     -- the C restatement, ``oracle/nrn_oracle.c``
                        (built into ``oracle/_lib/libnrn_oracle.so``);
* ``run_reference``  -- the reference implementation itself, compiled from
                        its own sources (``oracle/_ref/libnrn_ref.so``) and
                        driven by ``oracle/ref_harness.cpp``.

A network is a dict::

    {"pops":  [pop, ...], "projs": [proj, ...], "steps": T, "dt": 1e-4,
     "slow_ratio": 1, "seed": 7, "trace_ids": [...]}
    pop  = {"model": "lif"|"adex"|"izh", "n": n, "params": [...],
            "syn": None | [(kind "exp"|"dexp"|"ampa", tau_rise, tau_decay, e_rev), ...]
                   (synapse channels; receptor "chanK" delivers into channel K),
            "drive": None | ("poisson", lam, amp) | ("gauss", mean, std)
                        | ("poisson_gexc", lam, amp),
            "cond": None | [tau_e, tau_i, e_exc, e_inh],
            "init_v": None|f32[n], "init_aux": None|f32[n], "hp": None|f32[np,n]}
    proj = {"src": p, "tgt": p, "receptor": "current"|"gexc"|"ginh",
            "src_idx": i32[nnz] (sorted), "tgt_idx": i32[nnz], "w": f32[nnz],
            "delay": u8[nnz], "plastic": bool,
            "stdp": [tau_plus, tau_minus, a_plus, a_minus, w_min, w_max, lr]}
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(HERE, "_lib")
REF_DIR = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(LIB_DIR, "libnrn_oracle.so")
HARNESS_SO = os.path.join(REF_DIR, "libnrn_ref_harness.so")

MODELS = {"lif": 0, "adex": 1, "izh": 2}
NPARAM = {"lif": 7, "adex": 13, "izh": 5}
DRIVES = {None: 0, "poisson": 1, "gauss": 2, "poisson_gexc": 3}
RECEPTORS = {"current": 0, "gexc": 1, "ginh": 2, "chan0": 16, "chan1": 17, "chan2": 18, "chan3": 19}
SYN_KINDS = {"exp": 1, "dexp": 2, "ampa": 3}

# Default parameters of the reference's option structs
# (include/nrn/neuron/options.h:23-92).
LIF_DEFAULT = [-0.065, -0.050, -0.065, 0.010, 0.002, 250e-12, 0.0]
ADEX_DEFAULT = [-0.0706, -0.0504, -0.0706, 0.0, 9.37e-3, 0.144, 0.002, 281e-12,
                30e-9, 4e-9, 80.5e-12, 0.002, 0.0]
IZH_DEFAULT = [0.02, 0.2, -65.0, 8.0, 30.0]


class OrcPop(C.Structure):
    _fields_ = [("model", C.c_int32), ("n", C.c_int32), ("offset", C.c_int32),
                ("drive_kind", C.c_int32), ("p", C.c_double * 16), ("cond", C.c_double * 4),
                ("drive", C.c_double * 4), ("init_v", C.c_void_p), ("init_aux", C.c_void_p),
                ("hp", C.c_void_p), ("n_chan", C.c_int32), ("chan_kind", C.c_int32 * 4),
                ("chan_tau", (C.c_double * 2) * 4), ("chan_e", C.c_double * 4)]


class OrcProj(C.Structure):
    _fields_ = [("src_pop", C.c_int32), ("tgt_pop", C.c_int32), ("receptor", C.c_int32),
                ("plastic", C.c_int32), ("nnz", C.c_int64), ("src", C.c_void_p),
                ("tgt", C.c_void_p), ("w", C.c_void_p), ("delay", C.c_void_p),
                ("stdp", C.c_double * 7), ("w_out", C.c_void_p)]


class OrcNet(C.Structure):
    _fields_ = [("npop", C.c_int32), ("nproj", C.c_int32), ("pops", C.POINTER(OrcPop)),
                ("projs", C.POINTER(OrcProj)), ("steps", C.c_int32), ("slow_ratio", C.c_int32),
                ("dt", C.c_double), ("seed", C.c_uint64), ("spike_cap", C.c_int64),
                ("n_spikes", C.c_void_p), ("spike_step", C.c_void_p), ("spike_id", C.c_void_p),
                ("final_v", C.c_void_p), ("final_aux", C.c_void_p), ("final_ref", C.c_void_p),
                ("trace_n", C.c_int32), ("trace_ids", C.c_void_p), ("trace_v", C.c_void_p),
                ("threads", C.c_int32)]


def _ptr(a):
    return None if a is None else a.ctypes.data


# Where the reference's sources are read from when the reference is built:
# $NRN_REFERENCE_DIR, else the build container's copy.  The GPU box has no
# reference tree; it uses the libraries built here (oracle/_ref).
DEFAULT_REFERENCE_DIR = "/root/reference"


def reference_dir() -> str | None:
    """The reference source tree, or None (reported) when it is absent."""
    d = os.environ.get("NRN_REFERENCE_DIR", DEFAULT_REFERENCE_DIR)
    if os.path.isdir(os.path.join(d, "src")) and os.path.isdir(os.path.join(d, "include")):
        return d
    print(f"oracle: no reference sources at {d} (set NRN_REFERENCE_DIR); "
          "building the C restatement only", file=sys.stderr)
    return None


def build(reference: bool | None = None) -> None:
    """Builds the C restatement and, when the reference sources are present
    (reference=None: look for them; True: required), the reference itself
    from its unmodified sources into oracle/_ref (a parallel make: its CUDA
    files take minutes each through the LibTorch headers)."""
    ref = reference_dir() if reference is not False else None
    if reference is True and ref is None:
        raise FileNotFoundError("reference sources not found (NRN_REFERENCE_DIR)")
    targets = ["cport"] + (["ref"] if ref else [])
    jobs = str(max(2, min(16, os.cpu_count() or 2)))
    extra = [f"REF={ref}"] if ref else []
    subprocess.run(["make", "-s", "-j", jobs, "-C", HERE, f"PY={sys.executable}"] + extra + targets,
                   check=True, stdout=subprocess.DEVNULL)


_libs: dict = {}


def _lib(which: str):
    if which not in _libs:
        path = ORACLE_SO if which == "oracle" else HARNESS_SO
        if not os.path.exists(path):
            if which == "oracle":
                build(False)
            else:
                raise FileNotFoundError(f"reference harness not built: {path}")
        lib = C.CDLL(path)
        if which == "oracle":
            lib.orc_net_run.argtypes = [C.POINTER(OrcNet)]
            lib.orc_neuron_run.argtypes = [C.POINTER(OrcPop), C.c_int, C.c_double] + [C.c_void_p] * 5
            lib.orc_gen_fixed_degree.restype = C.c_int64
            lib.orc_gen_fixed_degree.argtypes = [C.c_int, C.c_uint64, C.c_uint32] + [C.c_int32] * 5 + \
                [C.c_int, C.c_int32, C.c_int32, C.c_float, C.c_float, C.c_int32, C.c_int32] + \
                [C.c_void_p] * 4
            lib.orc_init_uniform.argtypes = [C.c_uint64, C.c_uint32, C.c_int32, C.c_int32, C.c_float,
                                             C.c_float, C.c_void_p]
            lib.orc_drive_values.argtypes = [C.c_int, C.c_double, C.c_double, C.c_uint64,
                                             C.c_int32, C.c_int32, C.c_int32, C.c_void_p]
            lib.orc_philox.argtypes = [C.c_uint64] + [C.c_uint32] * 4 + [C.c_void_p]
            lib.orc_gen_random.restype = C.c_int64
            lib.orc_gen_random.argtypes = [C.c_int, C.c_uint64, C.c_uint32] + [C.c_int32] * 5 + [C.c_int] + \
                [C.c_double] * 4 + [C.c_int32, C.c_int32, C.c_float, C.c_float] + [C.c_void_p] * 4
            lib.orc_normal_from_words.restype = C.c_float
            lib.orc_normal_from_words.argtypes = [C.c_uint32, C.c_uint32]
        else:
            lib.ref_net_run.argtypes = [C.POINTER(OrcNet), C.c_int64, C.POINTER(C.c_double)]
            lib.ref_neuron_run.argtypes = [C.POINTER(OrcPop), C.c_int, C.c_double] + [C.c_void_p] * 5
            lib.ref_er_connect.restype = C.c_int64
            lib.ref_er_connect.argtypes = [C.c_int64, C.c_int64, C.c_int64, C.c_double, C.c_int,
                                           C.c_double, C.c_uint64, C.c_int] + [C.c_void_p] * 4 + [C.c_int64]
        _libs[which] = lib
    return _libs[which]


def reference_available() -> bool:
    return os.path.exists(HARNESS_SO)


def _fill_pop(pop: dict, offset: int, keep: list) -> OrcPop:
    P = OrcPop()
    P.model = MODELS[pop["model"]]
    P.n = int(pop["n"])
    P.offset = offset
    drive = pop.get("drive")
    kind = drive[0] if drive else None
    P.drive_kind = DRIVES[kind]
    for i, x in enumerate(pop["params"]):
        P.p[i] = float(x)
    if pop.get("cond") is not None:
        for i, x in enumerate(pop["cond"]):
            P.cond[i] = float(x)
    if drive:
        for i, x in enumerate(drive[1:]):
            P.drive[i] = float(x)
    # synapse channels: [(kind, tau_rise, tau_decay, e_rev), ...]
    for c, ch in enumerate(pop.get("syn") or []):
        P.chan_kind[c] = SYN_KINDS[ch[0]]
        P.chan_tau[c][0], P.chan_tau[c][1] = float(ch[1]), float(ch[2])
        P.chan_e[c] = float(ch[3])
        P.n_chan = c + 1
    for name in ("init_v", "init_aux", "hp"):
        a = pop.get(name)
        if a is not None:
            a = np.ascontiguousarray(a, dtype=np.float32)
            keep.append(a)
            setattr(P, name, a.ctypes.data)
    return P


def _prepare(net: dict, spike_cap: int | None = None):
    keep: list = []
    pops = net["pops"]
    offs = np.cumsum([0] + [p["n"] for p in pops])[:-1]
    N = int(sum(p["n"] for p in pops))
    parr = (OrcPop * len(pops))(*[_fill_pop(p, int(o), keep) for p, o in zip(pops, offs)])
    projs = net.get("projs", [])
    qarr = (OrcProj * max(1, len(projs)))()
    w_outs = []
    for i, q in enumerate(projs):
        Q = qarr[i]
        Q.src_pop, Q.tgt_pop = int(q["src"]), int(q["tgt"])
        Q.receptor = RECEPTORS[q.get("receptor", "current")]
        Q.plastic = int(bool(q.get("plastic", False)))
        arrs = [np.ascontiguousarray(q["src_idx"], np.int32), np.ascontiguousarray(q["tgt_idx"], np.int32),
                np.ascontiguousarray(q["w"], np.float32), np.ascontiguousarray(q["delay"], np.uint8)]
        keep.extend(arrs)
        Q.nnz = len(arrs[0])
        Q.src, Q.tgt, Q.w, Q.delay = (a.ctypes.data for a in arrs)
        for k, x in enumerate(q.get("stdp", [0.02, 0.02, 0.01, -0.012, 0.0, 1.0, 1.0])):
            Q.stdp[k] = float(x)
        wo = np.zeros(Q.nnz, np.float32)
        w_outs.append(wo)
        Q.w_out = wo.ctypes.data
    steps = int(net["steps"])
    cap = spike_cap if spike_cap is not None else max(1024, N * steps // 4)
    out = {
        "n_spikes": np.zeros(1, np.int64), "spike_step": np.zeros(cap, np.int32),
        "spike_id": np.zeros(cap, np.int32), "final_v": np.zeros(N, np.float32),
        "final_aux": np.zeros(N, np.float32), "final_ref": np.zeros(N, np.float32),
    }
    tids = np.ascontiguousarray(net.get("trace_ids", []), np.int32)
    out["trace_v"] = np.zeros((steps, len(tids)), np.float32)
    keep.append(tids)
    S = OrcNet()
    S.npop, S.nproj = len(pops), len(projs)
    S.pops, S.projs = parr, qarr
    S.steps = steps
    S.slow_ratio = int(net.get("slow_ratio", 1))
    S.dt = float(net["dt"])
    S.seed = int(net.get("seed", 0))
    S.spike_cap = cap
    for k in ("n_spikes", "spike_step", "spike_id", "final_v", "final_aux", "final_ref", "trace_v"):
        setattr(S, k, out[k].ctypes.data)
    S.trace_n = len(tids)
    S.trace_ids = tids.ctypes.data if len(tids) else None
    S.threads = int(net.get("threads", 0))
    return S, out, w_outs, (keep, parr, qarr)


def _finish(S, out, w_outs):
    n = int(out["n_spikes"][0])
    if n > S.spike_cap:
        raise RuntimeError("spike capacity exceeded")
    res = {k: out[k] for k in ("final_v", "final_aux", "final_ref", "trace_v")}
    res["spike_step"] = out["spike_step"][:n].copy()
    res["spike_id"] = out["spike_id"][:n].copy()
    res["w_out"] = w_outs
    return res


def run_oracle(net: dict, spike_cap: int | None = None) -> dict:
    """Runs the C restatement on the network description."""
    S, out, w_outs, _keep = _prepare(net, spike_cap)
    _lib("oracle").orc_net_run(C.byref(S))
    return _finish(S, out, w_outs)


def run_reference(net: dict, block: int = 64, spike_cap: int | None = None) -> dict:
    """Runs the reference implementation (compiled unmodified) on the network."""
    S, out, w_outs, _keep = _prepare(net, spike_cap)
    el = C.c_double(0.0)
    _lib("harness").ref_net_run(C.byref(S), int(block), C.byref(el))
    res = _finish(S, out, w_outs)
    res["elapsed_s"] = el.value
    return res


def _neuron(which: str, pop: dict, steps: int, dt: float, I=None):
    keep: list = []
    P = _fill_pop(pop, 0, keep)
    n = int(pop["n"])
    I = None if I is None else np.ascontiguousarray(I, np.float32).reshape(steps, n)
    o = {k: np.zeros((steps, n), np.float32) for k in ("v", "aux", "ref")}
    o["spike"] = np.zeros((steps, n), np.uint8)
    fn = _lib(which).orc_neuron_run if which == "oracle" else _lib(which).ref_neuron_run
    fn(C.byref(P), int(steps), float(dt), _ptr(I), o["v"].ctypes.data, o["aux"].ctypes.data,
       o["ref"].ctypes.data, o["spike"].ctypes.data)
    return o


def neuron_oracle(pop: dict, steps: int, dt: float, I=None) -> dict:
    return _neuron("oracle", pop, steps, dt, I)


def neuron_reference(pop: dict, steps: int, dt: float, I=None) -> dict:
    return _neuron("harness", pop, steps, dt, I)


def gen_fixed_degree(seed: int, gen: int, n_src: int, src_offset: int, n_tgt: int,
                     tgt_offset: int, degree: int, *, out_degree: bool = False,
                     no_autapses: bool = True, dmin: int = 1, dmax: int = 1,
                     w_lo: float = 1.0, w_span: float = 0.0, keep=None):
    """Fixed in-degree (or out-degree) synapse list in source-major order.

    Sources are local to [src_offset, src_offset + n_src); kept targets are
    local to keep = (lo, hi) (default: the whole target range)."""
    lo, hi = keep if keep is not None else (tgt_offset, tgt_offset + n_tgt)
    lib = _lib("oracle")
    args = (int(out_degree), seed, gen, n_src, src_offset, n_tgt, tgt_offset, degree,
            int(no_autapses), dmin, dmax, float(w_lo), float(w_span), lo, hi)
    total = lib.orc_gen_fixed_degree(*args, None, None, None, None)
    s = np.zeros(total, np.int32)
    t = np.zeros(total, np.int32)
    w = np.zeros(total, np.float32)
    d = np.zeros(total, np.uint8)
    lib.orc_gen_fixed_degree(*args, s.ctypes.data, t.ctypes.data, w.ctypes.data, d.ctypes.data)
    return s, t, w, d


def gen_random(rule: str, seed: int, gen: int, n_src: int, n_tgt: int, tgt_gid_offset: int, *,
               same_pop: bool, p: float = 0.0, sigma: float = 0.0, max_distance: float = 0.0,
               min_probability: float = 0.0, dmin: int = 1, dmax: int = 1, w_lo: float = 1.0,
               w_span: float = 0.0, keep=None):
    """Random ("er") or distance-dependent ("distance") synapse list, rows =
    target population indices keep = (lo, n) (default all), in row order;
    targets relative to lo."""
    lo, nr = keep if keep is not None else (0, n_tgt)
    lib = _lib("oracle")
    args = ({"er": 1, "distance": 2}[rule], seed, gen, n_src, n_tgt, lo, nr, tgt_gid_offset, int(same_pop),
            float(p), float(sigma), float(max_distance), float(min_probability), dmin, dmax, float(w_lo),
            float(w_span))
    total = lib.orc_gen_random(*args, None, None, None, None)
    s = np.zeros(total, np.int32)
    t = np.zeros(total, np.int32)
    w = np.zeros(total, np.float32)
    d = np.zeros(total, np.uint8)
    lib.orc_gen_random(*args, s.ctypes.data, t.ctypes.data, w.ctypes.data, d.ctypes.data)
    return s, t, w, d


def init_uniform(seed: int, which: int, offset: int, n: int, lo: float, span: float):
    out = np.zeros(n, np.float32)
    _lib("oracle").orc_init_uniform(seed, which, offset, n, float(lo), float(span), out.ctypes.data)
    return out


def drive_values(kind: str, d0: float, d1: float, seed: int, offset: int, n: int, step: int):
    out = np.zeros(n, np.float32)
    _lib("oracle").orc_drive_values(DRIVES[kind], d0, d1, seed, offset, n, step, out.ctypes.data)
    return out


def philox(seed: int, c0: int, c1: int, c2: int, c3: int):
    out = np.zeros(4, np.uint32)
    _lib("oracle").orc_philox(seed, c0, c1, c2, c3, out.ctypes.data)
    return out


def reference_er_connect(n_src: int, n_tgt: int, block: int, p: float, autapses: bool,
                         weight_scale: float, seed: int, same_population: bool):
    """The reference's connect() with its Erdos-Renyi generator, seeded."""
    ntb = (n_tgt + block - 1) // block
    nsb = (n_src + block - 1) // block
    nb = ntb * nsb
    rp = np.zeros(ntb + 1, np.int32)
    ci = np.zeros(nb, np.int32)
    W = np.zeros((nb, block, block), np.float32)
    M = np.zeros((nb, block, block), np.float32)
    got = _lib("harness").ref_er_connect(n_src, n_tgt, block, p, int(autapses), weight_scale, seed,
                                         int(same_population), rp.ctypes.data, ci.ctypes.data,
                                         W.ctypes.data, M.ctypes.data, nb)
    assert got == nb
    return rp, ci, W, M
