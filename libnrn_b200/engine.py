"""Host-side driver of the device engine (include/nrn_cuda.h, nrn_engine_*).

``Network`` holds a network resident on one GPU: population state lives in
torch CUDA tensors owned here (torch is the allocator only), synapses and
spike histories inside the engine.  It mirrors the reference's
sim_create / sim_run_steps / sim_get_spikes sequence
(src/simulation/runner.cpp:17-197) for Python callers: the test suite and
bench.py.  Every step runs in the CUDA library; nothing here computes.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native as N

NPARAM = {"lif": 7, "adex": 13, "izh": 5}


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


class Network:
    """A network on one GPU, or this rank's part of a network partitioned
    over GPUs: ``partition=(rank, world, nccl_unique_id, max_rate_hz)``
    (libnrn_b200.partition); populations are then added with their whole
    size ``n_global`` and this rank's slice."""

    def __init__(self, dt: float, slow_ratio: int = 1, device: int = 0, partition=None,
                 comm_timeout: float | None = None):
        self.L = N.lib()
        self.device = device
        self.dt = float(dt)
        self.dev = torch.device("cuda", device)
        h = C.c_void_p()
        N.check(self.L.nrn_engine_create(C.byref(h), device, self.dt, int(slow_ratio)), "nrn_engine_create")
        self.h = h
        self.rank, self.world = 0, 1
        if comm_timeout is not None:
            N.check(self.L.nrn_engine_set_comm_timeout(self.h, float(comm_timeout)), "nrn_engine_set_comm_timeout")
        if partition is not None:
            rank, world, uid, max_rate = partition
            buf = (C.c_uint8 * 128)(*bytes(uid))
            N.check(self.L.nrn_engine_set_partition(self.h, int(rank), int(world), C.byref(buf), float(max_rate)),
                    "nrn_engine_set_partition")
            self.rank, self.world = int(rank), int(world)
        self.pops: list[dict] = []
        self.projs: list[dict] = []
        self._keep: list = []
        self.finalized = False

    # -- construction -------------------------------------------------------
    def add_population(self, model: str, n: int, params, *, hp=None, drive=None, cond=None,
                       init_v=None, init_aux=None, record: bool = True, seed: int = 0,
                       n_global: int | None = None, local_offset: int = 0) -> int:
        """n neurons on this GPU: neurons [local_offset, local_offset + n) of a
        population of n_global (default n); per-neuron arrays are this
        slice's."""
        f32 = dict(dtype=torch.float32, device=self.dev)
        off = sum(p["n_global"] for p in self.pops)
        n_global = n if n_global is None else int(n_global)
        if init_v is None:
            v = torch.full((n,), -65.0 if model == "izh" else float(params[0]), **f32)
        else:
            v = torch.as_tensor(np.asarray(init_v, np.float32)).to(self.dev)
        aux = None
        if model != "lif":
            if init_aux is not None:
                aux = torch.as_tensor(np.asarray(init_aux, np.float32)).to(self.dev)
            elif model == "izh":
                aux = torch.full((n,), np.float32(float(params[1]) * -65.0), **f32)
            else:
                aux = torch.zeros(n, **f32)
        ref = torch.zeros(n, **f32) if model != "izh" else None
        spike = torch.zeros(n, **f32)
        i_syn = torch.zeros(n, **f32)
        d = N.PopDesc()
        d.model = N.MODEL[model]
        d.n = n
        d.gid_offset = off
        d.record = int(record)
        if n_global != n or local_offset:
            d.n_global = n_global
            d.local_offset = int(local_offset)
        d.v, d.aux, d.refractory, d.spike, d.i_syn = (_ptr(t) for t in (v, aux, ref, spike, i_syn))
        if cond is not None:
            d.tau_syn_exc, d.tau_syn_inh, d.e_exc, d.e_inh = (float(x) for x in cond)
        for k, x in enumerate(params):
            d.uniform[k] = float(x)
        hpt = None
        if hp is not None:
            hpt = torch.as_tensor(np.asarray(hp, np.float32)).to(self.dev).contiguous()
            for k in range(hpt.shape[0]):
                d.param[k] = hpt[k].data_ptr()
        if drive is not None:
            d.drive.kind = N.DRIVE[drive[0]]
            d.drive.p0 = float(drive[1])
            d.drive.p1 = float(drive[2])
            d.drive.seed = int(seed)
        pid = C.c_int32()
        N.check(self.L.nrn_engine_add_population(self.h, C.byref(d), C.byref(pid)), "add_population")
        self.pops.append({"model": model, "n": n, "n_global": n_global, "lo": int(local_offset),
                          "offset": off, "v": v, "aux": aux, "ref": ref,
                          "spike": spike, "i_syn": i_syn, "hp": hpt, "record": record})
        return pid.value

    def add_synapse_channel(self, pop: int, kind: str, tau_rise: float, tau_decay: float, e_rev: float = 0.0) -> int:
        """Synapse channel of population pop ("exp", "dexp" or "ampa",
        nrn_syn_desc_t); projections deliver into it with receptor
        "chan<k>"."""
        d = N.SynDesc()
        d.kind = N.SYN_KIND[kind]
        d.tau_rise, d.tau_decay, d.e_rev = float(tau_rise), float(tau_decay), float(e_rev)
        c = C.c_int32()
        N.check(self.L.nrn_engine_add_synapse_channel(self.h, int(pop), C.byref(d), C.byref(c)), "add_synapse_channel")
        return c.value

    def add_projection(self, src: int, tgt: int, src_idx, tgt_idx, w, delay, *, receptor="current",
                       mod=None) -> int:
        arrs = [np.ascontiguousarray(src_idx, np.int32), np.ascontiguousarray(tgt_idx, np.int32),
                np.ascontiguousarray(w, np.float32), np.ascontiguousarray(delay, np.uint8)]
        m = None if mod is None else np.ascontiguousarray(mod, np.float32)
        d = N.ProjDesc()
        d.src_pop, d.tgt_pop, d.receptor, d.on_device = src, tgt, N.RECEPTOR[receptor], 0
        d.nnz = len(arrs[0])
        d.src, d.tgt, d.w, d.delay = (a.ctypes.data for a in arrs)
        d.mod = None if m is None else m.ctypes.data
        qid = C.c_int32()
        N.check(self.L.nrn_engine_add_projection(self.h, C.byref(d), C.byref(qid)), "add_projection")
        self.projs.append({"src": src, "tgt": tgt, "nnz": d.nnz})
        return qid.value

    def generate_projection(self, src: int, tgt: int, *, out_degree: bool = False, degree: int = 0, gen_id: int,
                            dmin: int, dmax: int, w_lo: float, w_span: float, seed: int,
                            cols=None, receptor="current", rule: str = "fixed", p: float = 0.0,
                            sigma: float = 0.0, max_distance: float = 0.0, min_probability: float = 0.0) -> int:
        """Connectivity generated on the device (nrn_gen_desc_t): rule
        "fixed" (in/out-degree), "er" (probability p) or "distance"."""
        g = N.GenDesc()
        g.src_pop, g.tgt_pop, g.receptor = src, tgt, N.RECEPTOR[receptor]
        g.rule = {"fixed": 0, "er": 1, "distance": 2}[rule]
        g.p, g.sigma, g.max_distance, g.min_probability = float(p), float(sigma), float(max_distance), \
            float(min_probability)
        g.out_degree, g.degree, g.gen_id = int(out_degree), degree, gen_id
        g.col_offset, g.col_n = cols if cols is not None else (0, 0)
        g.dmin, g.dmax, g.w_lo, g.w_span, g.seed = dmin, dmax, w_lo, w_span, seed
        qid = C.c_int32()
        nnz = C.c_int64()
        N.check(self.L.nrn_engine_generate_projection(self.h, C.byref(g), C.byref(qid), C.byref(nnz)),
                "generate_projection")
        self.projs.append({"src": src, "tgt": tgt, "nnz": nnz.value})
        return qid.value

    def set_stdp(self, proj: int, params) -> None:
        arr = (C.c_double * 7)(*[float(x) for x in params])
        N.check(self.L.nrn_engine_set_stdp(self.h, proj, arr), "set_stdp")

    def set_deterministic(self, on: bool = True) -> None:
        """Deterministic delivery (nrn_engine_set_deterministic): inputs summed
        in the synapse-list order, before finalize."""
        N.check(self.L.nrn_engine_set_deterministic(self.h, int(on)), "set_deterministic")

    def finalize(self, init_update: bool = True) -> None:
        N.check(self.L.nrn_engine_finalize(self.h, int(init_update)), "finalize")
        self.finalized = True

    # -- running -----------------------------------------------------------
    def run(self, steps: int, chunk: int = 0) -> None:
        N.check(self.L.nrn_engine_run(self.h, int(steps), int(chunk)), "run")

    def profile(self, steps: int):
        """Runs steps eagerly; returns summed device ms of (delivery, neuron
        updates, plasticity) measured with CUDA events on the engine stream."""
        ms = (C.c_double * 3)()
        N.check(self.L.nrn_engine_profile(self.h, int(steps), ms), "profile")
        return tuple(ms)

    KERNEL_PHASES = ("drive", "static_delivery", "stdp_walks", "neuron_update", "stdp_step", "window_end")

    def profile_kernels(self, steps: int):
        """Runs steps with the kernels serialised on the engine stream; returns
        ({phase: summed device ms}, {"static_events", "walk_events",
        "windows", "steps"}) (nrn_engine_profile_kernels)."""
        ms = (C.c_double * 6)()
        cnt = (C.c_int64 * 4)()
        N.check(self.L.nrn_engine_profile_kernels(self.h, int(steps), ms, cnt), "profile_kernels")
        return (dict(zip(self.KERNEL_PHASES, list(ms))),
                dict(zip(("static_events", "walk_events", "windows", "steps"), list(cnt))))

    def sync(self) -> None:
        N.check(self.L.nrn_engine_sync(self.h), "sync")

    def stream(self) -> int:
        s = C.c_void_p()
        N.check(self.L.nrn_engine_stream(self.h, C.byref(s)), "stream")
        return s.value or 0

    @property
    def step(self) -> int:
        return int(self.L.nrn_engine_step(self.h))

    def prepare(self, first_step: int, steps: int, chunk: int = 0) -> None:
        """Captures the graphs a run of `steps` steps from `first_step` will
        replay, without running it (nrn_engine_prepare)."""
        N.check(self.L.nrn_engine_prepare(self.h, int(first_step), int(steps), int(chunk)), "prepare")

    def info(self) -> dict:
        """The window, raster capacity and recorded neuron count
        (nrn_engine_info)."""
        i = N.EngineInfo()
        N.check(self.L.nrn_engine_info(self.h, C.byref(i)), "info")
        return {f: int(getattr(i, f)) for f, _ in N.EngineInfo._fields_}

    def raster(self, cap: int | None = None, out=None):
        """Spikes recorded since the last call: (step, gid), sorted by step then
        id (the engine sorts on the device before the copy).  ``out``: two
        int32 arrays to copy into (for instance page-locked ones, which copy
        fastest); the result is then a prefix view of them."""
        n = C.c_int64()
        if out is not None:
            st, gd = out
            assert st.dtype == np.int32 and gd.dtype == np.int32 and st.flags.c_contiguous and gd.flags.c_contiguous
            cap = min(st.size, gd.size)
        else:
            cap = cap if cap is not None else 1 << 26
            st = np.empty(cap, np.int32)
            gd = np.empty(cap, np.int32)
        N.check(self.L.nrn_engine_raster(self.h, st.ctypes.data, gd.ctypes.data, cap, C.byref(n)), "raster")
        return st[:n.value], gd[:n.value]   # sorted on the device

    def weights(self, proj: int) -> np.ndarray:
        nnz = C.c_int64()
        N.check(self.L.nrn_engine_nnz(self.h, proj, C.byref(nnz)), "nnz")
        out = np.empty(nnz.value, np.float32)
        N.check(self.L.nrn_engine_weights(self.h, proj, out.ctypes.data, nnz.value), "weights")
        return out

    def counters(self):
        s, e = C.c_int64(), C.c_int64()
        N.check(self.L.nrn_engine_counters(self.h, C.byref(s), C.byref(e)), "counters")
        return s.value, e.value

    def enable_spike_stats(self) -> None:
        """Keep per-neuron spike statistics (before finalize)."""
        N.check(self.L.nrn_engine_enable_spike_stats(self.h), "enable_spike_stats")
        self._stats_from = None

    def spike_stats(self, pop: int) -> np.ndarray:
        """This rank's neurons' spike records of a population
        (libnrn_b200.stats.SPIKE_STAT)."""
        from .stats import SPIKE_STAT
        out = np.zeros(self.pops[pop]["n"], SPIKE_STAT)
        N.check(self.L.nrn_engine_spike_stats(self.h, pop, out.ctypes.data, out.size), "spike_stats")
        return out

    def reset_spike_stats(self) -> None:
        N.check(self.L.nrn_engine_spike_stats_reset(self.h), "spike_stats_reset")
        self._stats_from = self.step

    def population_stats(self, pop: int) -> dict:
        """Rate and CV of the inter-spike interval of a population's neurons on
        this rank since the statistics were enabled or reset."""
        from .stats import summarize
        start = getattr(self, "_stats_from", None) or 0
        return summarize(self.spike_stats(pop), self.step - start, self.dt)

    def checkpoint(self) -> bytes:
        """The engine's device state (neurons, spike histories, weights,
        plasticity state, step, counters, unread raster) as bytes; see
        nrn_engine_checkpoint_save."""
        n = C.c_int64()
        N.check(self.L.nrn_engine_checkpoint_size(self.h, C.byref(n)), "checkpoint_size")
        buf = np.empty(n.value, np.uint8)
        N.check(self.L.nrn_engine_checkpoint_save(self.h, buf.ctypes.data, n.value), "checkpoint_save")
        return buf.tobytes()

    def restore(self, ckpt: bytes) -> None:
        """Loads a checkpoint taken from an engine built from the same network."""
        buf = np.frombuffer(ckpt, np.uint8)
        N.check(self.L.nrn_engine_checkpoint_load(self.h, buf.ctypes.data, buf.size), "checkpoint_load")

    def state(self, name: str) -> np.ndarray:
        """Concatenated state variable over all populations (host copy)."""
        self.sync()
        parts = []
        for p in self.pops:
            t = p[name]
            parts.append(np.zeros(p["n"], np.float32) if t is None else t.cpu().numpy())
        return np.concatenate(parts)

    def close(self) -> None:
        if getattr(self, "h", None):
            self.L.nrn_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- builders ----------------------------------------------------------
    @classmethod
    def from_net(cls, net: dict, device: int = 0, record: bool = True, spike_stats: bool = False,
                 deterministic: bool = False) -> "Network":
        """From a network description with explicit synapse lists (the
        oracle's form)."""
        nw = cls(net["dt"], net.get("slow_ratio", 1), device)
        for p in net["pops"]:
            pid = nw.add_population(p["model"], p["n"], p["params"], hp=p.get("hp"), drive=p.get("drive"),
                                    cond=p.get("cond"), init_v=p.get("init_v"), init_aux=p.get("init_aux"),
                                    record=record, seed=net.get("seed", 0))
            for ch in p.get("syn") or []:
                nw.add_synapse_channel(pid, ch[0], ch[1], ch[2], ch[3])
        for q in net.get("projs", []):
            qid = nw.add_projection(q["src"], q["tgt"], q["src_idx"], q["tgt_idx"], q["w"], q["delay"],
                                    receptor=q.get("receptor", "current"), mod=q.get("mod"))
            if q.get("plastic"):
                nw.set_stdp(qid, q["stdp"])
        if spike_stats:
            nw.enable_spike_stats()
        if deterministic:
            nw.set_deterministic(True)
        nw.finalize(True)
        return nw

    @classmethod
    def from_spec(cls, spec: dict, device: int = 0, record: bool = True, partition=None,
                  spike_stats: bool = False, comm_timeout: float | None = None) -> "Network":
        """From a workload spec (libnrn_b200.workloads), connectivity
        generated on the device; with ``partition``, this rank's slice."""
        from . import workloads as W
        from .partition import partition_range

        nw = cls(spec["dt"], spec.get("slow_ratio", 1), device, partition=partition, comm_timeout=comm_timeout)
        for p in spec["pops"]:
            arr = W.population_arrays(spec, p)
            lo, n = partition_range(p["n"], nw.rank, nw.world)

            def cut(a):
                if a is None:
                    return None
                a = np.asarray(a)
                return a[..., lo:lo + n]

            nw.add_population(p["model"], n, p["params"], hp=cut(arr["hp"]), drive=p.get("drive"),
                              cond=p.get("cond"), init_v=cut(arr["init_v"]), init_aux=cut(arr["init_aux"]),
                              record=record, seed=spec["seed"], n_global=p["n"], local_offset=lo)
        for q in spec["projs"]:
            g = q["gen"]
            cols = (0, spec["n_total"]) if g.get("cols") == "all" else None
            rule = g["mode"] if g["mode"] in ("er", "distance") else "fixed"
            qid = nw.generate_projection(q["src"], q["tgt"], out_degree=g["mode"] == "out",
                                         degree=g.get("degree", 0), gen_id=g["id"], dmin=g["dmin"],
                                         dmax=g["dmax"], w_lo=g["w_lo"], w_span=g["w_span"], seed=spec["seed"],
                                         cols=cols, receptor=q["receptor"], rule=rule, p=g.get("p", 0.0),
                                         sigma=g.get("sigma", 0.0), max_distance=g.get("max_distance", 0.0),
                                         min_probability=g.get("min_probability", 0.0))
            if q.get("plastic"):
                nw.set_stdp(qid, q["stdp"])
        if spike_stats:
            nw.enable_spike_stats()
        nw.finalize(True)
        return nw
