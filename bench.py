"""Benchmark: synaptic events/s, neuron updates/s and real-time factor of the
per-timestep simulation loop on B200.

Workload (default): the Brunel balanced LIF network with pair STDP on E->E,
1,048,576 neurons per GPU (838,860 E + 209,716 I), fixed in-degree 1,000 E +
250 I (1.31e9 synapses per GPU), delay 15 steps, dt 0.1 ms, Poisson drive at
2 nu_thr, weights clipped to [0, 2J].  Connectivity is generated on the GPU
from Philox (synthetic, seeded).  One bench step = one simulation timestep.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload brunel_stdp|brunel|adex|izh|bsr]

`--workload bsr` is the batched-trial block-sparse product (64 trials, 262,144
neurons, 2% of 64x64 bf16 blocks) with its own metric line.

Prints one JSON line (rank 0).  `value` is delivered synaptic events per
second over the timed steps with the network resident in HBM; `e2e` is the
same run through the C ABI with the initial state uploaded from pinned host
memory and the spike raster downloaded, inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return PEAKS_FALLBACK, "fallback"


def workload_spec(name: str, world: int, steps: int, scale: float = 1.0):
    from libnrn_b200 import workloads as W

    def scaled(n):   # population sizes of a scaled-down network: multiples of 4
        return max(4, int(round(n * scale / 4)) * 4)

    if name == "brunel_stdp":
        if scale != 1.0:
            return W.brunel(scaled(838_860 * world), scaled(209_716 * world), 1_000, 250, steps=steps, stdp=True)
        return W.brunel_stdp_per_gpu(world, steps=steps)
    if name == "brunel":
        return W.brunel(10_000 * world, 2_500 * world, 1_000, 250, steps=steps)
    if name == "brunel_1m":
        # the bench network without plasticity: 1,048,576 LIF neurons and
        # 1.31e9 static synapses per GPU
        return W.brunel(scaled(838_860 * world), scaled(209_716 * world), 1_000, 250, steps=steps)
    if name == "adex":
        return W.adex_cond(1_048_576 * world, 1_000, steps=steps)
    if name == "izh":
        return W.izhikevich(1_000_000 * world, 1_000, steps=steps)
    raise SystemExit(f"unknown workload {name}")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def wait_first(self, limit_s: float) -> None:
        """Waits (at most limit_s) until nvidia-smi has printed a sample."""
        t0 = time.perf_counter()
        while self.proc and not self.rows and time.perf_counter() - t0 < limit_s:
            time.sleep(0.02)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                mhz.append(float(r[1]))
                mx = float(r[2])
                for k, nm in enumerate(names):
                    if r[5 + k].lower().startswith("active"):
                        reasons.add(nm)
            except Exception:
                continue
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(mhz)}


def cpu_reference(args, world_steps_hint=None):
    """The reference's own CPU implementation (compiled from its unmodified
    sources into oracle/_ref) on a bounded sample of the workload, with all
    host threads.  The reference stores every projection as dense B x B
    blocks (memory grows as N_src * N_tgt: about 4 TB at the bench's 1M
    neurons), so the sample is the 12,500-neuron Brunel network of the
    reference's own example configuration.  Without oracle/_ref (a snapshot
    built without the reference sources) the C restatement runs instead, on
    one thread, and the line says why."""
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import numpy as np
    from libnrn_b200 import workloads as W
    from oracle import oracle as O
    import specs as S

    threads = os.cpu_count() or 1
    if args.workload == "bsr":
        return cpu_bsr_sample(threads)
    steps = int(os.environ.get("NRN_CPU_SAMPLE_STEPS", "30"))
    if args.workload in ("brunel_stdp", "brunel", "brunel_1m"):
        spec = W.brunel(10_000, 2_500, 1_000, 250, steps=steps, stdp=args.workload == "brunel_stdp")
        sample = (f"Brunel LIF 10,000 E + 2,500 I, in-degree 1,000 + 250, delay 15, "
                  f"{'STDP on E->E, ' if args.workload == 'brunel_stdp' else ''}{steps} steps, block 256; "
                  f"events per step over the steps after the first delay")
    elif args.workload == "adex":
        spec = W.adex_cond(16_384, 1_000, steps=steps)
        sample = f"AdEx conductance network 16,384 neurons, in-degree 1,000, {steps} steps, block 256"
    else:
        spec = W.izhikevich(16_000, 1_000, dt=1e-3, steps=steps)
        sample = f"Izhikevich 16,000 neurons, out-degree 1,000, {steps} steps, block 256"
    net = S.realize(spec)
    net["threads"] = threads
    reason = None
    if O.reference_available():
        kind, cores = "reference", threads
        res = O.run_reference(net, block=256)
        elapsed = res["elapsed_s"]
    else:
        kind, cores = "port", 1
        reason = ("oracle/_ref was not built (the reference sources were absent when build() ran); "
                  "the single-threaded C restatement oracle/nrn_oracle.c ran instead")
        t0 = time.perf_counter()
        res = O.run_oracle(net)
        elapsed = time.perf_counter() - t0
    # delivered events: spikes whose delay has elapsed within the sample
    n_total = spec["n_total"]
    outdeg = np.zeros(n_total, np.int64)
    delay_of = {}
    for q, p in zip(net["projs"], spec["projs"]):
        off = spec["pops"][p["src"]]["offset"]
        np.add.at(outdeg, q["src_idx"] + off, 1)
        delay_of[p["src"]] = int(q["delay"].min()) if len(q["delay"]) else 1
    dmin = min(delay_of.values()) if delay_of else 1
    st, gid = res["spike_step"], res["spike_id"]
    ev = int(outdeg[gid[st + dmin < steps]].sum())
    # No spike can arrive in the first dmin steps of the sample, but the
    # reference spends the same time on every step (its block-dense product
    # runs regardless of spikes): events per step are taken over the steps
    # that deliver, time per step over all steps.
    per_step_s = elapsed / steps
    ev_per_step = ev / max(1, steps - dmin)
    out = {
        "events_per_s": ev_per_step / per_step_s, "neuron_updates_per_s": n_total * steps / elapsed,
        "rtf": elapsed / (steps * spec["dt"]), "elapsed_s": elapsed, "cores": cores, "kind": kind,
        "sample": sample, "same_config": False,
        "same_config_note": "the reference's dense-block storage cannot hold the bench network",
    }
    if reason:
        out["reason"] = reason
    return out


# dram__bytes_read.sum + dram__bytes_write.sum of one walk_kernel launch in an
# ncu capture of the bench network at 262,144 neurons (bench.py --scale 0.25
# --burn-in 200, launch 301), and the walk events of a step at that size;
# the bench line scales the bytes by its own walk events per step.
WALK_TRAFFIC_CAPTURED = 13.138432e6 + 0.0
WALK_EVENTS_CAPTURED = 632_380.0
# the same for the full-size block-sparse product (one launch, 262,144
# neurons, 64 trials)
BSR_TRAFFIC_CAPTURED = 2.854493e9 + 44.104192e6

BSR_N = 262_144          # pre = post neurons of the batched block-sparse workload
BSR_DENSITY = 0.02       # fraction of the 64x64 block slots present
BSR_P = 0.01             # spike probability per neuron, trial and step


def cpu_bsr_sample(threads: int) -> dict:
    """The batched block-sparse product on the host cores (torch fp32, all
    threads) for a sample of 64 block rows of the full-size workload (82
    blocks of 64x64 per row on average, 64 trials), scaled to one step of
    all 4,096 block rows."""
    import torch
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(4)
    nb_rows, nc, rows = BSR_N // 64, BSR_N // 64, 64
    per_row = int(round(BSR_DENSITY * nc))
    w = torch.randn(rows * per_row, 64, 64, generator=g) * 0.02
    cols = torch.randint(0, nc, (rows * per_row,), generator=g)
    s = (torch.rand(BSR_N, 64, generator=g) < BSR_P).float().view(nc, 64, 64)
    out = torch.zeros(rows, 64, 64)
    reps = 3
    t0 = time.perf_counter()
    for _ in range(reps):
        prod = torch.bmm(w, s[cols])
        out.index_add_(0, torch.arange(rows).repeat_interleave(per_row), prod)
    dt = (time.perf_counter() - t0) / reps * (nb_rows / rows)
    n_blocks = int(round(BSR_DENSITY * nb_rows * nc))
    return {"updates_per_s": n_blocks * 64 * 64 * 64 / dt, "step_s": dt, "cores": threads, "kind": "port",
            "sample": f"torch fp32 block product, 64 of 4,096 block rows ({per_row} blocks each, 64 trials), "
                      f"{reps} repetitions, scaled to all rows"}


def run_bsr(args, rank: int, world: int, local: int) -> None:
    """C4: 64 trials of a 262,144 x 262,144 network of 64x64 bf16 blocks at
    2% block density; Bernoulli(0.01) spikes per step.  The workload does not
    shard: at N GPUs each rank runs its own replica (`value` sums them)."""
    import torch

    from libnrn_b200 import bsr as B

    peaks, peaks_kind = load_peaks()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=600))

    def reduce(x: float, op: str) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
        return float(t.item())

    n = max(64, int(BSR_N * args.scale) // 64 * 64)
    w = B.BlockSparse.random(n, n, BSR_DENSITY, seed=4)
    tiles = B.spike_tiles(w.n_pre_blocks)
    cur = torch.zeros(n, 64, device="cuda")
    stream = torch.cuda.current_stream()

    def step(s: int) -> None:
        B.bernoulli_spikes(tiles, 5, s, BSR_P, stream)
        w.propagate(tiles, cur, stream)

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    w.check()
    if dist is not None:
        dist.barrier()
    with ClockSampler(local) as clk:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for s in range(args.steps):
            step(args.warmup + s)
        b.record(stream)
        torch.cuda.synchronize()
    w.check()
    ms = reduce(a.elapsed_time(b), "max")
    updates = w.n_blocks * 64 * 64 * 64   # (synapse, trial) pairs per step
    value = reduce(updates * args.steps / (ms / 1e3), "sum")
    # the dominant kernel alone (propagation), CUDA events on the same stream
    kp = max(10, args.steps // 10)
    a.record(stream)
    for _ in range(kp):
        w.propagate(tiles, cur, stream)
    b.record(stream)
    torch.cuda.synchronize()
    w.check()
    k_ms = a.elapsed_time(b) / kp
    alg_bytes = w.n_blocks * 8192 + n * 64 * 8 + n * 64 * 2   # weights, currents r/w, spikes once
    flops = 2.0 * 64 ** 3 * w.n_blocks
    achieved = alg_bytes / (k_ms / 1e3) / 1e9
    # e2e: each step's spike tiles from pinned host memory, the currents back at the end
    host_tiles = tiles.cpu().pin_memory()
    host_cur = torch.empty(cur.shape, dtype=cur.dtype).pin_memory()
    torch.cuda.synchronize()
    k_e2e = max(5, min(args.steps, 50))
    t0 = time.perf_counter()
    for _ in range(k_e2e):
        tiles.copy_(host_tiles, non_blocking=True)
        w.propagate(tiles, cur, stream)
    host_cur.copy_(cur, non_blocking=True)
    torch.cuda.synchronize()
    e2e_s = reduce(time.perf_counter() - t0, "max")
    e2e = reduce(updates * k_e2e, "sum") / e2e_s
    cpu = None
    if not args.no_cpu and rank == 0:
        try:
            cpu = cpu_bsr_sample(os.cpu_count() or 1)
        except Exception as ex:
            cpu = {"error": str(ex)[:200]}
    line = {
        "metric": "synapse_trial_updates_per_s", "value": value, "unit": "updates/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 x bf16 -> f32",
        "data": "synthetic (seeded block positions, N(0, 0.02) weights, Bernoulli spikes)",
        "config": {"workload": "bsr", "neurons": n, "trials": 64, "blocks": w.n_blocks, "block": 64,
                   "density": BSR_DENSITY, "p_spike": BSR_P,
                   "l2": f"inputs larger than L2 (weights {w.n_blocks * 8192 / 1e9:.2f} GB)",
                   "parallelism": "single GPU" if world == 1 else f"{world} independent replicas"},
        "kernel_ms": k_ms, "tflops": flops / (k_ms / 1e3) / 1e12,
        "gpu_launches": 2 * args.steps,
        "roofline": {"kernel": "bsr_kernel", "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "peak_kind": peaks_kind,
                     "traffic": BSR_TRAFFIC_CAPTURED if n == BSR_N else None,
                     "traffic_note": "DRAM bytes of one full-size bsr_kernel launch from an ncu capture",
                     "tensor_frac": flops / (k_ms / 1e3) / 1e12 / peaks.get("bf16_tflops", 1590.0)},
        "e2e": {"value": e2e, "unit": "updates/s", "h2d_bytes_per_step": tiles.numel() * 2,
                "d2h_bytes_per_step": cur.numel() * 4 / k_e2e},
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu if "error" in cpu else {
            "value": cpu["updates_per_s"], "unit": "updates/s", "cores": cpu["cores"], "kind": cpu["kind"],
            "sample": cpu["sample"]}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_reference_arm(args, rank: int):
    if rank != 0:
        return
    r = cpu_reference(args)
    if args.workload == "bsr":
        line = {"impl": "reference", "metric": "synapse_trial_updates_per_s", "value": r["updates_per_s"],
                "unit": "updates/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "dtype": "f32", "data": "synthetic", "config": {"workload": "bsr"},
                "cpu_baseline": {"value": r["updates_per_s"], "unit": "updates/s", "cores": r["cores"],
                                 "kind": r["kind"], "sample": r["sample"]},
                "e2e": {"value": r["updates_per_s"], "unit": "updates/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    line = {
        "impl": "reference", "metric": "synaptic_events_per_s", "value": r["events_per_s"],
        "unit": "events/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload + " (bounded CPU sample)"},
        "neuron_updates_per_s": r["neuron_updates_per_s"], "rtf": r["rtf"],
        "cpu_baseline": {k: r[k] for k in ("cores", "kind", "sample", "same_config", "same_config_note", "reason")
                         if k in r} | {"value": r["events_per_s"], "unit": "events/s"},
        "e2e": {"value": r["events_per_s"], "unit": "events/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_network(args, rank: int, world: int, local: int) -> None:
    """The spiking-network workloads (default: Brunel + STDP, 1,048,576
    neurons per GPU)."""
    import numpy as np
    import torch

    from libnrn_b200.engine import Network
    from libnrn_b200.partition import share_unique_id

    peaks, peaks_kind = load_peaks()
    torch.cuda.set_device(local)
    dist = None
    partition = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=600))
        partition = (rank, world, share_unique_id(), args.max_rate)

    def all_reduce(x: float, op: str) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
        return float(t.item())

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    spec = workload_spec(args.workload, world, args.steps, args.scale)
    t_setup = time.perf_counter()
    nw = Network.from_spec(spec, device=local, record=True, partition=partition)
    torch.cuda.synchronize()
    setup_s = all_reduce(time.perf_counter() - t_setup, "max")
    nnz = all_reduce(float(sum(p["nnz"] for p in nw.projs)), "sum")
    n_total = spec["n_total"]
    stream = torch.cuda.ExternalStream(nw.stream())

    # burn-in (untimed): the network leaves its start-up transient
    burn = max(0, args.burn_in)
    while burn > 0:
        k = min(burn, 2000)
        nw.run(k, args.chunk)
        nw.sync()
        nw.raster()
        burn -= k
    # The timed run starts on a window boundary (whole-window graphs first).
    win = nw.info()["window"]
    lead = (-(nw.step + args.warmup)) % win
    if lead:
        nw.run(lead, args.chunk)
    # Graphs (untimed): the engine runs every step inside CUDA graphs keyed
    # by the window phase and length of each piece of a run; the graphs the
    # warm-up and the timed run replay are captured and uploaded here without
    # running them, so none is captured inside the timed region.
    nw.prepare(nw.step, args.warmup, args.chunk)
    nw.prepare(nw.step + args.warmup, args.steps, args.chunk)
    nw.sync()
    nw.raster()
    # Clocks are sampled from the warm-up through the end-to-end run: a
    # short timed region (tens of steps) holds no sample of its own.
    with ClockSampler(local) as clk:
        clk.wait_first(2.0)
        nw.run(args.warmup, args.chunk)
        nw.sync()
        nw.raster()
        s0, e0 = nw.counters()
        barrier()
        ev_a = torch.cuda.Event(enable_timing=True)
        ev_b = torch.cuda.Event(enable_timing=True)
        ev_a.record(stream)
        nw.run(args.steps, args.chunk)
        ev_b.record(stream)
        torch.cuda.synchronize()
        ms = all_reduce(ev_a.elapsed_time(ev_b), "max")
        barrier()
        nw.sync()
        s1, e1 = nw.counters()
        nw.raster()
        events = all_reduce(float(e1 - e0), "sum")
        spikes = all_reduce(float(s1 - s0), "sum")
        sec = ms / 1e3
        value = events / sec

        # e2e: this rank's state from pinned host, run, raster to host, all
        # timed (wall clock, max over ranks).  The copies run on torch's
        # stream; the engine stream starts after them.  The host copy is the
        # state the engine holds when the timed region starts (a state from
        # an earlier step would put neurons out of step with their spike
        # history and traces).
        # the raster is read into page-locked host arrays allocated up front
        rcap = sum(p["n"] for p in nw.pops) * 64
        rcap = min(max(rcap, 1 << 20), 1 << 26)
        r_st = torch.empty(rcap, dtype=torch.int32).pin_memory().numpy()
        r_gid = torch.empty(rcap, dtype=torch.int32).pin_memory().numpy()
        nw.prepare(nw.step, args.steps, args.chunk)   # the end-to-end run's graphs, untimed
        nw.sync()
        nw.raster()
        host_state = []
        for p in nw.pops:
            for k in ("v", "ref"):
                t = p[k]
                if t is not None:
                    host_state.append((t, t.cpu().pin_memory()))
        h2d = sum(h.numel() * 4 for _, h in host_state)
        barrier()
        t0 = time.perf_counter()
        for dev_t, h in host_state:
            dev_t.copy_(h, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        t_up = time.perf_counter()
        e_s0, e_e0 = nw.counters()
        nw.run(args.steps, args.chunk)
        nw.sync()
        t_run = time.perf_counter()
        st2, gid2 = nw.raster(out=(r_st, r_gid))
        e_s1, e_e1 = nw.counters()
        t1 = time.perf_counter()
    e2e_s = all_reduce(t1 - t0, "max")
    e2e = all_reduce(float(e_e1 - e_e0), "sum") / e2e_s
    d2h = all_reduce(float(len(gid2) * 8), "sum")
    h2d = all_reduce(float(h2d), "sum")
    del host_state, r_st, r_gid, st2, gid2
    torch.cuda.synchronize()

    # Per-kernel device times: the same steps with the kernels serialised
    # on the engine stream, CUDA events between them (the timed run above
    # overlaps static delivery and the drive with the STDP walks).
    prof, cnt = nw.profile_kernels(args.profile_steps)
    finish_network_line(args, spec, nw, world, rank, dist, all_reduce, peaks, peaks_kind, clk, ms, value, events,
                        spikes, nnz, setup_s, prof, cnt, e2e, e2e_s, h2d, d2h, (t0, t_up, t_run, t1))


# Random-access ceilings of one B200, measured by libnrn_b200/csrc/l2_probe.cu
# (`bench.py --probe-l2`) with the delivery kernels' memory pattern and
# array sizes, and nothing else (no dependent chains, no STDP logic):
WALK_EVENTS_PER_S = 85.2e9     # a 16-byte and a 4-byte load and a reduction at one random
                               # target, with the synapse's 12 B sequential stream
STATIC_EVENTS_PER_S = 155.4e9  # a reduction at a random target with the 8 B sequential stream


def l2_floor(kernel, cnt, prof, steps):
    """The dominant kernel's floor: its events at the probe's rate for the
    same memory pattern.  A walk event is one 16-byte load (the target's
    newest spike steps), one 4-byte load (its trace at the source spike) and
    one reduction; a static event is one reduction."""
    if kernel == "walk_kernel":
        floor_s = cnt["walk_events"] / WALK_EVENTS_PER_S
        ms = prof["stdp_walks"]
    elif kernel == "deliver_kernel":
        floor_s = cnt["static_events"] / STATIC_EVENTS_PER_S
        ms = prof["static_delivery"]
    else:
        return None
    if ms <= 0 or steps <= 0:
        return None
    return {"floor_ms_per_launch": floor_s * 1e3 / steps, "ms_per_launch": ms / steps,
            "frac": floor_s * 1e3 / ms,
            "note": "the kernel's events at the measured rate of their memory pattern alone (walk event: "
                    "85.2 G/s; static event: 155.4 G/s): the bound of this kernel"}


def finish_network_line(args, spec, nw, world, rank, dist, all_reduce, peaks, peaks_kind, clk, ms, value, events,
                        spikes, nnz, setup_s, prof, cnt, e2e, e2e_s, h2d, d2h, tmarks):
    import numpy as np
    import torch

    P = max(1, cnt["steps"])
    _, gid_p = nw.raster()            # the profiled steps' spikes
    n_total = spec["n_total"]
    sec = ms / 1e3
    # Algorithmic HBM bytes per launch (one launch per step):
    #  walk_kernel: 12 B per event through a plastic segment (target index,
    #    weight read and write) + 32 B per arriving spike (segment bounds 16 B,
    #    segment state read and write 16 B);
    #  deliver_kernel: 8 B per static event (target, weight) + 16 B per
    #    (spike, delay segment) for its bounds;
    #  neuron update: 40 B per neuron (v, refractory, input read and zeroed,
    #    drive, spike flag, target trace ring read and write).
    pop_spikes = []
    for p_ in spec["pops"]:
        pop_spikes.append(int(np.count_nonzero((gid_p >= p_["offset"]) & (gid_p < p_["offset"] + p_["n"]))))
    arrivals, segs = 0.0, 0.0
    for q in spec["projs"]:
        g = q["gen"]
        nd = g["dmax"] - g["dmin"] + 1
        if q.get("plastic"):
            ps_, pt_ = spec["pops"][q["src"]], spec["pops"][q["tgt"]]
            mean_out = g["degree"] * (pt_["n"] / world) / ps_["n"] if g["mode"] == "in" else g["degree"] / world
            arrivals += cnt["walk_events"] / max(mean_out, 1e-9)
        else:
            segs += pop_spikes[q["src"]] * nd
    walk_bytes = 12.0 * cnt["walk_events"] + 32.0 * arrivals
    deliver_bytes = 8.0 * cnt["static_events"] + 16.0 * segs
    neuron_bytes = 40.0 * sum(p_["n"] for p_ in nw.pops) * P
    # the neuron update of uniform-parameter LIF populations runs four neurons
    # a thread (lif4_group_kernel); other models run pop_group_kernel
    neuron_kernel = "lif4_group_kernel" if all(p_["model"] == "lif" for p_ in spec["pops"]) else "pop_group_kernel"
    kern = {"walk_kernel": ("stdp_walks", walk_bytes), "deliver_kernel": ("static_delivery", deliver_bytes),
            neuron_kernel: ("neuron_update", neuron_bytes)}
    dom = max(kern, key=lambda k: prof[kern[k][0]])
    dom_ms = prof[kern[dom][0]]
    dom_bytes = kern[dom][1]
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9 if dom_ms > 0 else 0.0
    # Random L2 operations of the delivery: one reduction per event, plus per
    # plastic event two loads (the target's spike steps and its trace).
    l2_ops = cnt["static_events"] + cnt["walk_events"] * 3
    deliv_ms = prof["static_delivery"] + prof["stdp_walks"]
    traffic = None
    if args.workload == "brunel_stdp" and dom == "walk_kernel" and cnt["walk_events"] > 0:
        traffic = WALK_TRAFFIC_CAPTURED * (cnt["walk_events"] / P) / WALK_EVENTS_CAPTURED

    exch_ms = None
    if dist is not None:
        win = min(15, 32)
        block = sum(win + 1 + max(4096, int(-(-p_["n_global"] // world) * win * args.max_rate * spec["dt"] + 0.999999))
                    for p_ in nw.pops)
        sb = torch.zeros(block, dtype=torch.int32, device="cuda")
        rb = torch.zeros(block * world, dtype=torch.int32, device="cuda")
        for _ in range(3):
            dist.all_gather_into_tensor(rb, sb)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(20):
            dist.all_gather_into_tensor(rb, sb)
        a1.record()
        torch.cuda.synchronize()
        exch_ms = all_reduce(a0.elapsed_time(a1) / 20, "max")
        del sb, rb

    cpu = None
    if not args.no_cpu and rank == 0:
        try:
            cpu = cpu_reference(args)
        except Exception as ex:  # report, do not fail the GPU line
            cpu = {"error": str(ex)[:200]}

    n_walk = sum(1 for q in spec["projs"] if q.get("plastic"))
    windows = args.steps // 15 if (world > 1 or n_walk) else 0
    kernels_per_step = 3 + n_walk     # drive, static delivery, walks, one neuron launch (one model)
    chunk = args.chunk if args.chunk > 0 else 45
    t0, t_up, t_run, t1 = tmarks
    line = {
        "metric": "synaptic_events_per_s", "value": value, "unit": "events/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (Philox-generated connectivity and drive)",
        "config": {"workload": args.workload, "neurons": n_total, "synapses": int(nnz),
                   "dt_ms": spec["dt"] * 1e3, "burn_in_steps": max(0, args.burn_in),
                   "l2": f"inputs larger than L2 (synapse store {nnz * 8 / 1e9:.1f} GB)",
                   "parallelism": "single GPU" if world == 1 else
                   f"partitioned by neuron over {world} GPUs, NCCL all-gather of spike ids per 15-step window"},
        "neuron_updates_per_s": n_total * args.steps / sec,
        "rtf": sec / (args.steps * spec["dt"]),
        "spikes": int(spikes), "rate_hz": spikes / n_total / (args.steps * spec["dt"]),
        "setup_s": setup_s,
        "gpu_launches": kernels_per_step * args.steps + windows * (1 + len(nw.pops) * (2 if world > 1 else 0))
        + (args.steps + chunk - 1) // chunk,
        "kernel_ms_per_step": {k: v / P for k, v in prof.items()},
        "kernel_ms_note": "the kernels run one after the other with CUDA events between them over "
                          f"{P} further steps; the timed run overlaps static delivery and the drive with the walks",
        "exchange_ms_per_window": exch_ms,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_kind": peaks_kind,
                     "bytes_per_launch": dom_bytes / P, "ms_per_launch": dom_ms / P,
                     "counts_per_step": {"walk_events": cnt["walk_events"] / P,
                                         "static_events": cnt["static_events"] / P,
                                         "arriving_plastic_spikes": arrivals / P,
                                         "static_segments": segs / P, "profiled_steps": P},
                     "step_frac": (walk_bytes + deliver_bytes + neuron_bytes) / P / (ms / args.steps / 1e3) / 1e9
                     / peaks["hbm_gbs"],
                     "traffic": traffic,
                     "traffic_note": "DRAM bytes of one walk_kernel launch from an ncu capture at 262,144 neurons, "
                                     "scaled by walk events per step to this run" if traffic else None,
                     "l2_floor": l2_floor(dom, cnt, prof, P),
                     "l2_random_ops_per_s": l2_ops / (deliv_ms / 1e3) if deliv_ms > 0 else None,
                     "l2_note": "random L2 reductions and loads of static delivery + walks per second of their "
                                "serialised time; measured ceilings of one kind alone: 186 G/s reductions, 222 G/s "
                                "16-byte loads, 285 G/s 4-byte loads; mixed as in a walk event: 256 G/s"},
        "e2e": {"value": e2e, "unit": "events/s", "h2d_bytes_per_step": h2d / args.steps,
                "d2h_bytes_per_step": d2h / args.steps,
                "seconds": {"upload": t_up - t0, "run": t_run - t_up, "raster": t1 - t_run}},
        "clocks": clk.summary() | {"window": "sampled through the warm-up, timed and end-to-end runs"},
    }
    if cpu is not None:
        if "error" in cpu:
            line["cpu_baseline"] = cpu
        else:
            line["cpu_baseline"] = {k: cpu[k] for k in ("same_config", "same_config_note", "reason") if k in cpu}
            line["cpu_baseline"] |= {"value": cpu["events_per_s"], "unit": "events/s", "cores": cpu["cores"],
                                     "kind": cpu["kind"], "sample": cpu["sample"],
                                     "neuron_updates_per_s": cpu["neuron_updates_per_s"], "rtf": cpu["rtf"]}
    torch.cuda.synchronize()
    nw.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10_000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="brunel_stdp", choices=["brunel_stdp", "brunel_1m", "brunel", "adex", "izh", "bsr", "api_c1"])
    ap.add_argument("--chunk", type=int, default=0)
    ap.add_argument("--burn-in", type=int, default=1000,
                    help="untimed steps after set-up and before the warm-up, so that the timed steps see the "
                         "network's steady activity rather than its start-up transient")
    ap.add_argument("--profile-steps", type=int, default=300)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--max-rate", type=float, default=200.0,
                    help="mean firing rate bound (Hz) that sizes the multi-GPU spike exchange buffers")
    ap.add_argument("--scale", type=float, default=1.0,
                    help="network size factor (profiling of small cases only; the bench line uses 1)")
    ap.add_argument("--probe-l2", action="store_true",
                    help="run the random-access throughput probe (libnrn_b200/_lib/l2_probe) and exit")
    args = ap.parse_args()
    if args.probe_l2:
        from libnrn_b200 import build as B
        subprocess.run([B.build_probe()], check=True)
        return
    args.warmup = max(3, args.warmup)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank)
        return
    if args.workload == "bsr":
        run_bsr(args, rank, world, local)
        return
    if args.workload == "api_c1":
        run_api(args, rank)
        return
    run_network(args, rank, world, local)


def run_api(args, rank: int) -> None:
    """The reference's Brunel example configuration (10,000 E + 2,500 I,
    p = 0.1, STDP on E->E) through the nrn:: C++ API (libnrn.so): one
    sim_run_steps(K) call against K sim_step calls (tests/cpp/api_bench.cpp)."""
    if rank != 0:
        return
    exe = os.path.join(ROOT, "tests", "cpp", "_bin", "api_bench")
    if not os.path.exists(exe):
        raise SystemExit(f"{exe} not built (python -c 'import __graft_entry__ as g; g.build()')")
    out = subprocess.run([exe, str(args.steps)], capture_output=True, text=True, check=True).stdout
    line = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    line["n_gpus"] = 1
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
