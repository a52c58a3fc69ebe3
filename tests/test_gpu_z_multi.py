"""The network partitioned over 2, 4 or 8 GPUs (one process per GPU, spike
ids exchanged by NCCL all-gather once per window) gives the same spikes and
plastic weights as the same network on one GPU.  Each case needs as many
GPUs as ranks.  The file is collected after the single-GPU tests, so that
a run stopping at its first failure has run those."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

def needs(n):
    return pytest.mark.skipif(torch.cuda.device_count() < n, reason=f"needs {n} GPUs")


needs2 = needs(2)


def spec_of(name, steps):
    from libnrn_b200 import workloads as W
    if name == "brunel_stdp":
        return W.brunel(3000, 750, 200, 50, stdp=True, seed=3, steps=steps)
    if name == "brunel":
        return W.brunel(3000, 750, 200, 50, stdp=False, seed=4, steps=steps)
    # bursting sources: inter-spike intervals shorter than the delays
    spec = W.brunel(2000, 500, 100, 25, delay=8, stdp=True, seed=21, steps=steps)
    for p in spec["pops"]:
        p["params"][4] = 2e-4
        p["params"][2] = 0.018
        kind, lam, w = p["drive"]
        p["drive"] = (kind, lam * 2.0, w)
    return spec


def run_one(spec, device=0, partition=None):
    from libnrn_b200.engine import Network
    nw = None
    try:
        nw = Network.from_spec(spec, device=device, partition=partition)
        nw.run(spec["steps"])
        nw.sync()
        st, gid = nw.raster()
        w = [nw.weights(q) for q in range(len(spec["projs"]))]
        return {"st": st, "gid": gid, "w": w, "err": None}
    except Exception as ex:   # reported to the parent
        return {"err": f"{type(ex).__name__}: {ex}"}
    finally:
        if nw is not None:
            nw.close()


def _worker(rank, world, port, name, steps, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from libnrn_b200.partition import share_unique_id
        uid = share_unique_id()
        res = run_one(spec_of(name, steps), device=rank, partition=(rank, world, uid, 2000.0))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def run_partitioned(name, steps, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=300) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():   # a rank that did not finish: end it, report below
                p.kill()
    return [out[r] for r in range(world)]


def merged_raster(parts):
    st = np.concatenate([p["st"] for p in parts])
    gid = np.concatenate([p["gid"] for p in parts])
    o = np.lexsort((gid, st))
    return st[o], gid[o]


@pytest.mark.parametrize("world", [pytest.param(2, marks=needs(2)), pytest.param(4, marks=needs(4)),
                                   pytest.param(8, marks=needs(8))])
@pytest.mark.parametrize("name", ["brunel", "brunel_stdp"])
def test_partitioned_equals_one_gpu(name, world):
    steps = 600   # a whole number of 15-step windows
    ref = run_one(spec_of(name, steps))
    assert ref["err"] is None, ref["err"]
    parts = run_partitioned(name, steps, world)
    for p in parts:
        assert p["err"] is None, p["err"]
    st, gid = merged_raster(parts)
    assert len(gid) > 1000
    assert np.array_equal(st, ref["st"]) and np.array_equal(gid, ref["gid"])
    for q in range(len(ref["w"])):
        a = np.sort(np.concatenate([p["w"][q] for p in parts]))
        assert np.array_equal(a, np.sort(ref["w"][q]))


@needs2
def test_two_gpus_report_sources_faster_than_their_delay():
    # STDP across GPUs is exact when a plastic source does not spike twice
    # within its delay; otherwise the run reports it instead of diverging.
    parts = run_partitioned("burst", 240)
    errs = [p["err"] for p in parts]
    assert any(e is not None and "spiked twice within one synaptic delay" in e for e in errs)


# --- failure handling (no GPU is faulted: errors are made on the host) ------

def _fail_worker(rank, world, port, scenario, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from libnrn_b200 import _native as N
    from libnrn_b200.engine import Network
    from libnrn_b200.partition import StepAgreement, share_unique_id
    nw = None
    out = {"rank": rank}
    try:
        uid = share_unique_id()
        spec = spec_of("brunel", 60)
        max_rate = 2000.0 if not (scenario == "layout" and rank == 1) else 1000.0
        try:
            nw = Network.from_spec(spec, device=rank, partition=(rank, world, uid, max_rate), comm_timeout=10.0)
        except N.NrnError as ex:
            out["build"] = str(ex)
            q.put(out)
            return
        ag = StepAgreement(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=5.0,
                           prefix=f"nrn/{scenario}")
        ag.check(0, 30)
        nw.run(30)
        nw.sync()
        if scenario == "fake_error":
            if rank == 0:
                N.lib().nrn_comm_fake_async_error(6)   # ncclRemoteError, reported by the next wait
            try:
                nw.sync()
                out["sync"] = "ok"
            except N.NrnError as ex:
                out["sync"] = str(ex)
                try:
                    nw.run(15)
                    out["run_after"] = "ok"
                except N.NrnError as ex2:
                    out["run_after"] = str(ex2)
        elif scenario == "leave":
            if rank == 1:
                out["left"] = True       # between runs: nothing in flight
            else:
                try:
                    ag.check(30, 30)
                    out["check"] = "ok"
                except RuntimeError as ex:
                    out["check"] = str(ex)
        q.put(out)
    except Exception as ex:
        out["err"] = f"{type(ex).__name__}: {ex}"
        q.put(out)
    finally:
        if nw is not None:
            nw.close()
        if scenario == "leave" and rank == 0:
            import time
            time.sleep(1.0)
        dist.destroy_process_group()


def run_failure(scenario, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_fail_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = {}
        for _ in procs:
            r = q.get(timeout=180)
            out[r["rank"]] = r
    finally:
        for p in procs:
            p.join(timeout=90)
            if p.is_alive():
                p.kill()
    return out


@needs2
def test_nccl_error_aborts_communicator():
    out = run_failure("fake_error")
    assert "communicator aborted" in out[0]["sync"] or "NCCL reported" in out[0]["sync"]
    assert "aborted" in out[0]["run_after"]
    assert out[1]["sync"] == "ok"


@needs2
def test_ranks_disagreeing_on_layout_are_refused():
    out = run_failure("layout")
    for r in (0, 1):
        assert "disagree on the spike exchange" in out[r].get("build", ""), out[r]


@needs2
def test_rank_leaving_between_runs_is_found_on_the_host():
    out = run_failure("leave")
    assert out[1].get("left")
    assert "did not reach" in out[0]["check"]
