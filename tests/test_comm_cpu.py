"""Failure detection of a partitioned network, on CPU.

* The engine's bounded host wait (nrn_comm_bounded_wait), driven by fake
  poll functions: completion, an error code, and a wait that never ends.
* StepAgreement over world-size-2 gloo groups: ranks that agree pass; a rank
  that leaves between runs, or runs other steps, is reported on the host
  before the next run would be launched."""
import os
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from libnrn_b200 import _native as N

NRN_OK, NRN_ERR_COMM, NRN_ERR_TIMEOUT = 0, 6, 7


def _wait(poll, timeout):
    cb = N.POLL_FN(poll)
    return N.lib().nrn_comm_bounded_wait(cb, None, float(timeout))


def test_bounded_wait_completes():
    calls = []

    def poll(_):
        calls.append(1)
        return 1 if len(calls) >= 5 else 0

    assert _wait(poll, 5.0) == NRN_OK and len(calls) == 5


def test_bounded_wait_reports_failure():
    assert _wait(lambda _: -1, 5.0) == NRN_ERR_COMM


def test_bounded_wait_times_out():
    t0 = time.perf_counter()
    assert _wait(lambda _: 0, 0.3) == NRN_ERR_TIMEOUT
    el = time.perf_counter() - t0
    assert 0.29 <= el < 3.0
    assert b"timed out" in N.lib().nrn_last_error()


def test_fake_async_error_hook_is_exported():
    assert N.lib().nrn_comm_fake_async_error(0) == NRN_OK


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _agree_worker(rank, world, port, scenario, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    from libnrn_b200.partition import StepAgreement

    ag = StepAgreement(store, rank, world, timeout_s=3.0)
    ag.check(0, 15)
    ag.check(15, 30)
    if scenario == "leave" and rank == 1:
        q.put((rank, "left"))
        return                       # between runs, nothing in flight
    steps = 45 if (scenario == "mismatch" and rank == 1) else 30
    try:
        ag.check(45, steps)
        q.put((rank, "ok"))
    except RuntimeError as ex:
        q.put((rank, "error: " + str(ex)))
    if rank == 0:
        time.sleep(1.0)              # keep the store up while the peer reads


@pytest.mark.parametrize("scenario", ["agree", "leave", "mismatch"])
def test_step_agreement(scenario):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, 2, port, scenario, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    if scenario == "agree":
        assert res == {0: "ok", 1: "ok"}
    elif scenario == "leave":
        assert res[1] == "left"
        assert res[0].startswith("error") and "[1]" in res[0] and "did not reach" in res[0]
    else:
        assert res[0].startswith("error") and res[1].startswith("error")
        assert "runs steps" in res[0]
