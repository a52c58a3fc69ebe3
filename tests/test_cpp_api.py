"""The nrn:: C++ API (libnrn.so): the reference's suites re-expressed in C++
(tests/cpp/), Erdos-Renyi connect() parity with the reference, and one user
program built against both the reference and this library."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

import fixtures as F
from libnrn_b200 import build as B


@pytest.fixture(scope="module")
def bins():
    return B.build_cpp_tests()


def run(exe, *args, timeout=600):
    r = subprocess.run([exe, *map(str, args)], capture_output=True, text=True, timeout=timeout)
    return r.returncode, r.stdout + r.stderr


def test_core_suites_host(bins):
    rc, out = run(bins["test_core"])
    assert rc == 0, out


def test_erdos_renyi_connect_matches_reference(bins):
    ref = F.load("er_connect")
    d = F.desc(ref)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "er.bin")
        rc, out = run(bins["er_dump"], path, d["n"], d["block"], d["p"], d["weight_scale"], d["seed"])
        assert rc == 0, out
        raw = open(path, "rb").read()
    nr, nb = np.frombuffer(raw[:16], np.int64)
    body = raw[16:]
    rp = np.frombuffer(body[:4 * nr], np.int32)
    ci = np.frombuffer(body[4 * nr:4 * (nr + nb)], np.int32)
    rest = np.frombuffer(body[4 * (nr + nb):], np.float32)
    bb = d["block"] * d["block"]
    W, M = rest[:nb * bb], rest[nb * bb:]
    assert np.array_equal(rp, ref["row_ptr"]) and np.array_equal(ci, ref["col_idx"])
    assert np.array_equal(W, ref["weights"].reshape(-1))
    assert np.array_equal(M, ref["mask"].reshape(-1))


@pytest.mark.gpu
def test_gpu_api_suites(bins):
    rc, out = run(bins["test_gpu_api"])
    assert rc == 0, out


@pytest.mark.gpu
def test_dropin_program_matches_reference(bins):
    """tests/cpp/dropin_brunel.cpp built against the reference (run on its
    CPU path when the fixture was made) and against this library (GPU)."""
    ref = F.load("dropin_brunel")
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "ours.bin")
        rc, out = run(bins["dropin_brunel"], path, "cuda", 300)
        assert rc == 0, out
        raw = open(path, "rb").read()
    ne, ni, nw = (int(x) for x in np.frombuffer(raw[:12], np.int32))
    body = np.frombuffer(raw[12:], np.float32)
    exc = body[:2 * ne].reshape(-1, 2)
    inh = body[2 * ne:2 * (ne + ni)].reshape(-1, 2)
    w = body[2 * (ne + ni):]
    assert np.array_equal(exc, ref["exc"])
    assert np.array_equal(inh, ref["inh"])
    scale = float(np.abs(ref["w_ee"]).max())
    assert float(np.abs(w - ref["w_ee"]).max()) <= 1e-5 * scale
