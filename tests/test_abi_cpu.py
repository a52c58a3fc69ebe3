"""The C-ABI library loads, exports every entry point include/nrn_cuda.h
declares, and fails loudly (no fallback) where no GPU is present."""
import ctypes as C
import os
import re

import pytest
import torch

from libnrn_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "nrn_cuda.h")).read()
    return sorted(set(re.findall(r"^NRN_API [^(]*?\b(nrn_[a-z_]+)\(", src, re.M)))


def test_header_lists_match_binding():
    assert declared() == sorted(N.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    for name in declared():
        assert hasattr(lib, name), name


def test_status_strings_and_version():
    lib = N.lib()
    assert lib.nrn_status_string(0) == b"ok"
    assert b"sm_100a" in lib.nrn_version()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks behaviour without a GPU")
def test_engine_refuses_without_gpu():
    h = C.c_void_p()
    st = N.lib().nrn_engine_create(C.byref(h), 0, 1e-4, 1)
    assert st == 5   # NRN_ERR_UNSUPPORTED, no silent CPU path
    with pytest.raises(N.NrnError):
        N.check(st, "nrn_engine_create")


def test_invalid_arguments_rejected_before_launch():
    p = N.PopStep()
    p.model = 7
    p.n = 10
    assert N.lib().nrn_cuda_pop_step(C.byref(p), None) == 1
    assert b"unknown model" in N.lib().nrn_last_error()
