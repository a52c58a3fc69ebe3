"""Counter-based random numbers for set-up time values (numpy, vectorised).

Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11).  The device kernels
(``csrc/rng.cuh``) implement the same generator for per-step drive and for
connectivity generation; set-up values such as initial membrane potentials
and per-neuron parameters are drawn here, on the host, from the same
counters.  Counter words: (c0, c1, c2, c3) with c3 a stream identifier.
"""
from __future__ import annotations

import numpy as np

STREAM_DRIVE = 0x44524956
STREAM_CONN = 0x434F4E4E
STREAM_INIT = 0x494E4954

_M0 = np.uint64(0xD2511F53)
_M1 = np.uint64(0xCD9E8D57)
_W0 = 0x9E3779B9
_W1 = 0xBB67AE85
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(seed: int, c0, c1, c2, c3):
    """Vectorised Philox4x32-10; returns four uint32 arrays."""
    c0, c1, c2, c3 = np.broadcast_arrays(*(np.asarray(c, dtype=np.uint64) & _MASK
                                           for c in (c0, c1, c2, c3)))
    x0, x1, x2, x3 = (c.astype(np.uint64) for c in (c0, c1, c2, c3))
    k0 = seed & 0xFFFFFFFF
    k1 = (seed >> 32) & 0xFFFFFFFF
    for _ in range(10):
        p0 = _M0 * x0
        p1 = _M1 * x2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK
        x0, x1, x2, x3 = (hi1 ^ x1 ^ np.uint64(k0), lo1, hi0 ^ x3 ^ np.uint64(k1), lo0)
        k0 = (k0 + _W0) & 0xFFFFFFFF
        k1 = (k1 + _W1) & 0xFFFFFFFF
    return tuple(x.astype(np.uint32) for x in (x0, x1, x2, x3))


def u01(x):
    """Uniform in (0,1) from a uint32: odd multiples of 2^-24 (exact in fp32)."""
    x = np.asarray(x, dtype=np.uint32)
    return ((((x >> np.uint32(9)) << np.uint32(1)) | np.uint32(1)).astype(np.float32)
            * np.float32(5.9604644775390625e-8))


def init_uniform(seed: int, which: int, offset: int, n: int, lo: float, span: float):
    """Per-neuron lo + span * u01(Philox(seed; gid, which, 0, STREAM_INIT)[0])."""
    gid = np.arange(offset, offset + n, dtype=np.uint64)
    w0, _, _, _ = philox4x32_10(seed, gid, which, 0, STREAM_INIT)
    return (np.float32(lo) + np.float32(span) * u01(w0)).astype(np.float32)
