"""ctypes binding of the device layer's C ABI (include/nrn_cuda.h).

The shared library is libnrn_b200/_lib/libnrn_cuda.so, built in-tree by
``libnrn_b200.build``.  There is no fallback: if the library is missing or a
call fails, the error is raised.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# NRN_CUDA_LIB: another build of the same library (for example a debug build)
LIB_PATH = os.environ.get("NRN_CUDA_LIB") or os.path.join(HERE, "_lib", "libnrn_cuda.so")

NRN_MAX_PARAMS = 13
NRN_MAX_PROJ = 32
NRN_MAX_POPS = 32

MODEL = {"lif": 0, "adex": 1, "izh": 2}
DRIVE = {None: 0, "poisson": 1, "gauss": 2, "poisson_gexc": 3}
RECEPTOR = {"current": 0, "gexc": 1, "ginh": 2, "chan0": 16, "chan1": 17, "chan2": 18, "chan3": 19}
SYN_KIND = {"exp": 1, "dexp": 2, "ampa": 3}

# Public entry points of include/nrn_cuda.h (checked by the test suite).
EXPORTS = [
    "nrn_status_string", "nrn_last_error", "nrn_version",
    "nrn_cuda_pop_step", "nrn_cuda_deliver", "nrn_cuda_deliver_counted", "nrn_cuda_stdp_step",
    "nrn_cuda_clamp",
    "nrn_engine_create", "nrn_engine_destroy", "nrn_engine_add_population", "nrn_engine_set_params",
    "nrn_engine_add_projection", "nrn_engine_generate_projection", "nrn_engine_set_stdp",
    "nrn_engine_finalize", "nrn_engine_run", "nrn_engine_sync", "nrn_engine_stream", "nrn_engine_step",
    "nrn_engine_info", "nrn_engine_prepare",
    "nrn_engine_raster", "nrn_engine_weights", "nrn_engine_nnz", "nrn_engine_counters",
    "nrn_engine_profile", "nrn_engine_weights_device", "nrn_engine_set_state", "nrn_engine_set_step",
    "nrn_cuda_block_deliver", "nrn_cuda_block_stdp", "nrn_cuda_compact", "nrn_cuda_gather_ring",
    "nrn_cuda_scatter", "nrn_engine_raster_noalloc", "nrn_comm_unique_id", "nrn_engine_set_partition",
    "nrn_cuda_bsr_propagate", "nrn_cuda_bsr_pack", "nrn_cuda_bsr_pack_spikes", "nrn_cuda_bsr_unpack_spikes",
    "nrn_cuda_bsr_spikes", "nrn_cuda_drive_fill", "nrn_engine_checkpoint_size", "nrn_engine_checkpoint_save",
    "nrn_engine_checkpoint_load", "nrn_engine_enable_spike_stats", "nrn_engine_spike_stats",
    "nrn_engine_spike_stats_reset", "nrn_engine_set_comm_timeout", "nrn_comm_bounded_wait",
    "nrn_comm_fake_async_error", "nrn_engine_profile_kernels", "nrn_engine_add_synapse_channel",
    "nrn_engine_set_deterministic", "nrn_engine_add_probe", "nrn_engine_clear_probes",
]


class NrnError(RuntimeError):
    """A libnrn_b200 call failed (status code and message from the library)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Drive(C.Structure):
    _fields_ = [("kind", C.c_int32), ("p0", C.c_float), ("p1", C.c_float), ("seed", C.c_uint64)]


class PopStep(C.Structure):
    _fields_ = [
        ("model", C.c_int32), ("n", C.c_int32), ("gid_offset", C.c_int32), ("pad0", C.c_int32),
        ("dt", C.c_double), ("v", C.c_void_p), ("aux", C.c_void_p), ("refractory", C.c_void_p),
        ("spike", C.c_void_p), ("i_syn", C.c_void_p), ("g_exc", C.c_void_p), ("g_inh", C.c_void_p),
        ("gin_exc", C.c_void_p), ("gin_inh", C.c_void_p), ("tau_syn_exc", C.c_float),
        ("tau_syn_inh", C.c_float), ("e_exc", C.c_float), ("e_inh", C.c_float),
        ("param", C.c_void_p * NRN_MAX_PARAMS), ("uniform", C.c_float * NRN_MAX_PARAMS),
        ("drive", Drive), ("step", C.c_int64), ("step_base", C.c_void_p), ("spike_ids", C.c_void_p),
        ("spike_count", C.c_void_p), ("hist_depth", C.c_int32), ("hist_cap", C.c_int32),
        ("raster_step", C.c_void_p), ("raster_gid", C.c_void_p), ("raster_count", C.c_void_p),
        ("raster_cap", C.c_int64), ("n_traces", C.c_int32), ("trace_slow_ratio", C.c_int32),
        ("trace", C.c_void_p * 4), ("trace_decay", C.c_float * 4),
        ("trace_ring", C.c_void_p * 4), ("trace_ring_depth", C.c_int32), ("pad1", C.c_int32),
        ("post_recent", C.c_void_p), ("post_ring", C.c_void_p), ("post_cnt", C.c_void_p),
        ("post_ring_k", C.c_int32), ("id_offset", C.c_int32), ("win", C.c_int32),
        ("win_mask", C.c_void_p), ("send_hdr", C.c_void_p), ("send_ids", C.c_void_p),
        ("send_cap", C.c_int32), ("pad2", C.c_int32), ("err", C.c_void_p), ("drive_values", C.c_void_p),
        ("spike_stats", C.c_void_p), ("n_chan", C.c_int32), ("chan_kind", C.c_int32 * 4),
        ("chan_e_rev", C.c_float * 4), ("chan_tau_rise", C.c_double * 4), ("chan_tau_decay", C.c_double * 4),
        ("chan_in", C.c_void_p * 4), ("chan_s", C.c_void_p * 4), ("chan_r", C.c_void_p * 4),
    ]


class SynDesc(C.Structure):
    _fields_ = [("kind", C.c_int32), ("pad", C.c_int32), ("tau_rise", C.c_double), ("tau_decay", C.c_double),
                ("e_rev", C.c_double)]


class SpikeHist(C.Structure):
    _fields_ = [("ids", C.c_void_p), ("count", C.c_void_p), ("cap", C.c_int32), ("depth", C.c_int32)]


class Proj(C.Structure):
    _fields_ = [
        ("n_src", C.c_int32), ("n_tgt", C.c_int32), ("dmin", C.c_int32), ("nd", C.c_int32),
        ("src_hist", C.c_int32), ("max_seg", C.c_int32), ("seg_ptr", C.c_void_p), ("tgt", C.c_void_p),
        ("w", C.c_void_p), ("mod", C.c_void_p), ("acc", C.c_void_p),
    ]


class PopDesc(C.Structure):
    _fields_ = [
        ("model", C.c_int32), ("n", C.c_int32), ("gid_offset", C.c_int32), ("record", C.c_int32),
        ("n_global", C.c_int32), ("local_offset", C.c_int32), ("v", C.c_void_p), ("aux", C.c_void_p), ("refractory", C.c_void_p), ("spike", C.c_void_p),
        ("i_syn", C.c_void_p), ("tau_syn_exc", C.c_float), ("tau_syn_inh", C.c_float),
        ("e_exc", C.c_float), ("e_inh", C.c_float), ("param", C.c_void_p * NRN_MAX_PARAMS),
        ("uniform", C.c_float * NRN_MAX_PARAMS), ("drive", Drive),
    ]


class Bsr(C.Structure):
    _fields_ = [
        ("n_post_blocks", C.c_int32), ("n_pre_blocks", C.c_int32), ("n_blocks", C.c_int64),
        ("row_ptr", C.c_void_p), ("col_idx", C.c_void_p), ("tiles", C.c_void_p),
    ]


class ProjDesc(C.Structure):
    _fields_ = [
        ("src_pop", C.c_int32), ("tgt_pop", C.c_int32), ("receptor", C.c_int32), ("on_device", C.c_int32),
        ("nnz", C.c_int64), ("src", C.c_void_p), ("tgt", C.c_void_p), ("w", C.c_void_p),
        ("delay", C.c_void_p), ("mod", C.c_void_p),
    ]


class GenDesc(C.Structure):
    _fields_ = [
        ("src_pop", C.c_int32), ("tgt_pop", C.c_int32), ("receptor", C.c_int32), ("out_degree", C.c_int32),
        ("degree", C.c_int32), ("gen_id", C.c_int32), ("col_offset", C.c_int32), ("col_n", C.c_int32),
        ("dmin", C.c_int32), ("dmax", C.c_int32), ("w_lo", C.c_float), ("w_span", C.c_float),
        ("seed", C.c_uint64), ("rule", C.c_int32), ("pad", C.c_int32), ("p", C.c_double),
        ("sigma", C.c_double), ("max_distance", C.c_double), ("min_probability", C.c_double),
    ]


class EngineInfo(C.Structure):
    _fields_ = [
        ("window", C.c_int32), ("n_pops", C.c_int32), ("raster_capacity", C.c_int64),
        ("recorded_neurons", C.c_int64), ("step", C.c_int64),
    ]


_lib = None


# int (*poll)(void* ctx) of nrn_comm_bounded_wait
POLL_FN = C.CFUNCTYPE(C.c_int, C.c_void_p)


def lib() -> C.CDLL:
    """Loads libnrn_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NrnError(5, f"libnrn_b200 device library not built: {LIB_PATH} "
                              "(run `python -m libnrn_b200.build`)")
        L = C.CDLL(LIB_PATH)
        vp, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
        L.nrn_status_string.restype = C.c_char_p
        L.nrn_status_string.argtypes = [C.c_int]
        L.nrn_last_error.restype = C.c_char_p
        L.nrn_version.restype = C.c_char_p
        L.nrn_engine_step.restype = i64
        L.nrn_engine_step.argtypes = [vp]
        sig = {
            "nrn_cuda_pop_step": [C.POINTER(PopStep), vp],
            "nrn_cuda_drive_fill": [C.POINTER(PopStep), vp, vp],
            "nrn_cuda_deliver": [C.POINTER(Proj), i32, C.POINTER(SpikeHist), i32, i64, vp, vp],
            "nrn_cuda_deliver_counted": [C.POINTER(Proj), i32, C.POINTER(SpikeHist), i32, i64, vp, vp, vp],
            "nrn_cuda_clamp": [vp, i64, C.c_float, C.c_float, vp],
            "nrn_engine_create": [C.POINTER(vp), C.c_int, C.c_double, i32],
            "nrn_engine_destroy": [vp],
            "nrn_engine_add_population": [vp, C.POINTER(PopDesc), C.POINTER(i32)],
            "nrn_engine_set_params": [vp, i32, vp, vp],
            "nrn_engine_add_projection": [vp, C.POINTER(ProjDesc), C.POINTER(i32)],
            "nrn_engine_generate_projection": [vp, C.POINTER(GenDesc), C.POINTER(i32), C.POINTER(i64)],
            "nrn_engine_set_stdp": [vp, i32, C.POINTER(C.c_double)],
            "nrn_engine_finalize": [vp, i32],
            "nrn_comm_unique_id": [C.POINTER(C.c_uint8 * 128)],
            "nrn_cuda_bsr_propagate": [C.POINTER(Bsr), vp, vp, vp, vp],
            "nrn_cuda_bsr_pack": [vp, i64, vp, vp],
            "nrn_cuda_bsr_pack_spikes": [vp, i32, vp, vp],
            "nrn_cuda_bsr_unpack_spikes": [vp, i32, vp, vp],
            "nrn_cuda_bsr_spikes": [C.c_uint64, i64, C.c_float, i32, vp, vp],
            "nrn_engine_set_partition": [vp, i32, i32, C.POINTER(C.c_uint8 * 128), C.c_double],
            "nrn_engine_run": [vp, i64, i32],
            "nrn_engine_sync": [vp],
            "nrn_engine_stream": [vp, C.POINTER(vp)],
            "nrn_engine_raster": [vp, vp, vp, i64, C.POINTER(i64)],
            "nrn_engine_raster_noalloc": [vp, vp, vp, i64, C.POINTER(i64)],
            "nrn_engine_weights": [vp, i32, vp, i64],
            "nrn_engine_nnz": [vp, i32, C.POINTER(i64)],
            "nrn_engine_counters": [vp, C.POINTER(i64), C.POINTER(i64)],
            "nrn_engine_profile": [vp, i64, C.POINTER(C.c_double)],
            "nrn_engine_checkpoint_size": [vp, C.POINTER(i64)],
            "nrn_engine_checkpoint_save": [vp, vp, i64],
            "nrn_engine_checkpoint_load": [vp, vp, i64],
            "nrn_engine_enable_spike_stats": [vp],
            "nrn_engine_spike_stats": [vp, i32, vp, i64],
            "nrn_engine_spike_stats_reset": [vp],
            "nrn_engine_set_comm_timeout": [vp, C.c_double],
            "nrn_comm_bounded_wait": [POLL_FN, vp, C.c_double],
            "nrn_comm_fake_async_error": [i32],
            "nrn_engine_add_synapse_channel": [vp, i32, C.POINTER(SynDesc), C.POINTER(i32)],
            "nrn_engine_set_deterministic": [vp, i32],
            "nrn_engine_add_probe": [vp, i32, i32, vp, i32, C.POINTER(i32)],
            "nrn_engine_clear_probes": [vp],
            "nrn_engine_profile_kernels": [vp, i64, C.POINTER(C.c_double), C.POINTER(i64)],
            "nrn_engine_info": [vp, C.POINTER(EngineInfo)],
            "nrn_engine_prepare": [vp, i64, i64, i32],
        }
        for name, args in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = C.c_int
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.nrn_last_error().decode(errors="replace")
        kind = L.nrn_status_string(status).decode()
        raise NrnError(status, f"{what}: {kind}: {msg}")
