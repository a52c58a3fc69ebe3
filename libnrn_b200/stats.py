"""Population spike statistics from the per-neuron records the neuron
updates accumulate on the device (nrn_spike_stat_t: last spike step + 1,
spike count, sums of the inter-spike intervals and of their squares, in
steps): firing rate and coefficient of variation of the inter-spike
interval, per neuron and per population, without reading the raster."""
from __future__ import annotations

import numpy as np

# numpy layout of nrn_spike_stat_t (include/nrn_cuda.h)
SPIKE_STAT = np.dtype([("last", np.int32), ("count", np.int32), ("isi_sum", np.int64), ("isi_sum2", np.int64)])


def summarize(rec: np.ndarray, steps: int, dt: float) -> dict:
    """Statistics of one population over `steps` steps of `dt` seconds.

    rate_hz: spikes per neuron and second; cv: CV of the inter-spike
    interval of each neuron with at least two intervals (NaN otherwise);
    rate_mean_hz and cv_mean: population means (cv over the neurons that
    have one)."""
    rec = np.asarray(rec, SPIKE_STAT)
    count = rec["count"].astype(np.float64)
    rate = count / (steps * dt) if steps > 0 else np.zeros_like(count)
    m = count - 1.0
    ok = m >= 2
    mean = np.where(ok, rec["isi_sum"] / np.maximum(m, 1.0), np.nan)
    var = np.where(ok, rec["isi_sum2"] / np.maximum(m, 1.0) - mean * mean, np.nan)
    cv = np.where(ok, np.sqrt(np.maximum(var, 0.0)) / mean, np.nan)
    return {"rate_hz": rate, "cv": cv, "rate_mean_hz": float(rate.mean()) if rate.size else 0.0,
            "cv_mean": float(np.nanmean(cv)) if ok.any() else float("nan"), "n_cv": int(ok.sum())}


def records_from_raster(step: np.ndarray, idx: np.ndarray, n: int) -> np.ndarray:
    """The records the device keeps, rebuilt from a raster of (step, local
    index) pairs of one population (for checking)."""
    rec = np.zeros(n, SPIKE_STAT)
    order = np.lexsort((step, idx))
    s, i = np.asarray(step)[order].astype(np.int64), np.asarray(idx)[order]
    for k in range(len(i)):
        r = rec[i[k]]
        if r["last"] > 0:
            isi = s[k] + 1 - r["last"]
            rec["isi_sum"][i[k]] += isi
            rec["isi_sum2"][i[k]] += isi * isi
        rec["last"][i[k]] = s[k] + 1
        rec["count"][i[k]] += 1
    return rec
