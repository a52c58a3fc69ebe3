"""Host summary of the device's per-neuron spike records (rate and CV of
the inter-spike interval) against a direct computation from spike trains."""
import numpy as np

from libnrn_b200.stats import records_from_raster, summarize


def test_summary_equals_direct_isi_statistics():
    rng = np.random.default_rng(7)
    n, steps, dt = 300, 5000, 1e-4
    step, idx = [], []
    trains = {}
    for i in range(n):
        k = int(rng.integers(0, 60))
        t = np.unique(rng.integers(0, steps, k))
        trains[i] = t
        step.extend(t.tolist())
        idx.extend([i] * len(t))
    perm = rng.permutation(len(step))               # raster order does not matter
    rec = records_from_raster(np.asarray(step)[perm], np.asarray(idx)[perm], n)
    s = summarize(rec, steps, dt)
    for i in range(n):
        t = trains[i]
        assert rec["count"][i] == len(t)
        assert abs(s["rate_hz"][i] - len(t) / (steps * dt)) < 1e-9
        if len(t) >= 3:
            isi = np.diff(t).astype(np.float64)
            assert abs(s["cv"][i] - isi.std() / isi.mean()) < 1e-9
        else:
            assert np.isnan(s["cv"][i])
    assert s["n_cv"] == sum(len(t) >= 3 for t in trains.values())


def test_regular_train_has_zero_cv():
    step = np.arange(0, 1000, 10)
    rec = records_from_raster(step, np.zeros_like(step), 1)
    s = summarize(rec, 1000, 1e-3)
    assert s["cv"][0] == 0.0 and abs(s["rate_hz"][0] - 100.0) < 1e-9
