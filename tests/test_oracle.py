"""The CPU oracle against the reference's own pins (no GPU needed).

1. The golden b2-runner run (brian2-rust/tests/fixtures/reference-v1): the
   oracle must reproduce results.bin and events.bin byte for byte and the
   summary counts (155 spikes, 1,238 synaptic events).
2. Brian2's numpy runtime on the same lowered networks (the reference's
   cross-backend gate, brian2-rust/examples/cuba.py:140-160): identical spike
   rasters, states within the gate's tolerance.
3. Planted mistakes: a corrupted oracle output must fail the comparison
   (the reference tests its gates the same way, tests/test_gpu_comparison.py:55-71).
"""
from __future__ import annotations

import json
import shutil

import numpy as np
import pytest

from conftest import GOLDEN, MODELS, model_file, run_oracle
from b2results import load_model, read_results


def test_golden_results_bytes(oracle, tmp_path):
    out = run_oracle(oracle, GOLDEN / "reference-v1" / "model.json", tmp_path / "out")
    assert (out / "results.bin").read_bytes() == (GOLDEN / "reference-v1" / "results.bin").read_bytes()
    assert (out / "events.bin").read_bytes() == (GOLDEN / "reference-v1" / "events.bin").read_bytes()
    ours = json.loads((out / "summary.json").read_text())
    ref = json.loads((GOLDEN / "reference-v1" / "summary.json").read_text())
    for key in ("dump_bytes", "event_dump_bytes", "spike_count", "synaptic_events", "neuron_count",
                "population_count", "final_time_seconds", "schema"):
        assert ours[key] == ref[key], key


def test_golden_comparison_detects_corruption(oracle, tmp_path):
    out = run_oracle(oracle, GOLDEN / "reference-v1" / "model.json", tmp_path / "out")
    data = bytearray((out / "results.bin").read_bytes())
    data[len(data) // 2] ^= 1
    assert bytes(data) != (GOLDEN / "reference-v1" / "results.bin").read_bytes()


@pytest.mark.parametrize("name,rtol", [("cuba_small", 1e-12), ("cobahh_small", 1e-9), ("gap_junctions_small", 1e-9),
                                      ("timed_input_small", 1e-12)])
def test_oracle_matches_brian_numpy(oracle, tmp_path, name, rtol):
    model_path = model_file(name, tmp_path)
    out = run_oracle(oracle, model_path, tmp_path / "out")
    res = read_results(out, load_model(model_path))
    ref = np.load(GOLDEN / "brian_numpy" / f"{name}.npz")
    spikes = res.populations[0].spikes
    ticks = np.rint(ref["spike_t"] / 1e-4).astype(np.int64)
    order = np.lexsort((ref["spike_i"], ticks))
    assert len(spikes) == len(ticks)
    np.testing.assert_array_equal(spikes[:, 0], ticks[order])
    np.testing.assert_array_equal(spikes[:, 1], ref["spike_i"][order])
    np.testing.assert_allclose(res.populations[0].states["v"], ref["v"], rtol=rtol, atol=1e-18)


def test_oracle_rejects_existing_output_dir(oracle, tmp_path):
    import subprocess
    (tmp_path / "exists").mkdir()
    proc = subprocess.run([str(oracle), str(MODELS / "cuba_small.json"), str(tmp_path / "exists")],
                          capture_output=True, text=True)
    assert proc.returncode == 1
    assert "already exists" in proc.stderr


def test_oracle_synaptic_events_equal_outdegree_of_spikes(oracle, tmp_path):
    """summary.synaptic_events == sum of out-degrees of the delivered spikes
    (the reference's check in brian2-rust/examples/cuba.py:120-123)."""
    model_path = MODELS / "cuba_small.json"
    model = load_model(model_path)
    out = run_oracle(oracle, model_path, tmp_path / "out")
    res = read_results(out, model)
    spikes = res.populations[0].spikes
    total = 0
    for syn in model["instance"]["synapses"]:
        outdeg = np.bincount(np.asarray(syn["source"]), minlength=model["definition"]["populations"][0]["count"])
        total += int(outdeg[spikes[:, 1]].sum())
    assert sum(res.delivered) == total


def test_oracle_synapse_updates_match_brian_numpy(oracle, tmp_path):
    """Clock-driven synaptic traces (synapse_state_update every tick), a
    synaptic run_regularly and STDP pathways, against Brian2's numpy runtime
    on the same network (deterministic inputs): output spikes exact, weights
    and traces within 1e-12."""
    model_path = MODELS / "synapse_updates_small.json"
    out = run_oracle(oracle, model_path, tmp_path / "out")
    res = read_results(out, load_model(model_path))
    ref = np.load(GOLDEN / "brian_numpy" / "synapse_updates_small.npz")
    spikes = res.populations[1].spikes
    ticks = np.rint(ref["spike_t"] / 1e-4).astype(np.int64)
    order = np.lexsort((ref["spike_i"], ticks))
    assert len(spikes) == len(ticks) > 0
    np.testing.assert_array_equal(spikes[:, 0], ticks[order])
    np.testing.assert_array_equal(spikes[:, 1], ref["spike_i"][order])
    np.testing.assert_allclose(res.populations[1].states["v"], ref["v"], rtol=1e-12, atol=1e-18)
    for name in ("w", "Apre", "Apost"):
        np.testing.assert_allclose(res.synapse_states[0][name], ref[name], rtol=1e-12, atol=1e-18)


def test_oracle_random_draws_have_their_distributions(oracle, tmp_path):
    """The oracle's restated counter streams (executor.rs:209-222 polar
    normal, :290-336 Knuth below 10 and PTRS from 10) drawn through a model
    (random_draws_small, lowered by the reference frontend): every neuron's
    300 Poisson counts have mean lam and variance lam within 5 standard
    errors (both branches), and the membrane driven by white noise has the
    Ornstein-Uhlenbeck spread it implies.  The GPU engine must then equal
    these draws (tests/test_gpu_tolerance.py)."""
    path = MODELS / "random_draws_small.json"
    model = load_model(path)
    r = read_results(run_oracle(oracle, path, tmp_path / "ref"), model)
    names = [p["name"] for p in model["definition"]["populations"]]
    k = r.populations[names.index("draws")].samples["k"]  # (ticks, neurons)
    lam = np.linspace(0.5, 60.0, k.shape[1])
    assert np.all(k == np.floor(k)) and np.all(k >= 0)
    mean_err = (k.mean(axis=0) - lam) / np.sqrt(lam / k.shape[0])
    assert np.max(np.abs(mean_err)) < 5, mean_err
    var_ratio = k.var(axis=0, ddof=1) / lam
    assert np.all(np.abs(var_ratio - 1.0) < 5 * np.sqrt(2.0 / (k.shape[0] - 1)) + 0.05)
    # pooled: the z-scores of the means look standard normal
    assert abs(mean_err.mean()) < 0.5 and 0.6 < mean_err.std() < 1.4
    # white noise: v's increments over one tick below threshold have std
    # sigma * sqrt(dt / tau) (Euler-Maruyama), sigma = 0.5, dt/tau = 0.01
    v = r.populations[names.index("noisy")].samples["v"]
    dv = np.diff(v, axis=0)
    quiet = (v[:-1] > 0.05) & (v[1:] > 0.05) & (v[:-1] < 0.95)
    drift = (0.8 - v[:-1]) * 0.01
    noise = (dv - drift)[quiet]
    assert abs(noise.std() / 0.05 - 1.0) < 0.05 and abs(noise.mean()) < 0.002
