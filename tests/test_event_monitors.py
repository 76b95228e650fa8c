"""EventMonitors (record_events, brian2-rust/src/executor.rs:3053-3080) on a
fixture lowered by the reference frontend: CUBA with a custom event `near`
(v > -55 mV) monitored in the after_thresholds slot, and an EventMonitor on
`spike` scheduled in the start slot, before the thresholder, which records the
previous tick's spikes under the current tick (the reference's `fired` list
still holds them).  Oracle semantics on CPU; GPU = oracle bytes.
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

from conftest import GOLDEN, MODELS, run_oracle


def read_events(path, value_dtypes=None):
    """(event streams, monitors) of an events.bin; a monitor is its (k, 2)
    (tick, index) records, plus its value columns when `value_dtypes` gives
    the dtypes of each monitor's variables."""
    data = path.read_bytes()
    assert data[:8] == b"B2EVT001" and data[-8:] == b"B2EEND01"
    pos = 8

    def u64():
        nonlocal pos
        v = struct.unpack_from("<Q", data, pos)[0]
        pos += 8
        return v

    def pairs(n):
        nonlocal pos
        a = np.frombuffer(data, dtype="<u8", count=2 * n, offset=pos).reshape(n, 2)
        pos += 16 * n
        return a

    streams = [pairs(u64()) for _ in range(u64())]
    monitors = []
    for k in range(u64()):
        n, nvalues = u64(), u64()
        records = pairs(n)
        if value_dtypes is None:
            assert nvalues == 0
            monitors.append(records)
            continue
        assert nvalues == len(value_dtypes[k])
        columns = []
        for dt in value_dtypes[k]:
            columns.append(np.frombuffer(data, dtype=dt, count=n, offset=pos))
            pos += n * np.dtype(dt).itemsize
        monitors.append((records, columns))
    return streams, monitors


def test_oracle_event_monitor_semantics(oracle, tmp_path):
    out = run_oracle(oracle, MODELS / "cuba_events_small.json", tmp_path / "ref")
    streams, monitors = read_events(out / "events.bin")
    near_stream, spike_stream = streams  # events in definition order: near, spike
    near_monitor, late_spike_monitor = monitors
    assert len(near_monitor) > 0 and np.array_equal(near_monitor, near_stream)
    # the start-slot monitor sees tick t-1's spikes at tick t
    shifted = spike_stream.copy()
    shifted[:, 0] += 1
    last = int(spike_stream[:, 0].max()) if len(spike_stream) else 0
    shifted = shifted[shifted[:, 0] <= last]
    expect = shifted[np.lexsort((shifted[:, 1], shifted[:, 0]))]
    assert np.array_equal(late_spike_monitor[late_spike_monitor[:, 0] <= last], expect)


@pytest.mark.gpu
def test_gpu_event_monitors_match_oracle(pkg, oracle, tmp_path):
    path = MODELS / "cuba_events_small.json"
    with pkg.Engine(path.read_bytes(), device=0) as eng:
        eng.run()
        (tmp_path / "gpu").mkdir()
        eng.write_results(tmp_path / "gpu")
    ref = run_oracle(oracle, path, tmp_path / "ref")
    assert (tmp_path / "gpu" / "results.bin").read_bytes() == (ref / "results.bin").read_bytes()
    assert (tmp_path / "gpu" / "events.bin").read_bytes() == (ref / "events.bin").read_bytes()


# event_variables_small: `near` records (ge, v) after the thresholds and
# before the reset; the start-slot spike monitor records (v, vt0) of the
# previous tick's spikes after their reset (vt0 is a per-neuron parameter)
VARIABLE_DTYPES = [["<f8", "<f8"], ["<f8", "<f8"]]


def test_oracle_event_monitor_variables_match_brian_numpy(oracle, tmp_path):
    """Recorded variables against Brian2's numpy runtime on the same network
    (tests/golden/brian_numpy/event_variables_small.npz): identical records,
    values within 1e-12 relative."""
    out = run_oracle(oracle, MODELS / "event_variables_small.json", tmp_path / "ref")
    _, ((near, (near_ge, near_v)), (late, (late_v, late_vt0))) = read_events(out / "events.bin", VARIABLE_DTYPES)
    ref = np.load(GOLDEN / "brian_numpy" / "event_variables_small.npz")
    assert len(near) == int(ref["near_count"])
    k = len(ref["near_i"])
    np.testing.assert_array_equal(near[:k, 0], np.rint(ref["near_t"] / 1e-4).astype(np.int64))
    np.testing.assert_array_equal(near[:k, 1], ref["near_i"])
    np.testing.assert_allclose(near_v[:k], ref["near_v"], rtol=1e-12, atol=1e-18)
    np.testing.assert_allclose(near_ge[:k], ref["near_ge"], rtol=1e-12, atol=1e-18)
    assert len(late) == len(ref["late_i"]) > 0
    np.testing.assert_array_equal(late[:, 0], np.rint(ref["late_t"] / 1e-4).astype(np.int64))
    np.testing.assert_array_equal(late[:, 1], ref["late_i"])
    np.testing.assert_allclose(late_v, ref["late_v"], rtol=1e-12, atol=1e-18)
    np.testing.assert_array_equal(late_vt0, ref["late_vt0"])


@pytest.mark.gpu
def test_gpu_event_monitor_variables_match_oracle(pkg, oracle, tmp_path):
    path = MODELS / "event_variables_small.json"
    with pkg.Engine(path.read_bytes(), device=0) as eng:
        eng.run()
        (tmp_path / "gpu").mkdir()
        eng.write_results(tmp_path / "gpu")
    ref = run_oracle(oracle, path, tmp_path / "ref")
    assert (tmp_path / "gpu" / "results.bin").read_bytes() == (ref / "results.bin").read_bytes()
    assert (tmp_path / "gpu" / "events.bin").read_bytes() == (ref / "events.bin").read_bytes()
