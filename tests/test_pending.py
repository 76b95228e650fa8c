"""Pending (continuation) events: the delayed deliveries a segmented run hands
to its next segment (AtlasIR.md section 6; seeded into the ring by
PathwayQueue::new, executor.rs:6185-6212; validated by model.rs:4315-4337).

The golden fixture has per-edge delays of 1-4 ticks (pending items are edge
ids); the CUBA fixture has one uniform delay (items are source indices).  Both
get seeded pending events; the GPU engine must reproduce the oracle's bytes,
on one GPU and partitioned over GPUs.  Invalid pending lists are rejected with
the reference's message before any device work (CPU).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN, MODELS, encode_model, run_oracle


def with_pending(doc: dict, seed: int, per_pathway: int = 40) -> dict:
    rng = np.random.default_rng(seed)
    start = doc["run"]["clocks"][0]["start_tick"]
    for s, syn in enumerate(doc["instance"]["synapses"]):
        definition = doc["definition"]["synapses"][s]
        for pw in syn["pathways"]:
            delays = pw["delay_ticks"]
            uniform = all(d == delays[0] for d in delays)
            horizon = max(delays) + 1
            if uniform:
                count = definition["source_count"] if pw["kind"] == "pre" else definition["target_count"]
            else:
                count = len(syn["source"])
            ticks = np.sort(rng.integers(start, start + horizon, per_pathway))
            items = rng.integers(0, count, per_pathway)
            pw["pending"] = [{"delivery_tick": int(t), "item": int(i)} for t, i in zip(ticks, items)]
    return doc


def golden_with_pending(tmp_path, seed=1):
    doc = with_pending(json.loads((GOLDEN / "reference-v1" / "model.json").read_text()), seed)
    path = tmp_path / "golden_pending.json"
    path.write_bytes(encode_model(doc))
    return path


def cuba_with_pending(tmp_path, seed=2):
    doc = json.loads((MODELS / "cuba_small.json").read_text())
    # give the pathways a uniform 3-tick delay so pending items span slots
    for syn in doc["instance"]["synapses"]:
        for pw in syn["pathways"]:
            pw["delay_ticks"] = [3] * len(pw["delay_ticks"])
    doc = with_pending(doc, seed)
    path = tmp_path / "cuba_pending.json"
    path.write_bytes(encode_model(doc))
    return path


def test_oracle_delivers_pending_events(oracle, tmp_path):
    """Seeded pending events change the run (they are delivered at all)."""
    base = run_oracle(oracle, GOLDEN / "reference-v1" / "model.json", tmp_path / "base")
    seeded = run_oracle(oracle, golden_with_pending(tmp_path), tmp_path / "seeded")
    a = json.loads((base / "summary.json").read_text())["synaptic_events"]
    b = json.loads((seeded / "summary.json").read_text())["synaptic_events"]
    assert b > a


def test_invalid_pending_is_rejected(pkg, tmp_path):
    doc = json.loads((GOLDEN / "reference-v1" / "model.json").read_text())
    pw = doc["instance"]["synapses"][0]["pathways"][0]
    pw["pending"] = [{"delivery_tick": 5, "item": 0}, {"delivery_tick": 2, "item": 0}]  # not sorted
    with pytest.raises(pkg.B2GpuError, match="invalid pending synaptic pathway event"):
        pkg.codegen(encode_model(doc))
    pw["pending"] = [{"delivery_tick": 1, "item": len(doc["instance"]["synapses"][0]["source"])}]  # no such edge
    with pytest.raises(pkg.B2GpuError, match="invalid pending synaptic pathway event"):
        pkg.codegen(encode_model(doc))


def assert_same_files(a, b):
    assert (a / "results.bin").read_bytes() == (b / "results.bin").read_bytes()
    assert (a / "events.bin").read_bytes() == (b / "events.bin").read_bytes()


@pytest.mark.gpu
@pytest.mark.parametrize("make", [golden_with_pending, cuba_with_pending])
def test_gpu_matches_oracle_with_pending_events(pkg, oracle, tmp_path, make):
    path = make(tmp_path)
    with pkg.Engine(path.read_bytes(), device=0) as eng:
        eng.run()
        (tmp_path / "gpu").mkdir()
        eng.write_results(tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")
