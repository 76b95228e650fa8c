"""Canonical JSON layer hashes and the runner's non-run modes (CPU).

Pins: the reference's own golden hash corpus
(brian2-rust/tests/golden/{atlasir-v1,b2ir-v1}/{minimal-v1.json,hashes.json}
and the probe predecessors b2ir-v1/minimal-v34..v37.json, copied to
tests/golden/canonical/), Python's json.dumps(sort_keys=True,
separators=(",", ":"), ensure_ascii=False) for reals, escapes and non-ASCII
text, and the runner contract of `--canonical-hashes` / `--validate` /
"AtlasIR canonical layer hash mismatch" (brian2-rust/src/model.rs:4596-4677).
"""
from __future__ import annotations

import hashlib
import json
import subprocess

import pytest

from conftest import GOLDEN, MODELS, ROOT

CANON = GOLDEN / "canonical"


def runner(*args):
    exe = ROOT / "brian2-atlas_b200" / "bin" / "b2gpu-runner"
    return subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True)


@pytest.mark.parametrize("name", ["atlasir", "b2ir"])
def test_golden_corpus_hashes(name):
    proc = runner("--canonical-hashes", CANON / f"{name}-minimal-v1.json")
    assert proc.returncode == 0, proc.stderr
    want = json.loads((CANON / f"{name}-hashes.json").read_text())["layers"]
    assert json.loads(proc.stdout) == want
    assert proc.stdout.strip() == json.dumps(want, separators=(",", ":"))


def python_hash(value) -> str:
    text = json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=False)
    return hashlib.sha256(text.encode()).hexdigest()


def test_reals_escapes_and_unicode_match_python(tmp_path):
    doc = json.loads((MODELS / "cuba_small.json").read_text())
    doc["run"]["x_canonical_probe"] = {
        "reals": [0.1, 1e16, 1e15, 1e-5, 1.5e-4, 0.0001, 123456789012345678.0, 2.5, -0.0, 1e300, 5e-324,
                  0.30000000000000004, 12345.678, -7.25e-12, 1.7976931348623157e308, 100.0],
        "text": ["été", "☃", "tab\tnew\nline", "\x01\x1f", 'quote"back\\slash', "\x7f"],
        "nested": {"b": [1, -2, 18446744073709551615, -9223372036854775808], "a": None, "c": True},
    }
    want = python_hash(doc["run"])
    path = tmp_path / "probe.json"
    path.write_text(json.dumps(doc, ensure_ascii=False))
    proc = runner("--canonical-hashes", path)  # stale protocol: rejected, but only after hashing
    assert proc.returncode == 1 and "canonical layer hash mismatch" in proc.stderr
    import importlib
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    doc = synthetic.attach_protocol(doc)
    assert doc["protocol"]["layers"]["run"] == want
    path.write_text(json.dumps(doc, ensure_ascii=False))
    proc = runner("--canonical-hashes", path)
    assert proc.returncode == 0, proc.stderr
    assert json.loads(proc.stdout)["run"] == want


def test_tampered_document_is_refused(pkg, tmp_path):
    doc = json.loads((MODELS / "cuba_small.json").read_text())
    doc["instance"]["rng_seed"] = doc["instance"]["rng_seed"] + 1
    path = tmp_path / "tampered.json"
    path.write_text(json.dumps(doc))
    for mode in ("--validate", "--canonical-hashes"):
        proc = runner(mode, path)
        assert proc.returncode == 1
        assert proc.stderr.strip() == "b2-runner: AtlasIR canonical layer hash mismatch"
    proc = runner(path, tmp_path / "out")
    assert proc.returncode == 1 and not (tmp_path / "out").exists()
    with pytest.raises(pkg.B2GpuError, match="canonical layer hash mismatch"):
        pkg.codegen(path.read_bytes())


def test_validate_accepts_fixtures():
    for path in [GOLDEN / "reference-v1" / "model.json", MODELS / "cuba_small.json", MODELS / "brunel_small.json",
                 CANON / "atlasir-minimal-v1.json", CANON / "b2ir-minimal-v1.json"]:
        proc = runner("--validate", path)
        assert proc.returncode == 0 and proc.stdout.strip() == "validated AtlasIR", (path, proc.stderr)


@pytest.mark.parametrize("version", [34, 35, 36, 37])
def test_probe_predecessors_migrate(oracle, tmp_path, version):
    """b2ir-gate0-probe-v34..v37 documents are migrated as the reference's
    prepare_protocol does: their migrated layers hash like the current
    minimal document (the reference's Python migrate_model gives the same
    hashes), they validate, and they run to the same result bytes."""
    path = CANON / f"b2ir-minimal-v{version}.json"
    proc = runner("--canonical-hashes", path)
    assert proc.returncode == 0, proc.stderr
    assert json.loads(proc.stdout) == json.loads((CANON / "atlasir-hashes.json").read_text())["layers"]
    proc = runner("--validate", path)
    assert proc.returncode == 0 and proc.stdout.strip() == "validated AtlasIR", proc.stderr
    for name, model in (("probe", path), ("current", CANON / "atlasir-minimal-v1.json")):
        done = subprocess.run([str(oracle), str(model), str(tmp_path / name)], capture_output=True, text=True)
        assert done.returncode == 0, done.stderr
    assert (tmp_path / "probe" / "results.bin").read_bytes() == (tmp_path / "current" / "results.bin").read_bytes()


def test_probe_predecessor_envelopes_are_checked(tmp_path):
    doc = json.loads((CANON / "b2ir-minimal-v35.json").read_text())
    doc["instance"]["rng_seed"] += 1
    (tmp_path / "v35.json").write_text(json.dumps(doc))
    proc = runner("--validate", tmp_path / "v35.json")
    assert proc.returncode == 1 and "canonical layer hash mismatch" in proc.stderr
    doc = json.loads((CANON / "b2ir-minimal-v34.json").read_text())
    doc["protocol"] = json.loads((CANON / "b2ir-minimal-v35.json").read_text())["protocol"]
    (tmp_path / "v34.json").write_text(json.dumps(doc))
    proc = runner("--validate", tmp_path / "v34.json")
    assert proc.returncode == 1 and "legacy AtlasIR has a protocol envelope" in proc.stderr


@pytest.mark.parametrize("env,message", [
    ({"B2_MAX_IR_BYTES": "100"}, "IR exceeds the configured byte budget"),
    ({"B2_MAX_NEURONS": "10"}, "invalid neuron count"),
    ({"B2_MAX_NEURONS": "1e6"}, "B2_MAX_NEURONS requires decimal digits in 1..16000000"),
    ({"B2_MAX_IR_BYTES": "0"}, "B2_MAX_IR_BYTES requires decimal digits in 1..68719476736"),
    ({"B2_MAX_POPULATION_STEPS": "10"}, "positive population dt and valid Clock interval required"),
    ({"B2_MAX_POPULATION_STATES": "1"}, "population state arrays do not match definition"),
    ({"B2_MAX_POPULATION_PARAMETERS": "1"}, "population parameter arrays do not match definition"),
    ({"B2_MAX_STATEMENTS": "1"}, "too many statements"),
    ({"B2_MAX_STATEMENTS": "2000"}, "B2_MAX_STATEMENTS requires decimal digits in 1..1024"),
])
def test_runner_process_budgets(tmp_path, env, message):
    """The runner's opt-in budgets (brian2-rust/src/resource_limits.rs) with
    the reference's defaults, limits and messages; the library API has none."""
    import os
    exe = ROOT / "brian2-atlas_b200" / "bin" / "b2gpu-runner"
    for args in (["--validate", MODELS / "cuba_small.json"], [MODELS / "cuba_small.json", tmp_path / "out"]):
        proc = subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True, env=dict(os.environ, **env))
        assert proc.returncode == 1 and message in proc.stderr, proc.stderr
        assert not (tmp_path / "out").exists()
    proc = subprocess.run([str(exe), "--validate", str(MODELS / "cuba_small.json")], capture_output=True, text=True,
                          env=dict(os.environ, B2_MAX_NEURONS="400"))
    assert proc.returncode == 0, proc.stderr


@pytest.mark.parametrize("model,env,message", [
    (GOLDEN / "reference-v1" / "model.json", {"B2_MAX_EXPLICIT_SYNAPSES": "100"}, "invalid synaptic topology"),
    (MODELS / "timed_input_small.json", {"B2_MAX_TIMED_ARRAY_VALUES": "3"}, "invalid TimedArray layout"),
    (GOLDEN / "reference-v1" / "model.json", {"B2_MAX_INITIAL_VALUES": "1000"}, "probe array budget exceeded"),
])
def test_runner_model_budgets(model, env, message):
    import os
    exe = ROOT / "brian2-atlas_b200" / "bin" / "b2gpu-runner"
    proc = subprocess.run([str(exe), "--validate", str(model)], capture_output=True, text=True,
                          env=dict(os.environ, **env))
    assert proc.returncode == 1 and message in proc.stderr, proc.stderr
    proc = subprocess.run([str(exe), "--validate", str(model)], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr


def test_probe_function_migration_matches_reference():
    """The Function branch of the probe migration (abi set to
    b2ir-function-v1, empty backend_implementations added): the migrated
    layer hashes equal those of the reference's Python migrate_model
    (tests/golden/make_probe_function.py wrote both files)."""
    proc = runner("--canonical-hashes", CANON / "b2ir-probe-v37-function.json")
    assert proc.returncode == 0, proc.stderr
    want = json.loads((CANON / "b2ir-probe-v37-function-migrated-hashes.json").read_text())["layers"]
    assert json.loads(proc.stdout) == want
