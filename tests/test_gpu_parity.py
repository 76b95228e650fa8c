"""GPU engine against the oracle and the reference's golden output (needs a GPU).

Bar: byte-identical results.bin / events.bin where every per-lane operation is
exact IEEE arithmetic (CUBA, Brunel, CUBA+PoissonInput and the golden fixture:
their transcendentals fold to host constants computed with glibc).  Models
with per-neuron device transcendentals (COBAHH's exp/exprel, STDP's trace
decay, per-tick normal draws) are held to tolerances instead:
tests/test_gpu_tolerance.py.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import (GOLDEN, MODELS, encode_model, golden_procedural_initializers, model_file, procedural_variant,
                      run_oracle)
from b2results import describe_difference, load_model, read_results

pytestmark = pytest.mark.gpu

# gap_junctions_small: a `(summed)` synaptic current recomputed every tick;
# synapse_updates_small: clock-driven synaptic traces, a synaptic
# run_regularly and STDP pathways
# timed_input_small: two- and one-dimensional TimedArray inputs
EXACT = ["cuba_small", "cuba_poisson_small", "brunel_small", "gap_junctions_small", "synapse_updates_small",
         "timed_input_small"]


def gpu_run(pkg, model_path, outdir, **kw):
    data = model_path.read_bytes()
    with pkg.Engine(data, device=0, **kw) as eng:
        eng.run()
        outdir.mkdir()
        eng.write_results(outdir)
        return eng.stats()


def assert_same_files(a, b, model=None):
    same = (a / "results.bin").read_bytes() == (b / "results.bin").read_bytes()
    assert same, describe_difference(a, b, load_model(model)) if model else "results.bin differs"
    ea, eb = a / "events.bin", b / "events.bin"
    assert ea.exists() == eb.exists()
    if ea.exists():
        assert ea.read_bytes() == eb.read_bytes()


@pytest.mark.parametrize("targets,warps", [("1", "0"), ("1", "1"), ("1", "2"), ("1", "8"), ("0", "0")])
def test_golden_fixture_bytes(pkg, tmp_path, monkeypatch, targets, warps):
    """The reference's golden b2-runner run, reproduced on the GPU byte for
    byte, with the per-edge-delay pathways delivered target-ordered (1, 2 or
    8 warps per target, or the planner's choice) and by the single-thread
    fold."""
    monkeypatch.setenv("B2GPU_TARGETS", targets)
    monkeypatch.setenv("B2GPU_TARGETS_WARPS", warps)
    out = tmp_path / "gpu"
    gpu_run(pkg, GOLDEN / "reference-v1" / "model.json", out)
    assert (out / "results.bin").read_bytes() == (GOLDEN / "reference-v1" / "results.bin").read_bytes()
    assert (out / "events.bin").read_bytes() == (GOLDEN / "reference-v1" / "events.bin").read_bytes()
    summary = json.loads((out / "summary.json").read_text())
    assert summary["spike_count"] == 155 and summary["synaptic_events"] == 1238


@pytest.mark.parametrize("name", EXACT)
def test_exact_models_match_oracle(pkg, oracle, tmp_path, name):
    path = model_file(name, tmp_path)
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref", path)


@pytest.mark.parametrize("expr", ["v_pre", "current_pre"])
def test_golden_variants_match_oracle(pkg, oracle, tmp_path, expr):
    """projection_0_0 delivering current_post + w * <expr>: target-ordered
    for v_pre, the serial fold for current_pre (presynaptic state that the
    pathway writes); both byte-identical to the oracle."""
    from test_abi import golden_variant
    path = tmp_path / "model.json"
    path.write_bytes(golden_variant(expr))
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")


@pytest.mark.parametrize("name,indegree", [("gap_junctions_small", 15), ("synapse_updates_small", 40)])
def test_procedural_synapse_programs_match_oracle(pkg, oracle, tmp_path, name, indegree):
    """Summed variables, synaptic state updates, run_regularly, target-ordered
    on_pre and on_post over fixed in-degree topologies generated on the
    device, against the oracle's host-side generation, byte for byte."""
    path = tmp_path / f"{name}_fixed_indegree.json"
    path.write_bytes(procedural_variant(name, indegree))
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")


def test_single_delay_golden_variant_matches_oracle(pkg, oracle, tmp_path):
    """The golden network (projection_0_0 scaled by the source's v) with one
    3-tick delay per pathway: event buckets and atomics, nothing delivered
    before tick 3."""
    from test_abi import golden_uniform_variant
    path = tmp_path / "model.json"
    path.write_bytes(golden_uniform_variant())
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")


@pytest.mark.parametrize("normal", [False, True])
def test_procedural_initializers_match_oracle(pkg, oracle, tmp_path, normal):
    """Fixed in-degree edges generated on the device with uniform per-edge
    weights and delays (drawn on the device) or clipped-normal ones (drawn on
    the host), delivered by the target-ordered scan over per-edge delays,
    against the oracle's host-side materialisation, byte for byte."""
    path = tmp_path / "model.json"
    path.write_bytes(golden_procedural_initializers(normal=normal))
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")


def test_cuba_4k_full_second(pkg, oracle, tmp_path):
    """Config 0 (CUBA 4000 neurons, ~320k synapses, 10,000 ticks)."""
    path = model_file("cuba_4k", tmp_path)
    stats = gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")
    assert stats["ticks"] == 10000


@pytest.mark.parametrize("kw", [dict(chunk_ticks=1), dict(chunk_ticks=7), dict(use_graphs=False)])
def test_chunking_and_graphs_do_not_change_results(pkg, oracle, tmp_path, kw):
    path = MODELS / "cuba_poisson_small.json"
    gpu_run(pkg, path, tmp_path / "gpu", **kw)
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")


def test_stepwise_api_and_state_readback(pkg, oracle, tmp_path):
    path = MODELS / "cuba_small.json"
    model = load_model(path)
    run_oracle(oracle, path, tmp_path / "ref")
    ref = read_results(tmp_path / "ref", model)
    with pkg.Engine(path.read_bytes(), device=0) as eng:
        assert eng.step(250) is False
        assert eng.stats()["ticks"] == 250
        eng.run()
        v = np.frombuffer(eng.read_state(0, "v"), dtype=np.float64)
        np.testing.assert_array_equal(v, ref.populations[0].states["v"])
        last = ref.populations[0].spikes
        tick = int(last[-1, 0])
        assert eng.spikes(0, tick) == [int(i) for t, i in last if t == tick]


def test_summary_without_files(pkg, tmp_path):
    """b2g_summary_json gives summary.json's content (timings aside) without
    writing anything."""
    with pkg.Engine((MODELS / "cuba_small.json").read_bytes(), device=0) as eng:
        eng.run()
        summary = eng.summary()
        (tmp_path / "out").mkdir()
        eng.write_results(tmp_path / "out")
    written = json.loads((tmp_path / "out" / "summary.json").read_text())
    for doc in (summary, written):
        doc.pop("timings")
    assert summary == written and summary["synaptic_events"] > 0


def test_nonfinite_state_raises_instead_of_faulting(pkg):
    """A value the reference would reject (overflow to inf) sets the device
    error word; the host raises and poisons the engine."""
    doc = load_model(MODELS / "cuba_small.json")
    # ge <- ge * ge with ge0 = 1e200 overflows to +inf on the first tick
    update = doc["definition"]["populations"][0]["code_objects"][0]
    for st in update["vector"]:
        if st["target"] == "ge":
            st["value"] = {"op": "mul", "left": {"op": "load", "name": "ge"}, "right": {"op": "load", "name": "ge"}}
    doc["instance"]["populations"][0]["initial_state"]["ge"][5] = "6974e718d7d7625a"  # 1e200
    with pkg.Engine(encode_model(doc), device=0) as eng:
        with pytest.raises(pkg.B2GpuError, match="non-finite"):
            eng.run()
        with pytest.raises(pkg.B2GpuError, match="create a new executor"):
            eng.step(1)


def test_scaled_cuba_fixed_indegree_matches_oracle(pkg, oracle, tmp_path):
    """Config 2's network shape at 20k neurons (in-degree 1000, 2e7 synapses
    generated on the device) against the oracle's host-side generation."""
    import importlib
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    template = json.loads((MODELS / "cuba_poisson_small.json").read_text())
    doc = synthetic.cuba_fixed_indegree(template, n=20000, indegree=1000, ticks=300, seed=9)
    path = tmp_path / "c2_20k.json"
    path.write_bytes(synthetic.encode(doc))
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")


def test_cli_runner_drop_in(pkg, oracle, tmp_path):
    """b2gpu-runner honours the b2-runner argv/output contract."""
    import subprocess
    path = MODELS / "cuba_small.json"
    proc = subprocess.run([str(pkg.runner_path()), str(path), str(tmp_path / "gpu")], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr
    assert proc.stdout.startswith("completed 1 populations for 400 neurons")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")
    again = subprocess.run([str(pkg.runner_path()), str(path), str(tmp_path / "gpu")], capture_output=True, text=True)
    assert again.returncode == 1 and again.stderr.startswith("b2-runner: ")


def test_stdp_targets_equal_serial_fold(pkg, tmp_path, monkeypatch):
    """Scaled STDP feedforward network (2,000 Poisson inputs onto 200
    neurons, in-degree 200, 40k plastic synapses): the target-ordered on_pre
    delivery and the single-thread fold run the same arithmetic in the same
    per-target order, so every output byte agrees."""
    import gzip
    import importlib
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    with gzip.open(MODELS / "stdp_small.json.gz", "rb") as f:
        template = json.loads(f.read())
    path = tmp_path / "stdp_40k.json"
    path.write_bytes(synthetic.encode(synthetic.stdp_feedforward(template, 2000, 200, 200, ticks=1500, seed=11)))
    # serial fold; event buckets; bitmap scan with 1 and 4 warps per target
    variants = {"fold": dict(B2GPU_TARGETS="0"), "buckets": dict(B2GPU_TARGETS="1"),
                "scan1": dict(B2GPU_TARGETS="1", B2GPU_TARGETS_SCAN="1", B2GPU_TARGETS_WARPS="1"),
                "scan4": dict(B2GPU_TARGETS="1", B2GPU_TARGETS_SCAN="1", B2GPU_TARGETS_WARPS="4")}
    stats = {}
    for name, env in variants.items():
        for key in ("B2GPU_TARGETS", "B2GPU_TARGETS_SCAN", "B2GPU_TARGETS_WARPS"):
            monkeypatch.setenv(key, env.get(key, "0"))
        stats[name] = gpu_run(pkg, path, tmp_path / name)
    assert stats["fold"]["synaptic_events"] > 0
    for name in variants:
        assert stats[name]["synaptic_events"] == stats["fold"]["synaptic_events"]
        assert_same_files(tmp_path / name, tmp_path / "fold")


def test_bucket_delivery_of_crowded_targets(pkg, tmp_path, monkeypatch):
    """150 inputs firing with probability 0.4 per tick onto 4 neurons with
    in-degree 100: about 40 on_pre events reach each target every tick, past
    the 32 a delivery warp ranks by shuffles, so the in-place bucket sort
    runs; results equal the single-thread fold's byte for byte."""
    import gzip
    import importlib
    import struct
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    with gzip.open(MODELS / "stdp_small.json.gz", "rb") as f:
        template = json.loads(f.read())
    doc = synthetic.stdp_feedforward(template, 150, 4, 100, ticks=300, seed=13)
    rates = doc["instance"]["populations"][0]["parameters"]["rates"]
    doc["instance"]["populations"][0]["parameters"]["rates"] = [struct.pack(">d", 4000.0).hex()] * len(rates)
    path = tmp_path / "crowded.json"
    path.write_bytes(encode_model(doc))
    stats = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("B2GPU_TARGETS", mode)
        stats[mode] = gpu_run(pkg, path, tmp_path / f"gpu{mode}")
    assert stats["1"]["synaptic_events"] == stats["0"]["synaptic_events"] > 300 * 4 * 33
    assert_same_files(tmp_path / "gpu1", tmp_path / "gpu0")


@pytest.mark.parametrize("counted,warp,packed,hints", [("0", "1", "1", "1"), ("1", "1", "1", "1"), ("1", "0", "1", "1"),
                                                     ("1", "1", "0", "0")])
def test_brunel_counted_and_atomic_delivery_match_oracle(pkg, oracle, tmp_path, monkeypatch, counted, warp, packed,
                                                         hints):
    """Brunel's f32 constant-addend pathways delivered by per-event
    compare-and-swap (counted=0) or counted per target and applied by the
    PoissonInput kernel (counted=1, the default), with scatter items per warp
    (the default) or per block, E and I counts packed into one counter or
    not, L2 eviction hints or not: all byte-identical to the oracle, on the
    fixture and on a fixed in-degree variant at 20k neurons."""
    import importlib
    monkeypatch.setenv("B2GPU_COUNTED", counted)
    monkeypatch.setenv("B2GPU_SCATTER_WARP", warp)
    monkeypatch.setenv("B2GPU_PACK_COUNTS", packed)
    monkeypatch.setenv("B2GPU_L2_HINTS", hints)
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    template = json.loads((MODELS / "brunel_small.json").read_text())
    big = tmp_path / "brunel_20k.json"
    big.write_bytes(synthetic.encode(synthetic.brunel_fixed_indegree(template, n=20000, indegree=1000, ticks=300,
                                                                     seed=17)))
    for k, path in enumerate([MODELS / "brunel_small.json", big]):
        gpu_run(pkg, path, tmp_path / f"gpu{k}")
        run_oracle(oracle, path, tmp_path / f"ref{k}")
        assert_same_files(tmp_path / f"gpu{k}", tmp_path / f"ref{k}")


@pytest.mark.parametrize("fuse", ["1", "0"])
def test_brunel_list_layout_in_the_scatter_launch_matches_oracle(pkg, oracle, tmp_path, monkeypatch, fuse):
    """A population of more than 1024 tiles gets a layout kernel for its
    list; when the tick's list is read only 15 ticks later (Brunel), that
    layout runs in the first blocks of the delayed scatter's launch
    (fuse=1, the default) or as its own kernel (fuse=0).  40k neurons in
    tiles of 32 (1250 tiles): byte-identical to the oracle either way."""
    import importlib
    monkeypatch.setenv("B2GPU_TILE", "32")
    monkeypatch.setenv("B2GPU_FUSE_LAYOUT", fuse)
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    template = json.loads((MODELS / "brunel_small.json").read_text())
    path = tmp_path / "brunel_40k.json"
    path.write_bytes(synthetic.encode(synthetic.brunel_fixed_indegree(template, n=40000, indegree=1000, ticks=200,
                                                                      seed=23)))
    src = pkg.codegen(path.read_bytes())
    assert ("neurons_layout(" in src) == (fuse == "0") and "s_pre[" in src
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref", path)


def test_counted_f64_delivery_matches_oracle(pkg, oracle, tmp_path, monkeypatch):
    """Config 2's f64 constant-addend pathways counted per target instead of
    one red.add.f64 per event: the scatters end the tick, so the next tick's
    step applies the counts ahead of the PoissonInput program deferred into
    it (and the flush kernel after the last tick): byte-identical to the
    oracle on the fixture and on a fixed in-degree variant at 20k neurons."""
    import importlib
    monkeypatch.setenv("B2GPU_COUNTED_F64", "1")
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    template = json.loads((MODELS / "cuba_poisson_small.json").read_text())
    big = tmp_path / "c2_20k.json"
    big.write_bytes(synthetic.encode(synthetic.cuba_fixed_indegree(template, n=20000, indegree=1000, ticks=300,
                                                                   seed=9)))
    for k, path in enumerate([MODELS / "cuba_poisson_small.json", big]):
        src = pkg.codegen(path.read_bytes())
        assert "_count_atomic" in src or "_count(" in src, "the counted plan was not taken"
        gpu_run(pkg, path, tmp_path / f"gpu{k}")
        run_oracle(oracle, path, tmp_path / f"ref{k}")
        assert_same_files(tmp_path / f"gpu{k}", tmp_path / f"ref{k}")


@pytest.mark.parametrize("warp", ["0", "1"])
def test_unfused_scatter_matches_oracle(pkg, oracle, tmp_path, monkeypatch, warp):
    """Config 2's shape at 20k neurons with the step laying out its own list
    (B2GPU_FUSE_EXCHANGE=0) and a separate f64 constant-addend scatter, items
    per block (0) or per warp (1): byte-identical to the oracle."""
    import importlib
    monkeypatch.setenv("B2GPU_FUSE_EXCHANGE", "0")
    monkeypatch.setenv("B2GPU_SCATTER_WARP", warp)
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    template = json.loads((MODELS / "cuba_poisson_small.json").read_text())
    path = tmp_path / "c2_20k.json"
    path.write_bytes(synthetic.encode(synthetic.cuba_fixed_indegree(template, n=20000, indegree=1000, ticks=300, seed=9)))
    gpu_run(pkg, path, tmp_path / "gpu")
    run_oracle(oracle, path, tmp_path / "ref")
    assert_same_files(tmp_path / "gpu", tmp_path / "ref")
