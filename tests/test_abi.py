"""The C ABI boundary and the plan compiler, without a GPU.

* libb2gpu.so loads and exports every entry point include/b2gpu.h declares.
* b2g_codegen builds the plan of each fixture model and compiles the generated
  kernels for sm_100a with NVRTC (no GPU involved).
* The plan picks the delivery strategy the reference semantics allow
  (atomic only for constant-addend pathways) and fuses update/threshold/reset.
* Unsupported models fail at creation with a capability message, before any
  result file exists (brian2-rust/AtlasIR.md:66-70).
"""
from __future__ import annotations

import gzip
import json
import re

import pytest

from conftest import GOLDEN, MODELS, ROOT, encode_model, golden_procedural_initializers, procedural_variant


def declared_symbols():
    text = (ROOT / "include" / "b2gpu.h").read_text()
    return sorted(set(re.findall(r"\b(b2g_[a-z_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.library()
    names = declared_symbols()
    assert "b2g_create" in names and "b2g_step" in names and "b2g_run_cli" in names
    for name in names:
        assert hasattr(lib, name), name


def test_version(pkg):
    assert "sm_100a" in pkg.version()


def kernels(src):
    return re.findall(r"__global__ void __launch_bounds__\(\d+(?:, \d+)?\) (\w+)", src)


def load(name):
    path = MODELS / f"{name}.json"
    if path.exists():
        return path.read_bytes()
    with gzip.open(MODELS / f"{name}.json.gz", "rb") as f:
        return f.read()


@pytest.mark.parametrize("name,expected", [
    # E and I pathways write different variables: one merged scatter launch
    ("cuba_small", ["statemon", "step", "exc_pre_inh_pre_atomic"]),
    # PoissonInput commutes with everything up to the next tick's update: it
    # runs in the next step's prologue (plus a flush kernel for the last tick)
    ("cuba_poisson_small", ["step", "exc_pre_inh_pre_atomic", "flush_0_neurons"]),
    # both pathways write f32 v (order matters): counted delivery, both
    # counts in one launch, applied E then I by the PoissonInput work, which
    # also resets the lanes the tick fired; that work, the tick's last, runs
    # in the next tick's step prologue (plus a flush kernel for the last tick)
    ("brunel_small", ["step", "excitatory_synapses_pre_inhibitory_synap_atomic", "flush_0_neurons"]),
    ("cobahh_small", ["step", "exc_pre_inh_pre_atomic"]),
    # the two populations step in one launch; on_pre writes the target's
    # conductance and the edge's weight and traces: target-ordered delivery
    # (bucket scatter, then per-target delivery); on_post writes only
    # synapse state
    ("stdp_small", ["neurons_step_inputs_step", "stdp_pre_targets", "stdp_pre_deliver", "stdp_post_edges"]),
])
def test_codegen_plan(pkg, name, expected):
    src = pkg.codegen(load(name))
    names = kernels(src)
    assert len(names) == len(expected), names
    for kernel, suffix in zip(names, expected):
        assert kernel.endswith(suffix), (kernel, suffix)


def test_codegen_golden_fixture(pkg):
    src = pkg.codegen((GOLDEN / "reference-v1" / "model.json").read_bytes())
    names = kernels(src)
    # per-edge delays 1-4 ticks and per-edge weights: ordered delivery, one
    # warp per target
    assert sum(n.endswith("_targets") for n in names) == 4
    assert names[2].endswith("exc_step_inh_step")  # both populations in one launch


def golden_variant(expr):
    """The golden fixture with projection_0_0 (population 0 onto itself)
    delivering current_post + w * <expr>."""
    doc = json.loads((GOLDEN / "reference-v1" / "model.json").read_text())
    code = doc["definition"]["synapses"][0]["code_objects"][0]
    value = code["vector"][0]["value"]
    value["right"] = {"op": "mul", "left": value["right"], "right": {"op": "load", "name": expr}}
    code["effects"]["reads"] = sorted(set(code["effects"]["reads"]) | {expr})
    return encode_model(doc)


def test_codegen_ordered_pathway_fallbacks(pkg, monkeypatch):
    # reading presynaptic `current` while writing postsynaptic `current` of
    # the same population makes the order across targets observable: serial
    names = kernels(pkg.codegen(golden_variant("current_pre")))
    assert names[3].endswith("projection_0_0_pre_serial")
    assert sum(n.endswith("_targets") for n in names) == 3
    # presynaptic `v` is never written by the pathway: target-ordered
    names = kernels(pkg.codegen(golden_variant("v_pre")))
    assert sum(n.endswith("_targets") for n in names) == 4
    # diagnostic switch back to the single-thread fold
    monkeypatch.setenv("B2GPU_TARGETS", "0")
    names = kernels(pkg.codegen((GOLDEN / "reference-v1" / "model.json").read_bytes()))
    assert sum(n.endswith("_serial") for n in names) == 4


def test_exact_linear_update_is_pure_arithmetic(pkg):
    """CUBA's exp(-dt/tau) terms fold to host constants computed with glibc, so
    the per-neuron update issues no device transcendental."""
    src = pkg.codegen(load("cuba_small"))
    step = src[src.index("_neurons_step(RunCtl"):]
    step = step[:step.index("\n}\n")]
    assert "exp(" not in step and "log(" not in step


def test_unsupported_model_fails_before_results(pkg, tmp_path):
    doc = json.loads(load("cuba_small"))
    doc["definition"]["clocks"].append(dict(doc["definition"]["clocks"][0], name="second"))
    doc["run"]["clocks"].append(dict(doc["run"]["clocks"][0]))
    with pytest.raises(pkg.B2GpuError, match="single clock"):
        pkg.codegen(encode_model(doc))


def test_malformed_document_is_rejected(pkg):
    with pytest.raises(pkg.B2GpuError, match="JSON"):
        pkg.codegen(b"{not json")
    with pytest.raises(pkg.B2GpuError, match="schema"):
        pkg.codegen(json.dumps({"schema": "other"}).encode())


def test_codegen_procedural_synapse_programs(pkg):
    """Summed variables, synaptic state updates, run_regularly and on_post on
    fixed in-degree topologies: the engine derives their edge endpoints and
    destination-major rows from the device-built source-major CSR."""
    names = kernels(pkg.codegen(procedural_variant("gap_junctions_small", 15)))
    assert names[1].endswith("gaps_summed_variable_Igap_post")
    names = kernels(pkg.codegen(procedural_variant("synapse_updates_small", 40)))
    assert [n.split("_", 2)[2] for n in names] == ["decay", "inputs_step_neurons_step", "stdp_stateupdater",
                                                   "stdp_pre_targets", "stdp_pre_deliver", "stdp_post_edges"]


def golden_uniform_variant(ticks=3):
    """golden_variant("v_pre") with every pathway's per-edge delays replaced
    by one delay of `ticks` ticks (seconds taken from an edge that already
    had it): projection_0_0 (per-edge w times the source's v) is delivered
    through the event buckets, the constant-addend projections by atomics."""
    doc = json.loads(golden_variant("v_pre"))
    for inst in doc["instance"]["synapses"]:
        for pw in inst["pathways"]:
            k = pw["delay_ticks"].index(ticks)
            pw["delay"] = [pw["delay"][k]] * len(pw["delay"])
            pw["delay_ticks"] = [ticks] * len(pw["delay_ticks"])
    return encode_model(doc)


def test_codegen_single_delay_golden_uses_buckets(pkg):
    names = kernels(pkg.codegen(golden_uniform_variant()))
    assert [n.split("_", 2)[2] for n in names[3:]] == [
        "projection_0_0_pre_targets", "projection_0_0_pre_deliver", "projection_0_1_pre_atomic",
        "projection_1_0_pre_atomic", "projection_1_1_pre_atomic"]


def test_codegen_procedural_delay_initializers(pkg, oracle, tmp_path):
    """Uniform and clipped-normal delay initializers on fixed in-degree
    projections plan as per-edge delays (target-ordered scan); the oracle
    runs both."""
    import subprocess
    for normal in (False, True):
        data = golden_procedural_initializers(normal=normal)
        names = kernels(pkg.codegen(data))
        assert sum(n.endswith("_pre_targets") for n in names) == 4
        path = tmp_path / f"model{int(normal)}.json"
        path.write_bytes(data)
        proc = subprocess.run([str(oracle), str(path), str(tmp_path / f"out{int(normal)}")], capture_output=True,
                              text=True)
        assert proc.returncode == 0, proc.stderr


def test_invalid_uniform_delay_initializer_is_refused(pkg, oracle, tmp_path):
    """A negative minimum fails materialize_uniform_ticks' check, in the
    engine and in the oracle, with the reference's message."""
    import subprocess
    doc = json.loads(golden_procedural_initializers())
    doc["instance"]["synapses"][1]["pathways"][0]["delay_initializer"]["minimum"] = "bf1a36e2eb1c432d"  # -1e-4
    data = encode_model(doc)
    with pytest.raises(pkg.B2GpuError, match="invalid uniform delay initializer"):
        pkg.codegen(data)
    path = tmp_path / "model.json"
    path.write_bytes(data)
    proc = subprocess.run([str(oracle), str(path), str(tmp_path / "out")], capture_output=True, text=True)
    assert proc.returncode == 1 and "invalid uniform delay initializer" in proc.stderr


def test_no_cpu_fallback(pkg, tmp_path):
    """Without a usable GPU the engine raises instead of computing on the
    host, and without the built library the package refuses to load."""
    import os
    import subprocess
    import sys
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(pkg.B2GpuError, match="cuda"):
        pkg.Engine(load("cuba_small"), device=0)
    code = ("import importlib, sys; sys.path.insert(0, sys.argv[1]); "
            "pkg = importlib.import_module('brian2-atlas_b200'); pkg.LIBRARY = pkg.LIBRARY.with_name('absent.so'); "
            "pkg._lib = None\n"
            "try:\n    pkg.library()\nexcept pkg.B2GpuError as e:\n    print('refused:', e)\n")
    out = subprocess.run([sys.executable, "-c", code, str(ROOT)], capture_output=True, text=True,
                         env=dict(os.environ))
    assert out.stdout.startswith("refused:") and "build.py" in out.stdout, out.stdout + out.stderr


def test_counted_delivery_plan(pkg, monkeypatch):
    """Brunel (f32 membrane, E then I constant-addend pathways, then the
    PoissonInput): the two scatters only count events per target, in one
    launch; the PoissonInput work applies E's then I's map that many times
    before its own draw and resets the lanes the tick fired, and as the tick's
    last dense work it runs in the next tick's step prologue;
    B2GPU_COUNTED=0 keeps one compare-and-swap scatter per pathway."""
    import re
    src = pkg.codegen(load("brunel_small"))
    names = [n.split("_", 2)[2] for n in re.findall(r"__global__ void __launch_bounds__\([^)]*\) (\w+)", src)]
    assert len([n for n in names if n.endswith("_atomic")]) == 1 and "b2_atomic_add_f32_via_f64(" not in src.split(
        "__constant__ u64 g_ptr")[1]
    step = src[src.index("_neurons_step(RunCtl"):]
    step = step[:step.index("\n}\n")]
    applies = [m.start() for m in re.finditer(r"if \(run_deferred && cna", step)]
    draw = step.index("b2_binomial_thr")
    assert len(applies) == 2 and applies[-1] < draw < step.index("ls == t_prev") < step.index("d_ls = t - ls")
    assert "neurons_reset" not in names and "neurons_poisson_input" not in names
    monkeypatch.setenv("B2GPU_COUNTED", "0")
    src = pkg.codegen(load("brunel_small"))
    names = [n.split("_", 2)[2] for n in re.findall(r"__global__ void __launch_bounds__\([^)]*\) (\w+)", src)]
    assert len([n for n in names if n.endswith("_atomic")]) == 2 and "n_ev" not in src


def test_chunk_kernel_plan(pkg, monkeypatch):
    """B2GPU_MEGA: every kernel of the tick becomes a device function of a
    virtual block (no programmatic-launch instructions, no hardware block
    index, loads through L2 rather than the read-only path), called by one
    cooperative chunk kernel with a grid barrier after each op; a plan with an
    op that is not a single kernel (two populations stepped by one launch)
    keeps the per-op kernels."""
    monkeypatch.setenv("B2GPU_MEGA", "1")
    src = pkg.codegen(load("cuba_poisson_small"))
    assert "b2_chunk(" in src
    chunk = src[src.index("b2_chunk("):]
    ops = re.findall(r"(b2_\d+_\w+)_m\(ctl, k, vb, (\d+)u\); __syncthreads\(\); \}", chunk)
    assert [o[0] for o in ops] == kernels(src)[:len(ops)] and len(ops) == 2
    assert chunk.count("b2_grid_barrier(") == len(ops)
    for name, _ in ops:
        body = src[src.index(f"void {name}_m("):]
        body = body[:body.index("\n}\n")]
        for banned in ("griddepcontrol", "blockIdx.x", "gridDim.x", "__ldg("):
            assert banned not in body, (name, banned)
    assert "b2_chunk(" not in pkg.codegen(load("synapse_updates_small"))
    monkeypatch.delenv("B2GPU_MEGA")
    assert "b2_chunk(" not in pkg.codegen(load("cuba_poisson_small"))
