"""The benchmark-scale network generator against the reference's lowering."""
from __future__ import annotations

import importlib
import json

from conftest import MODELS, ROOT

synthetic = importlib.import_module("brian2-atlas_b200.synthetic")


def test_scaler_reproduces_reference_lowering():
    """Scaling the reference-lowered 1000-neuron template to its own size and
    seed reproduces the document exactly, including the canonical hashes."""
    template = json.loads((MODELS / "cuba_poisson_small.json").read_text())
    doc = synthetic.cuba_fixed_indegree(template, n=1000, indegree=100, ticks=1000, seed=3)
    assert doc == template


def test_scaled_document_shapes():
    template = json.loads((MODELS / "cuba_poisson_small.json").read_text())
    doc = synthetic.cuba_fixed_indegree(template, n=20000, indegree=1000, ticks=50, seed=7)
    pop = doc["definition"]["populations"][0]
    assert pop["count"] == 20000 and pop["steps"] == 50
    exc, inh = doc["instance"]["synapses"]
    assert exc["topology"]["indegree"] == 800 and inh["topology"]["indegree"] == 200
    assert exc["topology"]["edge_count"] == 800 * 20000
    assert len(doc["instance"]["populations"][0]["initial_state"]["v"]) == 20000
    assert doc["definition"] == synthetic.attach_protocol(doc)["definition"]


def test_brunel_scaler_keeps_f32_state_and_drive():
    template = json.loads((MODELS / "brunel_small.json").read_text())
    doc = synthetic.brunel_fixed_indegree(template, n=10000, indegree=1000, ticks=20, seed=4)
    v = doc["instance"]["populations"][0]["initial_state"]["v"]
    assert len(v) == 10000 and all(len(x) == 8 for x in v[:10])


def test_stdp_spliced_encoding_is_the_plain_encoding(pkg):
    """The scaled STDP network's array-rendered encoding (used at 1e7 edges)
    is byte-identical to encode(attach_protocol(doc)), canonical hashes
    included, and the engine's validator accepts it."""
    import gzip
    with gzip.open(MODELS / "stdp_small.json.gz", "rb") as f:
        template = json.loads(f.read())
    plain = synthetic.encode(synthetic.stdp_feedforward(template, 3000, 50, 40, ticks=100, seed=2))
    spliced = synthetic.stdp_feedforward(template, 3000, 50, 40, ticks=100, seed=2, spliced=True)
    assert plain == spliced
    doc = json.loads(spliced)
    inst = doc["instance"]["synapses"][0]
    assert len(inst["source"]) == len(inst["initial_state"]["w"]) == 50 * 40
    assert max(inst["source"]) < 3000 and inst["target"][:41] == [0] * 40 + [1]
    assert "stdp_pre_targets" in pkg.codegen(spliced)  # layer hashes verified on load
