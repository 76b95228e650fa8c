"""Seeded synthetic AtlasIR networks at benchmark scale.

The benchmark configurations (1M-neuron CUBA with fixed in-degree 1000 and
Poisson drive; 4M-neuron Brunel network with a 1.5 ms delay) are too large to
lower through the Brian2 frontend on every run, and the frontend is not
available where the benchmark runs.  Their definition layer does not depend on
the network size: it is taken verbatim from a small network lowered by the
reference's own frontend (tests/golden/models/*_small.json, produced by
tests/golden/make_fixtures.py with brian2_rust.export.lower_network).  This
module rescales only the size-dependent fields (counts, subgroup ranges,
procedural edge counts, run length) and draws new seeded initial state with the
same distributions, then re-attaches the canonical layer hashes exactly as the
reference writer does (brian2-rust/python/brian2_rust/protocol.py:104-112:
SHA-256 of sorted-key, compact, UTF-8 JSON per layer).
"""
from __future__ import annotations

import copy
import hashlib
import json

import numpy as np


def _hex64(values: np.ndarray) -> list:
    raw = np.ascontiguousarray(values, dtype=np.float64).view(np.uint64)
    return [f"{int(x):016x}" for x in raw]


def _hex32(values: np.ndarray) -> list:
    raw = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    return [f"{int(x):08x}" for x in raw]


def _f64(bits: str) -> float:
    return float(np.frombuffer(bytes.fromhex(bits), dtype=">f8")[0])


def attach_protocol(doc: dict) -> dict:
    layers = {}
    for layer in ("definition", "instance", "run"):
        text = json.dumps(doc[layer], sort_keys=True, separators=(",", ":"), ensure_ascii=False, allow_nan=False)
        layers[layer] = hashlib.sha256(text.encode()).hexdigest()
    doc["protocol"]["layers"] = layers
    return doc


def encode(doc: dict) -> bytes:
    return json.dumps(doc, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()


def _set_run(doc: dict, ticks: int) -> None:
    dt = _f64(doc["definition"]["clocks"][0]["dt"])
    doc["run"]["clocks"][0]["steps"] = ticks
    doc["run"]["duration"] = f"{np.float64(ticks * dt).view(np.uint64):016x}"
    for p in doc["definition"]["populations"]:
        p["steps"] = ticks
        p["monitor"]["window_steps"] = ticks


def _scale_single_population(doc: dict, n: int, indegree: int, exc_fraction: float) -> None:
    """One population split into an excitatory head and an inhibitory tail,
    two fixed in-degree projections from those subgroups onto everything."""
    d, inst = doc["definition"], doc["instance"]
    pop = d["populations"][0]
    pop["count"] = n
    inst["neuron_count"] = n
    n_e = int(n * exc_fraction)
    k_e = int(indegree * exc_fraction)
    k_i = indegree - k_e
    exc, inh = d["synapses"]
    exc.update(source_start=0, source_count=n_e, target_start=0, target_count=n)
    inh.update(source_start=n_e, source_count=n - n_e, target_start=0, target_count=n)
    for syn, k in zip(inst["synapses"], (k_e, k_i)):
        topo = syn["topology"]
        assert topo["kind"] == "fixed_indegree"
        topo["indegree"] = k
        topo["edge_count"] = k * n


def cuba_fixed_indegree(template: dict, n: int = 1_000_000, indegree: int = 1000, ticks: int = 10_000,
                        seed: int = 3) -> dict:
    """The scaled CUBA benchmark network: v0 ~ U[Vr, Vt], ge = gi = 0,
    80/20 excitatory/inhibitory in-degree, Poisson drive as in the template."""
    doc = copy.deepcopy(template)
    _scale_single_population(doc, n, indegree, 0.8)
    _set_run(doc, ticks)
    pin = doc["instance"]["populations"][0]
    params = pin["parameters"]
    vr, vt = _f64(params["Vr"][0]), _f64(params["Vt"][0])
    rng = np.random.default_rng(seed)
    v = vr + rng.random(n) * (vt - vr)
    zero = "0000000000000000"
    pin["initial_state"] = {"v": _hex64(v), "ge": [zero] * n, "gi": [zero] * n}
    refr = pin["refractory"]
    refr["initial_lastspike"] = [refr["initial_lastspike"][0]] * n
    refr["initial_not_refractory"] = [True] * n
    doc["instance"]["rng_seed"] = seed
    return attach_protocol(doc)


def brunel_fixed_indegree(template: dict, n: int = 4_000_000, indegree: int = 1000, ticks: int = 10_000,
                          seed: int = 4) -> dict:
    """The balanced Brunel network with a homogeneous delay (f32 membrane
    state): v0 ~ U[0, theta], in-degree split 80/20, Poisson drive at twice
    the threshold rate as in the template (N_ext = excitatory in-degree)."""
    doc = copy.deepcopy(template)
    _scale_single_population(doc, n, indegree, 0.8)
    _set_run(doc, ticks)
    pin = doc["instance"]["populations"][0]
    theta = _f64(pin["parameters"]["theta"][0])
    rng = np.random.default_rng(seed)
    v = (rng.random(n) * theta).astype(np.float32)
    pin["initial_state"] = {"v": _hex32(v)}
    refr = pin["refractory"]
    refr["initial_lastspike"] = [refr["initial_lastspike"][0]] * n
    refr["initial_not_refractory"] = [True] * n
    # PoissonInput: N_ext tracks the excitatory in-degree, the per-input
    # probability (rate * dt) is unchanged: rate = 2 * theta / (J * C_E * tau)
    # scales with 1/C_E, so rescale it with the in-degree.
    k_e_old = None
    for co in doc["definition"]["populations"][0]["code_objects"]:
        if co["kind"] == "poisson_input":
            for st in co["vector"]:
                node = st["value"]
                stack = [node]
                while stack:
                    e = stack.pop()
                    if e.get("op") == "binomial":
                        k_e_old = e["n"]
                        e["n"] = int(indegree * 0.8)
                    stack.extend(v for v in e.values() if isinstance(v, dict))
    if k_e_old:
        for name, vals in pin["parameters"].items():
            if name.startswith("b2_poisson_probability"):
                p = _f64(vals[0]) * k_e_old / int(indegree * 0.8)
                vals[0] = f"{np.float64(p).view(np.uint64):016x}"
    doc["instance"]["rng_seed"] = seed
    return attach_protocol(doc)


_HEX = np.frombuffer(b"0123456789abcdef", dtype=np.uint8)


def _json_hex64(values: np.ndarray) -> bytes:
    """JSON list of the f64 bit patterns as 16-digit hex strings (the same
    text as json.dumps(_hex64(values))), rendered with array operations."""
    raw = np.ascontiguousarray(values, dtype=np.float64).view(np.uint64)
    if raw.size == 0:
        return b"[]"
    out = np.empty((raw.size, 19), dtype=np.uint8)
    out[:, 0] = out[:, 17] = ord('"')
    out[:, 18] = ord(",")
    for k in range(16):
        out[:, 1 + k] = _HEX[((raw >> np.uint64(60 - 4 * k)) & np.uint64(15)).astype(np.intp)]
    return b"[" + out.tobytes()[:-1] + b"]"


def _json_ints(values: np.ndarray) -> bytes:
    return ("[" + ",".join(map(str, np.asarray(values).tolist())) + "]").encode()


def _json_repeat(item: str, n: int) -> bytes:
    return b"[" + (f'"{item}",'.encode() * n)[:-1] + b"]" if n else b"[]"


def _splice(text: bytes, arrays: dict) -> bytes:
    cuts = []
    for name in arrays:
        key = f'"@@splice:{name}@@"'.encode()
        at = text.find(key)
        assert at >= 0 and text.find(key, at + 1) < 0, name
        cuts.append((at, len(key), name))
    parts, pos = [], 0
    for at, n, name in sorted(cuts):
        parts += [text[pos:at], arrays[name]]
        pos = at + n
    parts.append(text[pos:])
    return b"".join(parts)


def encode_spliced(doc: dict, arrays: dict) -> bytes:
    """encode(attach_protocol(doc)) for a document whose large arrays are
    given pre-rendered: doc holds the string "@@splice:NAME@@" where array
    NAME goes, and arrays[NAME] is that array's compact JSON text.  The
    arrays sit in the instance layer, whose hash is taken over the spliced
    canonical text, as the reference writer hashes the whole layer."""
    layers = {}
    for layer in ("definition", "instance", "run"):
        text = json.dumps(doc[layer], sort_keys=True, separators=(",", ":"), ensure_ascii=False, allow_nan=False)
        data = text.encode()
        if layer == "instance":
            data = _splice(data, arrays)
        layers[layer] = hashlib.sha256(data).hexdigest()
    doc["protocol"]["layers"] = layers
    return _splice(encode(doc), arrays)


def stdp_feedforward(template: dict, n_inputs: int = 100_000, n_neurons: int = 10_000, indegree: int = 1000,
                     ticks: int = 10_000, seed: int = 5, spliced: bool = False):
    """The STDP-plastic feedforward network (the Song-Abbott example scaled
    up): n_inputs Poisson inputs at the template's rate drive n_neurons
    conductance-based LIF neurons, each receiving `indegree` inputs drawn
    uniformly (with replacement), edges in target-major creation order;
    w0 ~ U[0, gmax], traces and lastupdate zero, membrane at its template
    value.  The template is stdp_small (one input group, one target group,
    one explicit plastic projection with on_pre and on_post pathways)."""
    doc = copy.deepcopy(template)
    d, inst = doc["definition"], doc["instance"]
    src_pop, tgt_pop = d["populations"]
    src_pop["count"], tgt_pop["count"] = n_inputs, n_neurons
    inst["neuron_count"] = n_inputs + n_neurons
    syn = d["synapses"][0]
    syn.update(source_start=0, source_count=n_inputs, target_start=0, target_count=n_neurons)
    _set_run(doc, ticks)
    pin_src, pin_tgt = inst["populations"]
    pin_src["parameters"]["rates"] = [pin_src["parameters"]["rates"][0]] * n_inputs
    for name, values in pin_tgt["initial_state"].items():
        pin_tgt["initial_state"][name] = [values[0]] * n_neurons
    rng = np.random.default_rng(seed)
    E = n_neurons * indegree
    source = rng.integers(0, n_inputs, size=E, dtype=np.int64)
    target = np.repeat(np.arange(n_neurons, dtype=np.int64), indegree)
    si = inst["synapses"][0]
    gmax = _f64(si["parameters"]["gmax"][0])
    w = rng.random(E) * gmax
    inst["rng_seed"] = seed
    zero = "0000000000000000"
    per_edge = [name for name, values in si["parameters"].items() if len(values) > 1]
    if spliced:
        # the same document, encoded without materialising per-edge Python lists
        arrays = {"source": _json_ints(source), "target": _json_ints(target), "w": _json_hex64(w),
                  "zero": None}
        si["source"], si["target"] = "@@splice:source@@", "@@splice:target@@"
        si["initial_state"] = {"w": "@@splice:w@@"}
        for name in ("Apre", "Apost", "lastupdate"):
            si["initial_state"][name] = f"@@splice:{name}@@"
            arrays[name] = _json_repeat(zero, E)
        for name in per_edge:
            arrays[f"param_{name}"] = _json_repeat(si["parameters"][name][0], E)
            si["parameters"][name] = f"@@splice:param_{name}@@"
        del arrays["zero"]
        return encode_spliced(doc, arrays)
    si["source"], si["target"] = source.tolist(), target.tolist()
    zeros = [zero] * E
    si["initial_state"] = {"w": _hex64(w), "Apre": zeros, "Apost": zeros, "lastupdate": zeros}
    for name in per_edge:
        si["parameters"][name] = [si["parameters"][name][0]] * E
    return attach_protocol(doc)
