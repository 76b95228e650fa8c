"""Reader for the b2-runner result files, for the parity tests.

Layout of `results.bin` (B2DMP001 v3) and `events.bin` (B2EVT001) as written
by brian2-rust/src/executor.rs:3142-3405 (and read by the reference's
python/brian2_rust/results.py:191).  The per-population sample, state and
synapse-state arrays are typed; their dtypes come from the model document.
"""
from __future__ import annotations

import gzip
import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

NP_DTYPE = {"f64": np.float64, "f32": np.float32, "i32": np.int32, "i64": np.int64,
            "u32": np.uint32, "u64": np.uint64, "bool": np.uint8}


def load_model(path) -> dict:
    path = Path(path)
    if path.suffix == ".gz":
        with gzip.open(path, "rt") as f:
            return json.load(f)
    return json.loads(path.read_text())


def model_bytes(path) -> bytes:
    path = Path(path)
    if path.suffix == ".gz":
        with gzip.open(path, "rb") as f:
            return f.read()
    return path.read_bytes()


@dataclass
class Population:
    count: int
    steps: int
    samples: dict = field(default_factory=dict)
    spikes: np.ndarray = None          # (k, 2) int64: tick, index
    counts: np.ndarray = None
    last_fired: np.ndarray = None
    states: dict = field(default_factory=dict)
    lastspike: np.ndarray = None
    not_refractory: np.ndarray = None


@dataclass
class Results:
    populations: list
    synapse_states: list
    delivered: list
    final_time: float
    events: list = None  # per event stream: (k, 2) int64


class _Cursor:
    def __init__(self, data: bytes):
        self.data, self.pos = data, 0

    def u64(self):
        v = struct.unpack_from("<Q", self.data, self.pos)[0]
        self.pos += 8
        return v

    def array(self, dtype, n):
        dt = np.dtype(dtype).newbyteorder("<")
        a = np.frombuffer(self.data, dtype=dt, count=n, offset=self.pos).copy()
        self.pos += dt.itemsize * n
        return a

    def raw(self, n):
        b = self.data[self.pos:self.pos + n]
        self.pos += n
        return b


def read_results(directory, model: dict) -> Results:
    directory = Path(directory)
    c = _Cursor((directory / "results.bin").read_bytes())
    assert c.raw(8) == b"B2DMP001"
    version, marker = struct.unpack_from("<II", c.data, c.pos)
    c.pos += 8
    assert version == 3 and marker == 0x01020304
    n_pop, _neurons, size = c.u64(), c.u64(), c.u64()
    assert size == len(c.data)
    d = model["definition"]
    pops = []
    for p in range(n_pop):
        pd = d["populations"][p]
        count, steps, nrec, nvar, nstate, nspk, nlast, refr = (c.u64() for _ in range(8))
        pop = Population(count, steps)
        symbols = {s["name"]: s["dtype"] for s in pd["states"] + pd["parameters"]}
        for name in pd["monitor"]["variables"]:
            dt = NP_DTYPE[symbols[name]]
            total = None
            # sample count = ticks recorded * nrec; derive from remaining layout
            pop.samples[name] = (dt, None)
        # samples are laid out per variable; their length is ticks*nrec where
        # ticks = min(window, steps) for a single-clock model.
        window = min(pd["monitor"]["window_steps"], steps) if pd["state_monitors"] else 0
        for name in pd["monitor"]["variables"]:
            dt = NP_DTYPE[symbols[name]]
            pop.samples[name] = c.array(dt, window * nrec).reshape(window, nrec) if nrec else np.zeros((0, 0))
        pop.spikes = c.array(np.int64, 2 * nspk).reshape(nspk, 2)
        pop.counts = c.array(np.int64, count)
        pop.last_fired = c.array(np.int64, nlast)
        for s in pd["states"]:
            pop.states[s["name"]] = c.array(NP_DTYPE[s["dtype"]], count)
        if refr:
            pop.lastspike = c.array(np.float64, count)
            pop.not_refractory = c.array(np.uint8, count)
        pops.append(pop)
    n_syn = c.u64()
    syn_states, delivered = [], []
    for s in range(n_syn):
        sd = d["synapses"][s]
        nstate, edges = c.u64(), c.u64()
        st = {}
        for sym in sd["states"]:
            st[sym["name"]] = c.array(NP_DTYPE[sym["dtype"]], edges)
        syn_states.append(st)
        delivered.append(c.u64())
    final_time = struct.unpack_from("<d", c.data, c.pos)[0]
    c.pos += 8
    assert c.raw(8) == b"B2END001"
    events = None
    ev = directory / "events.bin"
    if ev.exists():
        e = _Cursor(ev.read_bytes())
        assert e.raw(8) == b"B2EVT001"
        events = []
        for _ in range(e.u64()):
            n = e.u64()
            events.append(e.array(np.int64, 2 * n).reshape(n, 2))
    return Results(pops, syn_states, delivered, final_time, events)


def describe_difference(a, b, model: dict) -> str:
    """First differences between two result directories, per section (for
    assertion messages when two runs that must be identical are not)."""
    try:
        ra, rb = read_results(a, model), read_results(b, model)
    except Exception as exc:  # a layout the reader rejects is itself the finding
        return f"unreadable results: {exc!r}"
    out = []
    names = [p["name"] for p in model["definition"]["populations"]]
    for name, pa, pb in zip(names, ra.populations, rb.populations):
        if pa.spikes.shape != pb.spikes.shape or not np.array_equal(pa.spikes, pb.spikes):
            n = min(len(pa.spikes), len(pb.spikes))
            bad = np.nonzero(np.any(pa.spikes[:n] != pb.spikes[:n], axis=1))[0]
            first = int(bad[0]) if len(bad) else n
            out.append(f"{name}: {len(pa.spikes)} vs {len(pb.spikes)} spikes, first difference at #{first}: "
                       f"{pa.spikes[first].tolist() if first < len(pa.spikes) else None} vs "
                       f"{pb.spikes[first].tolist() if first < len(pb.spikes) else None}")
        for var in pb.samples:
            sa, sb = pa.samples.get(var), pb.samples[var]
            if sa is None or sa.shape != sb.shape:
                out.append(f"{name}.{var} samples: shape {None if sa is None else sa.shape} vs {sb.shape}")
            elif not np.array_equal(sa, sb):
                t, r = (int(x[0]) for x in np.nonzero(sa != sb))
                out.append(f"{name}.{var} samples: first difference at tick {t}, record {r}: {sa[t, r]!r} vs {sb[t, r]!r}")
        for var in pb.states:
            if not np.array_equal(pa.states[var], pb.states[var]):
                i = int(np.nonzero(pa.states[var] != pb.states[var])[0][0])
                out.append(f"{name}.{var} final: {int(np.sum(pa.states[var] != pb.states[var]))} differ, first at {i}")
    for s, (sa, sb) in enumerate(zip(ra.synapse_states, rb.synapse_states)):
        for var in sb:
            if not np.array_equal(sa[var], sb[var]):
                out.append(f"synapse {s}.{var}: {int(np.sum(sa[var] != sb[var]))} differ")
    if ra.delivered != rb.delivered:
        out.append(f"delivered {ra.delivered} vs {rb.delivered}")
    return "; ".join(out) or "no difference in the decoded sections"
