"""`binary_csr` topologies: external B2CSR001 source-major graphs
(brian2-rust/src/binary_topology.rs, model.rs:2163-2205, executor.rs:35-57).

The golden fixture's projections are rewritten as B2CSR001 files (edges in
file order, random per-edge weights as value column 0, a scalar 2-tick
delay).  Pins: the oracle gives the same bytes for the binary model and for
the explicit model with the same edges, weights and delays; the GPU engine
gives the oracle's bytes; malformed files and mappings fail with the
reference's messages before any device work.
"""
from __future__ import annotations

import copy
import hashlib
import json
import struct

import numpy as np
import pytest

from conftest import GOLDEN, encode_model, run_oracle


def hexf(x: float) -> str:
    return struct.pack(">d", x).hex()


def b2csr_bytes(sources: int, targets: int, src: np.ndarray, tgt: np.ndarray, columns: list) -> bytes:
    counts = np.bincount(src, minlength=sources)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype("<u8")
    head = b"B2CSR001" + struct.pack("<4Q", sources, targets, len(tgt), len(columns))
    body = offsets.tobytes() + tgt.astype("<u4").tobytes()
    for col in columns:
        body += np.asarray(col, dtype="<f8").tobytes()
    return head + body


def models(tmp_path, seed=5):
    """(binary_csr model, equivalent explicit model) as documents."""
    rng = np.random.default_rng(seed)
    base = json.loads((GOLDEN / "reference-v1" / "model.json").read_text())
    dt = struct.unpack(">d", bytes.fromhex(base["definition"]["clocks"][0]["dt"]))[0]
    explicit, binary = copy.deepcopy(base), copy.deepcopy(base)
    for s, (si_e, si_b) in enumerate(zip(explicit["instance"]["synapses"], binary["instance"]["synapses"])):
        d = base["definition"]["synapses"][s]
        src = np.asarray(si_e["source"], dtype=np.int64)
        tgt = np.asarray(si_e["target"], dtype=np.int64)
        order = np.argsort(src, kind="stable")  # source-major, creation order within a row
        src, tgt = src[order], tgt[order]
        w0 = struct.unpack(">d", bytes.fromhex(si_e["parameters"]["w"][0]))[0]
        w = w0 * (0.5 + rng.random(len(src)))
        si_e["source"], si_e["target"] = src.tolist(), tgt.tolist()
        si_e["parameters"]["w"] = [hexf(x) for x in w]
        for pw_e, pw_b in zip(si_e["pathways"], si_b["pathways"]):
            for pw in (pw_e, pw_b):
                pw["delay"], pw["delay_ticks"], pw["pending"] = [hexf(2 * dt)], [2], []
        data = b2csr_bytes(d["source_count"], d["target_count"], src, tgt, [w])
        path = tmp_path / f"projection_{s}.b2csr"
        path.write_bytes(data)
        si_b["source"], si_b["target"] = [], []
        del si_b["parameters"]["w"]
        si_b["topology"] = {"kind": "binary_csr", "edge_count": int(len(src)), "path": str(path),
                            "sha256": hashlib.sha256(data).hexdigest(), "column_count": 1,
                            "initializers": {"w": 0}}
    return binary, explicit


def write(tmp_path, name, doc):
    path = tmp_path / name
    path.write_bytes(encode_model(doc))
    return path


def test_oracle_binary_equals_explicit(oracle, tmp_path):
    binary, explicit = models(tmp_path)
    a = run_oracle(oracle, write(tmp_path, "binary.json", binary), tmp_path / "a")
    b = run_oracle(oracle, write(tmp_path, "explicit.json", explicit), tmp_path / "b")
    assert (a / "results.bin").read_bytes() == (b / "results.bin").read_bytes()
    assert (a / "events.bin").read_bytes() == (b / "events.bin").read_bytes()


def test_invalid_files_and_mappings(pkg, tmp_path):
    binary, _ = models(tmp_path)
    topo = binary["instance"]["synapses"][0]["topology"]
    path = tmp_path / "projection_0.b2csr"
    good = path.read_bytes()
    path.write_bytes(good[:-8])
    with pytest.raises(pkg.B2GpuError, match="binary CSR file length mismatch"):
        pkg.codegen(encode_model(binary))
    path.write_bytes(good[:-1] + bytes([good[-1] ^ 1]))
    with pytest.raises(pkg.B2GpuError, match="binary CSR checksum mismatch"):
        pkg.codegen(encode_model(binary))
    # a target outside the population, with a matching checksum
    sources = binary["definition"]["synapses"][0]["source_count"]
    at = 40 + (sources + 1) * 8
    bad = good[:at] + struct.pack("<I", 10 ** 6) + good[at + 4:]
    path.write_bytes(bad)
    topo["sha256"] = hashlib.sha256(bad).hexdigest()
    with pytest.raises(pkg.B2GpuError, match="binary CSR target outside population"):
        pkg.codegen(encode_model(binary))
    path.write_bytes(good)
    topo["sha256"] = hashlib.sha256(good).hexdigest()
    topo["initializers"] = {"unknown": 0}
    with pytest.raises(pkg.B2GpuError, match="invalid binary CSR mapping/pathway"):
        pkg.codegen(encode_model(binary))


@pytest.mark.gpu
def test_gpu_matches_oracle_on_binary_csr(pkg, oracle, tmp_path):
    binary, _ = models(tmp_path)
    path = write(tmp_path, "binary.json", binary)
    with pkg.Engine(path.read_bytes(), device=0) as eng:
        eng.run()
        (tmp_path / "gpu").mkdir()
        eng.write_results(tmp_path / "gpu")
    ref = run_oracle(oracle, path, tmp_path / "ref")
    assert (tmp_path / "gpu" / "results.bin").read_bytes() == (ref / "results.bin").read_bytes()
    assert (tmp_path / "gpu" / "events.bin").read_bytes() == (ref / "events.bin").read_bytes()
