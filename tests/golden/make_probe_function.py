"""Generate tests/golden/canonical/b2ir-probe-v37-function.json and its
expected migrated layer hashes with the reference's own Python migration
(brian2_rust.protocol.migrate_model), for the Function branch of the probe
migration (`abi` set to b2ir-function-v1, empty `backend_implementations`).

    python tests/golden/make_probe_function.py --reference PATH
"""
from __future__ import annotations

import argparse
import copy
import json
from pathlib import Path

import make_fixtures

HERE = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    make_fixtures.prepare_frontend(Path(args.reference))
    from brian2_rust import protocol
    base = json.loads((HERE / "canonical" / "atlasir-minimal-v1.json").read_text())
    doc = copy.deepcopy(base)
    doc["schema"] = "b2ir-gate0-probe-v37"
    doc["definition"]["functions"] = [{
        "name": "twice", "semantic_version": "1.0.0",
        "arguments": [{"name": "x", "dtype": "f64", "dimensions": [0.0] * 7}],
        "return_dtype": "f64", "return_dimensions": [0.0] * 7,
        "effects": {"deterministic": True, "reads_rng": False, "stateful": False},
        "body": {"op": "mul", "left": {"op": "load", "name": "x"},
                 "right": {"op": "literal", "bits": "4000000000000000"}},
        "implementations": {}}]
    doc["protocol"]["name"] = "b2ir"
    doc["protocol"]["canonical_encoding"] = "b2ir-canonical-json-v1"
    doc["protocol"]["layers"] = protocol.layer_hashes(doc)
    migrated = protocol.migrate_model(doc)
    out = HERE / "canonical"
    (out / "b2ir-probe-v37-function.json").write_text(json.dumps(doc, sort_keys=True, indent=1) + "\n")
    (out / "b2ir-probe-v37-function-migrated-hashes.json").write_text(
        json.dumps({"layers": migrated["protocol"]["layers"]}, sort_keys=True, indent=1) + "\n")
    print("wrote", out / "b2ir-probe-v37-function.json")


if __name__ == "__main__":
    main()
