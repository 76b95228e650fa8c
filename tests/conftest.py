"""Shared pytest configuration: the `gpu` marker, the built library, the oracle."""
from __future__ import annotations

import gzip
import importlib
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
MODELS = GOLDEN / "models"
ORACLE = ROOT / "oracle" / "b2ref"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


@pytest.fixture(scope="session")
def pkg():
    """The engine package; the library must already be built."""
    return importlib.import_module("brian2-atlas_b200")


@pytest.fixture(scope="session")
def oracle():
    """Path of the CPU oracle binary, built on demand with make."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    return ORACLE


def model_file(name: str, tmp: Path) -> Path:
    """Plain-JSON path of a fixture model (decompressing .json.gz into tmp)."""
    plain = MODELS / f"{name}.json"
    if plain.exists():
        return plain
    gz = MODELS / f"{name}.json.gz"
    out = tmp / f"{name}.json"
    if not out.exists():
        with gzip.open(gz, "rb") as src, open(out, "wb") as dst:
            shutil.copyfileobj(src, dst)
    return out


def encode_model(doc: dict) -> bytes:
    """JSON bytes of an edited model document with its protocol layer hashes
    recomputed (the engine, like the reference runner, refuses stale hashes)."""
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    return synthetic.encode(synthetic.attach_protocol(doc))


def run_oracle(oracle: Path, model: Path, outdir: Path) -> Path:
    proc = subprocess.run([str(oracle), str(model), str(outdir)], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr
    return outdir
