"""Build libb2gpu.so and the b2gpu-runner CLI in-tree for sm_100a.

Outputs (git-ignored, shipped with the repository snapshot):
    brian2-atlas_b200/lib/libb2gpu.so
    brian2-atlas_b200/bin/b2gpu-runner

The per-model kernels are generated at engine creation and compiled with NVRTC
for the device's architecture; everything compiled here (host runtime, the
device topology builder with CUB) targets sm_100a explicitly.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libb2gpu.so"
BIN = PKG / "bin" / "b2gpu-runner"
INCLUDE = PKG.parent / "include"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXXFLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-Wall", "-Wno-unused-function"]

HOST_SOURCES = [
    CSRC / "common" / "ir.cpp",
    CSRC / "common" / "dump.cpp",
    CSRC / "common" / "canonical.cpp",
    CSRC / "engine" / "program.cpp",
    CSRC / "engine" / "engine.cpp",
    CSRC / "abi.cpp",
]
CUDA_SOURCES = [CSRC / "engine" / "topology.cu", CSRC / "engine" / "spikes.cu"]
HEADERS = sorted(CSRC.rglob("*.hpp")) + sorted(CSRC.rglob("*.cuh")) + [INCLUDE / "b2gpu.h"]


def _embed_device_lib() -> Path:
    """Embed kernels/device_lib.cuh as a C++ string for NVRTC."""
    src = (CSRC / "kernels" / "device_lib.cuh").read_text()
    out = BUILD / "device_lib_embed.cpp"
    delim = "B2LIB"
    assert f"){delim}\"" not in src
    text = (
        "// generated from csrc/kernels/device_lib.cuh by build.py\n"
        "namespace b2gpu {\n"
        f"extern const char* const kDeviceLibSource = R\"{delim}(\n{src}\n){delim}\";\n"
        "}\n"
    )
    if not out.exists() or out.read_text() != text:
        out.write_text(text)
    return out


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + proc.stdout + proc.stderr)


def _compile(src: Path) -> Path:
    obj = BUILD / (src.stem + (".cu.o" if src.suffix == ".cu" else ".o"))
    if not _stale(obj, [src] + HEADERS):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--fmad=false",
               f"-I{CUDA_HOME / 'include'}", "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXXFLAGS, f"-I{CUDA_HOME / 'include'}", "-c", str(src), "-o", str(obj)]
    _run(cmd)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    BIN.parent.mkdir(exist_ok=True)
    sources = HOST_SOURCES + CUDA_SOURCES + [_embed_device_lib()]
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objects = list(pool.map(_compile, sources))
    if _stale(LIB, objects):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objects),
              f"-L{CUDA_HOME / 'lib64'}", f"-L{CUDA_HOME / 'lib64' / 'stubs'}",
              "-cudart", "static", "-lnvrtc", "-Xlinker", "-rpath=" + str(CUDA_HOME / "lib64")])
    runner_src = CSRC / "runner_main.cpp"
    if _stale(BIN, [LIB, runner_src]):
        _run(["g++", "-O2", "-std=c++17", str(runner_src), "-o", str(BIN), f"-L{LIB.parent}", "-lb2gpu",
              "-Wl,-rpath,$ORIGIN/../lib",
              "-Wl,-rpath," + str(CUDA_HOME / "lib64")])
    if verbose:
        print(f"built {LIB} and {BIN}")
    return LIB


def clean() -> None:
    for p in (BUILD, LIB, BIN):
        if p.is_dir():
            shutil.rmtree(p)
        elif p.exists():
            p.unlink()


if __name__ == "__main__":
    if "clean" in sys.argv[1:]:
        clean()
    build(verbose=True)
