"""Compile and launch a small CUDA test kernel that includes the engine's
device library (brian2-atlas_b200/csrc/kernels/device_lib.cuh) with the same
NVRTC options the engine uses, so device helpers can be checked element by
element against plain CUDA arithmetic.  Test infrastructure only: torch owns
the device buffers, cuda-python's NVRTC and driver bindings compile and
launch.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
DEVICE_LIB = ROOT / "brian2-atlas_b200" / "csrc" / "kernels" / "device_lib.cuh"
OPTIONS = [b"--gpu-architecture=sm_100a", b"--std=c++17", b"--fmad=false", b"--prec-div=true",
           b"--prec-sqrt=true", b"--ftz=false", b"-default-device"]


def _check(result):
    err = result[0]
    if int(err) != 0:
        raise RuntimeError(f"CUDA call failed: {err}")
    return result[1:] if len(result) > 2 else (result[1] if len(result) == 2 else None)


class Kernel:
    def __init__(self, source: str, name: str):
        from cuda.bindings import driver, nvrtc
        self._driver = driver
        full = DEVICE_LIB.read_text() + "\n" + source
        prog = _check(nvrtc.nvrtcCreateProgram(full.encode(), b"test.cu", 0, [], []))
        res = nvrtc.nvrtcCompileProgram(prog, len(OPTIONS), OPTIONS)
        if int(res[0]) != 0:
            size = _check(nvrtc.nvrtcGetProgramLogSize(prog))
            log = b" " * size
            nvrtc.nvrtcGetProgramLog(prog, log)
            raise RuntimeError(log.decode())
        size = _check(nvrtc.nvrtcGetCUBINSize(prog))
        cubin = b" " * size
        _check(nvrtc.nvrtcGetCUBIN(prog, cubin))
        self._module = _check(driver.cuModuleLoadData(cubin))
        self._fn = _check(driver.cuModuleGetFunction(self._module, name.encode()))

    def launch(self, grid: int, block: int, args: list, types: list, stream: int = 0):
        _check(self._driver.cuLaunchKernel(self._fn, grid, 1, 1, block, 1, 1, 0, stream,
                                           (tuple(args), tuple(types)), 0))


def pointer(tensor) -> tuple:
    return tensor.data_ptr(), ctypes.c_void_p
