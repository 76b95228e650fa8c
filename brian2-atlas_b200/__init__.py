"""brian2-atlas_b200: B200 engine for Brian2 Atlas AtlasIR simulations.

Host-side mirror of the reference's runner interface.  The reference frontend
runs its engine as a subprocess (`b2-runner MODEL.json OUTDIR`,
brian2-rust/python/brian2_rust/device.py:1316-1365); this package exposes the
same operation in-process over the C ABI of lib/libb2gpu.so (include/b2gpu.h):

    run_model(model_json_bytes, outdir)    # == b2-runner MODEL.json OUTDIR
    Engine(model_json_bytes).step(ticks)    # == Runtime::new / Runtime::step
    runner_path()                           # B2_RUNNER drop-in binary

Every operation runs the compiled CUDA engine; there is no CPU fallback.  If
the library has not been built (`python brian2-atlas_b200/build.py`), loading
fails with an error instead of degrading.
"""
from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIBRARY = _PKG / "lib" / "libb2gpu.so"
RUNNER = _PKG / "bin" / "b2gpu-runner"
_lib = None


class B2GpuError(RuntimeError):
    """An engine call failed; the message is the engine's error text."""


class Options(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("device", ctypes.c_int32), ("chunk_ticks", ctypes.c_uint32),
                ("use_graphs", ctypes.c_uint32), ("ring_capacity", ctypes.c_uint64), ("rank", ctypes.c_int32),
                ("world_size", ctypes.c_int32), ("exchange_timeout_ms", ctypes.c_uint32), ("reserved0", ctypes.c_uint32)]


class Stats(ctypes.Structure):
    _fields_ = [("ticks", ctypes.c_uint64), ("synaptic_events", ctypes.c_uint64), ("spikes", ctypes.c_uint64),
                ("kernel_launches", ctypes.c_uint64), ("launches_per_tick", ctypes.c_uint64),
                ("simulation_seconds", ctypes.c_double), ("build_seconds", ctypes.c_double),
                ("compile_seconds", ctypes.c_double), ("device_seconds", ctypes.c_double),
                ("h2d_bytes", ctypes.c_uint64), ("d2h_bytes", ctypes.c_uint64)]


class KernelTime(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 64), ("launches", ctypes.c_uint64), ("total_ms", ctypes.c_double)]


def library() -> ctypes.CDLL:
    """Load libb2gpu.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise B2GpuError(f"{LIBRARY} is missing; run `python brian2-atlas_b200/build.py`")
    lib = ctypes.CDLL(str(LIBRARY))
    c = ctypes
    sig = {
        "b2g_default_options": (None, [c.POINTER(Options)]),
        "b2g_create": (c.c_void_p, [c.c_char_p, c.c_size_t, c.POINTER(Options), c.c_char_p, c.c_size_t]),
        "b2g_step": (c.c_int, [c.c_void_p, c.c_uint64, c.POINTER(c.c_int), c.c_char_p, c.c_size_t]),
        "b2g_write_results": (c.c_int, [c.c_void_p, c.c_char_p, c.c_char_p, c.c_size_t]),
        "b2g_summary_json": (c.c_int, [c.c_void_p, c.c_char_p, c.c_size_t, c.POINTER(c.c_size_t), c.c_char_p,
                                       c.c_size_t]),
        "b2g_get_stats": (c.c_int, [c.c_void_p, c.POINTER(Stats), c.c_char_p, c.c_size_t]),
        "b2g_read_state": (c.c_int, [c.c_void_p, c.c_uint32, c.c_char_p, c.c_void_p, c.c_size_t,
                                     c.POINTER(c.c_size_t), c.c_char_p, c.c_size_t]),
        "b2g_spikes": (c.c_int, [c.c_void_p, c.c_uint32, c.c_uint64, c.c_void_p, c.c_size_t,
                                 c.POINTER(c.c_size_t), c.c_char_p, c.c_size_t]),
        "b2g_generated_source": (c.c_int, [c.c_void_p, c.c_char_p, c.c_size_t, c.POINTER(c.c_size_t)]),
        "b2g_codegen": (c.c_int, [c.c_char_p, c.c_size_t, c.POINTER(Options), c.c_char_p, c.c_size_t,
                                  c.POINTER(c.c_size_t), c.c_char_p, c.c_size_t]),
        "b2g_partition": (None, [c.c_uint64, c.c_int32, c.c_int32, c.POINTER(c.c_uint64), c.POINTER(c.c_uint64)]),
        "b2g_ipc_handle": (c.c_int, [c.c_void_p, c.c_void_p, c.c_size_t, c.POINTER(c.c_size_t), c.c_char_p,
                                     c.c_size_t]),
        "b2g_connect": (c.c_int, [c.c_void_p, c.c_void_p, c.c_size_t, c.c_size_t, c.c_char_p, c.c_size_t]),
        "b2g_publish_results": (c.c_int, [c.c_void_p, c.c_char_p, c.c_size_t]),
        "b2g_spikes_scratch_bytes": (c.c_size_t, [c.c_uint64]),
        "b2g_spikes_from_bitmap_noalloc": (c.c_int, [c.c_void_p, c.c_uint64, c.c_void_p, c.c_void_p, c.c_void_p,
                                                     c.c_char_p, c.c_size_t]),
        "b2g_spikes_from_bitmap": (c.c_int, [c.c_void_p, c.c_uint64, c.c_void_p, c.c_void_p, c.c_void_p, c.c_size_t,
                                             c.c_void_p, c.c_char_p, c.c_size_t]),
        "b2g_profile": (c.c_int, [c.c_void_p, c.c_uint64, c.POINTER(KernelTime), c.c_size_t,
                                  c.POINTER(c.c_size_t), c.c_char_p, c.c_size_t]),
        "b2g_destroy": (None, [c.c_void_p]),
        "b2g_version": (c.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _err():
    return ctypes.create_string_buffer(4096)


def version() -> str:
    return library().b2g_version().decode()


def _options(device=-1, chunk_ticks=0, use_graphs=True, ring_capacity=0, rank=0, world_size=1,
             exchange_timeout_ms=0) -> Options:
    opt = Options()
    library().b2g_default_options(ctypes.byref(opt))
    opt.device = device
    if chunk_ticks:
        opt.chunk_ticks = chunk_ticks
    opt.use_graphs = 1 if use_graphs else 0
    opt.ring_capacity = ring_capacity
    opt.rank = rank
    opt.world_size = world_size
    opt.exchange_timeout_ms = exchange_timeout_ms
    return opt


def codegen(model_json: bytes, rank: int = 0, world_size: int = 1) -> str:
    """Compile a model's plan (of one rank of `world_size`) for sm_100a without
    a GPU and return the generated source."""
    lib = library()
    opt = _options(rank=rank, world_size=world_size)
    err, need = _err(), ctypes.c_size_t(0)
    if lib.b2g_codegen(model_json, len(model_json), ctypes.byref(opt), None, 0, ctypes.byref(need), err, len(err)):
        raise B2GpuError(err.value.decode())
    buf = ctypes.create_string_buffer(need.value)
    if lib.b2g_codegen(model_json, len(model_json), ctypes.byref(opt), buf, need, ctypes.byref(need), err, len(err)):
        raise B2GpuError(err.value.decode())
    return buf.value.decode()


def partition(count: int, rank: int, world_size: int) -> tuple:
    """Global index range [lo, hi) that `rank` of `world_size` owns (the
    reference's owner rule, brian2_rust/distributed.py:80-81)."""
    lo, hi = ctypes.c_uint64(0), ctypes.c_uint64(0)
    library().b2g_partition(count, rank, world_size, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def spikes_from_bitmap(d_words: int, nbits: int, d_ids: int, d_count: int, d_scratch: int, scratch_bytes: int,
                       stream: int = 0) -> None:
    """Device primitive (pointers are device addresses, e.g. tensor.data_ptr()):
    ascending indices of the set bits among the first `nbits` bits of the u32
    words at d_words into d_ids, their number into the u32 at d_count;
    asynchronous on `stream` (a cudaStream_t handle)."""
    lib = library()
    err = _err()
    if lib.b2g_spikes_from_bitmap(d_words, nbits, d_ids, d_count, d_scratch, scratch_bytes, stream or None, err,
                                  len(err)):
        raise B2GpuError(err.value.decode())


SPIKES_NOALLOC_MAX_BITS = 1 << 27


def spikes_from_bitmap_noalloc(d_words: int, nbits: int, d_ids: int, d_count: int, stream: int = 0) -> None:
    """spikes_from_bitmap without device allocation (the library's fixed
    scratch; nbits <= SPIKES_NOALLOC_MAX_BITS; overlapping calls on one GPU
    race; the first call on a device does a one-time set-up)."""
    lib = library()
    err = _err()
    if lib.b2g_spikes_from_bitmap_noalloc(d_words, nbits, d_ids, d_count, stream or None, err, len(err)):
        raise B2GpuError(err.value.decode())


def spikes_scratch_bytes(nbits: int) -> int:
    return library().b2g_spikes_scratch_bytes(nbits)


class Engine:
    """One AtlasIR run on one GPU (mirrors the reference `Runtime`)."""

    def __init__(self, model_json: bytes, device: int = -1, chunk_ticks: int = 0, use_graphs: bool = True,
                 ring_capacity: int = 0, rank: int = 0, world_size: int = 1, exchange_timeout_ms: int = 0):
        lib = library()
        opt = _options(device, chunk_ticks, use_graphs, ring_capacity, rank, world_size, exchange_timeout_ms)
        self.rank, self.world_size = rank, world_size
        err = _err()
        self._h = lib.b2g_create(model_json, len(model_json), ctypes.byref(opt), err, len(err))
        if not self._h:
            raise B2GpuError(err.value.decode())
        self._lib = lib

    def _call(self, name, *args):
        err = _err()
        if getattr(self._lib, name)(self._h, *args, err, len(err)):
            raise B2GpuError(err.value.decode())

    def step(self, max_ticks: int = 2 ** 63) -> bool:
        done = ctypes.c_int(0)
        self._call("b2g_step", ctypes.c_uint64(max_ticks), ctypes.byref(done))
        return bool(done.value)

    def run(self) -> None:
        while not self.step():
            pass

    def write_results(self, outdir) -> None:
        self._call("b2g_write_results", str(outdir).encode())

    def summary(self) -> dict:
        """summary.json of the completed run, without writing files."""
        need = ctypes.c_size_t(0)
        self._call("b2g_summary_json", None, 0, ctypes.byref(need))
        buf = ctypes.create_string_buffer(need.value + 1)
        self._call("b2g_summary_json", buf, need.value + 1, ctypes.byref(need))
        return json.loads(buf.value.decode())

    def stats(self) -> dict:
        s = Stats()
        self._call("b2g_get_stats", ctypes.byref(s))
        return {name: getattr(s, name) for name, _ in Stats._fields_}

    def read_state(self, population: int, name: str) -> bytes:
        need = ctypes.c_size_t(0)
        self._call("b2g_read_state", population, name.encode(), None, 0, ctypes.byref(need))
        buf = ctypes.create_string_buffer(need.value)
        self._call("b2g_read_state", population, name.encode(), buf, need, ctypes.byref(need))
        return buf.raw[:need.value]

    def spikes(self, population: int, tick: int) -> list:
        count = ctypes.c_size_t(0)
        self._call("b2g_spikes", population, ctypes.c_uint64(tick), None, 0, ctypes.byref(count))
        buf = (ctypes.c_uint32 * max(count.value, 1))()
        self._call("b2g_spikes", population, ctypes.c_uint64(tick), buf, count.value, ctypes.byref(count))
        return list(buf[:count.value])

    def profile(self, ticks: int) -> list:
        """Advance `ticks` ticks with per-kernel CUDA-event timing."""
        out = (KernelTime * 64)()
        count = ctypes.c_size_t(0)
        self._call("b2g_profile", ctypes.c_uint64(ticks), out, 64, ctypes.byref(count))
        return [{"name": out[i].name.decode(), "launches": out[i].launches, "total_ms": out[i].total_ms}
                for i in range(min(count.value, 64))]

    # ---- multi-GPU (see brian2-atlas_b200/distributed.py for the driver)
    def ipc_handle(self) -> bytes:
        """CUDA IPC handle of this rank's shared exchange/staging allocation."""
        buf = ctypes.create_string_buffer(256)
        n = ctypes.c_size_t(0)
        self._call("b2g_ipc_handle", buf, 256, ctypes.byref(n))
        return buf.raw[:n.value]

    def connect(self, handles: list) -> None:
        """Map every rank's allocation; `handles` = all ranks' ipc_handle() in rank order."""
        if len({len(h) for h in handles}) != 1:
            raise B2GpuError("IPC handles differ in length")
        blob = b"".join(handles)
        self._call("b2g_connect", blob, len(handles[0]), len(handles))

    def publish_results(self) -> None:
        """Stage this rank's final results for rank 0's write_results()."""
        self._call("b2g_publish_results")

    def generated_source(self) -> str:
        need = ctypes.c_size_t(0)
        self._lib.b2g_generated_source(self._h, None, 0, ctypes.byref(need))
        buf = ctypes.create_string_buffer(need.value)
        self._lib.b2g_generated_source(self._h, buf, need, ctypes.byref(need))
        return buf.value.decode()

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.b2g_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        self.close()


def run_model(model_json: bytes, outdir, device: int = -1) -> dict:
    """Run a whole model and write results.bin/events.bin/summary.json into the
    new directory `outdir` (the b2-runner contract: the directory must not
    exist beforehand)."""
    outdir = Path(outdir)
    if outdir.exists():
        raise B2GpuError("output directory already exists; choose a new directory")
    with Engine(model_json, device=device) as eng:
        eng.run()
        outdir.mkdir(parents=True)
        eng.write_results(outdir)
        return eng.stats()


def runner_path() -> Path:
    """Path of the b2-runner drop-in binary (export it as B2_RUNNER)."""
    if not RUNNER.exists():
        raise B2GpuError(f"{RUNNER} is missing; run `python brian2-atlas_b200/build.py`")
    return RUNNER


def package_dir() -> Path:
    return _PKG


__all__ = ["Engine", "B2GpuError", "run_model", "codegen", "partition", "spikes_from_bitmap", "spikes_scratch_bytes",
           "spikes_from_bitmap_noalloc", "SPIKES_NOALLOC_MAX_BITS", "version", "library", "runner_path", "LIBRARY", "RUNNER"]
