"""Multi-GPU runs: one process per GPU, launched by torchrun (or any launcher
that sets RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR / MASTER_PORT).

Replaces the reference's experimental MPI path (brian2_rust/distributed.py,
mpi_codegen.py, mpi_runtime/bridge.c:74-101), which partitions every
population by target ownership and all-gathers the global spike ids of every
tick over MPI, with rank 0 writing the results.  Here the partition is the
same (owner rule ((i+1)*G-1)//N), but the per-tick exchange happens inside the
GPUs' own kernels over NVLink; the host only trades CUDA IPC handles once and
synchronises before rank 0 assembles the results.  torch.distributed is the
rendezvous plumbing (a gloo group is enough); no NCCL call is on the tick path.

    from brian2_atlas_b200.distributed import run_model_distributed
    stats = run_model_distributed(model_json, "out")   # under torchrun

Every rank must make the same calls in the same order (the tick budgets of
step() included): a rank that stops stepping makes its peers' exchange waits
expire, which poisons their engines with an error instead of hanging.
"""
from __future__ import annotations

import os
from pathlib import Path

from . import B2GpuError, Engine


def _dist():
    import torch.distributed as dist
    if not dist.is_initialized():
        raise B2GpuError("torch.distributed is not initialised (call init_process_group first)")
    return dist


def exchange_handles(local: bytes, group=None) -> list:
    """All-gather one opaque handle per rank, in rank order."""
    dist = _dist()
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(local), group=group)
    return out


def connect(engine: Engine, group=None) -> None:
    """Trade IPC handles with every rank and map the peers' buffers."""
    handles = exchange_handles(engine.ipc_handle(), group)
    engine.connect(handles)
    _dist().barrier(group)


def create_engine(model_json: bytes, device: int | None = None, group=None, **options) -> Engine:
    """This rank's engine, connected to its peers.  `device` defaults to
    LOCAL_RANK."""
    dist = _dist()
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    if device is None:
        device = int(os.environ.get("LOCAL_RANK", rank))
    engine = Engine(model_json, device=device, rank=rank, world_size=world, **options)
    if world > 1:
        connect(engine, group)
    return engine


def write_results(engine: Engine, outdir, group=None) -> None:
    """Every rank stages its block; rank 0 writes the merged results into the
    new directory `outdir` (the b2-runner contract)."""
    dist = _dist()
    if engine.world_size > 1:
        engine.publish_results()
    dist.barrier(group)
    if dist.get_rank(group) == 0:
        outdir = Path(outdir)
        if outdir.exists():
            raise B2GpuError("output directory already exists; choose a new directory")
        outdir.mkdir(parents=True)
        engine.write_results(outdir)
    dist.barrier(group)


def run_model_distributed(model_json: bytes, outdir, device: int | None = None, group=None) -> dict:
    """Run a whole model on all ranks; rank 0 writes results.bin / events.bin /
    summary.json.  Returns this rank's statistics (its own deliveries)."""
    with create_engine(model_json, device, group) as engine:
        engine.run()
        write_results(engine, outdir, group)
        return engine.stats()


__all__ = ["exchange_handles", "connect", "create_engine", "write_results", "run_model_distributed"]
