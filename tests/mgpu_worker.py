"""One rank of a multi-GPU test run, launched by torch.distributed.run with one
process per GPU (rendezvous on 127.0.0.1, gloo for the host-side handshake).

    worker.py run MODEL OUTDIR [MODEL OUTDIR ...]
        run every model on all ranks; rank 0 writes each OUTDIR
    worker.py stall MODEL TICKS
        rank 1 stops after TICKS ticks while rank 0 keeps stepping: rank 0's
        exchange wait must expire (exchange timeout 1 s) and raise, with no
        kernel left running on either GPU
"""
from __future__ import annotations

import importlib
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main(argv):
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    pkg = importlib.import_module("brian2-atlas_b200")
    distributed = importlib.import_module("brian2-atlas_b200.distributed")
    rank = dist.get_rank()
    try:
        _run(argv, dist, pkg, distributed, rank)
    except Exception as exc:  # surface the failing rank's message to the test
        print(json.dumps({"error": f"rank {rank}: {type(exc).__name__}: {exc}"}), flush=True)
        raise
    finally:
        dist.destroy_process_group()


def _run(argv, dist, pkg, distributed, rank):
    if argv[0] == "run":
        for model, outdir in zip(argv[1::2], argv[2::2]):
            stats = distributed.run_model_distributed(Path(model).read_bytes(), outdir)
            events = [None] * dist.get_world_size()
            dist.all_gather_object(events, stats["synaptic_events"])
            if rank == 0:
                print(json.dumps({"model": model, "events_per_rank": events}), flush=True)
    elif argv[0] == "stall":
        model, ticks = Path(argv[1]).read_bytes(), int(argv[2])
        outcome = "no error"
        with distributed.create_engine(model, exchange_timeout_ms=1000) as eng:
            eng.step(ticks)
            if rank == 0:
                try:
                    eng.step(ticks)
                except pkg.B2GpuError as exc:
                    outcome = str(exc)
            dist.barrier()  # rank 1 waits here with nothing in flight
            # rank 0's engine is poisoned; its peers must also refuse
            if rank == 0:
                try:
                    eng.step(1)
                except pkg.B2GpuError as exc:
                    outcome += " | then: " + str(exc)
        if rank == 0:
            print(json.dumps({"outcome": outcome}), flush=True)
        dist.barrier()
    else:
        raise SystemExit(f"unknown mode {argv[0]}")


if __name__ == "__main__":
    main(sys.argv[1:])
