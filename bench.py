"""Benchmark: synaptic events/s and realtime factor of the per-tick AtlasIR path.

Workload (config 2 of the benchmark set, one GPU): CUBA LIF network of
1,000,000 neurons (80% excitatory), fixed in-degree 1000 (1e9 synapses stored
as int32 row entries, generated on the device), Poisson drive of 100 inputs at
10 Hz per neuron, dt = 0.1 ms, float64 state.  The definition layer comes from
the reference frontend's lowering of the same network at 1000 neurons
(tests/golden/models/cuba_poisson_small.json); brian2-atlas_b200/synthetic.py
rescales it with seeded synthetic initial state.

One bench step = TICKS_PER_STEP ticks (100 ms simulated).  `value` is
synaptic events / device seconds (CUDA events around the tick kernels on the
engine's stream) over the timed steps; `e2e` is the same count over the wall
time of the public C-ABI b2g_step calls, which include the per-chunk
host->device tick cursor and device->host spike-list drain.

`raster_sha256` is the SHA-256 of the timed window's spikes (little-endian
int64 (tick, index) pairs in tick, then index order, per population, the
layout of results.bin's spike records) and `final_state_sha256` that of the
membrane state `v` read right after the window, merged over ranks: the same
digests at every GPU count show that a partitioned run computes the one-GPU
network.

With N > 1 GPUs (torchrun, one process per GPU) the same network is split by
target ownership: rank r owns neurons [floor(N r/G), floor(N (r+1)/G)) and
their incoming edges, and the tick kernels exchange spike lists by storing
into the peers' memory over NVLink (strong scaling: the total work is fixed).
Every timed step is bracketed by a barrier and a device synchronisation on
every rank; the step's time is the maximum over ranks; `value` counts every
rank's deliveries.

CPU side (one figure, one window): the CPU restatement of the reference
executor (oracle/b2ref, single-threaded like b2-runner; its one-time topology
build uses every host thread) runs the SAME network (same size, seed and
parameters) from tick 0 for W warm-up and K timed steps of
REFERENCE_TICKS_PER_STEP ticks.  `--impl reference` prints that as the
reference arm; the default run reports the same measurement as
`cpu_baseline`.  Its window lies in the network's opening transient, where
activity (events per tick) is ~3x the steady state the GPU window sees, which
raises a per-event CPU rate: the comparison favours the CPU.

--workload stdp measures config 4 instead: 100,000 Poisson inputs at 15 Hz
onto 10,000 conductance-based LIF neurons, in-degree 1000 (1e7 plastic
synapses, f64 weights U[0, gmax], additive pre/post traces; definition layer
from the reference frontend's lowering of the Song-Abbott STDP example,
tests/golden/models/stdp_small.json.gz).  On N > 1 GPUs the inputs run whole
on every rank and the targets are partitioned.  Its CPU sample is the same
network at 10,000 inputs onto 1,000 neurons (1e6 synapses), because the full
network's 1 GB document and 1e7 interpreted synapses do not fit a bounded CPU
run.

--workload c0 / c1 measure configs 0 and 1 (CUBA and COBAHH, 4000 neurons
each, the committed networks lowered by the reference frontend); their CPU
arm runs the GPU arm's own window (same ticks), not a shortened one.

--workload brunel measures config 3: the balanced Brunel network of
4,000,000 f32 LIF neurons, fixed in-degree 800 + 200 (4e9 synapses), a
homogeneous 1.5 ms (15-tick) delay, J = 0.1 mV, g = 5, PoissonInput of 800
inputs at twice the threshold rate (definition layer from the reference
frontend's lowering of brunel_device.py's network at 2000 neurons,
tests/golden/models/brunel_small.json).
"""
from __future__ import annotations

import argparse
import gzip
import hashlib
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TICKS_PER_STEP = 1000
DT = 1e-4
METRIC = "synaptic events/s"
UNIT = "events/s"
# CPU window: ticks per step of the reference arm (and of cpu_baseline, which
# times the same window): W warm-up + K timed steps of this many ticks.
REFERENCE_TICKS_PER_STEP = 2

WORKLOADS = {
    "c0": {"neurons": 4000, "indegree": 80, "dtype": "f64", "state_bytes": 24, "target_bytes": 8, "delay": 0,
           "fixture": "cuba_4k"},
    "c1": {"neurons": 4000, "indegree": 80, "dtype": "f64", "state_bytes": 48, "target_bytes": 8, "delay": 0,
           "fixture": "cobahh_4k"},
    "c2": {"neurons": 1_000_000, "indegree": 1000, "dtype": "f64", "state_bytes": 24, "target_bytes": 8,
           "delay": 0},
    "brunel": {"neurons": 4_000_000, "indegree": 1000, "dtype": "f32", "state_bytes": 4, "target_bytes": 4,
               "delay": 15},
    "stdp": {"inputs": 100_000, "neurons": 10_000, "indegree": 1000, "rate_hz": 15.0, "dtype": "f64",
             "cpu_warm": 100, "cpu_ticks": 300},
}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# dominant kernel, from one ncu capture of that kernel at the bench's network
# size (profiles/*.md gives the command and the figures).  The C2 step
# kernel's traffic does not depend on the in-degree, so a capture at in-degree
# 300 (a smaller device footprint) stands for the full network.  The per-tick
# neuron state (56 MB) stays L2-resident within a bench step, so DRAM carries
# ~1 % of the algorithmic bytes.  None where no capture exists.
TRAFFIC = {("c2", "_step", 1): 34_048 + 14_251}


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def host_facts() -> dict:
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    mem = None
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    mem = round(int(line.split()[1]) / 2 ** 20, 1)
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count(), "cpus_usable": len(os.sched_getaffinity(0)),
            "mem_gib": mem}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.lines = device, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _synthetic():
    return importlib.import_module("brian2-atlas_b200.synthetic")


def build_model(n, indegree, ticks, seed=3):
    template = json.loads((ROOT / "tests" / "golden" / "models" / "cuba_poisson_small.json").read_text())
    return _synthetic().encode(_synthetic().cuba_fixed_indegree(template, n=n, indegree=indegree, ticks=ticks,
                                                                seed=seed))


def build_brunel(n, indegree, ticks, seed=4):
    template = json.loads((ROOT / "tests" / "golden" / "models" / "brunel_small.json").read_text())
    return _synthetic().encode(_synthetic().brunel_fixed_indegree(template, n=n, indegree=indegree, ticks=ticks,
                                                                  seed=seed))


def build_stdp(n_inputs, n_neurons, indegree, ticks, seed=5):
    with gzip.open(ROOT / "tests" / "golden" / "models" / "stdp_small.json.gz", "rb") as f:
        template = json.loads(f.read())
    return _synthetic().stdp_feedforward(template, n_inputs, n_neurons, indegree, ticks=ticks, seed=seed,
                                         spliced=True)


def build_fixture(name, ticks):
    """A committed network lowered by the reference frontend (configs 0 and
    1 at their full size), its run extended to `ticks`."""
    with gzip.open(ROOT / "tests" / "golden" / "models" / f"{name}.json.gz", "rb") as f:
        doc = json.loads(f.read())
    _synthetic()._set_run(doc, ticks)
    return _synthetic().encode(_synthetic().attach_protocol(doc))


def build_workload(args, ticks):
    w = WORKLOADS[args.workload]
    if "fixture" in w:
        return build_fixture(w["fixture"], ticks)
    if args.workload == "stdp":
        return build_stdp(w["inputs"], w["neurons"], w["indegree"], ticks)
    if args.workload == "brunel":
        return build_brunel(args.neurons, args.indegree, ticks)
    return build_model(args.neurons, args.indegree, ticks)


def describe(args, world):
    """The `config` object of both arms (identical, so the lines compare)."""
    w = WORKLOADS[args.workload]
    if "fixture" in w:
        what = ("config 0: CUBA 4000 neurons (examples/CUBA.py), p = 0.02 (~320k synapses), exact-linear, f64"
                if args.workload == "c0" else
                "config 1: COBAHH 4000 neurons (examples/COBAHH.py), p = 0.02, exponential Euler, f64")
        return {"workload": what, "neurons": w["neurons"], "ticks_per_step": TICKS_PER_STEP, "dt_s": DT,
                "parallelism": "single GPU" if world == 1 else f"{world} GPUs: target-owned partition",
                "l2": "256 MiB buffer written between timed steps; the network fits in L2"}
    if args.workload == "stdp":
        return {"workload": "config 4: STDP feedforward, 100k Poisson inputs at 15 Hz onto 10k COBA LIF neurons, "
                            "in-degree 1000 (1e7 plastic synapses, on_pre + on_post)",
                "inputs": w["inputs"], "neurons": w["neurons"], "indegree": w["indegree"],
                "synapses": w["neurons"] * w["indegree"], "ticks_per_step": TICKS_PER_STEP, "dt_s": DT,
                "parallelism": "single GPU" if world == 1 else
                f"{world} GPUs: inputs replicated on every rank, targets partitioned",
                "l2": "256 MiB buffer written between timed steps; the 1e7-edge synapse state (320 MB) exceeds L2"}
    if args.workload == "brunel":
        return {"workload": "config 3: Brunel balanced network, f32 LIF, fixed in-degree 800+200, 15-tick delay, "
                            "PoissonInput 800 at 2x threshold rate",
                "neurons": args.neurons, "indegree": args.indegree, "synapses": args.neurons * args.indegree,
                "delay_ticks": 15, "ticks_per_step": TICKS_PER_STEP, "dt_s": DT,
                "parallelism": "single GPU" if world == 1 else
                f"{world} GPUs: target-owned partition, spike lists exchanged by peer stores over NVLink",
                "l2": "256 MiB buffer written between timed steps; 16 GB of row targets exceed L2"}
    return {"workload": "config 2: CUBA 1M neurons, fixed in-degree 1000 (1e9 synapses), Poisson 100x10 Hz",
            "neurons": args.neurons, "indegree": args.indegree, "synapses": args.neurons * args.indegree,
            "ticks_per_step": TICKS_PER_STEP, "dt_s": DT,
            "parallelism": "single GPU" if world == 1 else
            f"{world} GPUs: target-owned partition, spike lists exchanged by peer stores over NVLink",
            "l2": "256 MiB buffer written between timed steps; per-tick neuron state (56 MB) stays "
                  "L2-resident within a step"}


def cpu_window(args, model=None):
    """The oracle (CPU restatement of b2-runner) over W warm-up and K timed
    steps of REFERENCE_TICKS_PER_STEP ticks of the workload's network, from
    tick 0.  `model`: the GPU arm's own document (its run is longer than the
    window; the oracle stops after the window), else one is built.  Returns
    the oracle's measurement plus a description."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    warm = REFERENCE_TICKS_PER_STEP * args.warmup
    timed = REFERENCE_TICKS_PER_STEP * args.steps
    if "fixture" in WORKLOADS[args.workload]:
        # a 4000-neuron network: the CPU runs the GPU arm's own window
        warm, timed = TICKS_PER_STEP * args.warmup, TICKS_PER_STEP * args.steps
    if args.workload == "brunel":
        # nothing is delivered before the 15-tick delay has passed, and a
        # tick of the full network (17M events) takes seconds on one core:
        # start after the delay, at most 10 timed ticks
        warm, timed = WORKLOADS["brunel"]["delay"] + 1 + args.warmup, min(args.steps, 10)
    if args.workload == "stdp":
        # the full network: its output neurons fire only after the inputs
        # have driven them for some ticks; ~60k events per tick after that
        warm, timed = WORKLOADS["stdp"]["cpu_warm"], WORKLOADS["stdp"]["cpu_ticks"]
    t0 = time.time()
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "cpu_window.json"
        path.write_bytes(model if model is not None else build_workload(args, warm + timed + 1))
        t_json = time.time() - t0
        out = subprocess.run([str(ROOT / "oracle" / "b2ref"), "--timed", str(warm), str(timed), str(path)],
                             check=True, capture_output=True, text=True)
    s = json.loads(out.stdout)
    w = WORKLOADS[args.workload]
    network = "the bench's own network (same size and seed)"
    if "fixture" in w:
        network += ", the GPU arm's own window"
    if args.workload == "brunel":
        network += ", after the 15-tick delay"
    s["sample"] = (f"ticks {warm}..{warm + timed} of {network}, from tick 0 (the opening transient); "
                   f"oracle/b2ref tick loop on one thread; {s['synaptic_events']} events and {s['spikes']} spikes "
                   f"in {s['seconds']:.3f} s; topology build {s['build_seconds']:.1f} s on every host thread, "
                   + ("the GPU arm's document" if model is not None else f"document {t_json:.1f} s"))
    s["host"] = host_facts()
    return s


def run_reference(args, world, rank):
    """CPU reference arm: rank 0 only (the others exit without work)."""
    if rank != 0:
        return
    s = cpu_window(args)
    value = s["synaptic_events"] / s["seconds"] if s["seconds"] > 0 else 0.0
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * s["seconds"] / max(args.steps, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": WORKLOADS[args.workload]["dtype"], "data": "synthetic",
        "config": describe(args, world),
        "realtime_factor": s["ticks"] * DT / s["seconds"] if s["seconds"] else None,
        "synaptic_events": s["synaptic_events"], "spikes": s["spikes"],
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": 1, "kind": "port", "sample": s["sample"],
                         "host": s["host"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def raster_bytes(eng, populations, t0, t1):
    """Per population: the window's spikes as little-endian int64 (tick,
    index) pairs, tick then index order, and the per-tick counts."""
    import numpy as np
    out = []
    for p in populations:
        ticks, ids = [], []
        for tick in range(t0, t1):
            s = eng.spikes(p, tick)
            if s:
                ticks.append(np.full(len(s), tick, dtype=np.int64))
                ids.append(np.asarray(s, dtype=np.int64))
        if ticks:
            pairs = np.stack([np.concatenate(ticks), np.concatenate(ids)], axis=1)
        else:
            pairs = np.zeros((0, 2), dtype=np.int64)
        out.append(pairs.astype("<i8"))
    return out


def merge_rasters(per_rank):
    """Rank 0's merge of every rank's rasters: a list that every rank holds
    whole is taken once; rank-local blocks (disjoint, in rank order) are
    merged by (tick, index)."""
    import numpy as np
    merged = []
    for p in range(len(per_rank[0])):
        lists = [r[p] for r in per_rank]
        if all(a.shape == lists[0].shape and np.array_equal(a, lists[0]) for a in lists):
            merged.append(lists[0])
        else:
            both = np.concatenate(lists)
            order = np.lexsort((both[:, 1], both[:, 0]))
            merged.append(both[order])
    return merged


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=sorted(WORKLOADS))
    ap.add_argument("--neurons", type=int, default=None)
    ap.add_argument("--indegree", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--chunk-ticks", type=int, default=0, help="ticks per CUDA-graph replay (0: the engine default)")
    ap.add_argument("--no-graphs", action="store_true", help="launch every kernel directly (diagnostics)")
    args = ap.parse_args()
    w = WORKLOADS[args.workload]
    if args.neurons is None:
        args.neurons = w["neurons"]
    if args.indegree is None:
        args.indegree = w["indegree"]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    pkg = importlib.import_module("brian2-atlas_b200")
    import numpy as np
    import torch  # plumbing: process group, barriers, an L2 flush buffer
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        from datetime import timedelta
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
        distributed = importlib.import_module("brian2-atlas_b200.distributed")

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def reduce(values, op):
        if dist is None:
            return values
        t = torch.tensor(values, dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=op)
        return t.tolist()

    def gather(obj):
        if dist is None:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    total_ticks = (args.warmup + args.steps) * TICKS_PER_STEP
    stdp = args.workload == "stdp"
    t0 = time.time()
    model = build_workload(args, total_ticks + 400)
    t_json = time.time() - t0
    eopt = dict(chunk_ticks=args.chunk_ticks, use_graphs=not args.no_graphs)
    if dist is not None:
        eng = pkg.Engine(model, device=local_rank, rank=rank, world_size=world, **eopt)
        distributed.connect(eng)
    else:
        eng = pkg.Engine(model, device=local_rank, **eopt)
    if args.no_cpu_baseline or world > 1:
        del model  # else kept for the CPU leg, which runs the same document
    n_pops = 2 if stdp else 1
    state_pop = 1 if stdp else 0
    st0 = eng.stats()
    for _ in range(args.warmup):
        barrier()
        eng.step(TICKS_PER_STEP)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")
    before = eng.stats()
    wall = 0.0
    dev = 0.0
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.steps):
            flush.fill_(1)
            barrier()
            s0 = eng.stats()
            w0 = time.perf_counter()
            eng.step(TICKS_PER_STEP)
            w1 = time.perf_counter() - w0
            s1 = eng.stats()
            barrier()
            # the step's time is the slowest rank's
            d, wt = reduce([s1["device_seconds"] - s0["device_seconds"], w1],
                           dist.ReduceOp.MAX if dist else None)
            dev += d
            wall += wt
    after = eng.stats()
    # deliveries and launches of every rank; spikes are global on every rank
    events, launches = reduce([after["synaptic_events"] - before["synaptic_events"],
                               after["kernel_launches"] - before["kernel_launches"]],
                              dist.ReduceOp.SUM if dist else None)
    events, launches = int(events), int(launches)
    spikes = after["spikes"] - before["spikes"]
    h2d = (after["h2d_bytes"] - before["h2d_bytes"]) / args.steps
    d2h = (after["d2h_bytes"] - before["d2h_bytes"]) / args.steps
    sim_seconds = args.steps * TICKS_PER_STEP * DT
    # digests of the timed window (host copies of the drained lists) and of
    # the membrane state right after it, merged over ranks on rank 0
    w_lo, w_hi = args.warmup * TICKS_PER_STEP, (args.warmup + args.steps) * TICKS_PER_STEP
    rasters = gather(raster_bytes(eng, range(n_pops), w_lo, w_hi))
    v_block = gather(eng.read_state(state_pop, "v"))
    # Per-kernel timing (events around each launch) over 400 further ticks.
    barrier()
    prof = eng.profile(400)
    prof_after = eng.stats()
    prof_spikes = prof_after["spikes"] - after["spikes"]
    prof_events = prof_after["synaptic_events"] - after["synaptic_events"]
    clock_summary = clocks.summary()
    barrier()
    eng.close()
    clock_all = gather(clock_summary)
    if dist is not None:
        dist.destroy_process_group()
        if rank != 0:
            return
        clock_summary = dict(clock_all[0], reasons=sorted({r for c in clock_all for r in c["reasons"]}),
                             sm_mhz_min_over_ranks=min((c["sm_mhz"] or 0) for c in clock_all))
    merged = merge_rasters(rasters)
    raster_sha = hashlib.sha256(b"".join(m.tobytes() for m in merged)).hexdigest()
    # a replicated population (one that no synapse targets) is whole on
    # every rank; a partitioned one is the concatenation of the rank blocks
    full = w["neurons"] * (4 if w["dtype"] == "f32" else 8) if stdp else \
        args.neurons * (4 if w["dtype"] == "f32" else 8)
    v_all = v_block[0] if len(v_block[0]) == full else b"".join(v_block)
    state_sha = hashlib.sha256(v_all).hexdigest()
    local_neurons = pkg.partition(w["neurons"] if stdp else args.neurons, rank, world)
    local_neurons = local_neurons[1] - local_neurons[0]
    hbm, peak_kind = peaks()
    ticks_prof = 400
    e_t = prof_events / ticks_prof  # this rank's deliveries per tick
    f_t = prof_spikes / ticks_prof  # spikes per tick (global list)
    kernels = []
    for k in prof:
        name = k["name"]
        if stdp:
            # on_pre events per tick on this rank: 15 Hz x dt x local edges
            pre = w["rate_hz"] * DT * local_neurons * w["indegree"]
            if name.endswith("_targets") and os.environ.get("B2GPU_TARGETS_SCAN", "0") != "0":
                per_launch = 4 * local_neurons * w["indegree"] + 8 * (local_neurons + 1)
            elif name.endswith("_targets"):
                # bucket scatter per event: 4 B row entry, 4+4 B count
                # atomic, 8 B bucket offset, 8 B bucket entry
                per_launch = 28 * pre
            elif name.endswith("_deliver"):
                # per event: 8 B bucket entry, 4 B edge id, the edge's f64
                # w, Apre, Apost, lastupdate read and w, Apre, lastupdate
                # written, the target's f64 ge read and written
                per_launch = (8 + 4 + 32 + 24 + 16) * pre
            else:
                per_launch = 0
        elif "_step" in name:
            # neuron update + threshold + compaction + reset: read and write
            # the state (S bytes) and read lastspike (8 B) per neuron, 4 B
            # per spike written to the list
            per_launch = local_neurons * (2 * w["state_bytes"] + 8) + 4 * f_t
        elif name.endswith("_atomic"):
            # constant-addend scatter: 4 B row entry per event; read + write
            # of each distinct (target, variable) touched, U = N (1 - (1 -
            # 1/N)^E) per pathway for uniformly drawn targets, the in-degree
            # split 80/20 between the two pathways (a kernel of one pathway
            # gets its share); per fired source its ring entry (4 B) and row
            # bounds (16 B)
            n = max(local_neurons, 1)
            shares = (0.8,) if "excitatory" in name else (0.2,) if "inhibitory" in name else (0.8, 0.2)
            u = sum(n * (1.0 - (1.0 - 1.0 / n) ** (share * e_t)) for share in shares)
            per_launch = 4 * sum(shares) * e_t + 2 * w["target_bytes"] * u + 20 * f_t
        else:
            per_launch = 0
        kernels.append({"name": name, "event_us": 1e3 * k["total_ms"] / max(k["launches"], 1),
                        "launches": k["launches"], "algorithmic_bytes": per_launch})
    # A kernel's duration inside the graph-replayed tick: its share of the
    # event-timed launch sum times the measured device time per tick (the
    # event-timed launches also hold launch latency and lose the
    # programmatic-dependent-launch overlap, so their sum exceeds the tick).
    ms_tick = 1e3 * dev / (args.steps * TICKS_PER_STEP)
    total = sum(k["event_us"] * k["launches"] for k in kernels) or 1.0
    per_tick_launches = {k["name"]: k["launches"] / ticks_prof for k in kernels}
    for k in kernels:
        k["share"] = k["event_us"] * k["launches"] / total
        k["avg_us"] = k["share"] * ms_tick * 1e3 / max(per_tick_launches[k["name"]], 1e-9)
        k["achieved_gbs"] = k["algorithmic_bytes"] / (k["avg_us"] * 1e-6) / 1e9 if k["avg_us"] > 0 else 0.0
    dominant = max(kernels, key=lambda k: k["share"]) if kernels else None
    traffic = None
    if dominant is not None:
        for (wl, frag, n_gpu), b in TRAFFIC.items():
            if wl == args.workload and frag in dominant["name"] and n_gpu == world and \
                    args.neurons == w["neurons"]:
                traffic = b
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        s = cpu_window(args, model)
        del model
        cpu = {"value": s["synaptic_events"] / s["seconds"], "unit": UNIT, "cores": 1, "kind": "port",
               "sample": s["sample"], "host": s["host"]}
    line = {
        "metric": METRIC, "value": events / dev if dev > 0 else 0.0, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dev / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": w["dtype"],
        "data": "synthetic (seeded; definition layer lowered by the reference frontend)",
        "config": describe(args, world),
        "realtime_factor": sim_seconds / dev if dev > 0 else None,
        "realtime_factor_e2e": sim_seconds / wall if wall > 0 else None,
        "synaptic_events": events, "spikes": spikes,
        "raster_sha256": raster_sha, "final_state_sha256": state_sha,
        "digest_window_ticks": [w_lo, w_hi],
        "e2e": {"value": events / wall if wall > 0 else 0.0, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches,
        "roofline": None if dominant is None else {
            "bound": "hbm", "kernel": dominant["name"], "achieved": dominant["achieved_gbs"], "peak": hbm,
            "peak_kind": peak_kind, "unit": "GB/s", "frac": dominant["achieved_gbs"] / hbm, "traffic": traffic,
            "kernel_us": dominant["avg_us"], "algorithmic_bytes": dominant["algorithmic_bytes"],
            "timing": "kernel share of the event-timed launches x graph-replayed device time per tick"},
        "kernels": kernels,
        "clocks": clock_summary,
        "build": {"json_seconds": t_json, "engine_build_seconds": st0["build_seconds"],
                  "nvrtc_seconds": st0["compile_seconds"]},
        "cpu_baseline": cpu,
        "host": host_facts(),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
