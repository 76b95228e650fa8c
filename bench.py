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

With N > 1 GPUs (torchrun, one process per GPU) the same network is split by
target ownership: rank r owns neurons [floor(N r/G), floor(N (r+1)/G)) and
their incoming edges, and the tick kernels exchange spikes by storing into the
peers' memory over NVLink (strong scaling: the total work is fixed).  Every
timed step is bracketed by a barrier and a device synchronisation on every
rank; the step's time is the maximum over ranks; `value` counts every rank's
deliveries.

--impl reference times the CPU restatement of the reference executor
(oracle/b2ref, single-threaded like b2-runner) on a bounded sample of the
same network (50,000 neurons, in-degree 1000).

--workload stdp measures config 4 instead: 100,000 Poisson inputs at 15 Hz
onto 10,000 conductance-based LIF neurons, in-degree 1000 (1e7 plastic
synapses, f64 weights U[0, gmax], additive pre/post traces; definition layer
from the reference frontend's lowering of the Song-Abbott STDP example,
tests/golden/models/stdp_small.json.gz).  On N > 1 GPUs the inputs run whole
on every rank and the targets are partitioned.  Its CPU sample is the same
network at 10,000 inputs onto 1,000 neurons (1e6 synapses).
"""
from __future__ import annotations

import argparse
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
N_NEURONS = 1_000_000
INDEGREE = 1000
CPU_SAMPLE_NEURONS = 50_000
CPU_SAMPLE_WARMUP = 50
CPU_SAMPLE_TICKS = 200
METRIC = "synaptic events/s"
UNIT = "events/s"


# DRAM bytes (read + write) per launch of the neuron step kernel on the
# default 1M-neuron network, from one ncu capture (dram__bytes_read.sum +
# dram__bytes_write.sum, warm cache as in the timed run; the step kernel's
# traffic does not depend on the in-degree, so the 1M-neuron in-degree-300
# capture stands for the full network): 74,624 + 507,904 bytes.  The 56 MB of
# per-tick neuron state stays L2-resident within a step, so DRAM carries ~1 %
# of the algorithmic bytes.  None for other workloads.
STEP_DRAM_BYTES = {1_000_000: 74_624 + 507_904}


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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


def build_model(n, indegree, ticks, seed=3):
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    template = json.loads((ROOT / "tests" / "golden" / "models" / "cuba_poisson_small.json").read_text())
    return synthetic.encode(synthetic.cuba_fixed_indegree(template, n=n, indegree=indegree, ticks=ticks, seed=seed))


STDP_INPUTS, STDP_NEURONS, STDP_INDEGREE, STDP_RATE_HZ = 100_000, 10_000, 1000, 15.0
STDP_SAMPLE_INPUTS, STDP_SAMPLE_NEURONS = 10_000, 1000


def build_stdp(n_inputs, n_neurons, indegree, ticks, seed=5):
    import gzip
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    with gzip.open(ROOT / "tests" / "golden" / "models" / "stdp_small.json.gz", "rb") as f:
        template = json.loads(f.read())
    return synthetic.stdp_feedforward(template, n_inputs, n_neurons, indegree, ticks=ticks, seed=seed, spliced=True)


def cpu_sample(workdir: Path, warmup_ticks: int, timed_ticks: int, workload: str = "c2"):
    """Oracle (CPU restatement of b2-runner) on the bounded sample network."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    path = workdir / "cpu_sample.json"
    ticks = warmup_ticks + timed_ticks + 1
    if workload == "stdp":
        path.write_bytes(build_stdp(STDP_SAMPLE_INPUTS, STDP_SAMPLE_NEURONS, STDP_INDEGREE, ticks))
    else:
        path.write_bytes(build_model(CPU_SAMPLE_NEURONS, INDEGREE, ticks))
    out = subprocess.run([str(ROOT / "oracle" / "b2ref"), "--timed", str(warmup_ticks), str(timed_ticks), str(path)],
                         check=True, capture_output=True, text=True)
    return json.loads(out.stdout)


REFERENCE_TICKS_PER_STEP = 20  # one reference step: 20 ticks of the CPU sample network


def run_reference(args, world, rank):
    """CPU reference arm: rank 0 only; W warm-up steps then K timed steps of
    REFERENCE_TICKS_PER_STEP ticks each, in one oracle process."""
    if rank != 0:
        return
    steps, warmup = args.steps, args.warmup
    with tempfile.TemporaryDirectory() as tmp:
        s = cpu_sample(Path(tmp), REFERENCE_TICKS_PER_STEP * warmup, REFERENCE_TICKS_PER_STEP * steps, args.workload)
    total_events, total_seconds = s["synaptic_events"], s["seconds"]
    value = total_events / total_seconds if total_seconds > 0 else 0.0
    sim_seconds = s["ticks"] * DT
    per_step = [s]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
        "warmup": warmup, "ms_per_step": 1e3 * total_seconds / max(steps, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"STDP feedforward sample: {STDP_SAMPLE_INPUTS} inputs onto {STDP_SAMPLE_NEURONS} "
                               f"neurons x {STDP_INDEGREE} in-degree (config 4 scaled for one CPU core)",
                   "inputs": STDP_SAMPLE_INPUTS, "neurons": STDP_SAMPLE_NEURONS, "indegree": STDP_INDEGREE,
                   "dt_s": DT} if args.workload == "stdp" else
                  {"workload": f"CUBA fixed in-degree sample: {CPU_SAMPLE_NEURONS} neurons x {INDEGREE} in-degree "
                               f"+ Poisson drive (config 2 scaled for one CPU core)",
                   "neurons": CPU_SAMPLE_NEURONS, "indegree": INDEGREE, "dt_s": DT},
        "realtime_factor": sim_seconds / total_seconds if total_seconds else None,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": 1, "kind": "port",
                         "sample": f"{per_step[0]['ticks']} ticks of the sample network after "
                                   f"{REFERENCE_TICKS_PER_STEP * warmup} warm-up ticks"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--neurons", type=int, default=N_NEURONS)
    ap.add_argument("--indegree", type=int, default=INDEGREE)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="c2", choices=["c2", "stdp"])
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    pkg = importlib.import_module("brian2-atlas_b200")
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

    total_ticks = (args.warmup + args.steps) * TICKS_PER_STEP
    t0 = time.time()
    stdp = args.workload == "stdp"
    if stdp:
        model = build_stdp(STDP_INPUTS, STDP_NEURONS, STDP_INDEGREE, total_ticks + 400)
    else:
        model = build_model(args.neurons, args.indegree, total_ticks + 400)
    t_json = time.time() - t0
    if world > 1:
        eng = pkg.Engine(model, device=local_rank, rank=rank, world_size=world)
        distributed.connect(eng)
    else:
        eng = pkg.Engine(model, device=local_rank)
    del model
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
            d, w = reduce([s1["device_seconds"] - s0["device_seconds"], w1],
                          dist.ReduceOp.MAX if dist else None)
            dev += d
            wall += w
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
    # Per-kernel timing (events around each launch) over 400 further ticks.
    barrier()
    prof = eng.profile(400)
    prof_after = eng.stats()
    prof_spikes = prof_after["spikes"] - after["spikes"]
    prof_events = prof_after["synaptic_events"] - after["synaptic_events"]
    clock_summary = clocks.summary()
    barrier()
    eng.close()
    if dist is not None:
        clock_all = [None] * world
        dist.all_gather_object(clock_all, clock_summary)
        dist.destroy_process_group()
        if rank != 0:
            return
        clock_summary = dict(clock_all[0], reasons=sorted({r for c in clock_all for r in c["reasons"]}),
                             sm_mhz_min_over_ranks=min((c["sm_mhz"] or 0) for c in clock_all))
    local_neurons = pkg.partition(STDP_NEURONS if stdp else args.neurons, rank, world)
    local_neurons = local_neurons[1] - local_neurons[0]
    hbm, peak_kind = peaks()
    ticks_prof = 400
    kernels = []
    for k in prof:
        avg_ms = k["total_ms"] / max(k["launches"], 1)
        if stdp:
            # on_pre events per tick on this rank: inputs x 15 Hz x dt x
            # out-degree, i.e. 15 Hz x dt x local edges (the expectation of
            # the Poisson drive; the run's own count is within a percent)
            pre = STDP_RATE_HZ * DT * local_neurons * STDP_INDEGREE
            if k["name"].endswith("_targets") and os.environ.get("B2GPU_TARGETS_SCAN", "0") != "0":
                # bitmap scan: the 4 B source id of every local in-edge and
                # the 8 B row offset of every local target
                per_launch = 4 * local_neurons * STDP_INDEGREE + 8 * (local_neurons + 1)
            elif k["name"].endswith("_targets"):
                # bucket scatter per event: 4 B row entry, 4+4 B count
                # atomic, 8 B bucket offset, 8 B bucket entry
                per_launch = 28 * pre
            elif k["name"].endswith("_deliver"):
                # per event: 8 B bucket entry, 4 B edge id, the edge's f64
                # w, Apre, Apost, lastupdate read and w, Apre, lastupdate
                # written, the target's f64 ge read and written
                per_launch = (8 + 4 + 32 + 24 + 16) * pre
            else:
                per_launch = 0
        elif "_step" in k["name"]:
            # neuron update + threshold + compaction + reset: read and write
            # v, ge, gi (f64) and read lastspike (f64) per neuron, 4 B per spike
            per_launch = local_neurons * (2 * 24 + 8) + 4 * prof_spikes / ticks_prof
        elif k["name"].endswith("_atomic"):
            # scatter: 4 B row entry per event, read+write of the f64 target per
            # event (upper bound of 2*8*U_t), 4 B per fired source
            per_launch = (4 + 16) * (prof_events / ticks_prof) / 2 + 4 * prof_spikes / ticks_prof
        elif "poisson_input" in k["name"]:
            per_launch = local_neurons * 16
        else:
            per_launch = 0
        kernels.append({"name": k["name"], "avg_us": 1e3 * avg_ms, "launches": k["launches"],
                        "share": 0.0, "algorithmic_bytes": per_launch,
                        "achieved_gbs": per_launch / (avg_ms * 1e-3) / 1e9 if avg_ms > 0 else 0.0})
    total = sum(k["avg_us"] * k["launches"] for k in kernels) or 1.0
    for k in kernels:
        k["share"] = k["avg_us"] * k["launches"] / total
    dominant = max(kernels, key=lambda k: k["share"]) if kernels else None
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        with tempfile.TemporaryDirectory() as tmp:
            s = cpu_sample(Path(tmp), CPU_SAMPLE_WARMUP, CPU_SAMPLE_TICKS, args.workload)
        sample = (f"config 4 scaled to {STDP_SAMPLE_INPUTS} inputs onto {STDP_SAMPLE_NEURONS} neurons (in-degree "
                  f"{STDP_INDEGREE})" if stdp else
                  f"config 2 scaled to {CPU_SAMPLE_NEURONS} neurons (in-degree {INDEGREE})")
        cpu = {"value": s["synaptic_events"] / s["seconds"], "unit": UNIT, "cores": 1, "kind": "port",
               "sample": f"{s['ticks']} ticks of {sample} after {CPU_SAMPLE_WARMUP} warm-up ticks; oracle/b2ref "
                         f"single thread; {s['synaptic_events']} events in {s['seconds']:.3f} s"}
    if stdp:
        config = {"workload": "config 4: STDP feedforward, 100k Poisson inputs at 15 Hz onto 10k COBA LIF neurons, "
                              "in-degree 1000 (1e7 plastic synapses, on_pre + on_post)",
                  "inputs": STDP_INPUTS, "neurons": STDP_NEURONS, "indegree": STDP_INDEGREE,
                  "synapses": STDP_NEURONS * STDP_INDEGREE, "ticks_per_step": TICKS_PER_STEP, "dt_s": DT,
                  "parallelism": "single GPU" if world == 1 else
                  f"{world} GPUs: inputs replicated on every rank, targets partitioned, target spikes exchanged "
                  f"by peer stores over NVLink",
                  "l2": "256 MiB buffer written between timed steps; the 1e7-edge synapse state (320 MB) exceeds L2"}
    else:
        config = {"workload": "config 2: CUBA 1M neurons, fixed in-degree 1000 (1e9 synapses), Poisson 100x10 Hz",
                  "neurons": args.neurons, "indegree": args.indegree, "synapses": args.neurons * args.indegree,
                  "ticks_per_step": TICKS_PER_STEP, "dt_s": DT,
                  "parallelism": "single GPU" if world == 1 else
                  f"{world} GPUs: target-owned partition, spikes exchanged by peer stores over NVLink",
                  "l2": "256 MiB buffer written between timed steps; per-tick neuron state (56 MB) stays "
                        "L2-resident within a step"}
    line = {
        "metric": METRIC, "value": events / dev if dev > 0 else 0.0, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dev / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded; definition layer lowered by the reference frontend)",
        "config": config,
        "realtime_factor": sim_seconds / dev if dev > 0 else None,
        "realtime_factor_e2e": sim_seconds / wall if wall > 0 else None,
        "synaptic_events": events, "spikes": spikes,
        "e2e": {"value": events / wall if wall > 0 else 0.0, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches,
        "roofline": None if dominant is None else {
            "bound": "hbm", "kernel": dominant["name"], "achieved": dominant["achieved_gbs"], "peak": hbm,
            "peak_kind": peak_kind, "unit": "GB/s", "frac": dominant["achieved_gbs"] / hbm,
            "traffic": STEP_DRAM_BYTES.get(local_neurons) if "_step" in dominant["name"] and world == 1 and not stdp
            else None},
        "kernels": kernels,
        "clocks": clock_summary,
        "build": {"json_seconds": t_json, "engine_build_seconds": st0["build_seconds"],
                  "nvrtc_seconds": st0["compile_seconds"]},
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
