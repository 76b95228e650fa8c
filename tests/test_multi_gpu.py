"""Multi-GPU partition and spike exchange.

CPU (no GPU): the owner rule against the reference's formula
(brian2_rust/distributed.py:80-81), the per-rank plans, capability errors,
and the host-side handshake over two gloo ranks.
GPU (>= 2 GPUs): torchrun ranks against the oracle, byte for byte, as the
reference's MPI equivalence tests demand of 1/2/3/4 ranks
(brian2-rust/tests/test_mpi.py:265-734); and a rank that stops stepping makes
its peer's bounded exchange wait expire with an error instead of a hang.
"""
from __future__ import annotations

import json
import os
import re
import socket
import subprocess
import sys

import pytest

from conftest import GOLDEN, MODELS, ROOT, model_file, run_oracle
from b2results import describe_difference, load_model


def owner(i, n, g):
    return ((i + 1) * g - 1) // n


@pytest.mark.parametrize("n,g", [(1, 1), (10, 3), (4000, 3), (100, 8), (1000003, 8), (7, 8)])
def test_partition_is_the_reference_owner_rule(pkg, n, g):
    covered = 0
    for r in range(g):
        lo, hi = pkg.partition(n, r, g)
        assert lo == covered
        for i in {lo, hi - 1} if hi > lo else set():
            assert owner(i, n, g) == r
        covered = hi
    assert covered == n


def kernels(src):
    return re.findall(r"__global__ void __launch_bounds__\(\d+(?:, \d+)?\) (\w+)", src)


@pytest.mark.parametrize("world", [2, 3])
def test_rank_plans(pkg, world, monkeypatch):
    data = (MODELS / "cuba_small.json").read_bytes()
    n = json.loads(data)["definition"]["populations"][0]["count"]
    for r in range(world):
        src = pkg.codegen(data, rank=r, world_size=world)
        names = kernels(src)
        # the step publishes its block's ascending list to every rank; the
        # scatter waits for every rank's list, delivers it straight from the
        # inbox and lays the global list out in the ring
        assert [k.split("_", 2)[2] for k in names][-2:] == ["neurons_step", "neurons_receive_exc_pre_inh_pre_atomic"]
        lo, hi = pkg.partition(n, r, world)
        step = src[src.index("neurons_step("):src.index("neurons_receive_exc_pre_inh_pre_atomic(")]
        assert f"i < {hi - lo}u" in step and "b2_ll_store" in step and "atomicAdd" not in step
        assert "b2_ll_wait" in src[src.index("neurons_receive_exc_pre_inh_pre_atomic("):]
    # a separate receive launch, then the scatter reads the ring
    monkeypatch.setenv("B2GPU_FUSE_EXCHANGE", "0")
    names = [k.split("_", 2)[2] for k in kernels(pkg.codegen(data, rank=0, world_size=world))]
    assert names[-3:] == ["neurons_step", "neurons_receive", "exc_pre_inh_pre_atomic"]


def test_delayed_receive_moves_after_the_delivery(pkg, tmp_path, monkeypatch):
    """Brunel (one 15-tick delay): no kernel reads the tick's own list (the
    reset runs inside the PoissonInput kernel, on the lanes the threshold
    just fired), so the receive moves behind the delayed delivery and joins
    its launch: the scatter's first blocks wait for the peers' lists and lay
    them out while the others deliver older ticks' spikes
    (B2GPU_FUSE_LAYOUT=0: a receive kernel of its own at the end of the
    tick); with no fusion at all (one kernel per node) it stays right after
    the step."""
    data = (MODELS / "brunel_small.json").read_bytes()
    src = pkg.codegen(data, rank=1, world_size=4)
    names = [k.split("_", 2)[2] for k in kernels(src) if not k.startswith("b2_flush_")]
    assert names[-1].endswith("_atomic") and "neurons_reset" not in names and "neurons_receive" not in names
    last = src[src.index(kernels(src)[-2] + "("):]
    assert "b2_ll_wait" in last and "s_pre[" in last and "b2_bid" in last
    monkeypatch.setenv("B2GPU_FUSE_LAYOUT", "0")
    names = [k.split("_", 2)[2] for k in kernels(pkg.codegen(data, rank=1, world_size=4)) if not k.startswith("b2_flush_")]
    assert names[-1] == "neurons_receive"
    monkeypatch.delenv("B2GPU_FUSE_LAYOUT")
    monkeypatch.setenv("B2GPU_NO_FUSE", "1")
    names = [k.split("_", 2)[2] for k in kernels(pkg.codegen(data, rank=1, world_size=4)) if not k.startswith("b2_flush_")]
    assert names.index("neurons_receive") == names.index("neurons_step") + 1


def test_multi_gpu_synapse_programs_and_presynaptic_replicas(pkg, tmp_path):
    """Synaptic state updates and run_regularly run over each rank's own
    edges; a summed variable that reads the presynaptic v of a partitioned
    population (gap junctions) reads a replica that a replicate kernel and a
    bounded wait refresh right before it (the reference's MPI path keeps
    read-only presynaptic replicas, distributed.py:255)."""
    names = kernels(pkg.codegen(model_file("synapse_updates_small", tmp_path).read_bytes(), rank=1, world_size=2))
    assert [n.split("_", 2)[2] for n in names][:3] == ["decay", "inputs_step_neurons_step", "stdp_stateupdater"]
    src = pkg.codegen(model_file("gap_junctions_small", tmp_path).read_bytes(), rank=1, world_size=3)
    names = [n.split("_", 2)[2] for n in kernels(src)]
    assert names[1:4] == ["neurons_v_replicate", "neurons_v_replica_wait", "gaps_summed_variable_Igap_post"]
    summed = src[src.index("gaps_summed_variable_Igap_post(RunCtl"):]
    assert "__ldcg(" in summed[:summed.index("\n}\n")] or "__ldcg(" in src[:src.index("gaps_summed_variable_Igap_post(RunCtl")]


def test_multi_gpu_capability_errors(pkg, tmp_path):
    with pytest.raises(pkg.B2GpuError, match="EventMonitor variables"):
        pkg.codegen(model_file("event_variables_small", tmp_path).read_bytes(), rank=0, world_size=2)
    from conftest import golden_procedural_initializers
    with pytest.raises(pkg.B2GpuError, match="procedural per-edge initializers"):
        pkg.codegen(golden_procedural_initializers(), rank=1, world_size=2)


@pytest.mark.parametrize("world", [2, 3])
def test_stdp_rank_plans_replicate_the_inputs(pkg, tmp_path, world):
    """The Poisson inputs, which no synapse targets, run whole on every rank
    (draws keyed by global index), so their spikes need no exchange and feed
    the target-ordered on_pre kernel over the rank's own targets; the target
    neurons are partitioned, and their spikes, which only on_post over the
    rank's own in-edges reads, stay local: no kernel of the tick waits on
    another GPU."""
    data = model_file("stdp_small", tmp_path).read_bytes()
    targets = json.loads(data)["definition"]["populations"][1]["count"]
    for r in range(world):
        src = pkg.codegen(data, rank=r, world_size=world)
        names = [k.split("_", 2)[2] for k in kernels(src)]
        assert names == ["neurons_step_inputs_step", "stdp_pre_targets", "stdp_pre_deliver", "stdp_post_edges"]
        assert "b2_ll_store(((u64*)" not in src  # no peer stores either
        lo, hi = pkg.partition(targets, r, world)
        assert f"__ldg(other + q) - {lo}u" in src[src.index("stdp_pre_targets("):]
        assert f"tj + {lo}u" in src[src.index("stdp_pre_deliver("):]
    # diagnostics: partition and exchange the inputs as well (the bucket
    # scatter reads the exchanged global list); exchange the targets too
    for env, expect in ((dict(B2GPU_REPLICATE="0"), ["neurons_step_inputs_step", "inputs_receive", "stdp_pre_targets",
                                                    "stdp_pre_deliver", "stdp_post_edges"]),
                        (dict(B2GPU_LOCAL_STREAMS="0"), ["neurons_step_inputs_step", "stdp_pre_targets",
                                                         "stdp_pre_deliver", "neurons_receive", "stdp_post_edges"])):
        os.environ.update(env)
        try:
            names = [k.split("_", 2)[2] for k in kernels(pkg.codegen(data, rank=0, world_size=world))]
        finally:
            for key in env:
                del os.environ[key]
        assert names == expect


def _gloo_rank(rank, world, port, q):
    import importlib
    from datetime import timedelta
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    sys.path.insert(0, str(ROOT))
    distributed = importlib.import_module("brian2-atlas_b200.distributed")

    class FakeEngine:  # stands in for a live engine: records what connect() receives
        world_size = world
        got = None

        def ipc_handle(self):
            return bytes([rank]) * 64

        def connect(self, handles):
            FakeEngine.got = handles

    eng = FakeEngine()
    distributed.connect(eng)
    q.put((rank, [h[0] for h in FakeEngine.got], [len(h) for h in FakeEngine.got]))
    dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_handle_exchange_over_gloo():
    """Two gloo ranks trade handles; each receives every rank's, in rank order."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert got == [(0, [0, 1], [64, 64]), (1, [0, 1], [64, 64])]


# ---------------------------------------------------------------- GPU
def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def torchrun(world, args, timeout=600):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(world),
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), str(ROOT / "tests" / "mgpu_worker.py"),
           *map(str, args)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
    errors = [line for line in proc.stdout.splitlines() if line.startswith('{"error"')]
    assert proc.returncode == 0, "\n".join(errors) + "\n" + proc.stdout[-2000:] + proc.stderr[-2000:]
    return [json.loads(line) for line in proc.stdout.splitlines() if line.startswith("{")]


def assert_same_files(a, b, model=None):
    same = (a / "results.bin").read_bytes() == (b / "results.bin").read_bytes()
    assert same, describe_difference(a, b, load_model(model)) if model else "results.bin differs"
    ea, eb = a / "events.bin", b / "events.bin"
    assert ea.exists() == eb.exists()
    if ea.exists():
        assert ea.read_bytes() == eb.read_bytes()
    sa = json.loads((a / "summary.json").read_text())
    sb = json.loads((b / "summary.json").read_text())
    assert sa["synaptic_events"] == sb["synaptic_events"] and sa["spike_count"] == sb["spike_count"]


@pytest.mark.gpu
@pytest.mark.parametrize("world,fuse", [(2, "1"), (2, "0"), (3, "1"), (4, "1"), (8, "1")])
def test_ranks_match_oracle(pkg, oracle, tmp_path, monkeypatch, world, fuse):
    """fuse=0: a separate receive launch before a scatter that reads the ring
    (the default delivers delay-0 constant-addend pathways from the inbox)."""
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    monkeypatch.setenv("B2GPU_FUSE_EXCHANGE", fuse)
    import importlib
    synthetic = importlib.import_module("brian2-atlas_b200.synthetic")
    template = json.loads((MODELS / "cuba_poisson_small.json").read_text())
    c2 = tmp_path / "c2_20k.json"
    c2.write_bytes(synthetic.encode(synthetic.cuba_fixed_indegree(template, n=20000, indegree=1000, ticks=300,
                                                                  seed=9)))
    models = [model_file(n, tmp_path) for n in ["cuba_small", "cuba_poisson_small", "brunel_small",
                                                "synapse_updates_small", "gap_junctions_small"]]
    models += [GOLDEN / "reference-v1" / "model.json", c2]
    args = []
    for k, m in enumerate(models):
        args += [m, tmp_path / f"gpu{k}"]
    lines = torchrun(world, ["run", *args])
    assert len(lines) == len(models)
    for k, m in enumerate(models):
        run_oracle(oracle, m, tmp_path / f"ref{k}")
        assert_same_files(tmp_path / f"gpu{k}", tmp_path / f"ref{k}", m)
        # every rank delivered to its own targets only
        total = json.loads((tmp_path / f"ref{k}" / "summary.json").read_text())["synaptic_events"]
        assert sum(lines[k]["events_per_rank"]) == total


@pytest.mark.gpu
@pytest.mark.parametrize("world,replicate,local", [(2, "1", "1"), (3, "1", "1"), (2, "0", "1"), (2, "1", "0")])
def test_stdp_ranks_match_one_gpu(pkg, tmp_path, monkeypatch, world, replicate, local):
    """STDP with on_pre and on_post on 2-3 ranks against the same network on
    one GPU, byte for byte (the device arithmetic is the same; the trace
    decay's exp rules out the oracle as a byte-exact reference)."""
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    model = model_file("stdp_small", tmp_path)
    with pkg.Engine(model.read_bytes(), device=0) as eng:
        eng.run()
        (tmp_path / "one").mkdir()
        eng.write_results(tmp_path / "one")
    monkeypatch.setenv("B2GPU_REPLICATE", replicate)
    monkeypatch.setenv("B2GPU_LOCAL_STREAMS", local)
    lines = torchrun(world, ["run", model, tmp_path / "many"])
    assert_same_files(tmp_path / "many", tmp_path / "one", model)
    total = json.loads((tmp_path / "one" / "summary.json").read_text())["synaptic_events"]
    assert sum(lines[0]["events_per_rank"]) == total


@pytest.mark.gpu
def test_stalled_rank_expires_the_exchange_wait(tmp_path):
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    lines = torchrun(2, ["stall", MODELS / "cuba_small.json", 50], timeout=300)
    outcome = lines[-1]["outcome"]
    assert "spike exchange with a peer GPU timed out" in outcome
    assert "then: execution failed" in outcome
