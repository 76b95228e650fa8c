"""Generate the committed AtlasIR fixtures from the reference's own frontend.

Run where the reference checkout is available (--reference names its root):

    python tests/golden/make_fixtures.py --reference PATH [--only NAME]

What it writes (all under tests/golden/):
  reference-v1/        the reference's golden b2-runner run, copied verbatim
                       (brian2-rust/tests/fixtures/reference-v1/): model.json,
                       results.bin, events.bin, summary.json
  canonical/           the reference's canonical-hash corpus
                       (brian2-rust/tests/golden/{atlasir-v1,b2ir-v1}/) and its
                       b2ir-gate0-probe-v34..v37 vectors, copied verbatim
  models/*.json[.gz]   AtlasIR documents lowered by the reference's
                       brian2_rust.export.lower_network (export.py:2540) from
                       small versions of the benchmark networks (CUBA, COBAHH,
                       STDP, Brunel, CUBA + PoissonInput on a fixed in-degree
                       topology) and the full-size CUBA 4k config
  brian_numpy/*.npz    spikes and final state of the same networks run by
                       Brian2's numpy runtime (the reference's cross-backend
                       gate, brian2-rust/examples/cuba.py:140-160)

The reference frontend needs two local build steps that this script performs
in tests/golden/_frontend/ (git-ignored): a `pyparsing` alias onto pip's
vendored copy, and a copy of brian2/ with its two Cython extensions built.
"""
from __future__ import annotations

import argparse
import gzip
import json
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
FRONTEND = HERE / "_frontend"


def prepare_frontend(reference: Path) -> None:
    shim = FRONTEND / "shim"
    shim.mkdir(parents=True, exist_ok=True)
    (shim / "pyparsing.py").write_text(
        "import sys\nimport pip._vendor.pyparsing as _p\nsys.modules[__name__] = _p\n")
    src = FRONTEND / "src"
    if not (src / "brian2" / "synapses").exists():
        shutil.copytree(reference / "brian2", src / "brian2")
        for p in (src / "brian2").rglob("*"):
            p.chmod(0o755 if p.is_dir() else 0o644)
    setup = src / "build_ext.py"
    setup.write_text(
        "import numpy\nfrom setuptools import setup, Extension\nfrom Cython.Build import cythonize\n"
        "exts=[Extension('brian2.synapses.cythonspikequeue',['brian2/synapses/cythonspikequeue.pyx'],"
        "include_dirs=[numpy.get_include()]),\n"
        "Extension('brian2.memory.cythondynamicarray',['brian2/memory/cythondynamicarray.pyx'],"
        "include_dirs=[numpy.get_include(),'brian2/devices/cpp_standalone/brianlib'])]\n"
        "setup(name='b2', ext_modules=cythonize(exts, language_level=3), script_args=['build_ext','--inplace'])\n")
    if not list((src / "brian2" / "synapses").glob("cythonspikequeue*.so")):
        subprocess.run([sys.executable, "build_ext.py"], cwd=src, check=True, capture_output=True)
    sys.path[:0] = [str(shim), str(src), str(reference / "brian2-rust" / "python")]


def write_model(model: dict, name: str) -> Path:
    out = HERE / "models"
    out.mkdir(exist_ok=True)
    text = json.dumps(model, sort_keys=True, separators=(",", ":"))
    if len(text) > 1_000_000:
        path = out / f"{name}.json.gz"
        with gzip.open(path, "wt") as f:
            f.write(text)
    else:
        path = out / f"{name}.json"
        path.write_text(text)
    return path


def event_variables(reference: Path) -> dict:
    """cuba_events with recorded variables: `near` events record v and ge
    (after the thresholds, before the reset), start-slot spike events record
    v (after the previous tick's reset) and the per-neuron parameter vt0;
    also runs Brian2's numpy runtime on the same network and saves the
    monitors' records."""
    return cuba_events(reference, seed=8, variables=True)


def cuba_events(reference: Path, n: int = 400, p: float = 0.1, ticks: int = 1000, seed: int = 6,
                variables: bool = False) -> dict:
    """CUBA with a custom event `near` (v > -55 mV) and two EventMonitors: one
    on `near` in the thresholds slot, one on `spike` in the start slot (which,
    in the reference's schedule, records the previous tick's spikes)."""
    import numpy as np
    import brian2 as b
    import brian2_rust  # noqa: F401
    from brian2_rust.export import lower_network
    b.start_scope()
    taum, taue, taui = 20 * b.ms, 5 * b.ms, 10 * b.ms
    Vt, Vr, El = -50 * b.mV, -60 * b.mV, -49 * b.mV
    eqs = """
    dv/dt  = (ge+gi-(v-El))/taum : volt (unless refractory)
    dge/dt = -ge/taue : volt
    dgi/dt = -gi/taui : volt
    """
    clock = b.Clock(dt=0.1 * b.ms, name="clock")
    if variables:
        eqs += "vt0 : volt (constant)\n"
    P = b.NeuronGroup(n, eqs, threshold="v>Vt", reset="v = Vr", refractory=5 * b.ms, method="exact",
                      events={"near": "v > -55*mV"}, name="neurons", clock=clock)
    rng = np.random.default_rng(seed)
    P.v = Vr + rng.random(n) * (Vt - Vr)
    if variables:
        P.vt0 = Vt + rng.random(n) * b.mV
    we, wi = (60 * 0.27 / 10) * b.mV, (-20 * 4.5 / 10) * b.mV
    Ce = b.Synapses(P, P, on_pre="ge += we", name="exc", clock=clock)
    Ci = b.Synapses(P, P, on_pre="gi += wi", name="inh", clock=clock)
    ne = int(n * 0.8)
    mask = rng.random((n, n)) < p
    src, tgt = np.nonzero(mask)
    e = src < ne
    Ce.connect(i=src[e], j=tgt[e])
    Ci.connect(i=src[~e], j=tgt[~e])
    spikes = b.SpikeMonitor(P, name="spikes")
    near = b.EventMonitor(P, "near", name="near_events", variables=["v", "ge"] if variables else None)
    late = b.EventMonitor(P, "spike", name="spike_events_at_start", when="start",
                          variables=["v", "vt0"] if variables else None)
    net = b.Network(P, Ce, Ci, spikes, near, late)
    ns = dict(taum=taum, taue=taue, taui=taui, Vt=Vt, Vr=Vr, El=El, we=we, wi=wi)
    model = lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)
    if variables:
        b.prefs.codegen.target = "numpy"
        net.run(ticks * 0.1 * b.ms, namespace=ns)
        # the first 20,000 `near` records (and their total) keep the fixture small
        k = 20000
        np.savez_compressed(HERE / "brian_numpy" / "event_variables_small.npz", near_count=len(near.i),
                            near_i=np.array(near.i[:k]), near_t=np.array(near.t[:k] / b.second),
                            near_v=np.array(near.v[:k] / b.volt), near_ge=np.array(near.ge[:k] / b.volt),
                            late_i=np.array(late.i[:]), late_t=np.array(late.t / b.second),
                            late_v=np.array(late.v / b.volt), late_vt0=np.array(late.vt0 / b.volt))
    return model


def gap_junctions(reference: Path, n: int = 300, p: float = 0.05, ticks: int = 1000, seed: int = 7) -> dict:
    """Brian's gap-junction network: a `(summed)` synaptic current into the
    target, recomputed from pre/post voltages every tick, plus per-edge
    weights, threshold and reset."""
    import numpy as np
    import brian2 as b
    import brian2_rust  # noqa: F401
    from brian2_rust.export import lower_network
    b.start_scope()
    clock = b.Clock(dt=0.1 * b.ms, name="clock")
    eqs = """
    dv/dt = (v0 - v + Igap) / tau : 1
    Igap : 1
    v0 : 1
    """
    P = b.NeuronGroup(n, eqs, threshold="v > 1", reset="v = 0", method="euler", name="neurons", clock=clock)
    rng = np.random.default_rng(seed)
    P.v0 = np.linspace(0.0, 1.5, n)
    P.v = rng.random(n)
    S = b.Synapses(P, P, """
                   w : 1
                   Igap_post = w * (v_pre - v_post) : 1 (summed)
                   """, name="gaps", clock=clock)
    mask = rng.random((n, n)) < p
    np.fill_diagonal(mask, False)
    src, tgt = np.nonzero(mask)
    S.connect(i=src, j=tgt)
    S.w = 0.02 + 0.02 * rng.random(len(src))
    spikes = b.SpikeMonitor(P, name="spikes")
    trace = b.StateMonitor(P, ["v", "Igap"], record=[0, n // 2, n - 1], name="trace", clock=clock)
    net = b.Network(P, S, spikes, trace)
    ns = dict(tau=10 * b.ms)
    model = lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)
    # Brian2's numpy runtime on the same network: the oracle's independent pin
    b.prefs.codegen.target = "numpy"
    net.run(ticks * 0.1 * b.ms, namespace=ns)
    np.savez_compressed(HERE / "brian_numpy" / "gap_junctions_small.npz", spike_i=np.array(spikes.i[:]),
                        spike_t=np.array(spikes.t / b.second), v=np.array(P.v[:]), Igap=np.array(P.Igap[:]))
    return model


def synapse_updates(reference: Path, n_in: int = 200, n_out: int = 50, p: float = 0.2, ticks: int = 1000,
                    seed: int = 8) -> dict:
    """STDP with clock-driven synaptic traces (a synapse state updater every
    tick) and a synaptic run_regularly, driven by deterministic periodic
    inputs."""
    import numpy as np
    import brian2 as b
    import brian2_rust  # noqa: F401
    from brian2_rust.export import lower_network
    b.start_scope()
    b.defaultclock.dt = 0.1 * b.ms  # one clock for every object (the generator keeps its default schedule)
    rng = np.random.default_rng(seed)
    # deterministic periodic inputs (integrators with seeded rates and
    # phases), so Brian2's numpy runtime sees exactly the same input
    inputs = b.NeuronGroup(n_in, "dv/dt = r : 1\nr : Hz", threshold="v > 1", reset="v = 0", method="euler",
                           name="inputs")
    inputs.r = (20 + 40 * rng.random(n_in)) * b.Hz
    inputs.v = rng.random(n_in)
    G = b.NeuronGroup(n_out, """
                      dv/dt = (ge - v) / (10*ms) : 1
                      dge/dt = -ge / (5*ms) : 1
                      """, threshold="v > 0.3", reset="v = 0", method="exact", name="neurons")
    S = b.Synapses(inputs, G, """
                   w : 1
                   dApre/dt = -Apre / (20*ms) : 1 (clock-driven)
                   dApost/dt = -Apost / (20*ms) : 1 (clock-driven)
                   """, on_pre="""
                   ge += w
                   Apre += 0.01
                   w = clip(w + Apost, 0, 0.2)
                   """, on_post="""
                   Apost -= 0.0105
                   w = clip(w + Apre, 0, 0.2)
                   """, method="exact", name="stdp")
    mask = rng.random((n_in, n_out)) < p
    src, tgt = np.nonzero(mask)
    S.connect(i=src, j=tgt)
    S.w = 0.1 * rng.random(len(src))
    S.run_regularly("w = w * 0.9999", name="decay")
    spikes = b.SpikeMonitor(G, name="spikes")
    net = b.Network(inputs, G, S, spikes)
    model = lower_network(net, ticks * 0.1 * b.ms, rng_seed=seed)
    b.prefs.codegen.target = "numpy"
    net.run(ticks * 0.1 * b.ms)
    np.savez_compressed(HERE / "brian_numpy" / "synapse_updates_small.npz", spike_i=np.array(spikes.i[:]),
                        spike_t=np.array(spikes.t / b.second), v=np.array(G.v[:]), w=np.array(S.w[:]),
                        Apre=np.array(S.Apre[:]), Apost=np.array(S.Apost[:]))
    return model


def timed_input(reference: Path, n: int = 100, ticks: int = 1000, seed: int = 9) -> dict:
    """Neurons driven by a two-dimensional TimedArray input (time x neuron,
    1 ms rows over a 0.1 ms clock) plus a one-dimensional TimedArray gain."""
    import numpy as np
    import brian2 as b
    import brian2_rust  # noqa: F401
    from brian2_rust.export import lower_network
    b.start_scope()
    b.defaultclock.dt = 0.1 * b.ms
    rng = np.random.default_rng(seed)
    stimulus = b.TimedArray(1.5 * rng.random((ticks // 10, n)), dt=1 * b.ms, name="stimulus")
    gain = b.TimedArray(0.5 + rng.random(ticks // 50), dt=5 * b.ms, name="gain")
    G = b.NeuronGroup(n, "dv/dt = (gain(t) * stimulus(t, i) - v) / (10*ms) : 1", threshold="v > 0.8",
                      reset="v = 0", method="euler", name="neurons")
    G.v = rng.random(n) * 0.5
    spikes = b.SpikeMonitor(G, name="spikes")
    net = b.Network(G, spikes)
    ns = dict(stimulus=stimulus, gain=gain)
    model = lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)
    b.prefs.codegen.target = "numpy"
    net.run(ticks * 0.1 * b.ms, namespace=ns)
    np.savez_compressed(HERE / "brian_numpy" / "timed_input_small.npz", spike_i=np.array(spikes.i[:]),
                        spike_t=np.array(spikes.t / b.second), v=np.array(G.v[:]))
    return model


COBAHH_STATES = ["v", "m", "n", "h", "ge", "gi"]


def cobahh_network(n: int, p: float, seed: int, trace: bool = False):
    """The COBAHH network (examples/COBAHH.py at n neurons, connection
    probability p): exponential Euler with exprel/exp rate functions,
    threshold without reset, 3 ms refractory.  trace: a StateMonitor on every
    state of every neuron.  Returns (network, group, spike monitor, state
    monitor or None, namespace)."""
    import numpy as np
    import brian2 as b
    b.start_scope()
    area = 20000 * b.umetre ** 2
    Cm = (1 * b.ufarad * b.cm ** -2) * area
    gl = (5e-5 * b.siemens * b.cm ** -2) * area
    El, EK, ENa = -60 * b.mV, -90 * b.mV, 50 * b.mV
    g_na = (100 * b.msiemens * b.cm ** -2) * area
    g_kd = (30 * b.msiemens * b.cm ** -2) * area
    VT, taue, taui, Ee, Ei = -63 * b.mV, 5 * b.ms, 10 * b.ms, 0 * b.mV, -80 * b.mV
    we, wi = 6 * b.nS, 67 * b.nS
    eqs = b.Equations("""
    dv/dt = (gl*(El-v)+ge*(Ee-v)+gi*(Ei-v)-g_na*(m*m*m)*h*(v-ENa)-g_kd*(n*n*n*n)*(v-EK))/Cm : volt
    dm/dt = alpha_m*(1-m)-beta_m*m : 1
    dn/dt = alpha_n*(1-n)-beta_n*n : 1
    dh/dt = alpha_h*(1-h)-beta_h*h : 1
    dge/dt = -ge*(1./taue) : siemens
    dgi/dt = -gi*(1./taui) : siemens
    alpha_m = 0.32*(mV**-1)*4*mV/exprel((13*mV-v+VT)/(4*mV))/ms : Hz
    beta_m = 0.28*(mV**-1)*5*mV/exprel((v-VT-40*mV)/(5*mV))/ms : Hz
    alpha_h = 0.128*exp((17*mV-v+VT)/(18*mV))/ms : Hz
    beta_h = 4./(1+exp((40*mV-v+VT)/(5*mV)))/ms : Hz
    alpha_n = 0.032*(mV**-1)*5*mV/exprel((15*mV-v+VT)/(5*mV))/ms : Hz
    beta_n = .5*exp((10*mV-v+VT)/(40*mV))/ms : Hz
    """)
    clock = b.Clock(dt=0.1 * b.ms, name="clock")
    P = b.NeuronGroup(n, model=eqs, threshold="v>-20*mV", refractory=3 * b.ms, method="exponential_euler",
                      name="neurons", clock=clock)
    ne = int(n * 0.8)
    Ce = b.Synapses(P[:ne], P, on_pre="ge+=we", name="exc", clock=clock)
    Ci = b.Synapses(P[ne:], P, on_pre="gi+=wi", name="inh", clock=clock)
    rng = np.random.default_rng(seed)
    mask = rng.random((n, n)) < p
    src, tgt = np.nonzero(mask)
    e = src < ne
    Ce.connect(i=src[e], j=tgt[e])
    Ci.connect(i=src[~e] - ne, j=tgt[~e])
    P.v = El + rng.normal(0, 5, n) * b.mV
    P.ge = (rng.normal(0, 1.5, n) + 4) * 10 * b.nS
    P.gi = (rng.normal(0, 12, n) + 20) * 10 * b.nS
    spikes = b.SpikeMonitor(P, name="spikes")
    mon = b.StateMonitor(P, COBAHH_STATES, record=True, name="trace", clock=clock) if trace else None
    net = b.Network(P, Ce, Ci, spikes, *([mon] if mon is not None else []))
    ns = dict(area=area, Cm=Cm, gl=gl, El=El, EK=EK, ENa=ENa, g_na=g_na, g_kd=g_kd, VT=VT, taue=taue,
              taui=taui, Ee=Ee, Ei=Ei, we=we, wi=wi)
    return net, P, spikes, mon, ns


def stdp_network(n_in: int, n_out: int, indegree: int, seed: int, trace: bool = False):
    """The Song-Abbott STDP feedforward network (examples/synapses/STDP.py
    scaled): Poisson inputs at 15 Hz, conductance LIF targets (Euler),
    plastic weights with event-driven pre/post traces.  trace: a
    StateMonitor on v and ge of every target.  Returns (network, namespace)."""
    import numpy as np
    import brian2 as b
    b.start_scope()
    taum, taupre, taupost = 10 * b.ms, 20 * b.ms, 20 * b.ms
    Ee, vt, vr, El, taue = 0 * b.mV, -54 * b.mV, -60 * b.mV, -74 * b.mV, 5 * b.ms
    gmax, dApre = 0.01, 0.01
    dApost = -dApre * taupre / taupost * 1.05
    dApost *= gmax
    dApre *= gmax
    clock = b.Clock(dt=0.1 * b.ms, name="clock")
    inputs = b.PoissonGroup(n_in, rates=15 * b.Hz, name="inputs", clock=clock)
    neurons = b.NeuronGroup(n_out, "dv/dt = (ge * (Ee-v) + El - v) / taum : volt\ndge/dt = -ge / taue : 1",
                            threshold="v>vt", reset="v = vr", method="euler", name="neurons", clock=clock)
    neurons.v = vr
    S = b.Synapses(inputs, neurons,
                   """w : 1
                      dApre/dt = -Apre / taupre : 1 (event-driven)
                      dApost/dt = -Apost / taupost : 1 (event-driven)""",
                   on_pre="ge += w\nApre += dApre\nw = clip(w + Apost, 0, gmax)",
                   on_post="Apost += dApost\nw = clip(w + Apre, 0, gmax)", name="stdp", clock=clock)
    rng = np.random.default_rng(seed)
    src = np.concatenate([rng.choice(n_in, indegree, replace=False) for _ in range(n_out)])
    tgt = np.repeat(np.arange(n_out), indegree)
    S.connect(i=src, j=tgt)
    S.w = rng.random(len(src)) * gmax
    spikes = b.SpikeMonitor(neurons, name="spikes")
    extra = [b.StateMonitor(neurons, ["v", "ge"], record=True, name="trace", clock=clock)] if trace else []
    net = b.Network(inputs, neurons, S, spikes, *extra)
    ns = dict(taum=taum, taupre=taupre, taupost=taupost, Ee=Ee, vt=vt, vr=vr, El=El, taue=taue, gmax=gmax,
              dApre=dApre, dApost=dApost)
    return net, ns


def cobahh_trace(reference: Path, n: int = 400, p: float = 0.1, ticks: int = 100, seed: int = 2) -> dict:
    """cobahh_small's network (same seed) over its first 100 ticks with every
    state of every neuron recorded every tick."""
    import brian2 as b
    import brian2_rust  # noqa: F401
    from brian2_rust.export import lower_network
    net, _, _, _, ns = cobahh_network(n, p, seed, trace=True)
    return lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)


def stdp_trace(reference: Path, n_in: int = 1000, n_out: int = 20, indegree: int = 1000, ticks: int = 100,
               seed: int = 5) -> dict:
    """stdp_small's network (same seed) over its first 100 ticks with v and ge
    of every target recorded every tick."""
    import brian2 as b
    import brian2_rust  # noqa: F401
    from brian2_rust.export import lower_network
    net, ns = stdp_network(n_in, n_out, indegree, seed, trace=True)
    return lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)


def random_draws(reference: Path, n: int = 200, ticks: int = 300, seed: int = 12) -> dict:
    """Per-tick random draws on the device: an Euler-Maruyama membrane with
    white noise (Brian's xi, lowered to randn()) and a run_regularly Poisson
    draw whose rates span both of the reference's branches (Knuth's product
    below 10, PTRS at 10 and above); both recorded every tick."""
    import numpy as np
    import brian2 as b
    import brian2_rust  # noqa: F401
    from brian2_rust.export import lower_network
    b.start_scope()
    clock = b.Clock(dt=0.1 * b.ms, name="clock")
    G = b.NeuronGroup(n, "dv/dt = (mu - v) / tau + sigma * xi * tau**-0.5 : 1", threshold="v > 1", reset="v = 0",
                      method="euler", name="noisy", clock=clock)
    G.v = np.linspace(0.0, 0.9, n)
    D = b.NeuronGroup(n, "lam : 1\nk : 1", name="draws", clock=clock)
    D.lam = np.linspace(0.5, 60.0, n)
    D.run_regularly("k = poisson(lam)", clock=clock, name="draw")
    spikes = b.SpikeMonitor(G, name="spikes")
    tv = b.StateMonitor(G, "v", record=True, name="trace_v", clock=clock)
    tk = b.StateMonitor(D, "k", record=True, name="trace_k", clock=clock)
    net = b.Network(G, D, spikes, tv, tk)
    ns = dict(mu=0.8, sigma=0.5, tau=10 * b.ms)
    return lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--only", default=None, help="write just this model (e.g. cobahh_trace_small)")
    args = ap.parse_args()
    if args.only:
        prepare_frontend(Path(args.reference))
        make = {"cuba_events_small": cuba_events, "event_variables_small": event_variables,
                "gap_junctions_small": gap_junctions, "cobahh_trace_small": cobahh_trace,
                "stdp_trace_small": stdp_trace, "random_draws_small": random_draws,
                "synapse_updates_small": synapse_updates, "timed_input_small": timed_input}[args.only]
        write_model(make(Path(args.reference)), args.only)
        print("wrote", args.only)
        return
    reference = Path(args.reference)
    golden = reference / "brian2-rust" / "tests" / "fixtures" / "reference-v1"
    dst = HERE / "reference-v1"
    dst.mkdir(exist_ok=True)
    for name in ("model.json", "reference/results.bin", "reference/events.bin", "reference/summary.json"):
        shutil.copyfile(golden / name, dst / Path(name).name)
    # canonical-hash corpus and the probe predecessors, renamed by schema
    corpus = reference / "brian2-rust" / "tests" / "golden"
    canon = HERE / "canonical"
    canon.mkdir(exist_ok=True)
    for schema in ("atlasir", "b2ir"):
        for name in ("minimal-v1.json", "hashes.json"):
            shutil.copyfile(corpus / f"{schema}-v1" / name, canon / f"{schema}-{name}")
    for version in (34, 35, 36, 37):
        shutil.copyfile(corpus / "b2ir-v1" / f"minimal-v{version}.json", canon / f"b2ir-minimal-v{version}.json")

    prepare_frontend(reference)
    import numpy as np
    import brian2 as b
    import brian2_rust  # noqa: F401  (registers the atlas device)
    from brian2_rust.export import lower_network

    b.prefs.codegen.target = "numpy"
    (HERE / "brian_numpy").mkdir(exist_ok=True)

    # ---------------------------------------------------------------- CUBA
    def cuba(n, p, ticks, seed, numpy_run):
        b.start_scope()
        taum, taue, taui = 20 * b.ms, 5 * b.ms, 10 * b.ms
        Vt, Vr, El = -50 * b.mV, -60 * b.mV, -49 * b.mV
        eqs = """
        dv/dt  = (ge+gi-(v-El))/taum : volt (unless refractory)
        dge/dt = -ge/taue : volt
        dgi/dt = -gi/taui : volt
        """
        clock = b.Clock(dt=0.1 * b.ms, name="clock")
        P = b.NeuronGroup(n, eqs, threshold="v>Vt", reset="v = Vr", refractory=5 * b.ms, method="exact",
                          name="neurons", clock=clock)
        rng = np.random.default_rng(seed)
        P.v = Vr + rng.random(n) * (Vt - Vr)
        we, wi = (60 * 0.27 / 10) * b.mV, (-20 * 4.5 / 10) * b.mV
        Ce = b.Synapses(P, P, on_pre="ge += we", name="exc", clock=clock)
        Ci = b.Synapses(P, P, on_pre="gi += wi", name="inh", clock=clock)
        ne = int(n * 0.8)
        mask = rng.random((n, n)) < p
        src, tgt = np.nonzero(mask)
        e = src < ne
        Ce.connect(i=src[e], j=tgt[e])
        Ci.connect(i=src[~e], j=tgt[~e])
        spikes = b.SpikeMonitor(P, name="spikes")
        trace = b.StateMonitor(P, ["v", "ge"], record=[0, 1, n // 2], name="trace", clock=clock)
        net = b.Network(P, Ce, Ci, spikes, trace)
        ns = dict(taum=taum, taue=taue, taui=taui, Vt=Vt, Vr=Vr, El=El, we=we, wi=wi)
        model = lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)
        if numpy_run:
            net.run(ticks * 0.1 * b.ms, namespace=ns)
            return model, dict(spike_i=np.array(spikes.i[:]), spike_t=np.array(spikes.t / b.second),
                               v=np.array(P.v[:] / b.volt), ge=np.array(P.ge[:] / b.volt),
                               trace_v=np.array(trace.v / b.volt))
        return model, None

    model, ref = cuba(400, 0.1, 1000, 1, True)
    write_model(model, "cuba_small")
    np.savez_compressed(HERE / "brian_numpy" / "cuba_small.npz", **ref)
    model, _ = cuba(4000, 0.02, 10000, 1, False)
    write_model(model, "cuba_4k")

    # ---------------------------------------------------------------- COBAHH
    def cobahh(n, p, ticks, seed, numpy_run):
        net, P, spikes, _, ns = cobahh_network(n, p, seed)
        model = lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)
        if numpy_run:
            net.run(ticks * 0.1 * b.ms, namespace=ns)
            return model, dict(spike_i=np.array(spikes.i[:]), spike_t=np.array(spikes.t / b.second),
                               v=np.array(P.v[:] / b.volt))
        return model, None

    model, ref = cobahh(400, 0.1, 1000, 2, True)
    write_model(model, "cobahh_small")
    np.savez_compressed(HERE / "brian_numpy" / "cobahh_small.npz", **ref)
    model, _ = cobahh(4000, 0.02, 10000, 2, False)
    write_model(model, "cobahh_4k")

    # ---------------------------------------------------------------- STDP
    def stdp(n_in, n_out, indegree, ticks, seed):
        net, ns = stdp_network(n_in, n_out, indegree, seed)
        return lower_network(net, ticks * 0.1 * b.ms, namespace=ns, rng_seed=seed)

    write_model(stdp(1000, 20, 1000, 2000, 5), "stdp_small")

    # ---------------------------------------------------------------- Brunel (f32 v, delay 1.5 ms)
    def brunel(n, indegree, ticks, seed):
        b.start_scope()
        b.set_device("atlas", build_on_run=False)
        dev = b.get_device()
        tau, theta, reset, J = 20 * b.ms, 20 * b.mV, 10 * b.mV, 0.1 * b.mV
        n_e = int(n * 0.8)
        c_e = int(indegree * 0.8)
        c_i = indegree - c_e
        nu_thr = theta / (J * c_e * tau)
        clock = b.Clock(dt=0.1 * b.ms, name="clock")
        P = b.NeuronGroup(n, "dv/dt = -v/tau : volt (unless refractory)", threshold="v > theta", reset="v = reset",
                          refractory=2 * b.ms, name="neurons", dtype={"v": np.float32}, clock=clock)
        rng = np.random.default_rng(seed)
        P.v = rng.random(n) * theta
        syns = []
        for name, src, k, w, s in (("excitatory", P[:n_e], c_e, J, seed + 1),
                                   ("inhibitory", P[n_e:], c_i, -5 * J, seed + 2)):
            S = b.Synapses(src, P, "weight : volt (constant, shared)", on_pre="v_post += weight",
                           delay=1.5 * b.ms, name=f"{name}_synapses", clock=clock)
            dev.connect_fixed_indegree(S, k, seed=s)
            S.weight = w
            syns.append(S)
        ext = b.PoissonInput(P, "v", N=c_e, rate=2 * nu_thr, weight=J)
        spikes = b.SpikeMonitor(P, name="spikes")
        net = b.Network(P, *syns, ext, spikes)
        model = lower_network(net, ticks * 0.1 * b.ms, namespace=dict(tau=tau, theta=theta, reset=reset),
                              rng_seed=seed)
        b.set_device("runtime")
        return model

    write_model(brunel(2000, 200, 1000, 4), "brunel_small")

    # ---------------------------------------------------------------- CUBA on fixed in-degree + PoissonInput (C2 shape)
    def cuba_poisson(n, indegree, ticks, seed):
        b.start_scope()
        b.set_device("atlas", build_on_run=False)
        dev = b.get_device()
        taum, taue, taui = 20 * b.ms, 5 * b.ms, 10 * b.ms
        Vt, Vr, El = -50 * b.mV, -60 * b.mV, -49 * b.mV
        eqs = """
        dv/dt  = (ge+gi-(v-El))/taum : volt (unless refractory)
        dge/dt = -ge/taue : volt
        dgi/dt = -gi/taui : volt
        """
        clock = b.Clock(dt=0.1 * b.ms, name="clock")
        P = b.NeuronGroup(n, eqs, threshold="v>Vt", reset="v = Vr", refractory=5 * b.ms, method="exact",
                          name="neurons", clock=clock)
        rng = np.random.default_rng(seed)
        P.v = Vr + rng.random(n) * (Vt - Vr)
        we, wi = (60 * 0.27 / 10) * b.mV, (-20 * 4.5 / 10) * b.mV
        ne = int(n * 0.8)
        Ce = b.Synapses(P[:ne], P, on_pre="ge += we", name="exc", clock=clock)
        Ci = b.Synapses(P[ne:], P, on_pre="gi += wi", name="inh", clock=clock)
        dev.connect_fixed_indegree(Ce, int(indegree * 0.8), seed=seed + 1)
        dev.connect_fixed_indegree(Ci, indegree - int(indegree * 0.8), seed=seed + 2)
        ext = b.PoissonInput(P, "ge", N=100, rate=10 * b.Hz, weight=we)
        spikes = b.SpikeMonitor(P, name="spikes")
        net = b.Network(P, Ce, Ci, ext, spikes)
        model = lower_network(net, ticks * 0.1 * b.ms,
                              namespace=dict(taum=taum, taue=taue, taui=taui, Vt=Vt, Vr=Vr, El=El, we=we, wi=wi),
                              rng_seed=seed)
        b.set_device("runtime")
        return model

    write_model(cuba_poisson(1000, 100, 1000, 3), "cuba_poisson_small")
    print("fixtures written under", HERE)


if __name__ == "__main__":
    main()
