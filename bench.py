"""Benchmark of the B200 batched rigid-body stepper.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2_chain32] [--precision f32|f64] [--horizon H]

One bench "step" is one rollout of the workload: every world of the config
(BASELINE.json configs[1] by default: the 32-link chain, 65536 worlds)
advanced `horizon` physics steps (the config's 1000) under per-step controls
N(0, sigma), starting from the seeded initial state. Metric: world-steps/s
of the whole job, device-timed with CUDA events on the launching stream,
max over ranks. Multi-GPU runs are weak-scaled: each rank owns its own
contiguous block of worlds (no per-step communication); one NCCL all-reduce
of the per-world objective closes every rollout.

`value` has the inputs (initial state, control schedule) resident in HBM;
where the schedule is smaller than L2, a 256 MB buffer is written between
rollouts and value counts the rollouts' own device time. `e2e` is the same
metric through the C ABI with host buffers: the initial state and every
step's controls copied in from pinned host memory and the final state read
back, inside the timed region. `roofline` is the fused kernel against the
measured FP32/FP64 FMA pipe, counting the flops the running kernel executes
on this rollout's states. `cpu_baseline` is the reference's own kernels
compiled as host C++ (oracle/_ref) on this host's cores, on a fixed sample
both arms time alike; f64 runs add the f64 oracle (`cpu_baseline_f64_oracle`).
`reference_gpu` is the reference's own CUDA kernels on this GPU in their
stock launch sequence. The default run also measures C1 (f64, its 4096
worlds split over the GPUs), C3 and C4 (f32) under `per_config`.
`--impl reference` times only the reference CPU path.

`--config c3_quadruped_impulse` runs C3's worlds with impulse-mode contact
(16 staged Coulomb sweeps per step) in place of the penalty law, 100 steps
per rollout by default; `--config c3_quadruped_terrain` runs them with the
penalty law over a seeded 64 x 64 heightfield.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

# DRAM traffic of one rollout_kernel launch measured by ncu on a smaller
# case of the same workload (dram__bytes_read.sum + dram__bytes_write.sum of
# one launch at 65536 worlds).
# A launch reads/writes each world's state once and streams one control row
# per step, so it is scaled to the bench's launch as
#   state bytes (q, v in and out) + per-world-step bytes x worlds x steps,
# with the per-world-step part taken from the capture after removing its
# state bytes.
NCU_DRAM_CAPTURES: dict = {
    # slice mode (PHYZB_SLICES=1: 3 runs of 10 steps), as the bench's launch
    # runs: the state a run writes is read back by the next run from L2, so
    # DRAM sees it about once, as in tile mode
    ("c2_chain32", "f32"): {"nworld": 65536, "horizon": 30, "bytes": 270.800640e6 + 18.190592e6},
    # the model-specialized kernel
    ("c3_quadruped", "f32"): {"nworld": 65536, "horizon": 20, "bytes": 80.932608e6 + 5.339904e6},
    # the generic impulse variant: its DRAM traffic is the state and the
    # control stream, as the specialized kernel's is
    ("c3_quadruped_impulse", "f32"): {"nworld": 65536, "horizon": 10, "bytes": 53.736192e6 + 1.875200e6},
}

# Workloads beyond BASELINE.json's configs: a config's model, worlds and
# initial state with impulse-mode contact (enable_contact_impulse, 16 sweeps
# per step) in place of the penalty law, over a shorter default horizon
# (every impulse step runs 17 backward sweeps); or with the penalty law over
# a seeded heightfield (enable_contact_terrain) instead of the flat ground.
IMPULSE_WORKLOADS = {"c3_quadruped_impulse": ("c3_quadruped", 100)}
TERRAIN_WORKLOADS = {"c3_quadruped_terrain": "c3_quadruped"}


def base_config(name):
    """(config name the model / state / contact come from, impulse?, default horizon or 0)."""
    if name in IMPULSE_WORKLOADS:
        base, horizon = IMPULSE_WORKLOADS[name]
        return base, True, horizon
    if name in TERRAIN_WORKLOADS:
        return TERRAIN_WORKLOADS[name], False, 0
    return name, False, 0


def bench_heightfield(name):
    """The seeded terrain of a heightfield workload (None for the others):
    64 x 64 nodes 0.25 m apart centred on the origin, heights N(0, 0.05) m."""
    if name not in TERRAIN_WORKLOADS:
        return None
    from phyz_b200 import Heightfield

    hf = Heightfield.new((-8.0, -8.0, 0.0), 0.25, 64, 64)
    hf.heights[:] = (0.05 * np.random.default_rng(0x7E55).standard_normal(64 * 64)).astype(np.float32)
    return hf


def ncu_traffic(config, prec, nv, esz, nworld, horizon):
    cap = NCU_DRAM_CAPTURES.get((config, prec))
    if cap is None:
        return None
    state = lambda n: 4 * nv * esz * n  # q, v read and written once per launch
    per_ws = (cap["bytes"] - state(cap["nworld"])) / (cap["nworld"] * cap["horizon"])
    return state(nworld) + per_ws * nworld * horizon


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=7)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2_chain32")
    ap.add_argument("--precision", default="f32", choices=["f32", "f64"])
    ap.add_argument("--horizon", type=int, default=0, help="physics steps per bench step (0: the config's)")
    ap.add_argument("--nworld", type=int, default=0, help="worlds per GPU (0: the config's)")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--e2e-horizon", type=int, default=0, help="steps of the e2e rollout (0: the full horizon)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lanes", type=int, default=0, choices=[0, 2, 4, 8],
                    help="threads per world for branching trees (0: one thread per world)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own CUDA kernels on this GPU")
    ap.add_argument("--per-config", type=int, default=1,
                    help="with the default workload, also measure C1 f64, C3 f32 and C4 f32 (0: off)")
    ap.add_argument("--specialize", default="auto", choices=["auto", "0", "1"],
                    help="rollout kernel: 1 compiled at run time for the model (tables literal, loops "
                         "unrolled), 0 the generic variant, auto 1 unless the model's longest chain "
                         "exceeds 16 bodies")
    return ap.parse_args()


# ── clocks during the timed region ─────────────────────────────────────────
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ── distributed plumbing ──────────────────────────────────────────────────
def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ── shared by both arms ───────────────────────────────────────────────────
L2_BYTES = 126 * 1024 * 1024  # B200 L2


def held_controls(workload):
    """Configs with zero control (C1) step under held zero controls: no
    per-step control input exists to stream."""
    from phyz_b200 import configs

    return configs.CONFIGS[base_config(workload)[0]].ctrl_sigma == 0.0


def schedule_bytes(model, nworld, horizon, prec):
    return horizon * model.nv * nworld * (4 if prec == "f32" else 8)


def l2_rule(workload, model, nworld, horizon, prec):
    """(flush between rollouts?, the note for `config.l2`)."""
    if held_controls(workload):
        b = 4 * model.nv * nworld * (4 if prec == "f32" else 8)
        return True, (f"zero controls held (no per-step input); inputs smaller than L2 ({b / 1e3:.0f} kB of "
                      "state): a 256 MB buffer is written between timed rollouts (L2 flushed) and value counts "
                      "the rollouts' own device time")
    b = schedule_bytes(model, nworld, horizon, prec)
    if b > L2_BYTES:
        return False, (f"inputs larger than L2: the per-step control schedule ({b / 1e9:.2f} GB) streams from HBM "
                       "every rollout")
    return True, (f"inputs smaller than L2 ({b / 1e6:.1f} MB schedule): a 256 MB buffer is written between timed "
                  "rollouts (L2 flushed) and value counts the rollouts' own device time")


def bench_config(workload, model, nworld, horizon, prec, n_gpus, strong=False):
    """The `config` block, identical in both arms for the same arguments."""
    cfg_name, impulse, _ = base_config(workload)
    from phyz_b200 import configs

    cfg = configs.CONFIGS[cfg_name]
    contact = None
    if cfg.contact:
        contact = ("impulse, 16 sweeps per step" if impulse else
                   ("penalty, 64 x 64 heightfield" if workload in TERRAIN_WORKLOADS else "penalty"))
    out = {"workload": workload, "nbodies": model.nbodies, "nv": model.nv, "horizon": horizon, "precision": prec,
           "contact": contact, "l2": l2_rule(workload, model, nworld, horizon, prec)[1]}
    if strong:
        out["nworld_total"] = nworld
        out["parallelism"] = f"{nworld} worlds split over {n_gpus} GPU(s) (strong scaling)"
    else:
        out["nworld_per_gpu"] = nworld
        out["parallelism"] = f"{nworld} worlds per GPU on each of {n_gpus} GPU(s) (weak scaling)"
    return out


# ── the reference's CPU path (oracle/_ref) and the f64 oracle ─────────────
CPU_CHUNK = 64  # steps per timed repetition


def _cpu_sample(workload, model, nworld, impulse):
    from phyz_b200 import configs

    cfg_name = base_config(workload)[0]
    cfg = configs.CONFIGS[cfg_name]
    n = min(nworld, 2048 if impulse else 16384)  # an impulse step costs ~17 plain ones
    q, v = configs.initial_state(cfg_name, model, np.arange(n))
    rng = np.random.default_rng(configs.CTRL_SEED)
    sched = (rng.standard_normal((CPU_CHUNK, n, model.nv)) * cfg.ctrl_sigma * configs.actuated(model)).astype(
        np.float32)
    return cfg, n, q, v, sched


def reference_cpu(workload, model, nworld, horizon, reps, warm=1):
    """The reference's own kernels compiled as host C++ on every host core,
    timed on a fixed sample of the workload: min(nworld, 16384) of its worlds
    (2048 in impulse mode) from their seeded initial states, 64 steps of
    seeded controls per repetition, `warm` untimed then `reps` timed
    repetitions, each from the same initial state. Both bench arms call this
    with the same arguments. Returns (median world-steps/s, threads, sample
    text, per-repetition values)."""
    from oracle.oracle import RefHost, cpu_threads

    _, impulse, _ = base_config(workload)
    cfg, n, q0, v0, sched = _cpu_sample(workload, model, nworld, impulse)
    ref = RefHost()
    ref.set_heightfield(bench_heightfield(workload))
    threads = cpu_threads()
    contact = None
    if cfg.contact:
        g, k, d, mu = cfg.contact
        contact = (g, mu, k, d)

    def once():
        t0 = time.perf_counter()
        if impulse:
            ref.rollout_impulse(model, q0, v0, sched, CPU_CHUNK, schedule=True, contact=(contact[0], contact[1]),
                                nthreads=threads)
        else:
            ref.rollout(model, q0, v0, sched, CPU_CHUNK, schedule=True, contact=contact, nthreads=threads)
        return n * CPU_CHUNK / (time.perf_counter() - t0)

    for _ in range(warm):
        once()
    vals = [once() for _ in range(reps)]
    ref.set_heightfield(None)
    mode = {True: ", impulse contact (16 sweeps)"}.get(impulse, "")
    if workload in TERRAIN_WORKLOADS:
        mode = ", heightfield terrain"
    sample = (f"{n} of {nworld} worlds x {CPU_CHUNK} of {horizon} steps, f32{mode}, {threads} threads, median of "
              f"{reps} repetitions after {warm} untimed")
    return statistics.median(vals), threads, sample, vals


def oracle_cpu(workload, model, nworld, horizon, reps):
    """The f64 oracle (this repository's C++ restatement of phyz-rigid's ABA
    and integrator with the reference GPU's penalty law) on every host core,
    on min(nworld, 2048) worlds x 64 steps per repetition, median of `reps`.
    None for impulse and terrain workloads."""
    from oracle.oracle import Oracle, cpu_threads

    _, impulse, _ = base_config(workload)
    if impulse or workload in TERRAIN_WORKLOADS:
        return None
    cfg, n, q0, v0, sched = _cpu_sample(workload, model, min(nworld, 2048), False)
    o = Oracle()
    threads = cpu_threads()
    contact = None
    if cfg.contact:
        g, k, d, mu = cfg.contact
        contact = (g, mu, k, d)
    sched = sched.astype(np.float64)

    def once():
        t0 = time.perf_counter()
        o.rollout(model, q0, v0, sched, CPU_CHUNK, schedule=True, contact=contact, nthreads=threads)
        return n * CPU_CHUNK / (time.perf_counter() - t0)

    once()
    vals = [once() for _ in range(reps)]
    return {"value": statistics.median(vals), "unit": "world-steps/s", "cores": threads, "kind": "port",
            "sample": f"{n} of {nworld} worlds x {CPU_CHUNK} of {horizon} steps, f64 oracle (phyz-rigid restated), "
                      f"{threads} threads, median of {reps} repetitions"}


def reference_gpu(workload, model, nworld, horizon):
    """The reference's own CUDA kernels (crates/phyz-gpu/cuda/phyz_kernels.cu
    built for sm_100a by oracle/Makefile) on this GPU, in its stock sequence
    (contact -> aba -> integrate per step, 64-thread blocks, the rollout
    replayed as one captured CUDA graph), f32, the same worlds and horizon,
    controls held at the first step's row. Best of 3 replays."""
    from oracle.oracle import RefCuda, RefHost
    from phyz_b200 import configs

    cfg_name, impulse, _ = base_config(workload)
    if impulse or workload in TERRAIN_WORKLOADS:
        return None
    cfg = configs.CONFIGS[cfg_name]
    q0, v0 = configs.initial_state(cfg_name, model, np.arange(nworld))
    rng = np.random.default_rng(configs.CTRL_SEED)
    ctrl = (rng.standard_normal((nworld, model.nv)) * cfg.ctrl_sigma * configs.actuated(model)).astype(np.float32)
    contact = None
    if cfg.contact:
        g, k, d, mu = cfg.contact
        contact = (g, mu, k, d)
    rc = RefCuda(RefHost())
    _, _, _, _, ms = rc.rollout(model, q0, v0, ctrl, horizon, contact=contact, reps=3)
    return {"value": nworld * horizon / (ms * 1e-3), "unit": "world-steps/s", "ms_per_rollout": ms,
            "path": "phyz_kernels.cu contact -> aba -> integrate, 64-thread blocks, one CUDA graph per rollout, "
                    "f32, controls held"}


def run_reference_impl(args, world, rank):
    from phyz_b200 import configs

    if rank != 0:
        return
    cfg_name, _, h_default = base_config(args.config)
    cfg = configs.CONFIGS[cfg_name]
    model = cfg.builder()
    nworld = args.nworld or cfg.nworld
    horizon = args.horizon or h_default or cfg.steps
    value, threads, sample, _ = reference_cpu(args.config, model, nworld, horizon, reps=max(args.steps, 1),
                                              warm=max(args.warmup, 1))
    line = {
        "impl": "reference", "metric": "world-steps/sec", "value": value, "unit": "world-steps/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": bench_config(args.config, model, nworld, horizon, args.precision, args.gpus),
        "cpu_baseline": {"value": value, "unit": "world-steps/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": "world-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own kernels (phyz_kernels.cu) compiled as host C++, f32; the reference has no "
                "f64 or multithreaded batch stepper of its own",
    }
    print(json.dumps(line), flush=True)


# ── our arm ────────────────────────────────────────────────────────────────
# Configs measured beside the headline in the default run (BASELINE.json
# configs[0], [2], [3]): (workload, precision, worlds, strong scaling?).
# C1's 4096 worlds are split over the GPUs (the north star's target is that
# batch on 8 GPUs); C3 and C4 keep their worlds per GPU.
PER_CONFIG = [("c1_double_pendulum", "f64", 4096, True), ("c3_quadruped", "f32", 262144, False),
              ("c4_humanoid", "f32", 131072, False)]


class Ctx:
    """Per-process state shared by the measured workloads."""

    def __init__(self, args, world, rank, local):
        import torch

        from phyz_b200.parallel import Comm, share_bytes

        self.args, self.world, self.rank, self.local = args, world, rank, local
        self.stream = torch.cuda.Stream()
        self.comm = Comm(rank, world, local, timeout=120.0,
                         id_channel=(lambda p, r: share_bytes(p, r)) if world > 1 else (lambda p, r: p))
        self.flush_buf = None

    def flush_l2(self):
        import torch

        if self.flush_buf is None:
            self.flush_buf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MB
        with torch.cuda.stream(self.stream):
            self.flush_buf.zero_()


def measure(ctx, workload, prec, nworld_arg, horizon_arg, steps, warmup, strong=False, e2e=False, cpu=False,
            ref_gpu=False, specialize="auto", lanes=0):
    """One workload on this rank: `steps` timed rollouts after `warmup`.
    Returns the entry (rank 0's view; times are max over ranks)."""
    import torch

    from phyz_b200 import BatchSim, configs
    from phyz_b200 import _lib as L
    from phyz_b200.parallel import shard_bounds, weak_block

    args, world, rank, local, stream = ctx.args, ctx.world, ctx.rank, ctx.local, ctx.stream
    cfg_name, impulse, h_default = base_config(workload)
    cfg = configs.CONFIGS[cfg_name]
    model = cfg.builder()
    total = nworld_arg or cfg.nworld
    horizon = horizon_arg or h_default or cfg.steps
    if strong:
        lo, hi = shard_bounds(total, rank, world)
        nworld, offset = hi - lo, lo
    else:
        nworld = total
        offset, _ = weak_block(nworld, rank)
    tdt = torch.float32 if prec == "f32" else torch.float64
    esz = 4 if prec == "f32" else 8
    nv = model.nv
    flush, l2_note = l2_rule(workload, model, nworld, horizon, prec)
    held = held_controls(workload)

    sim = BatchSim(model, nworld, device=local, precision=prec)
    sim.specialize = {"auto": "auto", "0": False, "1": True}[specialize]
    hf = bench_heightfield(workload)
    if cfg.contact and impulse:
        sim.enable_contact_impulse(cfg.contact[0], cfg.contact[3])
    elif cfg.contact and hf is not None:
        from phyz_b200 import BodyContactGains

        g, k, d, mu = cfg.contact
        sim.enable_contact_terrain(g, mu, [BodyContactGains(k, d)] * model.nbodies, heightfield=hf)
    elif cfg.contact:
        sim.enable_ground_contact(*cfg.contact)
    if lanes:
        sim.world_lanes = lanes
    sim.set_stream(stream.cuda_stream)

    # inputs resident in HBM: initial state (SoA) and the per-step controls
    q0, v0 = configs.initial_state(cfg_name, model, np.arange(offset, offset + nworld))
    sim.load_states(q0, v0)
    q0_dev = torch.tensor(q0.T.copy(), dtype=tdt, device="cuda")
    v0_dev = torch.tensor(v0.T.copy(), dtype=tdt, device="cuda")
    gen = torch.Generator(device="cuda")
    gen.manual_seed(configs.CTRL_SEED + rank)
    mask = torch.tensor(configs.actuated(model), dtype=tdt, device="cuda").view(1, nv, 1)
    c0_dev = torch.zeros(nv, nworld, dtype=tdt, device="cuda")
    with torch.cuda.stream(stream):
        sched = torch.randn(1 if held else horizon, nv, nworld, generator=gen, dtype=tdt, device="cuda") * (
            cfg.ctrl_sigma * mask)
    torch.cuda.synchronize()  # inputs written on torch's streams before the simulator's stream reads them
    objective = [0.0]
    obj_dev = torch.zeros(max(steps, 1), dtype=tdt, device="cuda")

    def rollout(ev=None, k=None):
        if ev is not None:
            ev[0].record(stream)
        # same start, same work each rollout
        sim.load_states_device(q0_dev.data_ptr(), v0_dev.data_ptr(), c0_dev.data_ptr() if held else None)
        if ev is not None:
            ev[1].record(stream)
        if held:
            sim.step_many(horizon)
        else:
            sim.step_device_controls(sched.data_ptr(), nv * nworld, horizon)
        if ev is not None:
            ev[2].record(stream)
        if k is None:
            objective[0] = ctx.comm.reduce_objective(sim, 0)
        else:
            # enqueued into a device scalar; one bounded wait after the loop
            ctx.comm.reduce_objective_device(sim, obj_dev[k].data_ptr(), 0)
        if ev is not None:
            ev[3].record(stream)

    for _ in range(warmup):
        rollout()
        if flush:
            ctx.flush_l2()
    stream.synchronize()
    sim.sync()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for k in range(steps):
            rollout(ev[k], k)
            if flush:
                ctx.flush_l2()
        t1.record(stream)
        ctx.comm.sync(sim)
        stream.synchronize()
    objective[0] = float(obj_dev[steps - 1].item())
    barrier(world)
    torch.cuda.synchronize()
    sim.sync()  # raises if any world went non-finite
    region_ms = allreduce_max(t0.elapsed_time(t1), world)
    rollout_ms = allreduce_max(sum(e[0].elapsed_time(e[3]) for e in ev), world)
    per_launch = sorted(e[1].elapsed_time(e[2]) for e in ev)
    kernel_ms = allreduce_max(sum(per_launch) / steps, world)
    kernel_ms_min = allreduce_max(per_launch[0], world)
    kernel_ms_median = allreduce_max(statistics.median(per_launch), world)
    world_steps = (total if strong else nworld * world) * horizon
    ms = rollout_ms if flush else region_ms
    value = world_steps * steps / (ms * 1e-3)

    # roofline of the fused kernel against the measured FMA pipe of this
    # precision: the flops the running kernel executes per world-step,
    # counted on this rank's first 16 worlds over the whole schedule (the
    # contact force law included where a body touches; the specialized
    # kernel without its products with zero table constants), beside the
    # generic formulation's steady-state count
    flops_gen, trans_ws = sim.flops_per_world_step()
    ns = min(16, nworld)
    ctrl_s = (np.zeros((horizon, ns, nv)) if held else sched[:, :, :ns].permute(0, 2, 1).double().cpu().numpy())
    try:
        flops_ex, _ = sim.flops_executed(q0[:ns], v0[:ns], ctrl_s, specialized=sim.specialized)
    except L.PhyzbError:
        flops_ex = None  # terrain: counted on the flat ground only
    flops_ws = flops_ex if flops_ex is not None else flops_gen
    pk = np.zeros(1)
    L.check(L.load().phyzb_measure_fma_peak(L.F32 if prec == "f32" else L.F64, L.dptr(pk)))
    achieved = flops_ws * nworld * horizon / (kernel_ms * 1e-3) / 1e12
    traffic = ncu_traffic(workload, prec, nv, esz, nworld, horizon)
    hbm_peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("hbm_gbs") \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 6650.0
    alg_bytes = (3 + 2) * nv * esz  # read q, v, ctrl; write q, v per world-step
    roofline = {
        "bound": "fma", "pipe": f"{'fp32' if prec == 'f32' else 'fp64'} FMA", "achieved": achieved,
        "peak": float(pk[0]), "unit": "TFLOP/s", "frac": achieved / float(pk[0]),
        "peak_source": "measured in this run (independent FMA chains over every SM, phyzb_measure_fma_peak)",
        "flops_per_world_step": flops_ws,
        "flops_counted": ("executed by the running kernel on this rollout's first 16 worlds (contact force law "
                          "where bodies touch" + ("; model-specialized: products with zero table constants left "
                                                  "out)" if sim.specialized else ")")
                          if flops_ex is not None else "generic formulation, steady state, contact force excluded"),
        "flops_per_world_step_generic": flops_gen,
        "frac_generic_count": flops_gen * nworld * horizon / (kernel_ms * 1e-3) / 1e12 / float(pk[0]),
        "transcendentals_per_world_step": trans_ws,
        "traffic": traffic, "kernel": "rollout_kernel", "kernel_ms_per_launch": kernel_ms,
        "kernel_ms_min": kernel_ms_min, "kernel_ms_median": kernel_ms_median,
        "algorithmic_bytes_per_world_step": alg_bytes,
        "hbm_gbs_algorithmic": alg_bytes * nworld * horizon / (kernel_ms * 1e-3) / 1e9,
        "hbm_gbs_measured_traffic": None if traffic is None else traffic / (kernel_ms * 1e-3) / 1e9,
        "hbm_peak_gbs": hbm_peak,
        "hbm_frac": None if traffic is None else traffic / (kernel_ms * 1e-3) / 1e9 / hbm_peak,
        "traffic_note": "ncu DRAM bytes of a capture at 65536 worlds (NCU_DRAM_CAPTURES) scaled to this "
                        "launch (state once + control stream per step); None where no capture exists for "
                        "this workload",
    }

    # e2e through the C ABI with host buffers: every step's controls copied
    # in from pinned host memory, held as a ring of at most ~4 GB of steps
    # that the rollout walks through (the full horizon for C2 f32 takes
    # three passes: 476 + 476 + 48 steps)
    e2e_out = None
    if e2e and held:
        q0_pin = torch.from_numpy(np.ascontiguousarray(q0, np.float64)).pin_memory().numpy()
        v0_pin = torch.from_numpy(np.ascontiguousarray(v0, np.float64)).pin_memory().numpy()
        c0_pin = torch.zeros((nworld, nv), dtype=torch.float64).pin_memory().numpy()
        hq = torch.zeros((nworld, nv), dtype=torch.float64).pin_memory().numpy()
        hv = torch.zeros((nworld, nv), dtype=torch.float64).pin_memory().numpy()

        def e2e_held():
            sim.load_states(q0_pin, v0_pin, c0_pin)
            sim.step_many(horizon)
            sim.readback_states(out=(hq, hv))

        e2e_held()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_held()
        e1.record(stream)
        stream.synchronize()
        barrier(world)
        ems = allreduce_max(e0.elapsed_time(e1), world)
        e2e_out = {"value": nworld * horizon * world * args.e2e_steps / (ems * 1e-3), "unit": "world-steps/s",
                   "h2d_bytes_per_step": int(3 * nworld * nv * 8), "d2h_bytes_per_step": int(2 * nworld * nv * 8),
                   "horizon": horizon, "path": "phyzb_load_states (zero controls held) + phyzb_step + "
                                                "phyzb_readback_states, pinned host buffers"}
    elif e2e:
        eh = min(args.e2e_horizon or horizon, horizon)
        ring = max(1, min(eh, (4 << 30) // (nworld * nv * esz)))
        host_ctrl = torch.empty((ring, nworld, nv), dtype=tdt, pin_memory=True)
        host_ctrl.copy_(sched[:ring].permute(0, 2, 1).cpu())
        # every host buffer of the e2e leg is pinned (page-locked), the form a
        # collector streaming rollouts keeps its rows in
        q0_pin = torch.from_numpy(np.ascontiguousarray(q0, np.float64)).pin_memory().numpy()
        v0_pin = torch.from_numpy(np.ascontiguousarray(v0, np.float64)).pin_memory().numpy()
        hq = torch.zeros((nworld, nv), dtype=torch.float64).pin_memory().numpy()
        hv = torch.zeros((nworld, nv), dtype=torch.float64).pin_memory().numpy()
        hdt = L.HOST_F32 if prec == "f32" else L.HOST_F64

        def e2e_step():
            sim.load_states(q0_pin, v0_pin)
            done = 0
            while done < eh:
                n = min(ring, eh - done)
                sim.step_with_controls_ptr(host_ctrl.data_ptr(), hdt, n)
                done += n
            sim.readback_states(out=(hq, hv))

        e2e_step()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        stream.synchronize()
        barrier(world)
        ems = allreduce_max(e0.elapsed_time(e1), world)
        e2e_out = {"value": nworld * eh * world * args.e2e_steps / (ems * 1e-3), "unit": "world-steps/s",
                   "h2d_bytes_per_step": int(2 * nworld * nv * 8 + eh * nworld * nv * esz),
                   "d2h_bytes_per_step": int(2 * nworld * nv * 8), "horizon": eh,
                   "path": f"phyzb_load_states + phyzb_step_with_controls + phyzb_readback_states, pinned host "
                           f"buffers; controls from a {ring}-step pinned ring walked to the horizon"}
        del host_ctrl

    cpu_out = oracle_out = None
    if cpu and rank == 0 and world == 1:
        try:
            v, threads, sample, _ = reference_cpu(workload, model, nworld, horizon, reps=7)
            cpu_out = {"value": v, "unit": "world-steps/s", "cores": threads, "kind": "reference",
                       "sample": sample}
        except Exception as ex:  # the baseline is reported, never required
            cpu_out = {"value": None, "unit": "world-steps/s", "cores": None, "kind": "reference",
                       "sample": f"unavailable: {ex}"}
        if prec == "f64":
            try:
                oracle_out = oracle_cpu(workload, model, nworld, horizon, reps=7)
            except Exception as ex:
                oracle_out = {"value": None, "kind": "port", "sample": f"unavailable: {ex}"}
    ref_gpu_out = None
    if ref_gpu and rank == 0 and world == 1:
        try:
            ref_gpu_out = reference_gpu(workload, model, nworld, horizon)
            if ref_gpu_out is not None:
                ref_gpu_out["ratio"] = value / ref_gpu_out["value"]
        except Exception as ex:
            ref_gpu_out = {"value": None, "note": f"unavailable: {ex}"}

    info = dict(sim.launch_info())
    # how the rollout launch runs: tile mode (steps_per_run 0) or slice mode
    # (warps take 32 worlds x steps_per_run jobs; worlds_per_block / blocks
    # of the slice launch)
    info["slices"] = sim.slice_plan(horizon)
    entry = {
        "value": value, "unit": "world-steps/s", "ms_per_step": ms / steps, "steps": steps, "warmup": warmup,
        "dtype": prec, "scaling": "strong" if strong else "weak",
        "config": bench_config(workload, model, total, horizon, prec, world, strong=strong),
        "launch": info,
        "kernel": (f"one world over {lanes} lanes (all but the last step of a rollout)" if lanes and
                   sim.lanes_active else ("model-specialized (compiled at run time for this model)"
                                          if sim.specialized else "generic variant")),
        "timed_region_ms": region_ms,
        "roofline": roofline, "cpu_baseline": cpu_out, "e2e": e2e_out, "clocks": clk.summary(),
        "gpu_launches": steps * 2,  # per rollout: rollout_kernel + objective_kernel
        "objective": objective[0],
    }
    if oracle_out is not None:
        entry["cpu_baseline_f64_oracle"] = oracle_out
    if ref_gpu_out is not None:
        entry["reference_gpu"] = ref_gpu_out
    del sched
    sim.close()
    torch.cuda.empty_cache()
    return entry


def main():
    args = parse()
    if args.impl == "reference":
        # CPU only: no process group; rank 0 runs, the other ranks exit 0
        run_reference_impl(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup(args)
    if args.config == "c5_quadruped_ppo":
        run_c5(args, world, rank, local)
        finish(world)
        return
    ctx = Ctx(args, world, rank, local)
    main_entry = measure(ctx, args.config, args.precision, args.nworld, args.horizon, args.steps, args.warmup,
                         e2e=not args.no_e2e, cpu=not args.no_cpu_baseline, ref_gpu=not args.no_reference_gpu,
                         specialize=args.specialize, lanes=args.lanes)
    per_config = {}
    if args.per_config and args.config == "c2_chain32" and not args.nworld and not args.horizon:
        for wl, prec, total, strong in PER_CONFIG:
            per_config[f"{wl}_{prec}"] = measure(ctx, wl, prec, total, 0, min(args.steps, 5), 3, strong=strong,
                                                 cpu=not args.no_cpu_baseline,
                                                 ref_gpu=not args.no_reference_gpu and prec == "f32",
                                                 specialize=args.specialize)
    if rank == 0:
        e = main_entry
        line = {
            "metric": "world-steps/sec", "value": e["value"], "unit": "world-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": e["ms_per_step"], "higher_is_better": True,
            "scaling": e["scaling"], "vs_baseline": None, "dtype": args.precision, "data": "synthetic (seeded)",
            "config": e["config"], "launch": e["launch"], "kernel": e["kernel"],
            "timed_region_ms": e["timed_region_ms"], "roofline": e["roofline"], "cpu_baseline": e["cpu_baseline"],
            "e2e": e["e2e"], "clocks": e["clocks"], "gpu_launches": e["gpu_launches"],
            "objective": e["objective"],
            "objective_reduce": "phyzb_reduce_objective (NCCL all-reduce over all ranks, once per rollout)",
        }
        for key in ("cpu_baseline_f64_oracle", "reference_gpu"):
            if key in e:
                line[key] = e[key]
        if per_config:
            line["per_config"] = per_config
        print(json.dumps(line), flush=True)
    ctx.comm.close()
    finish(world)


# ── C5: the quadruped batch under an on-device policy, with PPO updates ──
def run_c5(args, world, rank, local):
    """One bench step = one PPO iteration of BASELINE.json configs[4]: reset,
    64 control steps of the on-device policy driving the quadruped's PD
    servos (262144 worlds per GPU), returns on the device with the NCCL
    reduction of the advantage moments, and one PPO epoch (minibatches of
    65536, gradients all-reduced over ranks). Metric: simulated world-steps/s
    of the whole job, the update included."""
    import torch

    from phyz_b200.parallel import Comm, share_bytes
    from phyz_b200.rl import C5Cfg, OnDevicePpo

    cfg = C5Cfg(nworld=args.nworld or 262144, steps=args.horizon or 64, precision=args.precision)
    comm = Comm(rank, world, local, timeout=120.0,
                id_channel=(lambda p, r: share_bytes(p, r))) if world > 1 else None
    ppo = OnDevicePpo(cfg, device=local, rank=rank, comm=comm)
    stream = torch.cuda.Stream()
    ppo.sim.set_stream(stream.cuda_stream)
    for _ in range(args.warmup):
        ppo.iteration()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rollout_ms = 0.0
    stats = []
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for _ in range(args.steps):
            r0.record(stream)
            ppo.rollout()
            r1.record(stream)
            stats.append(ppo.update())
            r1.synchronize()
            rollout_ms += r0.elapsed_time(r1)
        t1.record(stream)
        stream.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ppo.sim.sync()
    ms = allreduce_max(t0.elapsed_time(t1), world)
    rollout_ms = allreduce_max(rollout_ms / args.steps, world)
    world_steps = cfg.nworld * cfg.steps * cfg.substeps * world
    value = world_steps * args.steps / (ms * 1e-3)
    flops_phys, _ = ppo.sim.flops_per_world_step()
    i, h, o = ppo.spec.n_in, ppo.spec.hidden, ppo.spec.n_out
    mlp = lambda out: 2 * (i * h + h * h + h * out)
    # per control step and world: policy forward, critic value, and one
    # epoch of update (forward + backward ~ 3x forward, actor and critic)
    flops_ctrl = mlp(o) + mlp(1) + 3 * (mlp(o) + mlp(1)) * cfg.epochs
    flops_ws = flops_phys + flops_ctrl / cfg.substeps
    pk = np.zeros(1)
    from phyz_b200 import _lib as L
    L.check(L.load().phyzb_measure_fma_peak(L.F32, L.dptr(pk)))
    achieved = flops_ws * world_steps / world * args.steps / (ms * 1e-3) / 1e12
    if rank == 0:
        ret_mean, adv_mean, adv_std = stats[-1][0]
        upd = stats[-1][1]
        line = {
            "metric": "world-steps/sec", "value": value, "unit": "world-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": cfg.precision, "data": "synthetic (seeded)",
            "config": {"workload": "c5_quadruped_ppo", "nworld_per_gpu": cfg.nworld, "control_steps": cfg.steps,
                       "substeps": cfg.substeps, "policy": f"{i}->{h}->{h} tanh->{o}", "minibatch": cfg.minibatch,
                       "epochs": cfg.epochs, "parallelism": f"worlds sharded over {world} GPU(s), "
                                                            "gradients all-reduced per minibatch"},
            "phases_ms": {"rollout": rollout_ms, "returns_and_update": ms / args.steps - rollout_ms},
            "roofline": {"bound": "fma", "pipe": "fp32 FMA", "achieved": achieved, "peak": float(pk[0]),
                         "unit": "TFLOP/s", "frac": achieved / float(pk[0]),
                         "flops_per_world_step": flops_ws, "peak_source": "measured in this run"},
            "clocks": clk.summary(), "gpu_launches": None,
            "last_iteration": {"mean_return": ret_mean, "adv_std": adv_std, **upd},
        }
        print(json.dumps(line), flush=True)
    ppo.close()
    if comm is not None:
        comm.close()


def finish(world):
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
