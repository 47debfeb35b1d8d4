"""Slice mode of the rollout kernel: every warp takes (32 worlds, a run of
steps) jobs from a device queue, the state going through q and v between
runs, so that warps which finish early take the remaining worlds' runs
instead of idling through a partial last wave (pz::plan_slices,
phyzb_slice_plan).

* The planner: the headline workload (C2 f32, 65536 worlds x 1000 steps:
  1.98 waves of the tile shape) runs in slice mode at 256 worlds per block;
  one step, a single wave and PHYZB_SLICES=0 run in tile mode.
* Slices against tiles on the same inputs (PHYZB_SLICES=1 slices every
  launch of two or more steps): a run starts from q, v (and the impulse
  buffer) where the one before ended and recomputes its first forward sweep,
  so the two modes agree to rounding (f64 <= 1e-12 relative), and the f64
  results match the oracle <= 1e-9, on the generic variants that have
  slice mode (Tensor-Memory records, no impulse contact or terrain): chains
  and free joints with penalty contact, f32 and f64; and on the
  model-specialized kernel's slice-mode twin (compiled on the first sliced
  launch). The generic shared-memory layout and impulse / terrain variants
  run tile mode only.
* Many rounds of jobs: C2 f64 at 65536 worlds, where a warp takes several
  tiles' runs and waits for runs other SMs ran.
* The bounded wait: PHYZB_SLICES_STALL=1 starts the queue past every tile's
  first run, so each later run waits for a run that never comes; the wait
  gives up after its bound, the status reports it, and the device stays
  usable (a later simulator steps normally).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err
from phyz_b200 import BatchSim, PhyzbError, configs

pytestmark = pytest.mark.gpu


def run(name, precision, n, steps, env, monkeypatch, layout=None, spec=False, impulse=False):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    if layout is not None:
        monkeypatch.setenv("PHYZB_TMEM", layout)
    cfg = configs.CONFIGS[name]
    model = cfg.builder()
    q0, v0 = configs.initial_state(name, model, range(n))
    sched = configs.control_schedule(name, model, range(n), steps)
    sim = BatchSim(model, n, precision=precision)
    sim.specialize = spec
    if cfg.contact is not None:
        if impulse:
            sim.enable_contact_impulse(0.0, 1.0)
        else:
            sim.enable_ground_contact(*cfg.contact)
    sim.load_states(q0, v0)
    # one launch of every step: the schedule on the device, [step][nv][nworld]
    import torch

    dev = torch.as_tensor(np.ascontiguousarray(sched.transpose(0, 2, 1)),
                          dtype=torch.float32 if precision == "f32" else torch.float64).cuda()
    torch.cuda.synchronize()
    sim.step_device_controls(dev.data_ptr(), model.nv * n, steps)
    sim.sync()
    del dev
    plan = sim.slice_plan(steps)
    q, v = sim.readback_states()
    qdd = sim.readback_qdd()
    sim.close()
    for k in list(env) + (["PHYZB_TMEM"] if layout is not None else []):
        monkeypatch.delenv(k)
    return plan, q0, v0, sched, q, v, qdd


def oracle_contact(cfg, model):
    if cfg.contact is None:
        return None
    g, k, d, mu = cfg.contact
    return g, mu, [k] * model.nbodies, [d] * model.nbodies


def test_plan_headline_and_tile_cases():
    model = configs.chain()
    sim = BatchSim(model, 65536, precision="f32")
    p = sim.slice_plan(1000)
    assert p["steps_per_run"] > 0 and p["worlds_per_block"] == 256 and p["blocks"] == 148, p
    assert sim.slice_plan(1)["steps_per_run"] == 0
    sim.close()
    small = BatchSim(model, 4096, precision="f32")  # one wave: nothing to share
    assert small.slice_plan(1000)["steps_per_run"] == 0
    small.close()


def test_plan_switches(monkeypatch):
    model = configs.chain()
    monkeypatch.setenv("PHYZB_SLICES", "0")
    sim = BatchSim(model, 65536, precision="f32")
    assert sim.slice_plan(1000)["steps_per_run"] == 0
    sim.close()
    monkeypatch.setenv("PHYZB_SLICES", "1")
    monkeypatch.setenv("PHYZB_TMEM", "1")
    sim = BatchSim(model, 300, precision="f32")
    assert sim.slice_plan(12)["steps_per_run"] == 4
    assert sim.slice_plan(1)["steps_per_run"] == 0
    sim.close()


# (config, precision, record layout, specialized kernel, impulse contact):
# the Tensor-Memory variants, which have slice mode compiled in
CASES = [
    ("c2_chain32", "f64", "1", False, False),
    ("c2_chain32", "f32", "1", False, False),
    ("c3_quadruped", "f64", "1", False, False),
    ("c4_humanoid", "f64", "1", False, False),
    ("c4_humanoid", "f32", "1", False, False),
    ("c3_quadruped", "f64", "1", True, False),
    ("c4_humanoid", "f32", "1", True, False),
]


@pytest.mark.parametrize("name,precision,layout,spec,impulse", CASES)
def test_slices_match_tiles(oracle, monkeypatch, name, precision, layout, spec, impulse):
    n, steps = 3000, 12
    pt, q0, v0, sched, qt, vt, qddt = run(name, precision, n, steps, {"PHYZB_SLICES": "0"}, monkeypatch,
                                          layout, spec, impulse)
    ps, _, _, _, qs, vs, qdds = run(name, precision, n, steps, {"PHYZB_SLICES": "1"}, monkeypatch, layout, spec,
                                    impulse)
    assert pt["steps_per_run"] == 0 and ps["steps_per_run"] == 4, (pt, ps)
    tol = 1e-12 if precision == "f64" else 1e-5
    for nm, a, b in (("q", qs, qt), ("v", vs, vt), ("qdd", qdds, qddt)):
        assert np.isfinite(a).all()
        assert rel_err(a, b) <= tol, f"{nm}: slices vs tiles {rel_err(a, b):.3e}"
    if precision == "f64" and not impulse:
        cfg = configs.CONFIGS[name]
        model = cfg.builder()
        ws = np.unique(np.concatenate([np.arange(0, 40), np.arange(n - 40, n),
                                       np.random.default_rng(5).integers(40, n - 40, 48)]))
        qo, vo, qddo, _ = oracle.rollout(model, q0[ws], v0[ws], sched[:, ws], steps, schedule=True,
                                         contact=oracle_contact(cfg, model), nthreads=8)
        for nm, a, b in (("q", qs[ws], qo), ("v", vs[ws], vo), ("qdd", qdds[ws], qddo)):
            assert rel_err(a, b) <= 1e-9, f"{nm}: slices vs oracle {rel_err(a, b):.3e}"


@pytest.mark.parametrize("kind", ["smem", "impulse"])
def test_tile_only_kernels(monkeypatch, kind):
    """The generic shared-memory layout and the impulse-contact variants
    are compiled for tile mode only: they report it and step correctly with
    PHYZB_SLICES=1 set."""
    monkeypatch.setenv("PHYZB_SLICES", "1")
    if kind == "smem":
        monkeypatch.setenv("PHYZB_TMEM", "0")
    model = configs.quadruped()
    sim = BatchSim(model, 300, precision="f32")
    if kind == "impulse":
        sim.enable_contact_impulse(0.0, 1.0)
    else:
        sim.enable_ground_contact(*configs.CONFIGS["c3_quadruped"].contact)
    sim.specialize = False
    sim.step_many(2)
    sim.sync()
    assert sim.slice_plan(12)["steps_per_run"] == 0
    sim.close()


def test_many_rounds_of_jobs(oracle, monkeypatch):
    """C2 f64 at 65536 worlds x 40 steps: the planner picks slices (3.5 tile
    waves), 2048 warp tiles over 592 warp slots."""
    n, steps = 65536, 40
    pt, q0, v0, sched, qt, vt, _ = run("c2_chain32", "f64", n, steps, {"PHYZB_SLICES": "0"}, monkeypatch)
    ps, _, _, _, qs, vs, _ = run("c2_chain32", "f64", n, steps, {}, monkeypatch)
    assert pt["steps_per_run"] == 0 and 0 < ps["steps_per_run"] < steps, (pt, ps)
    assert -(-n // 32) > ps["blocks"] * ps["worlds_per_block"] // 32, ps
    assert rel_err(qs, qt) <= 1e-12 and rel_err(vs, vt) <= 1e-12, (rel_err(qs, qt), rel_err(vs, vt))
    model = configs.chain()
    ws = np.unique(np.concatenate([np.arange(0, 32), np.arange(n - 32, n),
                                   np.random.default_rng(6).integers(32, n - 32, 64)]))
    qo, vo, _, _ = oracle.rollout(model, q0[ws], v0[ws], sched[:, ws], steps, schedule=True, nthreads=8)
    assert rel_err(qs[ws], qo) <= 1e-9 and rel_err(vs[ws], vo) <= 1e-9


def test_bounded_wait_reports_and_device_stays_usable(monkeypatch):
    model = configs.chain()
    n, steps = 640, 6
    q0, v0 = configs.initial_state("c2_chain32", model, range(n))
    sched = configs.control_schedule("c2_chain32", model, range(n), steps)
    monkeypatch.setenv("PHYZB_SLICES", "1")
    monkeypatch.setenv("PHYZB_TMEM", "1")
    monkeypatch.setenv("PHYZB_SLICES_STALL", "1")
    sim = BatchSim(model, n, precision="f32")
    sim.load_states(q0, v0)
    sim.step_with_controls(np.ascontiguousarray(sched))
    with pytest.raises(PhyzbError, match="slice-mode run waited"):
        sim.sync()
    sim.close()
    monkeypatch.delenv("PHYZB_SLICES_STALL")
    ok = BatchSim(model, n, precision="f32")
    ok.load_states(q0, v0)
    ok.step_with_controls(np.ascontiguousarray(sched))
    ok.sync()
    q, _ = ok.readback_states()
    ok.close()
    assert np.isfinite(q).all()
