"""The lanes kernel (phyzb_set_world_lanes: one world over 2, 4 or 8 threads
of a warp, limbs in parallel, the trunk's sums by warp shuffles) against the
f64 oracle and against one thread per world: every launch of two or more
steps runs all but its last step on the lanes kernel."""
import numpy as np
import pytest

from conftest import rel_err
from phyz_b200 import BatchSim, PdDof, PhyzbError, configs

pytestmark = pytest.mark.gpu


def inputs(name, n, steps):
    cfg = configs.CONFIGS[name]
    m = cfg.builder()
    q0, v0 = configs.initial_state(name, m, range(n))
    sched = configs.control_schedule(name, m, range(n), steps)
    return cfg, m, q0, v0, sched


def device(name, precision, lanes, n, steps):
    cfg, m, q0, v0, sched = inputs(name, n, steps)
    sim = BatchSim(m, n, precision=precision)
    if cfg.contact:
        sim.enable_ground_contact(*cfg.contact)
    sim.world_lanes = lanes
    assert sim.world_lanes == lanes and sim.lanes_active
    sim.load_states(q0, v0)
    sim.step_with_controls(np.ascontiguousarray(sched))
    sim.sync()
    q, v = sim.readback_states()
    qdd = sim.readback_qdd()
    sim.close()
    return cfg, m, q0, v0, sched, q, v, qdd


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
@pytest.mark.parametrize("lanes", [2, 4, 8])
def test_lanes_match_oracle_f64(oracle, name, lanes):
    n, steps = 70, 50  # a ragged last group of lanes
    cfg, m, q0, v0, sched, q, v, qdd = device(name, "f64", lanes, n, steps)
    oc = None if cfg.contact is None else (cfg.contact[0], cfg.contact[3], cfg.contact[1], cfg.contact[2])
    qo, vo, qddo, _ = oracle.rollout(m, q0, v0, sched, steps, schedule=True, contact=oc, nthreads=8)
    for nm, a, b in (("q", q, qo), ("v", v, vo), ("qdd", qdd, qddo)):
        assert rel_err(a, b) <= 1e-9, f"{name} lanes {lanes} {nm}: {rel_err(a, b):.3e}"


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
def test_lanes_f32_and_many_tiles(oracle, name):
    """f32 at 4 lanes over enough worlds that blocks walk several tiles."""
    n, steps = 6000, 20
    cfg, m, q0, v0, sched, q, v, _ = device(name, "f32", 4, n, steps)
    oc = None if cfg.contact is None else (cfg.contact[0], cfg.contact[3], cfg.contact[1], cfg.contact[2])
    ws = np.r_[0:64, n - 64:n]
    qo, vo, _, _ = oracle.rollout(m, q0[ws], v0[ws], sched[:, ws], steps, schedule=True, contact=oc, nthreads=8)
    assert rel_err(q[ws], qo) <= 1e-3 and rel_err(v[ws], vo) <= 1e-3, (rel_err(q[ws], qo), rel_err(v[ws], vo))


def test_lanes_are_deterministic_and_step_split():
    name = "c4_humanoid"
    outs = []
    for split in (False, False, True):
        cfg, m, q0, v0, sched = inputs(name, 64, 1)
        sim = BatchSim(m, 64, precision="f64")
        sim.enable_ground_contact(*cfg.contact)
        sim.world_lanes = 4
        sim.load_states(q0, v0, sched[0])
        if split:
            for _ in range(3):
                sim.step_many(10)
        else:
            sim.step_many(30)
        outs.append(sim.readback_states())
        sim.close()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    assert rel_err(outs[2][0], outs[0][0]) <= 1e-12


def test_lanes_settings():
    """A chain does not split; PD servos return the simulator to one thread
    per world (and it still steps correctly); 0 turns lanes off."""
    with pytest.raises(PhyzbError):
        BatchSim(configs.chain(), 8).world_lanes = 4
    m = configs.quadruped()
    sim = BatchSim(m, 32)
    with pytest.raises(PhyzbError):
        sim.world_lanes = 3
    sim.world_lanes = 2
    assert sim.lanes_active
    sim.enable_pd_control([PdDof(j, j, 20.0, 1.0, 20.0) for j in range(6, m.nv)])
    assert sim.world_lanes == 2 and not sim.lanes_active
    sim.step_many(5)
    sim.world_lanes = 0
    assert sim.world_lanes == 0 and not sim.lanes_active
    sim.close()
