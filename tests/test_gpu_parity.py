"""Parity of the sm_100a kernels (through the C ABI) with the f64 oracle.

Tolerances are the north star's: max relative error (normwise, conftest
rel_err) <= 1e-5 on q, v, qdd after one step in f64 mode, <= 1e-3 in f32
mode. The f64 checks below also hold a much tighter bound where the two
formulations can only differ by rounding, so a formulation slip cannot
hide under the stated tolerance.
"""
import numpy as np
import pytest

from conftest import rel_err
from fixture_models import (armature_chain, double_pendulum, featureful, free_sphere, single_step_cases)
from phyz_b200 import BatchSim, BodyContactGains, PdDof, PhyzbError, configs
from phyz_b200 import _lib

pytestmark = pytest.mark.gpu

F64_TOL, F32_TOL = 1e-5, 1e-3
F64_TIGHT = 1e-10


def run_device(model, q0, v0, ctrl, steps=1, precision="f64", contact=None, schedule=False):
    n = q0.shape[0]
    sim = BatchSim(model, n, precision=precision)
    if contact is not None:
        sim.enable_ground_contact(*contact)
    if schedule:
        sim.load_states(q0, v0)
        sim.step_with_controls(np.ascontiguousarray(ctrl))
    else:
        sim.load_states(q0, v0, ctrl)
        sim.step_many(steps)
    sim.sync()
    q, v = sim.readback_states()
    qdd = sim.readback_qdd()
    cs = sim.readback_contacts() if contact is not None else None
    sim.close()
    return q, v, qdd, cs


@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_reference_fixtures_one_step(oracle, precision):
    tol = F64_TIGHT if precision == "f64" else F32_TOL
    for label, m, q, v, _ in single_step_cases():
        q0, v0 = np.array([q], float), np.array([v], float)
        c0 = np.zeros_like(q0)
        qd, vd, qddd, _ = run_device(m, q0, v0, c0, precision=precision)
        qo, vo, qddo, _ = oracle.rollout(m, q0, v0, c0, 1)
        for name, a, b in (("q", qd, qo), ("v", vd, vo), ("qdd", qddd, qddo)):
            assert rel_err(a, b) <= tol, f"{label} {precision} {name}: {rel_err(a, b):.3e}"


@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_featureful_model(oracle, precision):
    """General axis, rotated joint frame, damping/spring/armature/limits/
    friction loss, prismatic, fixed, branch and ball joints together."""
    m = featureful()
    n = 16
    rng = np.random.default_rng(3)
    q0 = rng.uniform(-0.4, 0.4, (n, m.nv))
    q0[:, 6] = rng.uniform(-0.5, 0.5, n)  # drive the limited hinge past its limits
    v0 = rng.normal(0, 0.5, (n, m.nv))
    ctrl = rng.normal(0, 0.3, (n, m.nv))
    tol = 1e-9 if precision == "f64" else F32_TOL
    for steps in (1, 20):
        qd, vd, qddd, _ = run_device(m, q0, v0, ctrl, steps, precision)
        qo, vo, qddo, _ = oracle.rollout(m, q0, v0, ctrl, steps)
        assert rel_err(qd, qo) <= tol and rel_err(vd, vo) <= tol, (steps, rel_err(qd, qo), rel_err(vd, vo))
        assert rel_err(qddd, qddo) <= tol * 10, (steps, rel_err(qddd, qddo))


def config_inputs(name, n, steps):
    cfg = configs.CONFIGS[name]
    model = cfg.builder()
    q0, v0 = configs.initial_state(name, model, range(n))
    sched = configs.control_schedule(name, model, range(n), steps)
    contact = None
    if cfg.contact is not None:
        g, k, d, mu = cfg.contact
        contact = (g, k, d, mu)
    return model, q0, v0, sched, contact


@pytest.mark.parametrize("name", list(configs.CONFIGS))
@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_configs_one_step(oracle, name, precision):
    model, q0, v0, sched, contact = config_inputs(name, 64, 1)
    qd, vd, qddd, csd = run_device(model, q0, v0, sched[0], 1, precision, contact)
    oc = None if contact is None else (contact[0], contact[3], contact[1], contact[2])
    qo, vo, qddo, cso = oracle.rollout(model, q0, v0, sched[0], 1, contact=oc)
    tol = F64_TOL if precision == "f64" else F32_TOL
    for nm, a, b in (("q", qd, qo), ("v", vd, vo), ("qdd", qddd, qddo)):
        e = rel_err(a, b)
        assert e <= tol, f"{name} {precision} {nm}: {e:.3e}"
        if precision == "f64":
            assert e <= 1e-9, f"{name} f64 {nm}: {e:.3e} (formulations should agree to rounding)"
    if contact is not None and precision == "f64":
        assert rel_err(csd, cso) <= 1e-9


@pytest.mark.parametrize("name", list(configs.CONFIGS))
def test_configs_schedule_50_steps_f64(oracle, name):
    """50 steps with per-step controls through the bulk host path."""
    model, q0, v0, sched, contact = config_inputs(name, 32, 50)
    qd, vd, qddd, csd = run_device(model, q0, v0, sched, precision="f64", contact=contact, schedule=True)
    oc = None if contact is None else (contact[0], contact[3], contact[1], contact[2])
    qo, vo, qddo, cso = oracle.rollout(model, q0, v0, sched, 50, schedule=True, contact=oc)
    assert rel_err(qd, qo) <= 1e-7, rel_err(qd, qo)
    assert rel_err(vd, vo) <= 1e-7, rel_err(vd, vo)


def test_trajectory_no_aliasing(oracle):
    """cuda_vs_cpu.rs:246-270: 3 worlds x 200 steps, worlds stay apart."""
    m = double_pendulum()
    q0 = np.array([[0.4 + 0.2 * i, -0.3] for i in range(3)])
    v0 = np.zeros_like(q0)
    qd, vd, _, _ = run_device(m, q0, v0, np.zeros_like(q0), 200)
    qo, vo, _, _ = oracle.rollout(m, q0, v0, np.zeros_like(q0), 200)
    assert rel_err(qd, qo) <= 1e-9 and rel_err(vd, vo) <= 1e-9
    assert abs(qd[0, 0] - qd[1, 0]) > 1e-3


def test_armature(oracle):
    m = armature_chain()
    q0, v0 = np.array([[0.3, -0.7]]), np.array([[0.9, -1.4]])
    qd, vd, qddd, _ = run_device(m, q0, v0, np.zeros_like(q0))
    qo, vo, qddo, _ = oracle.rollout(m, q0, v0, np.zeros_like(q0), 1)
    assert rel_err(qddd, qddo) <= F64_TIGHT


def test_pd_servo(oracle):
    """cuda_vs_cpu.rs:272-317: PD servo, 100 steps, against the CPU loop."""
    from phyz_b200.model import ModelBuilder, SpatialInertia, Transform
    m = (ModelBuilder().gravity([0, 0, -9.81]).dt(0.002)
         .add_revolute_body("link", -1, Transform.identity(),
                            SpatialInertia.new(1.0, [0, 0, -0.5], np.eye(3) * 0.1)).build())
    kp, kd, mx, tgt = 30.0, 2.0, 25.0, 0.8
    pd = [PdDof(0, 0, kp, kd, mx)]
    sim = BatchSim(m, 4)
    sim.enable_pd_control(pd)
    sim.set_position_targets(np.full((4, 1), tgt))
    q0 = np.full((4, 1), 0.3)
    sim.load_states(q0, np.zeros((4, 1)))
    sim.step_many(100)
    q, _ = sim.readback_states()
    qo, _, _, _ = oracle.rollout(m, q0, np.zeros((4, 1)), np.zeros((4, 1)), 100, pd=pd,
                                 targets=np.full((4, 1), tgt))
    assert rel_err(q, qo) <= 1e-10
    assert abs(q[0, 0] - 0.3) > 0.05


def test_sphere_rests_on_ground():
    """cuda_vs_cpu.rs:319-367 behaviour, in both precisions."""
    for precision in ("f64", "f32"):
        mass, radius = 1.0, 0.1
        m = free_sphere(mass, radius)
        omega, zeta = 200.0, 1.0
        sim = BatchSim(m, 2, precision=precision)
        assert sim.enable_ground_contact(0.0, mass * omega ** 2, 2 * zeta * mass * omega, 0.5) == 1
        q0 = np.zeros((2, 6))
        q0[:, 5] = 0.5
        sim.load_states(q0, np.zeros((2, 6)))
        sim.step()
        assert sim.readback_contacts()[0, 0, 0] == 0.0, "airborne body reports contact"
        sim.step_many(2000)
        q, _ = sim.readback_states()
        assert abs(q[0, 5] - radius) < 0.02
        c = sim.readback_contacts()[1, 0]
        assert c[0] == 1.0
        weight = mass * 9.81
        assert abs(c[7] - weight) < 0.15 * weight
        assert abs(c[4]) < 1e-6
        sim2 = BatchSim(m, 1, precision=precision)
        gains = BodyContactGains.uniform_frequency(m, omega, zeta)
        assert sim2.enable_ground_contact_per_body(0.0, 0.5, gains) == 1
    bare = BatchSim(double_pendulum(), 1)
    with pytest.raises(PhyzbError):
        bare.enable_ground_contact(0.0, 1.0, 1.0, 0.5)
    with pytest.raises(PhyzbError):
        bare.readback_contacts()


def test_step_split_and_determinism():
    """step(n) == n x step(1) up to rounding, and a replay is bit-identical
    (the reference pins graph replay against direct launches,
    cuda_vs_cpu.rs:1295)."""
    model, q0, v0, sched, _ = config_inputs("c2_chain32", 64, 1)
    outs = []
    for split in (False, True, False):
        sim = BatchSim(model, 64)
        sim.load_states(q0, v0, sched[0])
        if split:
            for _ in range(30):
                sim.step()
        else:
            sim.step_many(30)
        outs.append(sim.readback_states())
    assert np.array_equal(outs[0][0], outs[2][0]) and np.array_equal(outs[0][1], outs[2][1])
    assert rel_err(outs[1][0], outs[0][0]) <= 1e-12


def test_double_pendulum_500_step_drift(oracle):
    """C1 drift bound: device-vs-oracle divergence after 500 steps stays
    within 100x the oracle's own 1-ulp-perturbation envelope
    (crates/phyz/src/determinism.rs:180,333 method)."""
    model = configs.double_pendulum()
    n = 256
    q0, v0 = configs.initial_state("c1_double_pendulum", model, range(n))
    c = np.zeros_like(q0)
    qd, vd, _, _ = run_device(model, q0, v0, c, 500)
    qo, vo, _, _ = oracle.rollout(model, q0, v0, c, 500)
    qp, vp, _, _ = oracle.rollout(model, np.nextafter(q0, np.inf), v0, c, 500)
    env = np.maximum(np.abs(qp - qo), 1e-15)
    dev = np.abs(qd - qo)
    assert np.all(dev <= 100 * env + 1e-12), float(np.max(dev / (100 * env + 1e-12)))


def test_nonfinite_state_is_reported():
    m = double_pendulum()
    sim = BatchSim(m, 4)
    q0 = np.zeros((4, 2))
    q0[2, 0] = np.nan
    sim.load_states(q0, np.zeros((4, 2)))
    sim.step()
    with pytest.raises(PhyzbError) as e:
        sim.sync()
    assert e.value.code == _lib.ERR_NONFINITE and "world 2" in e.value.message
    sim.clear_status()
    sim.load_states(np.zeros((4, 2)), np.zeros((4, 2)))
    sim.step()
    sim.sync()


def test_objective_matches_oracle_energy(oracle):
    import torch
    model, q0, v0, _, _ = config_inputs("c4_humanoid", 128, 1)
    sim = BatchSim(model, 128)
    sim.load_states(q0, v0 + 0.3)
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    sim.objective_device(0, out.data_ptr())
    torch.cuda.synchronize()
    ke, _ = oracle.energy(model, q0, v0 + 0.3)
    assert abs(out.item() - ke.sum()) <= 1e-10 * abs(ke.sum())


def test_device_schedule_matches_host_schedule():
    import torch
    name = "c3_quadruped"
    model, q0, v0, sched, contact = config_inputs(name, 64, 10)
    qh, vh, _, _ = run_device(model, q0, v0, sched, precision="f32", contact=contact, schedule=True)
    sim = BatchSim(model, 64, precision="f32")
    sim.enable_ground_contact(*contact)
    sim.load_states(q0, v0)
    dev = torch.tensor(sched.transpose(0, 2, 1).copy(), dtype=torch.float32, device="cuda")  # [step][nv][nworld]
    torch.cuda.synchronize()  # written on torch's stream, read on the simulator's
    sim.step_device_controls(dev.data_ptr(), 64 * model.nv, 10)
    sim.sync()
    qd, vd = sim.readback_states()
    assert np.array_equal(qd, qh) and np.array_equal(vd, vh)


@pytest.mark.parametrize("name", list(configs.CONFIGS))
@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_tensor_memory_layout(oracle, monkeypatch, name, precision):
    """The Tensor-Memory layout (hinge records in TMEM, one block per SM)
    forced at a ragged world count (the last warp partly idle) agrees with
    the oracle and with the shared-memory layout over a 30-step schedule."""
    n, steps = 70, 30
    model, q0, v0, sched, contact = config_inputs(name, n, steps)
    out = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("PHYZB_TMEM", mode)
        sim = BatchSim(model, n, precision=precision)
        if contact is not None:
            sim.enable_ground_contact(*contact)
        info = sim.launch_info()
        assert (info["tmem_cols"] > 0) == (mode == "1"), info
        sim.load_states(q0, v0)
        sim.step_with_controls(np.ascontiguousarray(sched))
        sim.sync()
        q, v = sim.readback_states()
        out[mode] = (q, v, sim.readback_qdd(), sim.readback_contacts() if contact is not None else None)
        sim.close()
    oc = None if contact is None else (contact[0], contact[3], contact[1], contact[2])
    qo, vo, qddo, cso = oracle.rollout(model, q0, v0, sched, steps, schedule=True, contact=oc)
    tol = 1e-7 if precision == "f64" else F32_TOL
    q, v, qdd, cs = out["1"]
    assert rel_err(q, qo) <= tol and rel_err(v, vo) <= tol, (rel_err(q, qo), rel_err(v, vo))
    same = 1e-12 if precision == "f64" else 1e-5
    for a, b in zip(out["1"], out["0"]):
        if a is not None:
            assert rel_err(a, b) <= same, rel_err(a, b)


def test_state_history():
    """mod.rs:1316-1376: snapshots recorded between launches read back as the
    states at those times; re-enabling with the same slot count keeps them."""
    name = "c3_quadruped"
    model, q0, v0, sched, contact = config_inputs(name, 40, 6)
    sim = BatchSim(model, 40, precision="f32")
    sim.enable_ground_contact(*contact)
    sim.load_states(q0, v0, sched[0])
    sim.enable_state_history(3)
    want = []
    for slot in range(3):
        sim.step_many(2)
        sim.record_state(slot)
        want.append(sim.readback_states())
    sim.enable_state_history(3)
    q, v = sim.readback_state_history(0, 3)
    for k in range(3):
        assert np.array_equal(q[k], want[k][0]) and np.array_equal(v[k], want[k][1])
    with pytest.raises(PhyzbError):
        sim.record_state(3)
    with pytest.raises(PhyzbError):
        sim.readback_state_history(2, 2)
    sim.close()
