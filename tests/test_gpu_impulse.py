"""Impulse-mode contact on the sm_100a kernels (phyzb_enable_contact_impulse
through the C ABI): parity with the f64 oracle (oracle/phyz_oracle.hpp
step_world_impulse) and, in f32, with the reference's own contact kernel
compiled for the host; the warm start carried across launches; both
record layouts; the sweep count."""
import numpy as np
import pytest

from conftest import rel_err
from fixture_models import free_box
from phyz_b200 import BatchSim, PhyzbError, _lib, configs

pytestmark = pytest.mark.gpu

BOXES = {  # contact_impulse_parity.rs:126-186: initial v, mass
    "dropped": ([0.0] * 6, 1.0),
    "sliding": ([0.0, 0.0, 0.0, 2.0, 0.0, 0.0], 1.0),
    "light": ([3.0, 0.0, 0.0, 2.0, 0.0, 0.0], 0.1),
}


def gpu_run(model, q0, v0, ctrl, chunks, per_chunk, precision, friction, sweeps=None):
    sim = BatchSim(model, q0.shape[0], precision=precision)
    sim.enable_contact_impulse(0.0, friction)
    if sweeps is not None:
        sim.contact_sweeps = sweeps
    sim.load_states(q0, v0, ctrl)
    traj = []
    for _ in range(chunks):
        sim.step_many(per_chunk)
        q, v = sim.readback_states()
        traj.append((q, v))
    cs = sim.readback_contacts()
    qdd = sim.readback_qdd()
    sim.close()
    return traj, qdd, cs


def host_run(engine, model, q0, v0, ctrl, chunks, per_chunk, friction, sweeps=16):
    st = None
    q, v = q0, v0
    traj = []
    for _ in range(chunks):
        q, v, qdd, cs, st = engine.rollout_impulse(model, q, v, ctrl, nsteps=per_chunk, contact=(0.0, friction),
                                                   state=st, sweeps=sweeps, nthreads=4)
        traj.append((q, v))
    return traj, qdd, cs


def box_inputs(name):
    v0, mass = BOXES[name]
    return free_box(mass=mass), np.zeros((1, 6)), np.array([v0], float), np.zeros((1, 6))


@pytest.mark.parametrize("name", list(BOXES))
def test_boxes_f64_match_the_oracle(oracle, name):
    m, q0, v0, c = box_inputs(name)
    tg, qddg, csg = gpu_run(m, q0, v0, c, 15, 100, "f64", 0.8)
    to, qddo, cso = host_run(oracle, m, q0, v0, c, 15, 100, 0.8)
    for (qg, vg), (qo, vo) in zip(tg, to):
        assert np.max(np.abs(qg - qo)) < 1e-8 and np.max(np.abs(vg - vo)) < 1e-7
    assert np.max(np.abs(qddg - qddo)) < 1e-5 * max(1.0, np.max(np.abs(qddo)))
    assert np.max(np.abs(csg - cso)) < 1e-6 * 9.81


@pytest.mark.parametrize("name", list(BOXES))
def test_boxes_f32_match_the_reference_kernel(refhost, name):
    m, q0, v0, c = box_inputs(name)
    tg, _, csg = gpu_run(m, q0, v0, c, 15, 100, "f32", 0.8)
    tr, _, csr = host_run(refhost, m, q0, v0, c, 15, 100, 0.8)
    for (qg, vg), (qr, vr) in zip(tg, tr):
        assert np.max(np.abs(qg - qr)) < 5e-5
    assert np.max(np.abs(csg - csr)) < 1e-3 * 9.81


def test_dropped_box_rests_and_carries_its_weight():
    m, q0, v0, c = box_inputs("dropped")
    tg, _, cs = gpu_run(m, q0, v0, c, 15, 100, "f32", 0.8)
    q, v = tg[-1]
    assert abs(0.5 + q[0, 5] - 0.1) < 1e-3 and np.max(np.abs(v)) < 1e-3
    assert cs[0, 0, 0] == 1.0 and abs(cs[0, 0, 7] - 9.81) < 1e-3


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
def test_articulated_f64_matches_the_oracle(oracle, name):
    m = configs.CONFIGS[name].builder()
    n = 16
    q0, v0 = configs.initial_state(name, m, range(n))
    if name == "c3_quadruped":
        q0[:, 5] = np.linspace(0.3, 0.5, n)
    c = np.zeros((n, m.nv))
    tg, qddg, csg = gpu_run(m, q0, v0, c, 6, 50, "f64", 1.0)
    to, qddo, cso = host_run(oracle, m, q0, v0, c, 6, 50, 1.0)
    assert cso[:, :, 0].sum() > 0  # contacts happen
    dq = np.stack([np.max(np.abs(qg - qo), axis=1) for (qg, _), (qo, _) in zip(tg, to)])
    # f64 against f64: rounding only, unless a point sits exactly at the margin
    assert np.mean(dq < 1e-8) >= 0.9, np.sort(dq.ravel())[-8:]
    assert np.max(dq) < 1e-3
    ok = dq[-1] < 1e-8
    assert np.max(np.abs(csg[ok] - cso[ok])) < 1e-6 * max(1.0, np.max(np.abs(cso)))


@pytest.mark.parametrize("precision,tol", [("f32", 1e-4), ("f64", 1e-9)])
def test_warm_start_carries_across_launches(precision, tol):
    """400 steps as one launch or as 40 launches of 10 agree up to rounding
    (the wrenches and staged impulses travel through the impulse buffer
    between launches); restarting the warm start every 10 steps instead
    (re-enabling contact) moves the result far more, at 2 sweeps per step."""
    m = configs.quadruped()
    n = 64
    q0, v0 = configs.initial_state("c3_quadruped", m, range(n))
    q0[:, 5] = np.linspace(0.3, 0.5, n)
    c = np.zeros((n, m.nv))
    one, _, cs1 = gpu_run(m, q0, v0, c, 1, 400, precision, 1.0, sweeps=2)
    many, _, cs2 = gpu_run(m, q0, v0, c, 40, 10, precision, 1.0, sweeps=2)
    sim = BatchSim(m, n, precision=precision)
    sim.contact_sweeps = 2
    sim.load_states(q0, v0, c)
    for _ in range(40):
        sim.enable_contact_impulse(0.0, 1.0)  # a fresh warm start
        sim.step_many(10)
    cold = sim.readback_states()[0]
    sim.close()
    split = rel_err(many[-1][0], one[-1][0])
    assert split <= tol, split
    assert rel_err(cold, one[-1][0]) > 100 * max(split, tol)


def test_tensor_memory_layout_agrees(monkeypatch):
    m = configs.quadruped()
    n = 256
    q0, v0 = configs.initial_state("c3_quadruped", m, range(n))
    q0[:, 5] = np.linspace(0.3, 0.5, n)
    c = np.zeros((n, m.nv))
    out = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("PHYZB_TMEM", mode)
        sim = BatchSim(m, n, precision="f32")
        sim.enable_contact_impulse(0.0, 1.0)
        out[mode] = sim.launch_info()["tmem_cols"]
        sim.load_states(q0, v0, c)
        sim.step_many(150)
        out[mode + "q"] = sim.readback_states()[0]
        sim.close()
    assert out["0"] == 0 and out["1"] > 0
    assert np.max(np.abs(out["0q"] - out["1q"])) < 1e-4


def test_sweep_count(oracle):
    m, q0, v0, c = box_inputs("sliding")
    tg, _, _ = gpu_run(m, q0, v0, c, 6, 100, "f64", 0.8, sweeps=4)
    to, _, _ = host_run(oracle, m, q0, v0, c, 6, 100, 0.8, sweeps=4)
    assert np.max(np.abs(tg[-1][0] - to[-1][0])) < 1e-8
    sim = BatchSim(m, 1)
    for bad in (0, _lib.MAX_CONTACT_SWEEPS + 1):
        with pytest.raises(PhyzbError) as e:
            sim.contact_sweeps = bad
        assert e.value.code == _lib.ERR_INVALID
    sim.close()


def test_switching_contact_modes():
    m, q0, v0, c = box_inputs("dropped")
    sim = BatchSim(m, 1)
    assert sim.enable_contact_impulse(0.0, 0.8) == 1
    sim.load_states(q0, v0, c)
    sim.step_many(600)
    z_imp = 0.5 + sim.readback_states()[0][0, 5]
    assert abs(z_imp - 0.1) < 2e-3
    # back to the penalty law: it sags mg/k into the ground
    sim.enable_ground_contact(0.0, 1e4, 100.0, 0.8)
    sim.step_many(600)
    z_pen = 0.5 + sim.readback_states()[0][0, 5]
    assert z_pen < z_imp - 1e-4
    sim.disable_contact()
    with pytest.raises(PhyzbError):
        sim.readback_contacts()
    sim.close()
    bare = BatchSim(configs.double_pendulum(), 1)
    with pytest.raises(PhyzbError) as e:
        bare.enable_contact_impulse(0.0, 1.0)
    assert e.value.code == _lib.ERR_INVALID
    bare.close()
