"""Pins the f64 oracle against the reference's own code run here: phyz's
crates/phyz-gpu/cuda/phyz_kernels.cu compiled as host C++ (f32), driven with
the reference step sequence (oracle/ref_host_driver.cpp). Tolerances are the
reference's own f32-kernel-vs-f64-CPU tolerances (cuda_vs_cpu.rs:199-244)
where it states them, 1e-3 relative otherwise.
"""
import numpy as np
import pytest

from conftest import rel_err
from fixture_models import double_pendulum, free_sphere, single_step_cases
from phyz_b200 import PdDof, configs


def test_reference_fixture_single_steps(oracle, refhost):
    for label, m, q, v, tol in single_step_cases():
        q0, v0 = np.array([q], float), np.array([v], float)
        c = np.zeros_like(q0)
        qo, vo, _, _ = oracle.rollout(m, q0, v0, c, 1)
        qr, vr, _, _ = refhost.rollout(m, q0, v0, c, 1)
        assert np.max(np.abs(qr - qo)) < tol and np.max(np.abs(vr - vo)) < tol, label


@pytest.mark.parametrize("name", list(configs.CONFIGS))
def test_configs_one_step(oracle, refhost, name):
    cfg = configs.CONFIGS[name]
    m = cfg.builder()
    q0, v0 = configs.initial_state(name, m, range(32))
    c = configs.controls(name, m, range(32), 0)
    contact = None
    if cfg.contact:
        g, k, d, mu = cfg.contact
        contact = (g, mu, k, d)
    qo, vo, qddo, cso = oracle.rollout(m, q0, v0, c, 1, contact=contact)
    qr, vr, qddr, csr = refhost.rollout(m, q0, v0, c, 1, contact=contact)
    assert rel_err(qr, qo) < 1e-3 and rel_err(vr, vo) < 1e-3, (rel_err(qr, qo), rel_err(vr, vo))
    assert rel_err(qddr, qddo) < 1e-3, rel_err(qddr, qddo)
    if contact:
        assert rel_err(csr, cso) < 1e-3


def test_trajectory(oracle, refhost):
    """cuda_vs_cpu.rs:246-270: 3 worlds x 200 steps at 5e-3."""
    m = double_pendulum()
    q0 = np.array([[0.4 + 0.2 * i, -0.3] for i in range(3)])
    z = np.zeros_like(q0)
    qo, vo, _, _ = oracle.rollout(m, q0, z, z, 200)
    qr, vr, _, _ = refhost.rollout(m, q0, z, z, 200)
    assert np.max(np.abs(qr - qo)) < 5e-3 and np.max(np.abs(vr - vo)) < 5e-3


def test_pd(oracle, refhost):
    from phyz_b200.model import ModelBuilder, SpatialInertia, Transform
    m = (ModelBuilder().gravity([0, 0, -9.81]).dt(0.002)
         .add_revolute_body("link", -1, Transform.identity(),
                            SpatialInertia.new(1.0, [0, 0, -0.5], np.eye(3) * 0.1)).build())
    pd = [PdDof(0, 0, 30.0, 2.0, 25.0)]
    q0, z = np.full((4, 1), 0.3), np.zeros((4, 1))
    t = np.full((4, 1), 0.8)
    qo, _, _, _ = oracle.rollout(m, q0, z, z, 100, pd=pd, targets=t)
    qr, _, _, _ = refhost.rollout(m, q0, z, z, 100, pd=pd, targets=t)
    assert np.max(np.abs(qr - qo)) < 1e-3


def test_contact_drop(oracle, refhost):
    """Penalty contact: the same 500-step sphere drop in both."""
    m = free_sphere(1.0, 0.1)
    q0 = np.zeros((2, 6))
    q0[:, 5] = 0.3
    z = np.zeros((2, 6))
    contact = (0.0, 0.5, 4e4, 400.0)
    qo, vo, _, cso = oracle.rollout(m, q0, z, z, 500, contact=contact)
    qr, vr, _, csr = refhost.rollout(m, q0, z, z, 500, contact=contact)
    assert abs(qo[0, 5] - 0.1) < 0.02
    assert np.max(np.abs(qr - qo)) < 1e-3
    assert abs(csr[0, 0, 7] - cso[0, 0, 7]) < 0.05 * abs(cso[0, 0, 7])
