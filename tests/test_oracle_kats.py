"""Pins the f64 oracle to the reference's own known-answer tests.

Each test restates one of phyz's CPU tests (cited) with its tolerance.
"""
import numpy as np
import pytest

from fixture_models import armature_chain, double_pendulum, free_base_with_limb, rod
from phyz_b200.model import GRAVITY, Joint, ModelBuilder, SpatialInertia, Transform

G = 9.81


def test_analytic_offset_double_pendulum(oracle):
    """tests/joint_offset_vs_cpu.rs:43-71: CPU ABA == closed form to 1e-9."""
    m = double_pendulum()
    theta = 0.4
    qdd = oracle.aba(m, np.array([[theta, 0.0]]), np.zeros((1, 2)))[0]
    m11, m12, m22 = 4.0 / 3.0, 0.5, 1.0 / 3.0
    t1, t2 = -1.5 * GRAVITY * np.sin(theta), -0.5 * GRAVITY * np.sin(theta)
    det = m11 * m22 - m12 * m12
    a1 = (m22 * t1 - m12 * t2) / det
    a2 = (m11 * t2 - m12 * t1) / det
    assert abs(qdd[0] - a1) < 1e-9 and abs(qdd[1] - (a2 - a1)) < 1e-9


def _aba_test_pendulum(nlinks):
    b = ModelBuilder().gravity([0.0, -GRAVITY, 0.0]).dt(0.001)
    b.add_revolute_body("link1", -1, Transform.identity(), rod(1.0, 0.5))
    if nlinks == 2:
        b.add_revolute_body("link2", 0, Transform.from_translation([0.0, -1.0, 0.0]), rod(1.0, 0.5))
    return b.build()


def test_double_pendulum_equilibrium(oracle):
    """aba.rs:523-530."""
    m = _aba_test_pendulum(2)
    qdd = oracle.aba(m, np.zeros((1, 2)), np.zeros((1, 2)))[0]
    assert np.all(np.abs(qdd) < 1e-10)


def test_aba_rnea_consistency(oracle):
    """aba.rs:532-548: RNEA(ABA(q, v, 0)) = 0 to 1e-10."""
    m = _aba_test_pendulum(2)
    q, v = np.array([[0.3, 0.2]]), np.array([[0.1, -0.1]])
    qdd = oracle.aba(m, q, v)
    tau = oracle.rnea(m, q, v, qdd)
    assert np.all(np.abs(tau) < 1e-10)


def test_aba_rnea_consistency_tree(oracle):
    """The same identity on a floating base with a limb (multi-DOF path)."""
    m = free_base_with_limb()
    q = np.array([[0.2, -0.1, 0.3, 0.1, 0.2, 0.5, 0.4]])
    v = np.array([[0.3, 0.1, -0.2, -0.2, 0.4, 0.1, 1.0]])
    ctrl = np.array([[0.0] * 6 + [0.7]])
    qdd = oracle.aba(m, q, v, ctrl)
    tau = oracle.rnea(m, q, v, qdd)
    assert np.all(np.abs(tau - ctrl) < 1e-10)


def test_single_pendulum(oracle):
    """aba.rs:550-578: qdd = -(m g L/2) / (m L^2/3) at pi/2."""
    m = _aba_test_pendulum(1)
    qdd = oracle.aba(m, np.array([[np.pi / 2]]), np.zeros((1, 1)))[0, 0]
    assert abs(qdd - (-(GRAVITY * 0.5) / (1.0 / 3.0))) < 1e-6


def test_free_fall(oracle):
    """aba.rs:580-608 and free_joint.rs:46-55."""
    m = (ModelBuilder().gravity([0, 0, -GRAVITY]).add_free_body("ball", -1, Transform.identity(),
                                                                 SpatialInertia.sphere(1.0, 0.1)).build())
    qdd = oracle.aba(m, np.zeros((1, 6)), np.zeros((1, 6)))[0]
    assert np.all(np.abs(qdd[:5]) < 1e-10) and abs(qdd[5] + GRAVITY) < 1e-6


def _unit_free_body(gravity, inertia=None):
    return (ModelBuilder().gravity(gravity).dt(0.001)
            .add_body("b", -1, Joint.free(), SpatialInertia.new(1.0, [0, 0, 0], inertia if inertia is not None
                                                               else np.eye(3))).build())


def test_free_body_falls_and_does_not_yaw(oracle):
    """free_joint.rs:57-85: z = 1 - g/2 (t^2 + t dt) to 1e-9, no yaw."""
    m = _unit_free_body([0, 0, -G])
    q = np.zeros((1, 6))
    q[0, 5] = 1.0
    steps = 200
    q1, v1, _, _ = oracle.rollout(m, q, np.zeros((1, 6)), np.zeros((1, 6)), steps)
    t = 0.2
    assert abs(q1[0, 5] - (1.0 - 0.5 * G * (t * t + t * m.dt))) < 1e-9
    assert np.all(np.abs(q1[0, :5]) < 1e-14)
    assert abs(v1[0, 5] + G * t) < 1e-9


def test_free_body_spin_is_exact(oracle):
    """free_joint.rs:87-132: torque-free spin about a principal axis."""
    m = _unit_free_body([0, 0, 0], np.diag([1.0, 1.0, 2.0]))
    v = np.zeros((1, 6))
    v[0, 2] = 3.0
    q1, v1, _, _ = oracle.rollout(m, np.zeros((1, 6)), v, np.zeros((1, 6)), 1000)
    assert np.all(np.abs(v1[0, :2]) < 1e-9) and abs(v1[0, 2] - 3.0) < 1e-9
    ang = q1[0, 2]
    wrapped = ((3.0 + np.pi) % (2 * np.pi)) - np.pi
    assert np.all(np.abs(q1[0, :2]) < 1e-9) and abs(ang - wrapped) < 1e-9
    assert np.all(np.abs(q1[0, 3:]) < 1e-12)


def test_free_joint_linear_velocity_is_body_frame(oracle):
    """free_joint.rs:134-156."""
    m = _unit_free_body([0, 0, 0])
    q = np.zeros((1, 6))
    q[0, 2] = np.pi / 2
    v = np.zeros((1, 6))
    v[0, 3] = 1.0
    q1 = oracle.integrate_configuration(m, q, v, 1.0)
    assert abs(q1[0, 3]) < 1e-12 and abs(q1[0, 4] - 1.0) < 1e-12 and abs(q1[0, 5]) < 1e-12


def test_hinge_integrates_scalar(oracle):
    """integrate.rs:100-117: v = 0.2, q = 0.02."""
    m = (ModelBuilder().dt(0.01).add_revolute_body("l", -1, Transform.identity(),
                                                   SpatialInertia.point_mass(1.0, [0, 0, -0.5])).build())
    q = oracle.integrate_configuration(m, np.zeros((1, 1)), np.array([[0.2]]), 0.1)
    assert abs(q[0, 0] - 0.02) < 1e-12


def test_armature_mass_matrix(oracle):
    """free_joint.rs:176-232: M qdd + bias = 0 with armature (M from RNEA
    columns: the armature is on the D diagonal of ABA, so add it here)."""
    m = armature_chain()
    q, v = np.array([[0.3, -0.7]]), np.array([[0.9, -1.4]])
    qdd = oracle.aba(m, q, v)[0]
    bias = oracle.rnea(m, q, v, np.zeros((1, 2)))[0]
    M = np.zeros((2, 2))
    for j in range(2):
        e = np.zeros((1, 2))
        e[0, j] = 1.0
        M[:, j] = oracle.rnea(m, q, np.zeros((1, 2)), e)[0] - oracle.rnea(m, q, np.zeros((1, 2)), np.zeros((1, 2)))[0]
    M += np.diag([0.37, 0.11])
    assert np.all(np.abs(M @ qdd + bias) < 1e-9)


def test_penalty_contact_rest_force(oracle):
    """A sphere resting exactly at depth f = m g / k gets the weight back
    (phyz_kernels.cu:939-965 law at rest)."""
    from fixture_models import free_sphere
    m = free_sphere(1.0, 0.1)
    k = 4e4
    depth = 9.81 / k
    q = np.zeros((1, 6))
    q[0, 5] = 0.1 - depth
    ext, cs = oracle.penalty_contact(m, q, np.zeros((1, 6)), 0.0, 0.5, k, 400.0)
    assert abs(ext[0, 0, 5] - 9.81) < 1e-9
    assert cs[0, 0, 0] == 1.0 and abs(cs[0, 0, 1] - depth) < 1e-15


@pytest.mark.parametrize("name", ["c1_double_pendulum", "c2_chain32", "c3_quadruped", "c4_humanoid"])
def test_energy_conserved_without_damping(oracle, name):
    """Sanity of every config model: with no control and no contact, total
    energy drifts by far less than its scale over 200 small steps."""
    from phyz_b200 import configs
    cfg = configs.CONFIGS[name]
    m = cfg.builder()
    m.dt = 1e-4
    q0, v0 = configs.initial_state(name, m, range(4))
    if name in ("c3_quadruped", "c4_humanoid"):
        q0[:, 5] += 10.0  # far above the ground
    ke0, pe0 = oracle.energy(m, q0, v0)
    q1, v1, _, _ = oracle.rollout(m, q0, v0, np.zeros_like(q0), 200)
    ke1, pe1 = oracle.energy(m, q1, v1)
    e0, e1 = ke0 + pe0, ke1 + pe1
    scale = np.abs(ke0) + np.abs(pe0) + 1.0
    assert np.all(np.abs(e1 - e0) / scale < 1e-3), (e0, e1)
