"""Heightfield terrain in the f64 oracle: its sampling pinned by the
reference's own heightfield tests (crates/phyz-model/src/heightfield.rs
flat / bilinear / clamp / ramp-normal / origin cases, which the GPU's
sampler phyz_kernels.cu:625-664 restates), and penalty and impulse contact
on a bumpy field against the reference's contact kernel compiled for the
host (oracle/_ref)."""
import numpy as np
import pytest

from phyz_b200 import Heightfield, configs
from test_impulse_oracle import as_ref_state


@pytest.fixture
def terrain(oracle, refhost):
    yield
    oracle.set_heightfield(None)
    refhost.set_heightfield(None)


def bumpy(seed=3, n=17):
    rng = np.random.default_rng(seed)
    hf = Heightfield.new((-2.0, -2.0, -0.05), 0.25, n, n)
    hf.heights[:] = (0.08 * rng.standard_normal(n * n)).astype(np.float32)
    return hf


def test_sampling_matches_the_reference_heightfield_tests(oracle, terrain):
    oracle.set_heightfield(Heightfield.flat(0.25))
    for x, y in ((0.0, 0.0), (-1e3, 42.0), (7.5, -7.5)):
        h, n = oracle.terrain_at(x, y)
        assert h == 0.25 and np.array_equal(n, [0.0, 0.0, 1.0])
    hf = Heightfield.new((0.0, 0.0, 0.0), 1.0, 2, 2)
    hf.heights[:] = [0.0, 1.0, 2.0, 3.0]  # h(x, y) = x + 2y on [0, 1]^2
    oracle.set_heightfield(hf)
    assert abs(oracle.terrain_at(0.5, 0.5)[0] - 1.5) < 1e-12
    assert abs(oracle.terrain_at(0.25, 0.75)[0] - 1.75) < 1e-12
    assert abs(oracle.terrain_at(5.0, 0.0)[0] - 1.0) < 1e-12  # clamped beyond the border
    assert abs(oracle.terrain_at(-5.0, -5.0)[0]) < 1e-12
    ramp = Heightfield.new((0.0, 0.0, 0.0), 1.0, 3, 2)
    ramp.heights[:] = [0.0, 1.0, 2.0, 0.0, 1.0, 2.0]  # 45 degrees along x
    oracle.set_heightfield(ramp)
    n = oracle.terrain_at(1.0, 0.5)[1]
    assert np.linalg.norm(n - np.array([-1.0, 0.0, 1.0]) / np.sqrt(2.0)) < 1e-12
    assert np.array_equal(oracle.terrain_at(100.0, 0.0)[1], [0.0, 0.0, 1.0])
    oracle.set_heightfield(Heightfield.new((10.0, -3.0, 2.0), 0.5, 1, 1))
    assert oracle.terrain_at(0.0, 0.0)[0] == 2.0


def test_flat_field_is_the_flat_ground(oracle, terrain):
    m = configs.quadruped()
    n = 8
    q0, v0 = configs.initial_state("c3_quadruped", m, range(n))
    c = np.zeros((n, m.nv))
    flat = oracle.rollout(m, q0, v0, c, nsteps=200, contact=(0.1, 1.0, 1e4, 100.0))
    oracle.set_heightfield(Heightfield.flat(0.1))
    field = oracle.rollout(m, q0, v0, c, nsteps=200, contact=(0.0, 1.0, 1e4, 100.0))
    assert np.array_equal(flat[0], field[0]) and np.array_equal(flat[3], field[3])


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
def test_penalty_on_a_heightfield_matches_the_reference_kernel(oracle, refhost, terrain, name):
    m = configs.CONFIGS[name].builder()
    n = 8
    q0, v0 = configs.initial_state(name, m, range(n))
    q0[:, 3] = np.linspace(-1.0, 1.0, n)  # spread over the bumps
    c = np.zeros((n, m.nv))
    hf = bumpy()
    oracle.set_heightfield(hf)
    refhost.set_heightfield(hf)
    qo, vo, _, cso = oracle.rollout(m, q0, v0, c, nsteps=100, contact=(0.0, 1.0, 1e4, 100.0))
    qr, vr, _, csr = refhost.rollout(m, q0, v0, c, nsteps=100, contact=(0.0, 1.0, 1e4, 100.0))
    assert cso[:, :, 0].sum() > 0 and np.array_equal(cso[:, :, 0], csr[:, :, 0])
    assert np.max(np.abs(qo - qr)) < 1e-4
    # the contact point sits on the terrain, not on the plane z = 0
    touching = cso[:, :, 0] == 1.0
    assert np.max(np.abs(cso[touching][:, 4])) > 1e-3
    assert np.max(np.abs(cso[:, :, 2:5] - csr[:, :, 2:5])) < 1e-4


def test_impulse_on_a_heightfield_matches_the_reference_kernel(oracle, refhost, terrain):
    m = configs.quadruped()
    n, nb = 8, m.nbodies
    q, v = configs.initial_state("c3_quadruped", m, range(n))
    q[:, 3] = np.linspace(-1.0, 1.0, n)
    c = np.zeros((n, m.nv))
    hf = bumpy()
    oracle.set_heightfield(hf)
    refhost.set_heightfield(hf)
    st = None
    dq_all, touched = [], 0.0
    for _ in range(4):
        q, v, _, _, st = oracle.rollout_impulse(m, q, v, c, nsteps=50, contact=(0.0, 1.0), state=st)
        qo, _, _, cso, _ = oracle.rollout_impulse(m, q, v, c, nsteps=10, contact=(0.0, 1.0), state=st)
        qr, _, _, csr, _ = refhost.rollout_impulse(m, q, v, c, nsteps=10, contact=(0.0, 1.0),
                                                   state=as_ref_state(st, n, nb))
        touched += cso[:, :, 0].sum()
        dq_all.append(np.max(np.abs(qo - qr), axis=1))
    dq = np.concatenate(dq_all)
    assert touched > 0
    assert np.mean(dq < 2e-6) >= 0.9 and np.max(dq) < 1e-3, np.sort(dq)[-6:]
