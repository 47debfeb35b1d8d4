"""Heightfield terrain on the sm_100a kernels (phyzb_enable_contact_terrain,
phyzb_enable_contact_impulse with a heightfield, phyzb_set_heightfield):
parity with the f64 oracle and, in f32, with the reference's contact kernel
compiled for the host; the 1 x 1 field against the flat ground; replacing
the field in place; both record layouts."""
import numpy as np
import pytest

from conftest import rel_err
from phyz_b200 import BatchSim, BodyContactGains, Heightfield, PhyzbError, _lib, configs

pytestmark = pytest.mark.gpu

K, D = 1e4, 100.0


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


def inputs(name, n):
    m = configs.CONFIGS[name].builder()
    q0, v0 = configs.initial_state(name, m, range(n))
    q0[:, 3] = np.linspace(-1.0, 1.0, n)  # spread over the bumps
    return m, q0, v0, np.zeros((n, m.nv))


def gains(m):
    return [BodyContactGains(K, D)] * m.nbodies


def gpu(m, q0, v0, c, hf, chunks, per, precision="f64", impulse=False):
    sim = BatchSim(m, q0.shape[0], precision=precision)
    if impulse:
        sim.enable_contact_impulse(0.0, 1.0, heightfield=hf)
    else:
        sim.enable_contact_terrain(0.0, 1.0, gains(m), heightfield=hf)
    sim.load_states(q0, v0, c)
    traj = []
    for _ in range(chunks):
        sim.step_many(per)
        traj.append(sim.readback_states()[0])
    cs = sim.readback_contacts()
    sim.close()
    return traj, cs


def host(engine, m, q0, v0, c, chunks, per, impulse=False):
    traj, st, q, v = [], None, q0, v0
    for _ in range(chunks):
        if impulse:
            q, v, _, cs, st = engine.rollout_impulse(m, q, v, c, nsteps=per, contact=(0.0, 1.0), state=st)
        else:
            q, v, _, cs = engine.rollout(m, q, v, c, nsteps=per, contact=(0.0, 1.0, K, D))
        traj.append(q)
    return traj, cs


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
@pytest.mark.parametrize("impulse", [False, True])
def test_f64_matches_the_oracle(oracle, terrain, name, impulse):
    m, q0, v0, c = inputs(name, 16)
    hf = bumpy()
    oracle.set_heightfield(hf)
    tg, csg = gpu(m, q0, v0, c, hf, 4, 50, impulse=impulse)
    to, cso = host(oracle, m, q0, v0, c, 4, 50, impulse=impulse)
    assert cso[:, :, 0].sum() > 0
    dq = np.stack([np.max(np.abs(a - b), axis=1) for a, b in zip(tg, to)])
    assert np.mean(dq < 1e-8) >= 0.9, np.sort(dq.ravel())[-6:]
    assert np.max(dq) < 1e-3
    ok = dq[-1] < 1e-8
    assert np.max(np.abs(csg[ok] - cso[ok])) < 1e-6 * max(1.0, np.max(np.abs(cso)))


def test_f32_matches_the_reference_kernel(refhost, terrain):
    m, q0, v0, c = inputs("c3_quadruped", 64)
    hf = bumpy()
    refhost.set_heightfield(hf)
    tg, csg = gpu(m, q0, v0, c, hf, 1, 100, precision="f32")
    tr, csr = host(refhost, m, q0, v0, c, 1, 100)
    assert csr[:, :, 0].sum() > 0 and np.array_equal(csg[:, :, 0], csr[:, :, 0])
    assert rel_err(tg[-1], tr[-1]) < 1e-3


def test_one_node_field_is_the_flat_ground():
    m, q0, v0, c = inputs("c3_quadruped", 32)
    out = []
    for hf in (None, Heightfield.flat(0.1)):
        sim = BatchSim(m, 32)
        sim.enable_contact_terrain(0.1, 1.0, gains(m), heightfield=hf)
        sim.load_states(q0, v0, c)
        sim.step_many(200)
        out.append((sim.readback_states()[0], sim.readback_contacts()))
        sim.close()
    assert rel_err(out[1][0], out[0][0]) < 1e-10
    assert np.max(np.abs(out[1][1] - out[0][1])) < 1e-6


def test_set_heightfield_replaces_the_terrain():
    m, q0, v0, c = inputs("c3_quadruped", 16)
    a, b = bumpy(3), bumpy(4)
    sim = BatchSim(m, 16)
    with pytest.raises(PhyzbError) as e:
        sim.set_heightfield(a)  # contact off
    assert e.value.code == _lib.ERR_STATE
    sim.enable_contact_terrain(0.0, 1.0, gains(m), heightfield=a)
    sim.set_heightfield(b)
    sim.load_states(q0, v0, c)
    sim.step_many(150)
    swapped = sim.readback_states()[0]
    with pytest.raises(PhyzbError) as e:
        sim.set_heightfield(Heightfield.new((0.0, 0.0, 0.0), 0.1, 18, 18))  # larger than the first field
    assert e.value.code == _lib.ERR_INVALID
    sim.close()
    fresh, _ = gpu(m, q0, v0, c, b, 1, 150)
    assert np.array_equal(swapped, fresh[-1])
    other, _ = gpu(m, q0, v0, c, a, 1, 150)
    assert np.max(np.abs(other[-1] - fresh[-1])) > 1e-3


def test_tensor_memory_layout_agrees(monkeypatch):
    m, q0, v0, c = inputs("c3_quadruped", 256)
    hf = bumpy()
    res = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("PHYZB_TMEM", mode)
        for impulse in (False, True):
            tr, _ = gpu(m, q0, v0, c, hf, 1, 100, precision="f32", impulse=impulse)
            res[(mode, impulse)] = tr[-1]
    for impulse in (False, True):
        assert rel_err(res[("1", impulse)], res[("0", impulse)]) < 1e-3
