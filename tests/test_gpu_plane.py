"""The body-attached contact plane on the sm_100a kernels
(phyzb_enable_contact_terrain / phyzb_enable_contact_impulse with a
phyzb_body_plane): parity with the f64 oracle and, in f32, with the
reference's contact kernel compiled for the host; the reference's own
plane tests (body_plane_contact.rs) on the device; the plane impulses
carried across launches; argument checks."""
import numpy as np
import pytest

from conftest import rel_err
from fixture_models import deck_and_riders, seesaw_and_riders
from phyz_b200 import BatchSim, BodyContactGains, BodyPlane, PhyzbError, _lib
from test_plane_oracle import DECK, PEN, RIDER, deck_rider

pytestmark = pytest.mark.gpu


@pytest.fixture
def plane(oracle, refhost):
    yield
    oracle.set_plane(None)
    refhost.set_plane(None)


def scene(name, n=8):
    if name == "deck":
        m = deck_and_riders(2)
        pl = BodyPlane(body=0, offset=0.02, max_depth=0.05, half_x=0.3, half_y=0.15)
    else:
        m = seesaw_and_riders()
        pl = BodyPlane(body=0, offset=0.02, max_depth=0.05, half_x=0.4, half_y=0.1)
    q0, v0 = np.zeros((n, m.nv)), np.zeros((n, m.nv))
    v0[:, 9] = np.linspace(-0.5, 0.5, n)
    return m, pl, q0, v0, np.zeros((n, m.nv))


def gpu(m, pl, q0, v0, c, chunks, per, precision="f64", impulse=False, k=None, d=None, ground=0.0):
    sim = BatchSim(m, q0.shape[0], precision=precision)
    if impulse:
        sim.enable_contact_impulse(ground, 0.8, plane=pl)
    else:
        kk = k if k is not None else [PEN[2]] * m.nbodies
        dd = d if d is not None else [PEN[3]] * m.nbodies
        sim.enable_contact_terrain(ground, 0.8, [BodyContactGains(a, b) for a, b in zip(kk, dd)], plane=pl)
    sim.load_states(q0, v0, c)
    traj = []
    for _ in range(chunks):
        sim.step_many(per)
        traj.append(sim.readback_states())
    sim.close()
    return traj


@pytest.mark.parametrize("name", ["deck", "seesaw"])
def test_f64_penalty_matches_the_oracle(oracle, plane, name):
    """20-step windows along a 500-step oracle run, the device restarted from
    the oracle's state each time (riders bouncing on stiff springs amplify
    rounding over longer stretches)."""
    m, pl, q, v, c = scene(name)
    oracle.set_plane(pl, m.nbodies)
    sim = BatchSim(m, q.shape[0])
    sim.enable_contact_terrain(0.0, 0.8, [BodyContactGains(PEN[2], PEN[3])] * m.nbodies, plane=pl)
    worst = 0.0
    for _ in range(25):
        sim.load_states(q, v, c)
        sim.step_many(20)
        qg, vg = sim.readback_states()
        q, v, _, _ = oracle.rollout(m, q, v, c, nsteps=20, contact=PEN)
        worst = max(worst, float(np.max(np.abs(qg - q))))
    sim.close()
    assert worst < 1e-9, worst


@pytest.mark.parametrize("name", ["deck", "seesaw"])
def test_f64_impulse_matches_the_oracle(oracle, plane, name):
    m, pl, q, v, c = scene(name)
    oracle.set_plane(pl, m.nbodies)
    tg = gpu(m, pl, q, v, c, 5, 100, impulse=True)
    st, dq = None, []
    for (qg, _) in tg:
        q, v, _, _, st = oracle.rollout_impulse(m, q, v, c, nsteps=100, contact=(0.0, 0.8), state=st)
        dq.append(np.max(np.abs(qg - q), axis=1))
    dq = np.concatenate(dq)
    assert np.mean(dq < 1e-8) >= 0.9 and np.max(dq) < 1e-3, np.sort(dq)[-6:]


@pytest.mark.parametrize("impulse", [False, True])
def test_f32_matches_the_reference_kernel(refhost, plane, impulse):
    m, pl, q, v, c = scene("seesaw", 16)
    refhost.set_plane(pl)
    (qg, _), = gpu(m, pl, q, v, c, 1, 200, precision="f32", impulse=impulse)
    if impulse:
        qr, _, _, _, _ = refhost.rollout_impulse(m, q, v, c, nsteps=200, contact=(0.0, 0.8))
    else:
        qr, _, _, _ = refhost.rollout(m, q, v, c, nsteps=200, contact=PEN)
    assert rel_err(qg, qr) < 1e-3


def test_reference_plane_scenarios_on_the_device():
    """body_plane_contact.rs: the face does not hold what is past its edge,
    a rider settles on the deck, the deck feels the rider (momentum)."""
    m, pl, k, d = deck_rider(-9.81)
    q, v = np.zeros((1, 12)), np.zeros((1, 12))
    q[0, 9] = DECK[0] + RIDER[0] + 0.05
    q[0, 11] = DECK[2] + RIDER[2]
    (_, vo), = gpu(m, pl, q, v, np.zeros((1, 12)), 1, 300, k=k, d=d, ground=-100.0)
    assert vo[0, 11] < -1e-3
    q, v = np.zeros((1, 12)), np.zeros((1, 12))
    q[0, 5] = DECK[2]
    q[0, 11] = 2 * DECK[2] + RIDER[2] + 0.02
    (qo, vo), = gpu(m, pl, q, v, np.zeros((1, 12)), 1, 1500, k=k, d=d)
    assert abs(qo[0, 5] - DECK[2]) < 0.02 and abs(qo[0, 11] - (qo[0, 5] + DECK[2] + RIDER[2])) < 0.02
    assert np.linalg.norm(vo) < 0.05
    m, pl, k, d = deck_rider(0.0)
    q, v = np.zeros((1, 12)), np.zeros((1, 12))
    q[0, 11] = DECK[2] + RIDER[2] + 0.005
    v[0, 11] = -0.5
    (_, vo), = gpu(m, pl, q, v, np.zeros((1, 12)), 1, 400, k=k, d=d, ground=-100.0)
    vd, vr = vo[0, 5], vo[0, 11]
    assert vd < -1e-3 and vr > -0.5 and abs(4.0 * vd + vr + 0.5) < 0.05 * 0.5


def test_plane_impulses_carry_across_launches():
    m, pl, q, v, c = scene("seesaw", 32)
    one = gpu(m, pl, q, v, c, 1, 300, impulse=True)[-1][0]
    many = gpu(m, pl, q, v, c, 30, 10, impulse=True)[-1][0]
    assert rel_err(many, one) < 1e-9


def test_plane_arguments_are_checked():
    m, pl, q, v, c = scene("deck", 2)
    sim = BatchSim(m, 2)
    gains = [BodyContactGains(*PEN[2:])] * m.nbodies
    for bad in (BodyPlane(body=7), BodyPlane(body=0, exclude=(9,))):
        with pytest.raises(PhyzbError) as e:
            sim.enable_contact_terrain(0.0, 0.8, gains, plane=bad)
        assert e.value.code == _lib.ERR_INVALID
    sim.close()
