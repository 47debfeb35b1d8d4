"""The body-attached contact plane (BodyPlane, contact_pipeline.rs:318-355;
phyz_kernels.cu:983-1132) in the f64 oracle, pinned against the reference's
contact kernel compiled for the host (oracle/_ref): a free deck with riders
and a hinged plank (whose frame the kernel relabels), penalty and impulse
mode, over 100-step windows restarted from the oracle's state; plus the
plane's own rules (the face's extent, the exclude list, the depth guard)."""
import numpy as np
import pytest

from fixture_models import deck_and_riders, seesaw_and_riders
from phyz_b200 import BodyPlane
from test_impulse_oracle import as_ref_state

PEN = (0.0, 0.8, 2e3, 40.0)


@pytest.fixture
def plane(oracle, refhost):
    yield
    oracle.set_plane(None)
    refhost.set_plane(None)


def scene(name):
    if name == "deck":
        m = deck_and_riders(2)
        pl = BodyPlane(body=0, offset=0.02, max_depth=0.05, half_x=0.3, half_y=0.15)
    else:
        m = seesaw_and_riders()
        pl = BodyPlane(body=0, offset=0.02, max_depth=0.05, half_x=0.4, half_y=0.1)
    n = 4
    q0, v0 = np.zeros((n, m.nv)), np.zeros((n, m.nv))
    v0[:, 9] = np.linspace(-0.5, 0.5, n)  # the first rider's sideways speed
    return m, pl, q0, v0, np.zeros((n, m.nv))


@pytest.mark.parametrize("name", ["deck", "seesaw"])
@pytest.mark.parametrize("impulse", [False, True])
def test_matches_the_reference_kernel(oracle, refhost, plane, name, impulse):
    """10-step windows along a 500-step oracle run, the reference restarted
    from the oracle's state each time: riders bouncing on stiff contacts
    amplify f32-vs-f64 rounding over longer stretches, so nearly every world
    agrees to rounding and none by more than a small bound."""
    m, pl, q, v, c = scene(name)
    n, nb = q.shape[0], m.nbodies
    oracle.set_plane(pl, nb)
    refhost.set_plane(pl)
    st = None
    dq = []
    for _ in range(50):
        if impulse:
            qr, _, _, _, _ = refhost.rollout_impulse(m, q, v, c, nsteps=10, contact=(0.0, 0.8),
                                                     state=None if st is None else as_ref_state(st, n, nb))
            q, v, _, _, st = oracle.rollout_impulse(m, q, v, c, nsteps=10, contact=(0.0, 0.8), state=st)
        else:
            qr, _, _, _ = refhost.rollout(m, q, v, c, nsteps=10, contact=PEN)
            q, v, _, _ = oracle.rollout(m, q, v, c, nsteps=10, contact=PEN)
        dq.append(np.max(np.abs(q - qr), axis=1))
    dq = np.concatenate(dq)
    assert np.mean(dq < 1e-6) >= 0.9 and np.max(dq) < 1e-3, np.sort(dq)[-6:]


# The reference's own plane tests (crates/phyz-gpu/tests/body_plane_contact.rs),
# restated on the oracle: a deck box (0.8 x 0.4 x 0.1 m, 4 kg) and a rider
# cube (0.2 m, 1 kg), both free, penalty gains BodyContactGains::
# uniform_frequency(omega = 50, zeta = 1): k = m omega^2, d = 2 zeta m omega.
DECK, RIDER = (0.4, 0.2, 0.05), (0.1, 0.1, 0.1)


def deck_rider(gravity):
    from phyz_b200.model import Geometry, Joint, ModelBuilder, SpatialInertia

    def box(mass, h):
        lx, ly, lz = 2 * h[0], 2 * h[1], 2 * h[2]
        return SpatialInertia.new(mass, np.zeros(3), np.diag([mass / 12 * (ly * ly + lz * lz),
                                                              mass / 12 * (lx * lx + lz * lz),
                                                              mass / 12 * (lx * lx + ly * ly)]))

    b = ModelBuilder().gravity([0.0, 0.0, gravity]).dt(0.001)
    b.add_body("deck", -1, Joint.free(), box(4.0, DECK), geometry=Geometry.box(*DECK))
    b.add_body("rider", -1, Joint.free(), box(1.0, RIDER), geometry=Geometry.box(*RIDER))
    m = b.build()
    k = np.array([4.0 * 50.0 ** 2, 1.0 * 50.0 ** 2])
    d = np.array([2.0 * 4.0 * 50.0, 2.0 * 1.0 * 50.0])
    return m, BodyPlane(body=0, offset=DECK[2], max_depth=0.05, half_x=DECK[0], half_y=DECK[1]), k, d


def test_the_face_does_not_support_what_is_past_its_edge(oracle, plane):
    m, pl, k, d = deck_rider(-9.81)
    oracle.set_plane(pl, m.nbodies)
    q, v = np.zeros((1, 12)), np.zeros((1, 12))
    q[0, 9] = DECK[0] + RIDER[0] + 0.05
    q[0, 11] = DECK[2] + RIDER[2]
    q, v, _, _ = oracle.rollout(m, q, v, np.zeros((1, 12)), nsteps=300, contact=(-100.0, 0.8, k, d))
    assert v[0, 11] < -1e-3


def test_a_rider_settles_on_the_deck(oracle, plane):
    m, pl, k, d = deck_rider(-9.81)
    oracle.set_plane(pl, m.nbodies)
    q, v = np.zeros((1, 12)), np.zeros((1, 12))
    q[0, 5] = DECK[2]
    q[0, 11] = 2 * DECK[2] + RIDER[2] + 0.02
    q, v, _, _ = oracle.rollout(m, q, v, np.zeros((1, 12)), nsteps=1500, contact=(0.0, 0.8, k, d))
    deck_z, rider_z = q[0, 5], q[0, 11]
    assert abs(deck_z - DECK[2]) < 0.02
    assert abs(rider_z - (deck_z + DECK[2] + RIDER[2])) < 0.02
    assert np.linalg.norm(v) < 0.05


def test_the_deck_feels_the_rider(oracle, plane):
    m, pl, k, d = deck_rider(0.0)
    oracle.set_plane(pl, m.nbodies)
    q, v = np.zeros((1, 12)), np.zeros((1, 12))
    q[0, 11] = DECK[2] + RIDER[2] + 0.005
    v[0, 11] = -0.5
    q, v, _, _ = oracle.rollout(m, q, v, np.zeros((1, 12)), nsteps=400, contact=(-100.0, 0.8, k, d))
    vd, vr = v[0, 5], v[0, 11]
    assert vd < -1e-3 and vr > -0.5
    p0, p1 = 1.0 * -0.5, 4.0 * vd + 1.0 * vr
    assert abs(p1 - p0) < 0.05 * abs(p0)


def test_exclude_list(oracle, plane):
    m, pl, k, d = deck_rider(-9.81)
    pl.exclude = (1,)
    oracle.set_plane(pl, m.nbodies)
    q, v = np.zeros((1, 12)), np.zeros((1, 12))
    q[0, 5] = DECK[2]
    q[0, 11] = 2 * DECK[2] + RIDER[2] + 0.02
    q, v, _, _ = oracle.rollout(m, q, v, np.zeros((1, 12)), nsteps=1500, contact=(0.0, 0.8, k, d))
    assert q[0, 11] < RIDER[2] + 0.01  # the excluded rider falls through the deck to the ground
