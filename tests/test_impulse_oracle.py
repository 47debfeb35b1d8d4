"""The impulse-mode contact restatement (oracle/phyz_oracle.hpp, f64)
pinned against the reference's own contact kernel compiled for the host
(phyz_kernels.cu, f32, solve_mode 1, the sweep sequence of cuda/mod.rs:
902-927), and the behaviour the reference's impulse parity tests assert
(crates/phyz-gpu/tests/contact_impulse_parity.rs): a dropped box lands and
rests, a sliding box stops, a light body stays finite. The reference's CPU
convex solver those tests compare with (phyz-contact) cannot be built here,
so its resting place is not a pin; the reference kernel is."""
import numpy as np
import pytest

from fixture_models import free_box
from oracle.oracle import IMPULSE_PTS, impulse_material, solref_erp_from
from phyz_b200 import _lib, configs

SCENARIOS = {  # contact_impulse_parity.rs:126-186: initial v, mass
    "dropped": ([0.0] * 6, 1.0),
    "sliding": ([0.0, 0.0, 0.0, 2.0, 0.0, 0.0], 1.0),
    "light": ([3.0, 0.0, 0.0, 2.0, 0.0, 0.0], 0.1),
}


def test_constants_match_the_reference():
    # DEFAULT_CONTACT_SWEEPS (gpu_batch_simulator.rs:31); solref error
    # reduction (contact_pipeline.rs:229-237) with MuJoCo's default SolRef
    assert _lib.DEFAULT_CONTACT_SWEEPS == 16
    for dt in (1e-4, 1e-3, 2e-3, 1e-2):
        assert abs(solref_erp_from(0.02, 1.0, dt) - dt / (0.04 + dt)) < 1e-15
    # GroundContactParams::default's value, evaluated at dt = 1 ms
    assert abs(solref_erp_from(0.02, 1.0, 0.001) - 0.001 / (2.0 * 0.02 + 0.001)) < 1e-18
    assert impulse_material(0.002)[1:] == [0.001, 0.0, 0.05, 0.9, 0.95, 0.001, 0.5, 2.0]


def roll_box(engine, name, steps, chunk=100, sweeps=16):
    v0, mass = SCENARIOS[name]
    m = free_box(mass=mass)
    q, v = np.zeros((1, 6)), np.array([v0], float)
    ctrl = np.zeros((1, 6))
    st = None
    traj = []
    for _ in range(steps // chunk):
        q, v, _, cs, st = engine.rollout_impulse(m, q, v, ctrl, nsteps=chunk, contact=(0.0, 0.8), state=st,
                                                 sweeps=sweeps)
        traj.append(q[0, 3:6].copy())
    return np.array(traj), v, cs


@pytest.mark.parametrize("name", list(SCENARIOS))
def test_box_scenarios_match_the_reference_kernel(oracle, refhost, name):
    to, vo, cso = roll_box(oracle, name, 1500)
    tr, vr, csr = roll_box(refhost, name, 1500)
    assert np.all(np.isfinite(to)) and np.all(np.isfinite(tr))
    # f64 restatement vs the f32 reference kernel over 1500 steps
    assert np.max(np.abs(to - tr)) < 2e-5
    assert np.max(np.abs(cso - csr)) < 1e-3 * 9.81


def test_dropped_box_rests_on_its_face(oracle):
    traj, v, cs = roll_box(oracle, "dropped", 1500)
    # joint frame at z = 0.5: the box centre rests at its half extent, inside
    # the contact margin, holding its weight (no mg/k sag of a penalty spring)
    z = 0.5 + traj[-1, 2]
    assert abs(z - 0.1) < 1e-3
    assert np.max(np.abs(v)) < 1e-3
    assert cs[0, 0, 0] == 1.0 and abs(cs[0, 0, 7] - 9.81) < 1e-6


def test_sliding_box_stops(oracle):
    traj, v, _ = roll_box(oracle, "sliding", 1500)
    assert np.max(np.abs(v)) < 1e-3  # real stiction, no creep
    assert abs(traj[-1, 0] - traj[-5, 0]) < 1e-6


def test_sweep_count_changes_the_solve_and_both_engines_agree(oracle, refhost):
    for sweeps in (1, 4):
        to, _, _ = roll_box(oracle, "sliding", 600, sweeps=sweeps)
        tr, _, _ = roll_box(refhost, "sliding", 600, sweeps=sweeps)
        assert np.max(np.abs(to - tr)) < 2e-5
    a, _, _ = roll_box(oracle, "sliding", 600, sweeps=1)
    b, _, _ = roll_box(oracle, "sliding", 600, sweeps=16)
    assert np.max(np.abs(a - b)) > 1e-4


def as_ref_state(st, n, nb):
    """The oracle's warm-start state in the reference's buffers: ext_forces
    [n][nb][6] and contact_state [n][nb][56] with the ground impulses at
    CS_IMPULSE_OFF = 8 and the plane's at CS_PLANE_OFF = 32
    (phyz_kernels.cu:502-505)."""
    ext = st[:, :nb * 6].reshape(n, nb, 6).astype(np.float32)
    cs = np.zeros((n, nb, 56), np.float32)
    g = nb * 6 + nb * 3 * IMPULSE_PTS
    cs[:, :, 8:8 + 3 * IMPULSE_PTS] = st[:, nb * 6:g].reshape(n, nb, 3 * IMPULSE_PTS)
    cs[:, :, 32:32 + 3 * IMPULSE_PTS] = st[:, g:].reshape(n, nb, 3 * IMPULSE_PTS)  # CS_PLANE_OFF
    return ext, cs


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
def test_articulated_contact_matches_the_reference_kernel(oracle, refhost, name):
    """Every 50 steps of an oracle run, the reference kernel restarts from the
    oracle's state and warm start, and both take 10 steps. A contact point
    whose depth sits at the margin (or a tangential impulse at the cone's
    edge) can switch one way in f32 and the other in f64, and a run of many
    contacts amplifies that, so the agreement is checked over short windows
    along the trajectory: nearly every world agrees to f32 rounding, and a
    world that met such a switch stays within a small bound."""
    m = configs.CONFIGS[name].builder()
    n, nb = 12, m.nbodies
    q, v = configs.initial_state(name, m, range(n))
    if name == "c3_quadruped":
        q[:, 5] = np.linspace(0.3, 0.5, n)  # feet reach the ground within the run
    ctrl = np.zeros((n, m.nv))
    st = None
    touched = 0.0
    dq_all = []
    for _ in range(6):
        q, v, _, _, st = oracle.rollout_impulse(m, q, v, ctrl, nsteps=50, contact=(0.0, 1.0), state=st, nthreads=4)
        qo, vo, _, cso, _ = oracle.rollout_impulse(m, q, v, ctrl, nsteps=10, contact=(0.0, 1.0), state=st,
                                                   nthreads=4)
        qr, vr, _, csr, _ = refhost.rollout_impulse(m, q, v, ctrl, nsteps=10, contact=(0.0, 1.0),
                                                    state=as_ref_state(st, n, nb), nthreads=4)
        touched += cso[:, :, 0].sum()
        dq_all.append(np.max(np.abs(qo - qr), axis=1))
    dq = np.concatenate(dq_all)
    assert touched > 0
    assert np.mean(dq < 2e-6) >= 0.9, np.sort(dq)[-8:]
    assert np.max(dq) < 1e-3, np.sort(dq)[-8:]
    # the warm-start state has the layout the oracle documents
    assert st.shape == (n, nb * 6 + 2 * nb * IMPULSE_PTS * 3)
