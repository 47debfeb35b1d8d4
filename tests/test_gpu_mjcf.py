"""A model ingested from MJCF (phyz_b200/mjcf.py) stepping on the sm_100a
kernels: penalty and impulse contact, against the f64 oracle on the same
loaded model."""
import numpy as np
import pytest

from phyz_b200 import BatchSim
from phyz_b200.mjcf import MjcfLoader
from test_mjcf import ROBOT

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("impulse", [False, True])
def test_mjcf_quadruped_matches_the_oracle(oracle, impulse):
    m = MjcfLoader.from_xml_str(ROBOT).build_model()
    n = 16
    q0, v0 = np.zeros((n, m.nv)), np.zeros((n, m.nv))
    q0[:, 5] = np.linspace(0.3, 0.6, n)
    rng = np.random.default_rng(5)
    q0[:, 6:] = rng.uniform(-0.3, 0.3, (n, m.nv - 6))
    c = np.zeros((n, m.nv))
    sim = BatchSim(m, n)
    if impulse:
        sim.enable_contact_impulse(0.0, 1.0)
    else:
        sim.enable_ground_contact(0.0, 2e4, 400.0, 1.0)
    sim.load_states(q0, v0, c)
    q, v, st, dq = q0, v0, None, []
    for _ in range(4):
        sim.step_many(50)
        qg = sim.readback_states()[0]
        if impulse:
            q, v, _, cs, st = oracle.rollout_impulse(m, q, v, c, nsteps=50, contact=(0.0, 1.0), state=st)
        else:
            q, v, _, cs = oracle.rollout(m, q, v, c, nsteps=50, contact=(0.0, 1.0, 2e4, 400.0))
        dq.append(np.max(np.abs(qg - q), axis=1))
    sim.close()
    dq = np.concatenate(dq)
    assert cs[:, :, 0].sum() > 0
    assert np.mean(dq < 1e-8) >= 0.9 and np.max(dq) < 1e-3, np.sort(dq)[-6:]
