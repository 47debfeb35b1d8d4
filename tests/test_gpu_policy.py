"""The on-device control loop through the C ABI (phyzb_enable_policy ...
phyzb_policy_rollout) against the f64 oracle (oracle/policy_oracle.py) and
the reference's own f32 kernels compiled as host C++: kinematics readout,
observation row, policy step (actions, log-prob, PD targets, the random
stream), and closed-loop control steps."""
import numpy as np
import pytest

from conftest import rel_err
from oracle import policy_oracle as po
from phyz_b200 import BatchSim, ObsOp, PhyzbError, PolicySpec, configs
from phyz_b200 import _lib
from phyz_b200.policy import pack_obs_ops, random_weights

pytestmark = pytest.mark.gpu


def c5_sim(n, precision, seed=7):
    m = configs.quadruped()
    q, v = configs.initial_state("c3_quadruped", m, range(n))
    rng = np.random.default_rng(seed)
    q[:, :3] = rng.uniform(-0.4, 0.4, (n, 3))
    q[:, 3:5] = rng.uniform(-1, 1, (n, 2))
    v = rng.normal(0, 0.5, v.shape)
    sim = BatchSim(m, n, precision=precision)
    pd = configs.c5_pd_dofs(m)
    sim.enable_pd_control(pd)
    spec = configs.c5_policy_spec(m)
    spec.history_steps = 8
    spec.input_noise = [0.0] * 20 + [0.05] * 10
    spec.noise_rho = 0.5
    sim.enable_policy(spec)
    w = random_weights(spec, 5, scale=1.5)
    std = np.linspace(0.1, 0.6, spec.n_out)
    base = rng.normal(0, 0.2, (n, len(pd)))
    sim.set_policy_weights(w)
    sim.set_policy_std(std)
    sim.set_policy_base_targets(base)
    sim.seed_policy(1234)
    sim.load_states(q, v)
    return m, sim, spec, pd, w, std, base, q, v


@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_kinematics_readout(oracle, precision):
    m, sim, *_ , q, v = c5_sim(40, precision)
    xf = sim.readback_kinematics()
    xw, vel = oracle.forward_kinematics(m, q, v)
    tol = 1e-12 if precision == "f64" else 2e-6
    assert rel_err(xf[:, :, :12], xw) <= tol
    assert rel_err(xf[:, :, 12:], vel) <= tol * 10
    sim.close()


@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_policy_step_matches_oracle_and_reference(oracle, refhost, precision):
    n = 48
    m, sim, spec, pd, w, std, base, q, v = c5_sim(n, precision)
    for step in range(3):  # the stream and the AR(1) state carry across calls
        sim.run_policy(step)
    obs, out = sim.readback_policy_history(0, 3)
    targets = sim.readback_targets()
    # oracle: the same three policy calls on the unchanged state
    obs0 = po.observe(oracle, m, q, v, spec.obs)
    for i in range(n):
        r = po.KernelRng(po.world_seed(1234, i))
        z = np.zeros(spec.n_out)
        tg = np.zeros(len(pd))
        for step in range(3):
            o = obs0[i].copy()
            act, logp = po.policy_reference(spec, w, std, r, o, z, base[i], tg)
            assert np.max(np.abs(obs[step, i] - o)) < 5e-5, (step, i)
            assert np.max(np.abs(out[step, i, :spec.n_out] - act)) < 5e-4, (step, i)
            assert abs(out[step, i, -1] - logp) < 5e-4 * max(1, abs(logp))
        assert np.max(np.abs(targets[i] - tg)) < 5e-4
    # the reference's own f32 kernels, first call
    table, aux = pack_obs_ops(spec.obs)
    ref_obs = refhost.observe(m, q, v, table, aux)
    st = np.array([po.world_seed(1234, i) for i in range(n)], np.uint64)
    _, ref_out, ref_obs_noised, _, _ = refhost.policy(spec, w, std, ref_obs, st, np.zeros((n, spec.n_out)), base)
    assert np.max(np.abs(obs[0] - ref_obs_noised)) < 5e-5
    assert np.max(np.abs(out[0] - ref_out)) < 5e-4
    sim.close()


def test_policy_rollout_closed_loop(oracle):
    """Control steps on device (policy -> PD targets -> 2 physics steps) vs
    the same loop on the host with the oracle's dynamics and policy."""
    n, steps, sub = 24, 4, 2
    m, sim, spec, pd, w, std, base, q, v = c5_sim(n, "f64")
    sim.policy_rollout(0, steps, sub)
    qd, vd = sim.readback_states()
    qo, vo = q.copy(), v.copy()
    rngs = [po.KernelRng(po.world_seed(1234, i)) for i in range(n)]
    z = np.zeros((n, spec.n_out))
    tg = np.zeros((n, len(pd)))
    for c in range(steps):
        ob = po.observe(oracle, m, qo, vo, spec.obs)
        for i in range(n):
            po.policy_reference(spec, w, std, rngs[i], ob[i], z[i], base[i], tg[i])
        qo, vo, _, _ = oracle.rollout(m, qo, vo, np.zeros_like(qo), sub, pd=pd, targets=tg)
    assert rel_err(qd, qo) < 1e-4, rel_err(qd, qo)
    assert rel_err(vd, vo) < 1e-3, rel_err(vd, vo)
    sim.close()


def test_policy_errors():
    m = configs.quadruped()
    sim = BatchSim(m, 8, precision="f32")
    spec = configs.c5_policy_spec(m)
    with pytest.raises(PhyzbError) as e:
        sim.enable_policy(spec)
    assert e.value.code == _lib.ERR_STATE  # needs PD
    sim.enable_pd_control(configs.c5_pd_dofs(m))
    bad = PolicySpec(obs=[ObsOp.v(99)], hidden=8, act_slots=[0], input_noise=[0.0])
    with pytest.raises(PhyzbError) as e:
        sim.enable_policy(bad)
    assert e.value.code == _lib.ERR_INVALID
    wide = PolicySpec(obs=[ObsOp.const(1.0)], hidden=200, act_slots=[0], input_noise=[0.0])
    with pytest.raises(PhyzbError) as e:
        sim.enable_policy(wide)
    assert e.value.code == _lib.ERR_UNSUPPORTED
    spec.history_steps = 2
    sim.enable_policy(spec)
    with pytest.raises(PhyzbError) as e:
        sim.run_policy(0)
    assert e.value.code == _lib.ERR_STATE  # no weights yet
    sim.set_policy_weights(random_weights(spec, 1))
    sim.set_policy_std(np.full(spec.n_out, 0.2))
    with pytest.raises(PhyzbError) as e:
        sim.run_policy(2)
    assert e.value.code == _lib.ERR_INVALID
    with pytest.raises(PhyzbError):
        sim.set_policy_weights(np.zeros(5))
    sim.run_policy(1)
    sim.sync()
    sim.close()
