"""The control-loop oracle (oracle/policy_oracle.py, f64) pinned against the
reference's own observation and policy kernels compiled as host C++
(phyz_host_fk / phyz_host_obs / phyz_host_policy, phyz_kernels.cu:1809-1835):
the random stream exactly, the observation row and the policy step to f32
rounding."""
import numpy as np
import pytest

from oracle import policy_oracle as po
from phyz_b200 import ObsOp, PolicySpec, configs
from phyz_b200.policy import pack_obs_ops, random_weights


def c5_state(n, seed=7):
    m = configs.quadruped()
    q, v = configs.initial_state("c3_quadruped", m, range(n))
    rng = np.random.default_rng(seed)
    q[:, :3] = rng.uniform(-0.4, 0.4, (n, 3))  # tilted torso: every op reads something non-trivial
    q[:, 3:5] = rng.uniform(-1, 1, (n, 2))
    v = rng.normal(0, 0.5, v.shape)
    return m, q, v


def test_world_seed_and_stream_match_the_reference_kernel(refhost):
    """Zero weights, unit std, no AR(1): each action is one draw of the
    world's stream, cast to f32 -- identical to the oracle's KernelRng."""
    n, k = 16, 6
    spec = PolicySpec(obs=[ObsOp.const(0.0)], hidden=2, act_slots=list(range(k)), act_clamp=10.0,
                      input_noise=[0.0])
    w = np.zeros(spec.n_weights())
    for seed in (0, 0x5EED, 2 ** 63 + 12345):
        st = np.array([po.world_seed(seed, i) for i in range(n)], np.uint64)
        _, out, _, st_after, _ = refhost.policy(spec, w, np.ones(k), np.zeros((n, 1)), st, np.zeros((n, k)),
                                                np.zeros((n, k)))
        for i in range(n):
            r = po.KernelRng(po.world_seed(seed, i))
            draws = np.array([r.normal() for _ in range(k)], np.float32)
            assert np.array_equal(out[i, :k], draws)
            assert int(st_after[i]) == r.s


def test_observation_row_matches_the_reference_kernel(oracle, refhost):
    m, q, v = c5_state(32)
    spec = configs.c5_policy_spec(m)
    table, aux = pack_obs_ops(spec.obs)
    ref = refhost.observe(m, q, v, table, aux)
    ours = po.observe(oracle, m, q, v, spec.obs)
    assert np.max(np.abs(ref - ours)) < 2e-5, np.max(np.abs(ref - ours))


def test_policy_step_matches_the_reference_kernel(refhost):
    n = 24
    spec = PolicySpec(obs=[ObsOp.const(0.0)] * 10, hidden=48, act_slots=[3, 0, 5, 1], act_clamp=0.4,
                      act_clamp_slots=[0.3, 0.5, 0.2, 1.0], noise_rho=0.6,
                      input_noise=[0.0, 0.1, 0.0, 0.2, 0.0, 0.0, 0.05, 0.0, 0.0, 0.3])
    w = random_weights(spec, 11, scale=2.0)
    w[-4:] = [0.1, -0.2, 0.3, 0.0]
    std = np.array([0.2, 0.5, 0.3, 0.8])
    rng = np.random.default_rng(3)
    obs = rng.normal(0, 1, (n, 10))
    z = rng.normal(0, 1, (n, 4))
    base = rng.normal(0, 0.5, (n, 6))
    st = np.array([po.world_seed(99, i) for i in range(n)], np.uint64)
    t_ref, out_ref, obs_ref, st_ref, z_ref = refhost.policy(spec, w, std, obs, st, z, base)
    for i in range(n):
        r = po.KernelRng(po.world_seed(99, i))
        o, zi, tg = obs[i].copy(), z[i].copy(), np.zeros(6)
        act, logp = po.policy_reference(spec, w, std, r, o, zi, base[i], tg)
        assert int(st_ref[i]) == r.s
        assert np.max(np.abs(obs_ref[i] - o)) < 1e-6
        assert np.max(np.abs(out_ref[i, :4] - act)) < 2e-5 * max(1.0, np.max(np.abs(act)))
        assert abs(out_ref[i, 4] - logp) < 2e-5 * max(1.0, abs(logp))
        assert np.max(np.abs(t_ref[i] - tg)) < 2e-5
        assert np.max(np.abs(z_ref[i] - zi)) < 1e-6
