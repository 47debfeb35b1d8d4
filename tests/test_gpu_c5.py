"""The on-device PPO iteration (phyz_b200/rl.py over the C ABI): returns on
the device against numpy GAE over the read-back history, device-shuffled
updates against host-ordered ones, and whole iterations of the C5 loop."""
import numpy as np
import pytest
import torch

from phyz_b200 import configs
from phyz_b200.rl import C5Cfg, OnDevicePpo
from phyz_b200.train import NetDims, PpoCfg, Trainer

pytestmark = pytest.mark.gpu


def gae_np(r, V, gamma, lam):
    T = r.shape[0]
    adv = np.zeros_like(r)
    A = np.zeros(r.shape[1])
    for t in range(T - 1, -1, -1):
        A = r[t] + gamma * V[t + 1] - V[t] + gamma * lam * A
        adv[t] = A
    return adv, adv + V[:T]


def test_advantages_match_numpy():
    cfg = C5Cfg(nworld=96, steps=6, minibatch=256, epochs=1, precision="f64")
    ppo = OnDevicePpo(cfg)
    ppo.rollout()
    N, T = cfg.nworld, cfg.steps
    for normalize in (False, True):
        st = ppo.sim.policy_advantages(ppo.trainer, None, ppo.coef, cfg.action_penalty, cfg.gamma, cfg.lam, T,
                                       ppo.adv.data_ptr(), ppo.ret.data_ptr(), normalize=normalize)
        obs, out = ppo.sim.readback_policy_history(0, T + 1)  # [t][w][k]
        r = np.einsum("twk,k->tw", obs[1:].astype(np.float64), ppo.coef) - cfg.action_penalty * np.sum(
            out[:T, :, :-1].astype(np.float64) ** 2, axis=2)
        V = torch.zeros((T + 1) * N, dtype=torch.float32, device="cuda")
        h = ppo.sim.policy_history_view()
        ppo.trainer.evaluate(1, (h["obs"], N, h["n_obs"]), (T + 1) * N, V.data_ptr())
        V = V.cpu().numpy().reshape(T + 1, N).astype(np.float64)
        adv, ret = gae_np(r, V, cfg.gamma, cfg.lam)
        assert abs(st[0] - r.sum(0).mean()) <= 1e-4 * abs(st[0]) + 1e-6
        assert abs(st[1] - adv.mean()) <= 1e-4 and abs(st[2] - adv.std()) <= 1e-4 * adv.std()
        got = ppo.adv.cpu().numpy().reshape(T, N)
        want = (adv - adv.mean()) / (adv.std() + 1e-8) if normalize else adv
        assert np.max(np.abs(got - want)) <= 2e-4 * max(1.0, np.max(np.abs(want)))
        assert np.max(np.abs(ppo.ret.cpu().numpy().reshape(T, N) - ret)) <= 2e-4 * np.max(np.abs(ret))
    ppo.close()


def test_shuffled_update_equals_host_ordered_update():
    rng = np.random.default_rng(2)
    A, Cn = NetDims(8, 32, 3), NetDims(8, 32, 1)
    n = 384
    batch = [rng.normal(0, 1, (n, 8)), rng.normal(0, 1, (n, 8)), rng.normal(0, 0.5, (n, 3)),
             rng.normal(-2, 0.3, n), rng.normal(0, 1, n), rng.normal(0, 1, n)]
    pa = np.concatenate([rng.normal(0, 0.3, A.param_count()), np.full(3, -0.7)])
    pc = rng.normal(0, 0.3, Cn.param_count())
    out = []
    for mode in ("host", "device"):
        t = Trainer(A, Cn, n, n)
        t.set_params(0, pa)
        t.set_params(1, pc)
        t.upload_batch(*batch)
        cfg = PpoCfg(minibatch=n, epochs=1)  # one minibatch: the order only permutes rows
        if mode == "host":
            t.update(np.arange(n, dtype=np.uint32)[None], cfg)
        else:
            t.update_shuffled(cfg, seed=77)
        out.append((t.params(0), t.params(1)))
        t.close()
    for a, b in zip(out[0], out[1]):
        assert np.max(np.abs(a - b)) <= 1e-7  # the row order changes only the f32 stage rounding


def test_c5_iterations_run_and_learn_nothing_nonfinite():
    cfg = C5Cfg(nworld=512, steps=8, minibatch=1024, epochs=2)
    ppo = OnDevicePpo(cfg)
    p0 = ppo.trainer.params(0)
    used = []  # the actor each iteration's rollout ran with
    for _ in range(2):
        used.append(ppo.trainer.params(0))
        (ret_mean, adv_mean, adv_std), upd = ppo.iteration()
        assert np.isfinite([ret_mean, adv_mean, adv_std, upd["policy_loss"], upd["value_loss"]]).all()
        assert upd["grad_steps"] == 2 * 4
    assert np.max(np.abs(ppo.trainer.params(0) - p0)) > 0
    ppo.sim.sync()
    # the second rollout's policy is the trainer's actor after the first
    # update: its log-prob of the recorded actions at the bootstrap row
    # matches the f64 MLP of those weights
    p1 = used[1]
    from oracle.policy_oracle import mlp_forward

    obs, out = ppo.sim.readback_policy_history(cfg.steps, 1)
    spec = ppo.spec
    w = p1[:spec.n_weights()]
    std = np.exp(p1[spec.n_weights():])
    # out = mean + std * z; with the recorded z unknown, check the log-prob
    # consistency instead: logp = sum(-0.5 z^2 - log std - 0.5 log 2pi)
    for i in range(8):
        mean = mlp_forward(spec.n_in, spec.hidden, spec.n_out, w, obs[0, i].astype(np.float64))
        z = (out[0, i, :-1] - mean) / std
        logp = np.sum(-0.5 * z * z - np.log(std) - 0.5 * np.log(2 * np.pi))
        assert abs(logp - out[0, i, -1]) <= 1e-3 * max(1, abs(logp))
    ppo.close()
