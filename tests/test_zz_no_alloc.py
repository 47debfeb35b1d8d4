"""phyzb_gae_noalloc, the returns entry point that allocates no device memory
(for callers whose framework owns the GPU's memory or whose loop must not
stall on cudaMalloc/cudaFree), against phyzb_policy_advantages, the entry
point that computes the same GAE with scratch it allocates itself.

Collected last on purpose (the name sorts after every other test file): the
entry point keeps its scratch in one static device array shared by every
call, so this file also checks that two calls in a row -- the second one
reading the array the first one left behind -- give the same answers as the
allocating path, after whatever the other tests did on the device."""
import ctypes as C

import numpy as np
import pytest

from phyz_b200 import _lib
from phyz_b200.train import gae_noalloc


def test_sizes_past_the_static_limit_are_rejected_before_device_use():
    lib = _lib.load()
    st = np.zeros(3)
    # non-null stand-ins: the call rejects the size before it looks at the
    # device or at these addresses
    fake = C.c_void_p(16)
    code = lib.phyzb_gae_noalloc(fake, fake, _lib.GAE_NOALLOC_MAX_WORLDS + 1, 4, 0.99, 0.95, 1, 0, None, fake,
                                 fake, _lib.dptr(st))
    assert code == _lib.ERR_TOO_LARGE
    assert b"static scratch limit" in lib.phyzb_last_error()
    assert lib.phyzb_gae_noalloc(None, fake, 8, 4, 0.99, 0.95, 1, 0, None, fake, fake, None) == _lib.ERR_INVALID
    assert lib.phyzb_gae_noalloc(fake, fake, 8, 0, 0.99, 0.95, 1, 0, None, fake, fake, None) == _lib.ERR_INVALID


def gae_np(r, V, gamma, lam):
    """GAE over [t][w] rows in f64 (the recursion of phyz_train.cu's returns)."""
    adv = np.zeros_like(r)
    A = np.zeros(r.shape[1])
    for t in range(r.shape[0] - 1, -1, -1):
        A = r[t] + gamma * V[t + 1] - V[t] + gamma * lam * A
        adv[t] = A
    return adv, adv + V[:r.shape[0]]


@pytest.mark.gpu
def test_two_calls_in_a_row_match_the_allocating_entry_point():
    """1000 worlds (four GAE blocks of partial sums in the static array), then
    300 worlds (two blocks: the partials the first batch left past them must
    be ignored); two calls per batch, each against the allocating entry
    point and against numpy GAE."""
    import torch

    from phyz_b200.rl import C5Cfg, OnDevicePpo

    for N in (1000, 300):
        cfg = C5Cfg(nworld=N, steps=6, minibatch=2 * N, epochs=1)
        ppo = OnDevicePpo(cfg)
        ppo.rollout()
        # reward = torso height of the next observation and no action penalty:
        # with a one-hot coefficient the allocating path's reward kernel yields
        # that observation column exactly, so both paths see identical rewards
        j = int(np.flatnonzero(ppo.coef)[0])
        assert ppo.coef[j] == 1.0 and np.count_nonzero(ppo.coef) == 1
        h = ppo.sim.policy_history_view()
        for steps, normalize in ((cfg.steps, False), (cfg.steps - 2, True)):
            adv_ref = torch.zeros(steps * N, dtype=torch.float32, device="cuda")
            ret_ref = torch.zeros_like(adv_ref)
            st_ref = ppo.sim.policy_advantages(ppo.trainer, None, ppo.coef, 0.0, cfg.gamma, cfg.lam, steps,
                                               adv_ref.data_ptr(), ret_ref.data_ptr(), normalize=normalize)
            obs, _ = ppo.sim.readback_policy_history(0, steps + 1)  # [t][w][k]
            r_host = np.ascontiguousarray(obs[1:, :, j])
            rewards = torch.from_numpy(r_host).cuda()
            values = torch.zeros((steps + 1) * N, dtype=torch.float32, device="cuda")
            ppo.trainer.evaluate(1, (h["obs"], N, h["n_obs"]), (steps + 1) * N, values.data_ptr())
            adv = torch.full_like(adv_ref, float("nan"))
            ret = torch.full_like(adv_ref, float("nan"))
            stream = torch.cuda.current_stream().cuda_stream
            torch.cuda.synchronize()
            st = gae_noalloc(rewards.data_ptr(), values.data_ptr(), N, steps, cfg.gamma, cfg.lam, adv.data_ptr(),
                             ret.data_ptr(), normalize=normalize, stream=stream)
            torch.cuda.synchronize()
            # the same kernels on the same inputs: equal up to the tolerance the
            # returns tests use for device-vs-device comparisons
            a, ar = adv.cpu().numpy(), adv_ref.cpu().numpy()
            r, rr = ret.cpu().numpy(), ret_ref.cpu().numpy()
            assert np.all(np.isfinite(a)) and np.all(np.isfinite(r))
            assert np.max(np.abs(a - ar)) <= 1e-6 * max(1.0, np.max(np.abs(ar)))
            assert np.max(np.abs(r - rr)) <= 1e-6 * max(1.0, np.max(np.abs(rr)))
            np.testing.assert_allclose(st, st_ref, rtol=1e-9, atol=1e-12)
            # and on its own against numpy GAE in f64 (test_gpu_c5's tolerances)
            V = values.cpu().numpy().reshape(steps + 1, N).astype(np.float64)
            adv_np, ret_np = gae_np(r_host.astype(np.float64), V, cfg.gamma, cfg.lam)
            want = (adv_np - adv_np.mean()) / (adv_np.std() + 1e-8) if normalize else adv_np
            assert np.max(np.abs(a.reshape(steps, N) - want)) <= 2e-4 * max(1.0, np.max(np.abs(want)))
            assert np.max(np.abs(r.reshape(steps, N) - ret_np)) <= 2e-4 * np.max(np.abs(ret_np))
            assert abs(st[1] - adv_np.mean()) <= 1e-4 and abs(st[2] - adv_np.std()) <= 1e-4 * adv_np.std()
        ppo.close()
