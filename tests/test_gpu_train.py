"""The device PPO update (phyzb_trainer_*) against the reference's own update
kernels run on the host (oracle/train_oracle.py over phyz_train.cu compiled
as host C++), at the reference's train_parity tolerances
(crates/phyz-gpu/tests/train_parity.rs:440-500): weight deltas within 2e-4
relative after one update and 1e-3 after three, losses within 1e-4, and the
KL brake stopping both sides on the same minibatch."""
import numpy as np
import pytest

from oracle.train_oracle import RefTrainer
from phyz_b200 import PhyzbError
from phyz_b200 import _lib
from phyz_b200.train import AdamCfg, NetDims, PpoCfg, Trainer

pytestmark = pytest.mark.gpu

ACTOR = NetDims(10, 32, 4)
CRITIC = NetDims(12, 24, 1)


def make(seed=0, n=600):
    rng = np.random.default_rng(seed)
    pa = np.concatenate([rng.normal(0, 0.4, ACTOR.param_count()), np.full(ACTOR.n_out, -0.5)])
    pc = rng.normal(0, 0.4, CRITIC.param_count())
    batch = (rng.normal(0, 1, (n, ACTOR.n_in)), rng.normal(0, 1, (n, CRITIC.n_in)),
             rng.normal(0, 0.6, (n, ACTOR.n_out)), rng.normal(-3.0, 0.5, n), rng.normal(0, 1, n),
             rng.normal(0, 2, n))
    return pa, pc, [np.asarray(x, np.float32) for x in batch]


def gap(before, a, b):
    da, db = a - before, b - before
    return np.linalg.norm(da - db) / max(np.linalg.norm(db), 1e-30)


def run_both(refhost, iters, cfg, seed=0):
    pa, pc, batch = make(seed)
    n = batch[0].shape[0]
    dev = Trainer(ACTOR, CRITIC, n, cfg.minibatch)
    ref = RefTrainer(refhost, ACTOR, CRITIC)
    for t in (dev, ref):
        t.set_params(0, pa)
        t.set_params(1, pc)
        t.set_adam(AdamCfg(lr=1e-3), AdamCfg(lr=2e-3))
    dev.upload_batch(*batch)
    rng = np.random.default_rng(seed + 1)
    out = []
    for it in range(iters):
        order = np.stack([rng.permutation(n) for _ in range(cfg.epochs)]).astype(np.uint32)
        sd = dev.update(order, cfg)
        sr = ref.update(batch, order, cfg)
        out.append((sd, sr))
    res = (pa, pc, dev.params(0), dev.params(1), ref.params(0), ref.params(1), out)
    dev.close()
    return res


def test_one_update_matches_the_reference(refhost):
    cfg = PpoCfg(clip=0.2, entropy_coef=0.01, vdelta=1.5, minibatch=128, epochs=2)
    pa, pc, da, dc, ra, rc, st = run_both(refhost, 1, cfg)
    assert gap(pa, da, ra) < 2e-4, gap(pa, da, ra)
    assert gap(pc, dc, rc) < 2e-4, gap(pc, dc, rc)
    sd, sr = st[0]
    assert sd["grad_steps"] == sr["grad_steps"] == 10
    assert abs(sd["policy_loss"] - sr["policy_loss"]) <= 1e-4 * max(abs(sr["policy_loss"]), 1e-12)
    assert abs(sd["value_loss"] - sr["value_loss"]) <= 1e-4 * abs(sr["value_loss"])
    assert abs(sd["kl"] - sr["kl"]) <= 1e-3 * max(abs(sr["kl"]), 1e-9)


def test_three_updates_track_the_reference(refhost):
    cfg = PpoCfg(clip=0.2, entropy_coef=0.0, vdelta=float("inf"), minibatch=256, epochs=3)
    pa, pc, da, dc, ra, rc, st = run_both(refhost, 3, cfg, seed=4)
    assert gap(pa, da, ra) < 1e-3 and gap(pc, dc, rc) < 1e-3
    for sd, sr in st:
        assert abs(sd["policy_loss"] - sr["policy_loss"]) <= 1e-3 * max(abs(sr["policy_loss"]), 1e-9)
        assert abs(sd["value_loss"] - sr["value_loss"]) <= 1e-3 * abs(sr["value_loss"])


def test_kl_brake_stops_both_sides_on_the_same_minibatch(refhost):
    cfg = PpoCfg(clip=0.2, minibatch=64, epochs=4, target_kl=0.002, kl_mode=1)
    *_, st = run_both(refhost, 1, cfg, seed=9)
    sd, sr = st[0]
    assert sr["stopped_early"] and sd["stopped_early"]
    assert sd["grad_steps"] == sr["grad_steps"] < 40


def test_trainer_errors():
    with pytest.raises(PhyzbError) as e:
        Trainer(ACTOR, NetDims(12, 24, 2), 100, 32)
    assert e.value.code == _lib.ERR_INVALID
    t = Trainer(ACTOR, CRITIC, 100, 32)
    with pytest.raises(PhyzbError):
        t.set_params(0, np.zeros(3))
    pa, pc, batch = make(n=100)
    t.upload_batch(*batch)
    with pytest.raises(PhyzbError):
        t.update(np.zeros((1, 100), np.uint32), PpoCfg(minibatch=64, epochs=2))
    with pytest.raises(PhyzbError):
        t.update(np.zeros((1, 100), np.uint32), PpoCfg(minibatch=64000, epochs=1))
    t.close()
