"""One PPO iteration of the C5 workload entirely on the device: the
quadruped batch under the on-device policy for T control steps, the
returns (rewards, critic values, GAE, advantage normalization over every
rank), and the PPO update of actor and critic on the policy history -- no
sample leaves the GPU. Multi-GPU: one process per GPU, each with its own
block of worlds; NCCL sums the advantage moments, the gradients and the
minibatch statistics, so every rank holds the same networks.

The pieces are the library's (phyz-gpu's policy pass, cuda/mod.rs:1209-1271,
and TrainPipeline, cuda/train.rs); this module only sequences them. The
reward is this workload's own choice: torso height minus 1e-3 |action|^2.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import configs
from .batch_sim import BatchSim
from .parallel import weak_block
from .policy import random_weights
from .train import AdamCfg, NetDims, PpoCfg, Trainer


@dataclass
class C5Cfg:
    nworld: int = 262144
    steps: int = configs.C5_STEPS       # control steps per rollout
    substeps: int = configs.C5_SUBSTEPS  # physics steps per control step
    minibatch: int = 65536
    epochs: int = 1
    gamma: float = 0.99
    lam: float = 0.95
    lr: float = 3e-4
    action_penalty: float = 1e-3
    precision: str = "f32"
    seed: int = configs.C5_SEED


class OnDevicePpo:
    def __init__(self, cfg: C5Cfg, device: int = 0, rank: int = 0, comm=None):
        import torch

        self.cfg, self.comm = cfg, comm
        self.model = configs.quadruped()
        m = self.model
        N, T = cfg.nworld, cfg.steps
        self.sim = BatchSim(m, N, device=device, precision=cfg.precision)
        g, k, d, mu = configs.CONFIGS["c3_quadruped"].contact
        self.sim.enable_ground_contact(g, k, d, mu)
        self.pd = configs.c5_pd_dofs(m)
        self.sim.enable_pd_control(self.pd)
        self.spec = configs.c5_policy_spec(m)
        self.spec.history_steps = T + 1  # + the bootstrap observation
        self.sim.enable_policy(self.spec)
        self.sim.set_policy_base_targets(np.zeros((N, len(self.pd))))
        self.sim.seed_policy(cfg.seed + 0x10001 * rank)
        n_in, n_out = self.spec.n_in, self.spec.n_out
        self.trainer = Trainer(NetDims(n_in, self.spec.hidden, n_out), NetDims(n_in, self.spec.hidden, 1), T * N,
                               cfg.minibatch, device)
        self.trainer.set_adam(AdamCfg(lr=cfg.lr), AdamCfg(lr=cfg.lr))
        # identical random-init weights on every rank
        actor = np.concatenate([random_weights(self.spec, cfg.seed), np.full(n_out, np.log(configs.C5_STD))])
        cspec = type(self.spec)(obs=self.spec.obs, hidden=self.spec.hidden, act_slots=[0], input_noise=None)
        self.trainer.set_params(0, actor)
        self.trainer.set_params(1, random_weights(cspec, cfg.seed + 1))
        if comm is not None:
            self.trainer.set_comm(comm)
        self.sim.policy_sync_from_trainer(self.trainer)
        lo, hi = weak_block(N, rank)
        q0, v0 = configs.initial_state("c3_quadruped", m, np.arange(lo, hi))
        tdt = torch.float32 if cfg.precision == "f32" else torch.float64
        self.q0 = torch.tensor(q0.T.copy(), dtype=tdt, device=f"cuda:{device}")
        self.v0 = torch.tensor(v0.T.copy(), dtype=tdt, device=f"cuda:{device}")
        self.adv = torch.zeros(T * N, dtype=torch.float32, device=f"cuda:{device}")
        self.ret = torch.zeros(T * N, dtype=torch.float32, device=f"cuda:{device}")
        # written on torch's stream; the simulator and trainer use their own
        torch.cuda.synchronize(device)
        self.coef = np.zeros(n_in)
        self.coef[24] = 1.0  # BodyPosZ(torso)
        self.iter = 0
        h = self.sim.policy_history_view()
        b = N
        self.cols = [(h["obs"], b, n_in), (h["obs"], b, n_in), (h["out"], b, n_out + 1),
                     (h["out"] + n_out * N * 4, b, n_out + 1), (self.adv.data_ptr(), b, 1),
                     (self.ret.data_ptr(), b, 1)]

    def rollout(self):
        """Reset to the seeded start state, T control steps, and the bootstrap
        observation (policy row T)."""
        c = self.cfg
        self.sim.load_states_device(self.q0.data_ptr(), self.v0.data_ptr())
        self.sim.policy_rollout(0, c.steps, c.substeps)
        self.sim.run_policy(c.steps)

    def update(self):
        c = self.cfg
        ret_stats = self.sim.policy_advantages(self.trainer, self.comm, self.coef, c.action_penalty, c.gamma, c.lam,
                                               c.steps, self.adv.data_ptr(), self.ret.data_ptr())
        self.trainer.set_batch_device(c.steps * c.nworld, self.cols)
        upd = self.trainer.update_shuffled(PpoCfg(clip=0.2, entropy_coef=0.0, minibatch=c.minibatch,
                                                  epochs=c.epochs), seed=c.seed + self.iter)
        self.sim.policy_sync_from_trainer(self.trainer)
        self.iter += 1
        return ret_stats, upd

    def iteration(self):
        self.rollout()
        return self.update()

    def close(self):
        self.trainer.close()
        self.sim.close()
