"""Host side of the device-resident PPO update (TrainPipeline,
crates/phyz-gpu/src/cuda/train.rs:474-810) over the C ABI's phyzb_trainer."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check


@dataclass
class NetDims:
    n_in: int
    n_h: int
    n_out: int

    def param_count(self) -> int:
        i, h, o = self.n_in, self.n_h, self.n_out
        return h * i + h + h * h + h + o * h + o


@dataclass
class AdamCfg:
    lr: float = 3e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.0


KL_CUMULATIVE, KL_MINIBATCH = 0, 1


@dataclass
class PpoCfg:
    clip: float = 0.2
    entropy_coef: float = 0.0
    vdelta: float = float("inf")
    minibatch: int = 4096
    epochs: int = 4
    target_kl: float = float("inf")
    kl_scale: float = 1.0
    kl_mode: int = KL_CUMULATIVE


class Trainer:
    """Actor (with a trailing log_std block) and critic MLPs on one GPU."""

    def __init__(self, actor: NetDims, critic: NetDims, capacity: int, max_minibatch: int, device: int = 0):
        self._lib = _lib.load()
        self.actor, self.critic = actor, critic
        h = C.c_void_p()
        d = lambda n: _lib.PhyzbNetDims(n.n_in, n.n_h, n.n_out)
        check(self._lib.phyzb_trainer_create(int(device), d(actor), d(critic), int(capacity), int(max_minibatch),
                                             C.byref(h)))
        self._h = h

    def n_params(self, which: int) -> int:
        return self.actor.param_count() + self.actor.n_out if which == 0 else self.critic.param_count()

    def set_adam(self, actor: AdamCfg, critic: AdamCfg) -> None:
        a = _lib.PhyzbAdamCfg(actor.lr, actor.beta1, actor.beta2, actor.eps, actor.weight_decay)
        c = _lib.PhyzbAdamCfg(critic.lr, critic.beta1, critic.beta2, critic.eps, critic.weight_decay)
        check(self._lib.phyzb_trainer_set_adam(self._h, C.byref(a), C.byref(c)))

    def set_params(self, which: int, flat) -> None:
        f = np.ascontiguousarray(flat, np.float64)
        check(self._lib.phyzb_trainer_set_params(self._h, int(which), _lib.dptr(f), int(f.size)))

    def params(self, which: int) -> np.ndarray:
        out = np.zeros(self.n_params(which))
        check(self._lib.phyzb_trainer_params(self._h, int(which), _lib.dptr(out), int(out.size)))
        return out

    def upload_batch(self, obs_a, obs_c, act, logp_old, adv, ret) -> None:
        cols = [np.ascontiguousarray(x, np.float32) for x in (obs_a, obs_c, act, logp_old, adv, ret)]
        fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))
        check(self._lib.phyzb_trainer_upload_batch(self._h, int(cols[0].shape[0]), *[fp(c) for c in cols]))

    def update(self, order, cfg: PpoCfg) -> dict:
        o = np.ascontiguousarray(order, np.uint32)
        c = _lib.PhyzbPpoCfg(cfg.clip, cfg.entropy_coef, cfg.vdelta, int(cfg.minibatch), int(cfg.epochs),
                             cfg.target_kl, cfg.kl_scale, int(cfg.kl_mode))
        st = _lib.PhyzbUpdateStats()
        check(self._lib.phyzb_trainer_update(self._h, o.ctypes.data_as(C.POINTER(C.c_uint32)), int(o.shape[0]),
                                             C.byref(c), C.byref(st)))
        return {"policy_loss": st.policy_loss, "value_loss": st.value_loss, "kl": st.kl,
                "grad_steps": st.grad_steps, "stopped_early": bool(st.stopped_early)}

    # ── device-resident batches (the collector feeding the update) ─────────
    def set_batch_device(self, n_rows: int, cols) -> None:
        """cols: 6 (device_ptr, block, features) triples: obs_a, obs_c, act,
        logp_old, adv, ret in blocked SoA (pz BatchCol)."""
        arr = (_lib.PhyzbBatchCol * 6)(*[_lib.PhyzbBatchCol(int(p), int(b), int(f)) for p, b, f in cols])
        check(self._lib.phyzb_trainer_set_batch_device(self._h, int(n_rows), arr))

    def update_shuffled(self, cfg: PpoCfg, seed: int) -> dict:
        c = _lib.PhyzbPpoCfg(cfg.clip, cfg.entropy_coef, cfg.vdelta, int(cfg.minibatch), int(cfg.epochs),
                             cfg.target_kl, cfg.kl_scale, int(cfg.kl_mode))
        st = _lib.PhyzbUpdateStats()
        check(self._lib.phyzb_trainer_update_shuffled(self._h, C.byref(c), C.c_uint64(seed & (2 ** 64 - 1)),
                                                      C.byref(st)))
        return {"policy_loss": st.policy_loss, "value_loss": st.value_loss, "kl": st.kl,
                "grad_steps": st.grad_steps, "stopped_early": bool(st.stopped_early)}

    def evaluate(self, which: int, x_col, n_rows: int, out_ptr: int) -> None:
        p, b, f = x_col
        check(self._lib.phyzb_trainer_evaluate(self._h, int(which), _lib.PhyzbBatchCol(int(p), int(b), int(f)),
                                               int(n_rows), C.c_void_p(int(out_ptr))))

    def set_comm(self, comm) -> None:
        check(self._lib.phyzb_trainer_set_comm(self._h, comm._h if comm is not None else None))

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.phyzb_trainer_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gae_noalloc(rewards_ptr: int, values_ptr: int, nworld: int, steps: int, gamma: float, lam: float, adv_ptr: int,
                ret_ptr: int, normalize: bool = True, device: int = 0, stream: int = 0) -> tuple:
    """GAE and advantage normalization over caller-owned device float
    buffers (rewards [steps][nworld], values [steps + 1][nworld], adv and ret
    [steps][nworld]) without any device allocation by the library: for
    callers whose framework owns the GPU's memory or whose loop must not stall
    on cudaMalloc/cudaFree. Scratch is a fixed static device array, so nworld
    is capped at _lib.GAE_NOALLOC_MAX_WORLDS, and calls that overlap on one
    device race on it. Returns (mean return per world, advantage mean,
    advantage std before normalization)."""
    lib = _lib.load()
    st = np.zeros(3)
    check(lib.phyzb_gae_noalloc(C.c_void_p(int(rewards_ptr)), C.c_void_p(int(values_ptr)), int(nworld), int(steps),
                                float(gamma), float(lam), int(bool(normalize)), int(device),
                                C.c_void_p(int(stream)) if stream else None, C.c_void_p(int(adv_ptr)),
                                C.c_void_p(int(ret_ptr)), _lib.dptr(st)))
    return tuple(st)
