"""TEST INFRASTRUCTURE ONLY -- the reference's PPO update run on the host:
TrainPipeline::update and DeviceNet::backward_and_step
(crates/phyz-gpu/src/cuda/train.rs:390-472, 655-795) restated as a Python
loop over the reference's own kernel bodies, crates/phyz-gpu/cuda/
phyz_train.cu compiled as host C++ (phyz_train_host_*, walking each grid
serially -- the form the reference's train_parity test pins against its f64
CPU optimizer). Row-major host arrays, as the reference lays them out."""
from __future__ import annotations

import ctypes as C

import numpy as np

_F = C.POINTER(C.c_float)
_D = C.POINTER(C.c_double)
_U = C.POINTER(C.c_uint32)
u = C.c_uint32


def _f(a):
    return a.ctypes.data_as(_F)


def _d(a):
    return a.ctypes.data_as(_D)


class RefTrainer:
    def __init__(self, refhost, actor, critic):
        L = refhost.lib
        self.L = L
        L.phyz_train_host_fwd.argtypes = [u, u, u, u, u, _F, _F, _U, _F, _F, _F]
        L.phyz_train_host_ppo_grad.argtypes = [u, u, u, C.c_float, C.c_float, _F, _F, _F, _F, _F, _U, _F, _F, _F]
        L.phyz_train_host_value_grad.argtypes = [u, u, C.c_float, _F, _F, _U, _F, _F]
        L.phyz_train_host_bwd_hidden.argtypes = [u, u, u, u, _F, _F, _F, _F]
        L.phyz_train_host_grad_w_idx.argtypes = [u, u, u, u, _F, _F, _U, _F, u]
        L.phyz_train_host_grad_w.argtypes = [u, u, u, u, _F, _F, _F, u]
        L.phyz_train_host_grad_b.argtypes = [u, u, u, _F, _F, u]
        L.phyz_train_host_adam.argtypes = [u, u, C.c_double, C.c_double, C.c_double, C.c_double, C.c_double,
                                           C.c_double, C.c_double, _F, _D, _D, _D, _F]
        L.phyz_train_host_reduce_stats.argtypes = [u, u, _F, _F]
        self.nets = [self._net(actor, actor.n_out), self._net(critic, 0)]

    @staticmethod
    def _net(d, extra):
        n = d.param_count() + extra
        return {"d": d, "n": n, "p": np.zeros(n), "m": np.zeros(n), "v": np.zeros(n), "w": np.zeros(n, np.float32),
                "g": np.zeros(n, np.float32), "t": 0, "adam": (3e-4, 0.9, 0.999, 1e-8, 0.0)}

    def set_params(self, which, flat):
        net = self.nets[which]
        net["p"] = np.array(flat, np.float64)
        net["w"] = net["p"].astype(np.float32)

    def params(self, which):
        return self.nets[which]["p"].copy()

    def set_adam(self, actor, critic):
        for net, a in zip(self.nets, (actor, critic)):
            net["adam"] = (a.lr, a.beta1, a.beta2, a.eps, a.weight_decay)

    def _offs(self, d):
        i, h, o = d.n_in, d.n_h, d.n_out
        b1 = h * i
        w2 = b1 + h
        b2 = w2 + h * h
        w3 = b2 + h
        b3 = w3 + o * h
        return b1, w2, b2, w3, b3

    def _fwd(self, net, x, idx, b):
        d = net["d"]
        h1 = np.zeros((b, d.n_h), np.float32)
        h2 = np.zeros((b, d.n_h), np.float32)
        out = np.zeros((b, d.n_out), np.float32)
        self.L.phyz_train_host_fwd(b, b, d.n_in, d.n_h, d.n_out, _f(net["w"]), _f(x), idx.ctypes.data_as(_U),
                                   _f(h1), _f(h2), _f(out))
        return h1, h2, out

    def _backward_and_step(self, net, b, x, idx, h1, h2, dout):
        L, d = self.L, net["d"]
        n_in, n_h, n_out = d.n_in, d.n_h, d.n_out
        ob1, ow2, ob2, ow3, ob3 = self._offs(d)
        w, g = net["w"], net["g"]
        wp = lambda off: w[off:].ctypes.data_as(_F)
        L.phyz_train_host_grad_w(n_out * n_h, b, n_out, n_h, _f(dout), _f(h2), _f(g), ow3)
        L.phyz_train_host_grad_b(n_out, b, n_out, _f(dout), _f(g), ob3)
        dh = np.zeros((b, n_h), np.float32)
        L.phyz_train_host_bwd_hidden(b * n_h, b, n_out, n_h, _f(dout), wp(ow3), _f(h2), _f(dh))
        dout = dh
        L.phyz_train_host_grad_w(n_h * n_h, b, n_h, n_h, _f(dout), _f(h1), _f(g), ow2)
        L.phyz_train_host_grad_b(n_h, b, n_h, _f(dout), _f(g), ob2)
        dh = np.zeros((b, n_h), np.float32)
        L.phyz_train_host_bwd_hidden(b * n_h, b, n_h, n_h, _f(dout), wp(ow2), _f(h1), _f(dh))
        dout = dh
        L.phyz_train_host_grad_w_idx(n_h * n_in, b, n_h, n_in, _f(dout), _f(x), idx.ctypes.data_as(_U), _f(g), 0)
        L.phyz_train_host_grad_b(n_h, b, n_h, _f(dout), _f(g), ob1)
        net["t"] += 1
        lr, b1, b2, eps, wd = net["adam"]
        bc1, bc2 = 1.0 - b1 ** net["t"], 1.0 - b2 ** net["t"]
        L.phyz_train_host_adam(net["n"], net["n"], lr, b1, b2, eps, wd, bc1, bc2, _f(g), _d(net["m"]),
                               _d(net["v"]), _d(net["p"]), _f(w))

    def update(self, batch, order, cfg):
        """batch: (obs_a, obs_c, act, logp_old, adv, ret) row-major f32."""
        obs_a, obs_c, act, logp, adv, ret = [np.ascontiguousarray(x, np.float32) for x in batch]
        n_rows = obs_a.shape[0]
        actor, critic = self.nets
        ad = actor["d"]
        logstd_off = ad.param_count()
        acc = {"policy": 0.0, "value": 0.0, "brake": 0.0, "kl": 0.0, "rows": 0, "batches": 0}
        stopped = False
        for ep in range(cfg.epochs):
            o = np.ascontiguousarray(order[ep], np.uint32)
            for start in range(0, n_rows, cfg.minibatch):
                idx = np.ascontiguousarray(o[start:start + cfg.minibatch])
                b = idx.size
                h1, h2, mean = self._fwd(actor, obs_a, idx, b)
                dmean = np.zeros((b, ad.n_out), np.float32)
                dls = np.zeros((b, ad.n_out), np.float32)
                stats = np.zeros((b, 4), np.float32)
                self.L.phyz_train_host_ppo_grad(b, b, ad.n_out, cfg.clip, cfg.entropy_coef, _f(mean),
                                                actor["w"][logstd_off:].ctypes.data_as(_F), _f(act), _f(logp),
                                                _f(adv), idx.ctypes.data_as(_U), _f(dmean), _f(dls), _f(stats))
                self.L.phyz_train_host_grad_b(ad.n_out, b, ad.n_out, _f(dls), _f(actor["g"]), logstd_off)
                self._backward_and_step(actor, b, obs_a, idx, h1, h2, dmean)
                ch1, ch2, vals = self._fwd(critic, obs_c, idx, b)
                dv = np.zeros((b, 1), np.float32)
                self.L.phyz_train_host_value_grad(b, b, cfg.vdelta, _f(vals), _f(ret), idx.ctypes.data_as(_U),
                                                  _f(dv), _f(stats))
                self._backward_and_step(critic, b, obs_c, idx, ch1, ch2, dv)
                red = np.zeros(4, np.float32)
                self.L.phyz_train_host_reduce_stats(4, b, _f(stats), _f(red))
                ploss, kl_sum, k3_sum, vloss = (float(x) for x in red)
                acc["policy"] += ploss / b
                acc["value"] += vloss / b
                acc["kl"] += kl_sum
                acc["rows"] += b
                brake = (abs(acc["kl"] / max(acc["rows"], 1)) if cfg.kl_mode == 0 else k3_sum / b) / cfg.kl_scale
                acc["brake"] += brake
                acc["batches"] += 1
                if brake > cfg.target_kl:
                    stopped = True
                    break
            if stopped:
                break
        nb = max(acc["batches"], 1)
        return {"policy_loss": acc["policy"] / nb, "value_loss": acc["value"] / nb, "kl": acc["brake"] / nb,
                "grad_steps": acc["batches"], "stopped_early": stopped}
