"""TEST INFRASTRUCTURE ONLY -- f64 restatement of phyz-gpu's on-device
control loop (crates/phyz-gpu/src/policy_pipeline.rs): the per-world random
stream (world_seed, KernelRng: :420-471), the observation ops (ObsOp::eval:
:180-245, centre_of_mass: :255-270), the MLP forward (mlp_forward: :475-497)
and one world's policy step (policy_reference: :505-539). Kinematics come
from the f64 oracle (forward_kinematics, phyz-rigid's FK). Plain numpy and
Python loops: small cases only. Used by tests/ only."""
from __future__ import annotations

import math

import numpy as np

MASK = (1 << 64) - 1


def world_seed(seed: int, world: int) -> int:
    """policy_pipeline.rs:420-428: SplitMix64 of (seed, world), zero-guarded."""
    z = (seed + 0x9E3779B97F4A7C15 * (world + 1)) & MASK
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK
    z ^= z >> 31
    return z if z else 1


class KernelRng:
    """policy_pipeline.rs:434-471: xorshift64 + Box-Muller."""

    def __init__(self, state: int):
        self.s = state & MASK

    def next_u64(self) -> int:
        x = self.s
        x ^= (x << 13) & MASK
        x ^= x >> 7
        x ^= (x << 17) & MASK
        self.s = x
        return x

    def uniform(self) -> float:
        return (self.next_u64() >> 11) / float(1 << 53)

    def normal(self) -> float:
        u1 = self.uniform()
        u2 = self.uniform()
        return math.sqrt(-2.0 * math.log(max(u1, 1e-300))) * math.cos(2.0 * math.pi * u2)


def _point(xw, b, o):
    """Body-frame point of body b in world (rot is world->body)."""
    R = xw[b, :9].reshape(3, 3)
    return xw[b, 9:12] + R.T @ np.asarray(o, np.float64)


def centre_of_mass(model, xw):
    num, den = np.zeros(3), 0.0
    for i, b in enumerate(model.bodies):
        m = b.inertia.mass
        if m <= 0.0:
            continue
        num += _point(xw, i, b.inertia.com) * m
        den += m
    return num / den if den > 0 else np.zeros(3)


def eval_op(op, model, q, v, xw) -> float:
    """ObsOp::eval for one world (policy_pipeline.rs:180-245)."""
    k = op.kind
    if k == 0:
        return op.c
    if k == 1:
        return q[int(op.a)] - op.c
    if k == 2:
        return v[int(op.a)]
    R = xw[int(op.a), :9].reshape(3, 3) if k in (3, 4, 5) else None
    if k == 3:
        return math.atan2(-R[0, 2], R[2, 2])
    if k == 4:
        return math.atan2(R[1, 2], R[2, 2])
    if k == 5:
        e = op.c - math.atan2(R[0, 1], R[0, 0])
        while e > math.pi:
            e -= 2 * math.pi
        while e < -math.pi:
            e += 2 * math.pi
        return e
    if k == 6:
        return xw[int(op.a), 11]
    if k == 7:
        return xw[int(op.a), 9 + min(int(op.b), 2)]
    if k == 8:
        if not op.support:
            return 0.0
        tgt = sum(_point(xw, b, o) for b, o in op.support) / len(op.support)
        e = centre_of_mass(model, xw) - tgt
        axis = int(op.c)
        if op.heading_body is None:
            return e[axis]
        Rh = xw[op.heading_body, :9].reshape(3, 3)
        yaw = math.atan2(Rh[0, 1], Rh[0, 0])
        sy, cy = math.sin(yaw), math.cos(yaw)
        return [cy * e[0] + sy * e[1], -sy * e[0] + cy * e[1], e[2]][axis]
    raise ValueError(k)


def observe(oracle, model, q, v, ops) -> np.ndarray:
    """observe_reference for every world: FK, then the ops. [n][n_in]."""
    xw, _ = oracle.forward_kinematics(model, q, v)
    return np.array([[eval_op(op, model, q[w], v[w], xw[w]) for op in ops] for w in range(q.shape[0])])


def mlp_forward(n_in, n_h, n_out, weights, x):
    w = np.asarray(weights, np.float64)
    o = 0
    W1 = w[o:o + n_h * n_in].reshape(n_h, n_in); o += n_h * n_in
    b1 = w[o:o + n_h]; o += n_h
    W2 = w[o:o + n_h * n_h].reshape(n_h, n_h); o += n_h * n_h
    b2 = w[o:o + n_h]; o += n_h
    W3 = w[o:o + n_out * n_h].reshape(n_out, n_h); o += n_out * n_h
    b3 = w[o:o + n_out]
    h1 = np.tanh(b1 + W1 @ x)
    h2 = np.tanh(b2 + W2 @ h1)
    return b3 + W3 @ h2


def policy_reference(spec, weights, std, rng: KernelRng, obs, z, base_targets, targets):
    """One world (policy_pipeline.rs:505-539): obs, z, targets updated in
    place; returns (actions, logp)."""
    noise = spec.input_noise if spec.input_noise is not None else [0.0] * spec.n_in
    for i in range(spec.n_in):
        if noise[i] != 0.0:
            obs[i] += noise[i] * rng.normal()
    targets[:] = base_targets
    mean = mlp_forward(spec.n_in, spec.hidden, spec.n_out, weights, obs)
    rho = spec.noise_rho
    keep = math.sqrt(max(1.0 - rho * rho, 0.0))
    clamp = spec.clamp_row()
    logp, act = 0.0, []
    for k in range(spec.n_out):
        z[k] = rho * z[k] + keep * rng.normal()
        a = mean[k] + std[k] * z[k]
        zi = (a - mean[k]) / std[k]
        logp += -0.5 * zi * zi - math.log(std[k]) - 0.5 * math.log(2.0 * math.pi)
        slot = spec.act_slots[k]
        targets[slot] = base_targets[slot] + min(max(a, -clamp[k]), clamp[k])
        act.append(a)
    return np.array(act), logp
