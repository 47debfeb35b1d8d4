"""Host side of the on-device control loop: phyz-gpu's observation op table
and PolicySpec (crates/phyz-gpu/src/policy_pipeline.rs), packed for the C
ABI's phyzb_policy_spec. BatchSim's policy methods take a PolicySpec."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _lib

OBS_OP_STRIDE = 4
SUPPORT_STRIDE = 4


@dataclass(frozen=True)
class ObsOp:
    """One observation feature (policy_pipeline.rs:57-110 ObsOp). Build with
    the constructors below; `kind`, `a`, `b`, `c` are its table row."""
    kind: int
    a: float = 0.0
    b: float = 0.0
    c: float = 0.0
    support: tuple = ()
    heading_body: Optional[int] = None

    @staticmethod
    def const(c: float) -> "ObsOp":
        return ObsOp(0, c=c)

    @staticmethod
    def q_minus(i: int, ref: float = 0.0) -> "ObsOp":
        return ObsOp(1, a=i, c=ref)

    @staticmethod
    def v(i: int) -> "ObsOp":
        return ObsOp(2, a=i)

    @staticmethod
    def body_pitch(b: int) -> "ObsOp":
        return ObsOp(3, a=b)

    @staticmethod
    def body_roll(b: int) -> "ObsOp":
        return ObsOp(4, a=b)

    @staticmethod
    def body_yaw_error(b: int, cmd: float) -> "ObsOp":
        return ObsOp(5, a=b, c=cmd)

    @staticmethod
    def body_pos_z(b: int) -> "ObsOp":
        return ObsOp(6, a=b)

    @staticmethod
    def body_pos(b: int, axis: int) -> "ObsOp":
        return ObsOp(7, a=b, b=axis)

    @staticmethod
    def com_over_support(support: Sequence[tuple], axis: int, heading_body: Optional[int] = None) -> "ObsOp":
        """support: [(body, (ox, oy, oz)), ...] body-frame points."""
        sup = tuple((int(b), tuple(float(x) for x in o)) for b, o in support)
        return ObsOp(8, c=axis, support=sup, heading_body=heading_body)

    def row(self, aux_off: int) -> list:
        if self.kind == 8:
            return [8.0, float(aux_off), float(len(self.support)), float(self.c)]
        return [float(self.kind), float(self.a), float(self.b), float(self.c)]

    def aux(self) -> list:
        if self.kind != 8:
            return []
        out = [1.0 if self.heading_body is not None else 0.0, float(self.heading_body or 0)]
        for b, o in self.support:
            out += [float(b), *o]
        return out


def pack_obs_ops(ops: Sequence[ObsOp]):
    """(table [n][4] f32, aux f32) as pack_obs_ops (policy_pipeline.rs:272-281)."""
    table, aux = [], []
    for op in ops:
        table += op.row(len(aux))
        aux += op.aux()
    return np.asarray(table, np.float32), np.asarray(aux, np.float32)


@dataclass
class PolicySpec:
    """policy_pipeline.rs:285-320."""
    obs: list
    hidden: int
    act_slots: list
    act_clamp: float = 1.0
    act_clamp_slots: Optional[list] = None
    noise_rho: float = 0.0
    input_noise: Optional[list] = None
    history_steps: int = 1

    @property
    def n_in(self) -> int:
        return len(self.obs)

    @property
    def n_out(self) -> int:
        return len(self.act_slots)

    def n_weights(self) -> int:
        i, h, o = self.n_in, self.hidden, self.n_out
        return i * h + h + h * h + h + h * o + o

    def clamp_row(self) -> np.ndarray:
        if self.act_clamp_slots is not None:
            return np.asarray(self.act_clamp_slots, np.float64)
        return np.full(self.n_out, self.act_clamp, np.float64)

    def to_c(self):
        """(phyzb_policy_spec, keep-alive arrays)."""
        table, aux = pack_obs_ops(self.obs)
        slots = np.asarray(self.act_slots, np.int32)
        noise = np.asarray(self.input_noise if self.input_noise is not None else [0.0] * self.n_in, np.float64)
        clamp = None if self.act_clamp_slots is None else np.asarray(self.act_clamp_slots, np.float64)
        keep = [table, aux, slots, noise, clamp]
        fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))
        spec = _lib.PhyzbPolicySpec(
            n_obs=self.n_in, obs_ops=fp(table), n_aux=int(aux.size),
            obs_aux=fp(aux) if aux.size else C.POINTER(C.c_float)(),
            hidden=int(self.hidden), n_act=self.n_out,
            act_slots=slots.ctypes.data_as(C.POINTER(C.c_int32)), act_clamp=float(self.act_clamp),
            act_clamp_slots=clamp.ctypes.data_as(C.POINTER(C.c_double)) if clamp is not None
            else C.POINTER(C.c_double)(),
            noise_rho=float(self.noise_rho), input_noise=noise.ctypes.data_as(C.POINTER(C.c_double)),
            history_steps=int(self.history_steps))
        return spec, keep


def random_weights(spec: PolicySpec, seed: int, scale: float = 1.0) -> np.ndarray:
    """Seeded random-init weights in the kernel's flat order (uniform in
    +-scale/sqrt(fan_in) per layer, zero biases)."""
    rng = np.random.default_rng(seed)
    i, h, o = spec.n_in, spec.hidden, spec.n_out
    parts = [rng.uniform(-1, 1, h * i) * scale / np.sqrt(i), np.zeros(h),
             rng.uniform(-1, 1, h * h) * scale / np.sqrt(h), np.zeros(h),
             rng.uniform(-1, 1, o * h) * scale / np.sqrt(h), np.zeros(o)]
    return np.concatenate(parts)
