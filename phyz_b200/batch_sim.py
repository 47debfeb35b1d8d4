"""BatchSim: the batched-simulation surface of phyz-gpu over libphyzb200.

Method for method this mirrors phyz_gpu::cuda::BatchSim
(crates/phyz-gpu/src/cuda/mod.rs:430-1377): build from a Model and a world
count, optionally enable ground contact and PD servos, then
load_states / set_controls / step / readback_states. Errors raise
PhyzbError where the reference returns Err(String); `try_step` returns the
error instead of raising, like the reference's try_step.

Host arrays are numpy float64, world-major (nworld x width), as phyz's
State rows (layout.rs:340-372).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import PhyzbError, check, dptr
from .model import Model


@dataclass
class PdDof:
    """phyz_gpu::PdDof (crates/phyz-gpu/src/pd_pipeline.rs)."""

    q_index: int
    v_index: int
    kp: float
    kd: float
    max_force: float


@dataclass
class BodyPlane:
    """phyz_gpu::BodyPlane (contact_pipeline.rs:318-355): a contact face at
    `offset` along body `body`'s +z, `half_x` x `half_y` in its x/y;
    penetrations beyond `max_depth` are ignored; `exclude` never touch it."""

    body: int
    offset: float = 0.0
    max_depth: float = 0.05
    half_x: float = 0.5
    half_y: float = 0.5
    exclude: tuple = ()


@dataclass
class BodyContactGains:
    """phyz_gpu::BodyContactGains (contact_pipeline.rs:277-305)."""

    stiffness: float
    damping: float

    @staticmethod
    def uniform_frequency(model: Model, omega: float, zeta: float) -> list:
        return [
            BodyContactGains(b.inertia.mass * omega * omega, 2.0 * zeta * b.inertia.mass * omega)
            for b in model.bodies
        ]


def _rows(a, nworld: int, width: int) -> np.ndarray:
    """pack_rows semantics (layout.rs:327-337): zero-pad / truncate rows.
    An array already of exactly that shape, C-contiguous f64, is used in
    place (no copy: pinned host memory stays pinned)."""
    if (isinstance(a, np.ndarray) and a.dtype == np.float64 and a.shape == (nworld, width)
            and a.flags.c_contiguous):
        return a
    out = np.zeros((nworld, width), np.float64)
    if a is None:
        return out
    if isinstance(a, np.ndarray) and a.ndim == 2:
        r, c = min(a.shape[0], nworld), min(a.shape[1], width)
        out[:r, :c] = a[:r, :c]
        return out
    for w, row in enumerate(list(a)[:nworld]):
        row = np.asarray(row, np.float64).reshape(-1)[:width]
        out[w, : row.size] = row
    return out


class BatchSim:
    """N independent worlds of one model on one GPU."""

    def __init__(self, model: Model, nworld: int, device: int = 0, precision: str = "f64"):
        self._lib = _lib.load()
        self.model = model
        self.nworld = int(nworld)
        self.device = int(device)
        self.precision = precision
        prec = {"f32": _lib.F32, "f64": _lib.F64}[precision]
        self._cmodel, self._cbodies = model.to_c()
        h = C.c_void_p()
        check(self._lib.phyzb_create(C.byref(self._cmodel), self.nworld, self.device, prec, C.byref(h)))
        self._h = h
        self.nv = model.nv
        self.nb = model.nbodies

    # ── construction (cuda/mod.rs:470-498) ────────────────────────────────
    @classmethod
    def new(cls, model: Model, nworld: int, precision: str = "f64") -> "BatchSim":
        return cls(model, nworld, 0, precision)

    @classmethod
    def on_device(cls, model: Model, nworld: int, ordinal: int, precision: str = "f64") -> "BatchSim":
        return cls(model, nworld, ordinal, precision)

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.phyzb_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_model(self, model: Model) -> None:
        cm, cb = model.to_c()
        check(self._lib.phyzb_set_model(self._h, C.byref(cm)))
        self.model, self._cmodel, self._cbodies = model, cm, cb

    # ── contact (cuda/mod.rs:596-700) ─────────────────────────────────────
    def enable_ground_contact(self, ground_height: float, stiffness: float, damping: float,
                              friction: float) -> int:
        n = C.c_int32()
        check(self._lib.phyzb_enable_ground_contact(self._h, ground_height, stiffness, damping, friction,
                                                    C.byref(n)))
        return n.value

    def enable_ground_contact_per_body(self, ground_height: float, friction: float, gains) -> int:
        k = np.ascontiguousarray([g.stiffness for g in gains], np.float64)
        d = np.ascontiguousarray([g.damping for g in gains], np.float64)
        if k.size != self.nb:
            raise PhyzbError(_lib.ERR_INVALID, f"need {self.nb} body gains, got {k.size}")
        n = C.c_int32()
        check(self._lib.phyzb_enable_ground_contact_per_body(self._h, ground_height, friction, dptr(k), dptr(d),
                                                             C.byref(n)))
        return n.value

    def _gains(self, gains):
        if gains is None:
            return None, None
        k = np.ascontiguousarray([g.stiffness for g in gains], np.float64)
        d = np.ascontiguousarray([g.damping for g in gains], np.float64)
        if k.size != self.nb:
            raise PhyzbError(_lib.ERR_INVALID, f"need {self.nb} body gains, got {k.size}")
        return k, d

    @staticmethod
    def _plane(plane):
        if plane is None:
            return None, None
        ex = np.ascontiguousarray(list(plane.exclude), np.int32)
        c = _lib.PhyzbBodyPlane(int(plane.body), float(plane.offset), float(plane.max_depth), float(plane.half_x),
                                float(plane.half_y), ex.ctypes.data_as(C.POINTER(C.c_int32)), int(ex.size))
        return c, ex

    def enable_contact_terrain(self, ground_height: float, friction: float, gains, plane=None,
                               heightfield=None) -> int:
        """Penalty contact with per-body gains against a heightfield
        (cuda/mod.rs:656-676; `ground_height` is ignored while one is
        loaded) and an optional body-attached plane."""
        k, d = self._gains(gains)
        pc, keep_p = self._plane(plane)
        hc, keep_h = heightfield.to_c() if heightfield is not None else (None, None)
        n = C.c_int32()
        check(self._lib.phyzb_enable_contact_terrain(self._h, ground_height, friction, dptr(k), dptr(d),
                                                     C.byref(pc) if pc is not None else None,
                                                     C.byref(hc) if hc is not None else None, C.byref(n)))
        return n.value

    def set_heightfield(self, heightfield) -> None:
        """Replace the terrain in place (cuda/mod.rs:741-759)."""
        hc, keep = heightfield.to_c()
        check(self._lib.phyzb_set_heightfield(self._h, C.byref(hc)))

    def enable_contact_impulse(self, ground_height: float, friction: float, gains=None, plane=None,
                               heightfield=None) -> int:
        """Contact as the velocity-level impulse solve (cuda/mod.rs:680-701):
        `contact_sweeps` staged Coulomb updates per step, warm-started from
        the previous step. `gains` (BodyContactGains per body) only matter to
        a later penalty enable."""
        k, d = self._gains(gains)
        pc, keep_p = self._plane(plane)
        hc, keep_h = heightfield.to_c() if heightfield is not None else (None, None)
        n = C.c_int32()
        check(self._lib.phyzb_enable_contact_impulse(self._h, ground_height, friction,
                                                     dptr(k) if k is not None else None,
                                                     dptr(d) if d is not None else None,
                                                     C.byref(pc) if pc is not None else None,
                                                     C.byref(hc) if hc is not None else None, C.byref(n)))
        return n.value

    @property
    def contact_sweeps(self) -> int:
        """Contact sweeps per step in impulse mode (the reference's public
        `contact_sweeps` field, default 16)."""
        return getattr(self, "_sweeps", _lib.DEFAULT_CONTACT_SWEEPS)

    @contact_sweeps.setter
    def contact_sweeps(self, n: int) -> None:
        check(self._lib.phyzb_set_contact_sweeps(self._h, int(n)))
        self._sweeps = int(n)

    def disable_contact(self) -> None:
        check(self._lib.phyzb_disable_contact(self._h))

    def collidable_bodies(self) -> int:
        return self._lib.phyzb_collidable_bodies(self._h)

    # ── PD (cuda/mod.rs:771-801) ───────────────────────────────────────────
    def enable_pd_control(self, dofs) -> None:
        arr = (_lib.PhyzbPdDof * max(len(dofs), 1))()
        for i, d in enumerate(dofs):
            arr[i] = _lib.PhyzbPdDof(d.q_index, d.v_index, d.kp, d.kd, d.max_force)
        check(self._lib.phyzb_enable_pd(self._h, arr, len(dofs)))
        self._npd = len(dofs)

    def set_position_targets(self, targets) -> None:
        t = _rows(targets, self.nworld, getattr(self, "_npd", 0))
        check(self._lib.phyzb_set_position_targets(self._h, dptr(t)))

    # ── state (cuda/mod.rs:804-821) ────────────────────────────────────────
    def load_states(self, q, v, ctrl=None) -> None:
        qa = _rows(q, self.nworld, self.nv)
        va = _rows(v, self.nworld, self.nv)
        ca = None if ctrl is None else _rows(ctrl, self.nworld, self.nv)
        check(self._lib.phyzb_load_states(self._h, dptr(qa), dptr(va), None if ca is None else dptr(ca)))

    def set_controls(self, controls) -> None:
        c = _rows(controls, self.nworld, self.nv)
        check(self._lib.phyzb_set_controls(self._h, dptr(c)))

    # ── stepping (cuda/mod.rs:818-875) ─────────────────────────────────────
    def step(self) -> None:
        self.step_many(1)

    def try_step(self):
        try:
            self.step_many(1)
            return None
        except PhyzbError as e:
            return e

    def step_many(self, n: int) -> None:
        check(self._lib.phyzb_step(self._h, int(n)))

    def step_with_controls(self, ctrl_seq: np.ndarray) -> None:
        """len(ctrl_seq) steps, step t under controls ctrl_seq[t] (nworld x nv),
        host float32 or float64 — the same as set_controls + step per row."""
        a = np.ascontiguousarray(ctrl_seq)
        if a.ndim != 3 or a.shape[1:] != (self.nworld, self.nv):
            raise PhyzbError(_lib.ERR_INVALID, f"ctrl_seq must be (n, {self.nworld}, {self.nv})")
        dt = {np.dtype(np.float32): _lib.HOST_F32, np.dtype(np.float64): _lib.HOST_F64}[a.dtype]
        check(self._lib.phyzb_step_with_controls(self._h, a.ctypes.data_as(C.c_void_p), dt, a.shape[0]))

    def step_with_controls_ptr(self, ptr: int, host_dtype: int, n: int) -> None:
        """Raw form of step_with_controls for pinned host buffers (e.g. torch)."""
        check(self._lib.phyzb_step_with_controls(self._h, C.c_void_p(ptr), host_dtype, int(n)))

    def step_device_controls(self, ptr: int, step_stride: int, n: int) -> None:
        check(self._lib.phyzb_step_device_controls(self._h, C.c_void_p(ptr), int(step_stride), int(n)))

    def sync(self) -> None:
        check(self._lib.phyzb_sync(self._h))

    def status(self) -> None:
        check(self._lib.phyzb_status(self._h))

    def clear_status(self) -> None:
        check(self._lib.phyzb_clear_status(self._h))

    # ── readback (cuda/mod.rs:978-996) ─────────────────────────────────────
    def readback_states(self, out=None):
        """(q, v) rows; `out` = a caller's (q, v) pair of (nworld, nv) C-contiguous
        f64 arrays (e.g. pinned) to fill instead of new ones."""
        if out is not None:
            q, v = out
            if not all(isinstance(a, np.ndarray) and a.dtype == np.float64 and a.shape == (self.nworld, self.nv)
                       and a.flags.c_contiguous for a in (q, v)):
                raise ValueError("out must be two C-contiguous float64 arrays of shape (nworld, nv)")
        else:
            q = np.zeros((self.nworld, self.nv))
            v = np.zeros((self.nworld, self.nv))
        check(self._lib.phyzb_readback_states(self._h, dptr(q), dptr(v)))
        return q, v

    def readback_qdd(self) -> np.ndarray:
        qdd = np.zeros((self.nworld, self.nv))
        check(self._lib.phyzb_readback_qdd(self._h, dptr(qdd)))
        return qdd

    def readback_contacts(self) -> np.ndarray:
        """(nworld, nbodies, 8): touching, depth, point xyz, force xyz."""
        cs = np.zeros((self.nworld, self.nb, _lib.CONTACT_STRIDE))
        check(self._lib.phyzb_readback_contacts(self._h, dptr(cs)))
        return cs

    # ── device-resident path ───────────────────────────────────────────────
    def device_view(self) -> dict:
        v = _lib.PhyzbDeviceView()
        check(self._lib.phyzb_device_view_get(self._h, C.byref(v)))
        return {k: getattr(v, k) for k, _ in _lib.PhyzbDeviceView._fields_}

    def load_states_device(self, q_ptr: int, v_ptr: int, ctrl_ptr: int | None = None) -> None:
        """Device SoA ([nv][nworld], sim precision) state upload, asynchronous."""
        check(self._lib.phyzb_load_states_device(self._h, C.c_void_p(q_ptr), C.c_void_p(v_ptr),
                                                 C.c_void_p(ctrl_ptr or 0)))

    def set_stream(self, stream_ptr: int | None) -> None:
        check(self._lib.phyzb_set_stream(self._h, C.c_void_p(stream_ptr or 0)))

    def objective_device(self, kind: int, out_ptr: int) -> None:
        check(self._lib.phyzb_objective_device(self._h, int(kind), C.c_void_p(out_ptr)))

    # ── state history (cuda/mod.rs:1316-1376) ───────────────────────────────
    def enable_state_history(self, slots: int) -> None:
        check(self._lib.phyzb_enable_state_history(self._h, int(slots)))
        self._hist = int(slots)

    def record_state(self, slot: int) -> None:
        check(self._lib.phyzb_record_state(self._h, int(slot)))

    def readback_state_history(self, slot0: int, n: int):
        """(q, v) rows [n][nworld][nv]."""
        q = np.zeros((n, self.nworld, self.nv))
        v = np.zeros((n, self.nworld, self.nv))
        check(self._lib.phyzb_readback_state_history(self._h, int(slot0), int(n), dptr(q), dptr(v)))
        return q, v

    # ── on-device control loop (cuda/mod.rs:1081-1313) ─────────────────────
    def enable_policy(self, spec) -> None:
        cs, keep = spec.to_c()
        check(self._lib.phyzb_enable_policy(self._h, C.byref(cs)))
        self._policy = spec

    def set_policy_weights(self, weights) -> None:
        w = np.ascontiguousarray(weights, np.float64)
        check(self._lib.phyzb_set_policy_weights(self._h, dptr(w), int(w.size)))

    def set_policy_std(self, std) -> None:
        s = np.ascontiguousarray(std, np.float64)
        check(self._lib.phyzb_set_policy_std(self._h, dptr(s), int(s.size)))

    def set_policy_base_targets(self, rows) -> None:
        r = _rows(rows, self.nworld, getattr(self, "_npd", 0))
        check(self._lib.phyzb_set_policy_base_targets(self._h, dptr(r)))

    def seed_policy(self, seed: int) -> None:
        check(self._lib.phyzb_seed_policy(self._h, C.c_uint64(int(seed) & 0xFFFFFFFFFFFFFFFF)))

    def run_policy(self, step: int) -> None:
        check(self._lib.phyzb_run_policy(self._h, int(step)))

    def policy_rollout(self, step0: int, n_control: int, substeps: int) -> None:
        check(self._lib.phyzb_policy_rollout(self._h, int(step0), int(n_control), int(substeps)))

    def readback_policy_history(self, step0: int, n: int):
        """(obs [n][nworld][n_in], out [n][nworld][n_out + 1]) float32."""
        sp = self._policy
        obs = np.zeros((n, self.nworld, sp.n_in), np.float32)
        out = np.zeros((n, self.nworld, sp.n_out + 1), np.float32)
        fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))
        check(self._lib.phyzb_readback_policy_history(self._h, int(step0), int(n), fp(obs), fp(out)))
        return obs, out

    def readback_targets(self) -> np.ndarray:
        t = np.zeros((self.nworld, getattr(self, "_npd", 0)))
        check(self._lib.phyzb_readback_targets(self._h, dptr(t)))
        return t

    def readback_kinematics(self) -> np.ndarray:
        """[nworld][nbodies][18]: world->body rot, origin, body-frame w, v."""
        xf = np.zeros((self.nworld, self.nb, _lib.KINEMATICS_STRIDE))
        check(self._lib.phyzb_readback_kinematics(self._h, dptr(xf)))
        return xf

    def policy_history_view(self) -> dict:
        h = _lib.PhyzbPolicyHistory()
        check(self._lib.phyzb_policy_history_view(self._h, C.byref(h)))
        return {"obs": h.obs, "out": h.out, "n_obs": h.n_obs, "n_act": h.n_act, "nworld": h.nworld,
                "steps": h.steps}

    def policy_advantages(self, trainer, comm, reward_coef, action_penalty: float, gamma: float, lam: float,
                          steps: int, adv_ptr: int, ret_ptr: int, normalize: bool = True):
        """Rewards, critic values, GAE and (global) advantage normalization of
        the last `steps` control steps, on the device. Returns (mean return
        per world, advantage mean, advantage std) over every rank."""
        coef = np.ascontiguousarray(reward_coef, np.float64)
        cfg = _lib.PhyzbReturnCfg(dptr(coef), float(action_penalty), float(gamma), float(lam), int(steps),
                                  int(bool(normalize)))
        st = np.zeros(3)
        check(self._lib.phyzb_policy_advantages(self._h, trainer._h, comm._h if comm is not None else None,
                                                C.byref(cfg), C.c_void_p(int(adv_ptr)), C.c_void_p(int(ret_ptr)),
                                                dptr(st)))
        return tuple(st)

    def policy_sync_from_trainer(self, trainer) -> None:
        check(self._lib.phyzb_policy_sync_from_trainer(self._h, trainer._h))

    def flops_per_world_step(self):
        f, t = C.c_double(), C.c_double()
        check(self._lib.phyzb_flops_per_world_step(self._h, C.byref(f), C.byref(t)))
        return f.value, t.value

    def flops_executed(self, q, v, ctrl=None, specialized: bool = False):
        """Flops per world-step the kernel executes from these states
        (q, v [n][nv] rows; ctrl [steps][n][nv] or None for one zero-control
        step), the contact force law included where a body touches; with
        `specialized`, as a model-specialized kernel executes them (products
        with zero table constants left out). Returns (flops, transcendentals)."""
        q = np.ascontiguousarray(q, np.float64)
        v = np.ascontiguousarray(v, np.float64)
        n = q.shape[0]
        steps = 1 if ctrl is None else int(np.shape(ctrl)[0])
        c = None if ctrl is None else np.ascontiguousarray(ctrl, np.float64)
        f, t = C.c_double(), C.c_double()
        check(self._lib.phyzb_flops_executed(self._h, dptr(q), dptr(v), None if c is None else dptr(c), n, steps,
                                             int(bool(specialized)), C.byref(f), C.byref(t)))
        return f.value, t.value

    @property
    def specialize(self):
        """Kernel specialization mode: False (generic variants), True (the
        rollout kernel compiled at run time for this model: tables literal,
        body loops unrolled) or "auto" (True for branching models whose
        longest chain has at most 16 bodies). The compile happens at the
        next launch after any table change and is cached in-process and on
        disk."""
        mode = C.c_int32()
        check(self._lib.phyzb_get_kernel_specialization(self._h, C.byref(mode), None))
        return {0: False, 1: True, 2: "auto"}[mode.value]

    @specialize.setter
    def specialize(self, mode) -> None:
        code = 2 if mode == "auto" else (1 if mode else 0)
        check(self._lib.phyzb_set_kernel_specialization(self._h, code))

    @property
    def world_lanes(self) -> int:
        """Threads per world (2, 4, 8; 0: one thread per world): for branching
        trees, each lane steps the trunk and its share of the limbs and the
        backward sweep sums the limbs' contributions over the lanes."""
        n = C.c_int32()
        check(self._lib.phyzb_get_world_lanes(self._h, C.byref(n), None))
        return n.value

    @world_lanes.setter
    def world_lanes(self, lanes: int) -> None:
        check(self._lib.phyzb_set_world_lanes(self._h, int(lanes)))

    @property
    def lanes_active(self) -> bool:
        """Whether a launch of two or more steps runs the lanes kernel."""
        n, a = C.c_int32(), C.c_int32()
        check(self._lib.phyzb_get_world_lanes(self._h, C.byref(n), C.byref(a)))
        return bool(a.value)

    @property
    def specialized(self) -> bool:
        """Whether the next rollout launch runs the model-specialized kernel."""
        mode, active = C.c_int32(), C.c_int32()
        check(self._lib.phyzb_get_kernel_specialization(self._h, C.byref(mode), C.byref(active)))
        return bool(active.value)

    def slice_plan(self, nsteps: int) -> dict:
        """How a rollout launch of nsteps steps runs: steps_per_run 0 = tile
        mode, else slice mode (warps take 32 worlds x steps_per_run jobs)."""
        vals = [C.c_int32() for _ in range(3)]
        check(self._lib.phyzb_slice_plan(self._h, int(nsteps), *[C.byref(x) for x in vals]))
        return dict(zip(("steps_per_run", "worlds_per_block", "blocks"), [x.value for x in vals]))

    def launch_info(self) -> dict:
        vals = [C.c_int32() for _ in range(5)]
        check(self._lib.phyzb_launch_info(self._h, *[C.byref(x) for x in vals]))
        return dict(zip(("worlds_per_block", "blocks", "smem_bytes", "scratch_per_world", "tmem_cols"),
                        [x.value for x in vals]))
