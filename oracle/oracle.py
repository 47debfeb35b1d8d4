"""TEST INFRASTRUCTURE ONLY — ctypes face of the CPU checkers.

* `Oracle`: the f64 C++ restatement of phyz's CPU path (phyz_oracle.hpp,
  built into _build/libphyz_oracle.so).
* `RefHost`: the reference's own crates/phyz-gpu/cuda/phyz_kernels.cu
  compiled as host C++ (f32), built into _ref/libphyz_ref_host.so by the
  Makefile from the reference tree; the prebuilt object travels with the
  repository snapshot, the reference tree does not.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
this module, and only as the checker / the timed CPU reference.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libphyz_oracle.so"
REF_SO = HERE / "_ref" / "libphyz_ref_host.so"

_D = C.POINTER(C.c_double)
_F = C.POINTER(C.c_float)
_I = C.POINTER(C.c_int32)


def build() -> None:
    """Run the Makefile (oracle always; the reference build when its tree exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _d(a):
    return None if a is None else a.ctypes.data_as(_D)


def _f(a):
    return None if a is None else a.ctypes.data_as(_F)


class Oracle:
    def __init__(self):
        if not ORACLE_SO.exists():
            build()
        self.lib = C.CDLL(str(ORACLE_SO))
        L = self.lib
        MP = C.c_void_p
        L.oracle_aba.argtypes = [MP, C.c_int64, _D, _D, _D, _D, _D]
        L.oracle_rnea.argtypes = [MP, C.c_int64, _D, _D, _D, _D]
        L.oracle_integrate_configuration.argtypes = [MP, C.c_int64, _D, _D, C.c_double]
        L.oracle_forward_kinematics.argtypes = [MP, C.c_int64, _D, _D, _D, _D]
        L.oracle_energy.argtypes = [MP, C.c_int64, _D, _D, _D, _D]
        L.oracle_penalty_contact.argtypes = [MP, C.c_int64, _D, _D, C.c_double, C.c_double, _D, _D, _D, _D]
        L.oracle_rollout.argtypes = [MP, C.c_int64, _D, _D, _D, C.c_int64, C.c_int32, C.c_int32, C.c_double,
                                     C.c_double, _D, _D, C.c_int32, _I, _D, _D, _D, _D, C.c_int32]
        L.oracle_set_heightfield.argtypes = [C.c_int32, C.c_int32, C.c_double, C.c_double, C.c_double,
                                             C.c_double, _F]
        L.oracle_rollout_impulse.argtypes = [MP, C.c_int64, _D, _D, _D, C.c_int64, C.c_int32, _D, C.c_int32,
                                             C.c_int32, _I, _D, _D, _D, _D, _D, C.c_int32]
        for f in ("oracle_aba", "oracle_rnea", "oracle_integrate_configuration", "oracle_forward_kinematics",
                  "oracle_energy", "oracle_penalty_contact", "oracle_rollout", "oracle_rollout_impulse"):
            getattr(L, f).restype = C.c_int

    @staticmethod
    def _m(model):
        cm, keep = model.to_c()
        return cm, keep

    def aba(self, model, q, v, ctrl=None, ext=None):
        cm, keep = self._m(model)
        q, v = np.ascontiguousarray(q, np.float64), np.ascontiguousarray(v, np.float64)
        ctrl = None if ctrl is None else np.ascontiguousarray(ctrl, np.float64)
        ext = None if ext is None else np.ascontiguousarray(ext, np.float64)
        out = np.zeros_like(q)
        self.lib.oracle_aba(C.addressof(cm), q.shape[0], _d(q), _d(v), _d(ctrl), _d(ext), _d(out))
        return out

    def rnea(self, model, q, v, qdd):
        cm, keep = self._m(model)
        q, v, qdd = (np.ascontiguousarray(a, np.float64) for a in (q, v, qdd))
        out = np.zeros_like(q)
        self.lib.oracle_rnea(C.addressof(cm), q.shape[0], _d(q), _d(v), _d(qdd), _d(out))
        return out

    def integrate_configuration(self, model, q, v, dt):
        cm, keep = self._m(model)
        q = np.array(q, np.float64, copy=True, order="C")
        v = np.ascontiguousarray(v, np.float64)
        self.lib.oracle_integrate_configuration(C.addressof(cm), q.shape[0], _d(q), _d(v), dt)
        return q

    def forward_kinematics(self, model, q, v):
        cm, keep = self._m(model)
        q, v = np.ascontiguousarray(q, np.float64), np.ascontiguousarray(v, np.float64)
        n, nb = q.shape[0], model.nbodies
        xw = np.zeros((n, nb, 12))
        vel = np.zeros((n, nb, 6))
        self.lib.oracle_forward_kinematics(C.addressof(cm), n, _d(q), _d(v), _d(xw), _d(vel))
        return xw, vel

    def energy(self, model, q, v):
        cm, keep = self._m(model)
        q, v = np.ascontiguousarray(q, np.float64), np.ascontiguousarray(v, np.float64)
        ke, pe = np.zeros(q.shape[0]), np.zeros(q.shape[0])
        self.lib.oracle_energy(C.addressof(cm), q.shape[0], _d(q), _d(v), _d(ke), _d(pe))
        return ke, pe

    def penalty_contact(self, model, q, v, ground, friction, k, d):
        cm, keep = self._m(model)
        q, v = np.ascontiguousarray(q, np.float64), np.ascontiguousarray(v, np.float64)
        n, nb = q.shape[0], model.nbodies
        k = np.ascontiguousarray(np.broadcast_to(k, (nb,)), np.float64)
        d = np.ascontiguousarray(np.broadcast_to(d, (nb,)), np.float64)
        ext = np.zeros((n, nb, 6))
        cs = np.zeros((n, nb, 8))
        self.lib.oracle_penalty_contact(C.addressof(cm), n, _d(q), _d(v), ground, friction, _d(k), _d(d),
                                        _d(ext), _d(cs))
        return ext, cs

    def rollout(self, model, q, v, ctrl=None, nsteps=1, schedule=False, contact=None, pd=None, targets=None,
                nthreads=1):
        """nsteps of [PD ->] [contact ->] ABA -> semi-implicit Euler.
        ctrl: (nworld, nv) held, or with schedule=True (nsteps, nworld, nv).
        contact: (ground, friction, k[nb], d[nb]); pd: list of PdDof."""
        cm, keep = self._m(model)
        q = np.array(q, np.float64, copy=True, order="C")
        v = np.array(v, np.float64, copy=True, order="C")
        n, nv, nb = q.shape[0], model.nv, model.nbodies
        stride = 0
        if ctrl is not None:
            ctrl = np.ascontiguousarray(ctrl, np.float64)
            stride = n * nv if schedule else 0
        qdd = np.zeros((n, nv))
        cs = np.zeros((n, nb, 8))
        has_c = contact is not None
        g, fr, k, d = (contact if has_c else (0.0, 0.0, None, None))
        if has_c:
            k = np.ascontiguousarray(np.broadcast_to(k, (nb,)), np.float64)
            d = np.ascontiguousarray(np.broadcast_to(d, (nb,)), np.float64)
        npd = 0
        pidx = pg = tg = None
        if pd:
            npd = len(pd)
            pidx = np.ascontiguousarray([[p.q_index, p.v_index] for p in pd], np.int32)
            pg = np.ascontiguousarray([[p.kp, p.kd, p.max_force] for p in pd], np.float64)
            tg = np.ascontiguousarray(targets, np.float64)
        self.lib.oracle_rollout(C.addressof(cm), n, _d(q), _d(v), _d(ctrl), stride, nsteps, int(has_c), g, fr,
                                _d(k), _d(d), npd, None if pidx is None else pidx.ctypes.data_as(_I), _d(pg),
                                _d(tg), _d(qdd), _d(cs), nthreads)
        return q, v, qdd, cs


def solref_erp_from(timeconst, dampratio, dt):
    """contact_pipeline.rs:229-237."""
    if dt <= 0.0:
        return 0.0
    tau, zeta = max(timeconst, 0.0), max(dampratio, 1e-6)
    denom = 2.0 * tau * zeta * zeta + dt
    return 1.0 if denom <= 0.0 else dt / denom


def impulse_material(dt):
    """enable_contact_impulse's material (cuda/mod.rs:680-701) over
    GroundContactParams::default (contact_pipeline.rs:199-218): erp, margin,
    restitution, restitution_threshold, solimp dmin, dmax, width, mid, power."""
    return [solref_erp_from(0.02, 1.0, dt), 0.001, 0.0, 0.05, 0.9, 0.95, 0.001, 0.5, 2.0]


IMPULSE_PTS = 8


def _rollout_impulse(self, model, q, v, ctrl=None, nsteps=1, schedule=False, contact=(0.0, 0.0), sweeps=16,
                     pd=None, targets=None, state=None, nthreads=1):
    """nsteps impulse-mode steps (step_world_impulse). contact: (ground,
    friction). state: per world nb*6 wrenches + nb*8*3 impulses (None: zeros);
    returns (q, v, qdd, contact_state [n][nb][8], state)."""
    cm, keep = self._m(model)
    q = np.array(q, np.float64, copy=True, order="C")
    v = np.array(v, np.float64, copy=True, order="C")
    n, nv, nb = q.shape[0], model.nv, model.nbodies
    stride = 0
    if ctrl is not None:
        ctrl = np.ascontiguousarray(ctrl, np.float64)
        stride = n * nv if schedule else 0
    per = nb * 6 + 2 * nb * IMPULSE_PTS * 3
    st = np.zeros((n, per)) if state is None else np.array(state, np.float64, copy=True, order="C")
    ground, fr = contact
    m = impulse_material(model.dt)
    params = np.array([ground, fr, m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7], m[8]], np.float64)
    npd = 0
    pidx = pg = tg = None
    if pd:
        npd = len(pd)
        pidx = np.ascontiguousarray([[p.q_index, p.v_index] for p in pd], np.int32)
        pg = np.ascontiguousarray([[p.kp, p.kd, p.max_force] for p in pd], np.float64)
        tg = np.ascontiguousarray(targets, np.float64)
    qdd = np.zeros((n, nv))
    cs = np.zeros((n, nb, 8))
    self.lib.oracle_rollout_impulse(C.addressof(cm), n, _d(q), _d(v), _d(ctrl), stride, nsteps, _d(params),
                                    int(sweeps), npd, None if pidx is None else pidx.ctypes.data_as(_I), _d(pg),
                                    _d(tg), _d(st), _d(qdd), _d(cs), nthreads)
    return q, v, qdd, cs, st


Oracle.rollout_impulse = _rollout_impulse


def _set_heightfield(self, hf=None):
    """The terrain the following contact rollouts sample (a
    phyz_b200.Heightfield; None: the flat plane at their ground height)."""
    if hf is None:
        self.lib.oracle_set_heightfield(0, 0, 0.0, 0.0, 0.0, 1.0, None)
        return
    h = np.ascontiguousarray(hf.heights, np.float32).reshape(-1)
    self.lib.oracle_set_heightfield(hf.nx, hf.ny, *[float(x) for x in hf.origin], float(hf.cell), _f(h))


Oracle.set_heightfield = _set_heightfield


def _terrain_at(self, x, y):
    """(height, unit normal) of the current terrain at world (x, y)."""
    self.lib.oracle_terrain_at.restype = C.c_double
    self.lib.oracle_terrain_at.argtypes = [C.c_double, C.c_double, _D]
    n = np.zeros(3)
    h = self.lib.oracle_terrain_at(float(x), float(y), _d(n))
    return h, n


Oracle.terrain_at = _terrain_at


def _set_plane(self, plane=None, nbodies=0):
    """The body-attached plane of the following contact rollouts (a
    phyz_b200.BodyPlane; None: no plane)."""
    L = self.lib
    L.oracle_set_plane.argtypes = [C.c_int32, C.c_double, C.c_double, C.c_double, C.c_double, _I, C.c_int32,
                                   C.c_int32]
    if plane is None:
        L.oracle_set_plane(-1, 0.0, 0.0, 0.0, 0.0, None, 0, 0)
        return
    ex = np.ascontiguousarray(list(plane.exclude) or [-1], np.int32)
    L.oracle_set_plane(int(plane.body), float(plane.offset), float(plane.max_depth), float(plane.half_x),
                       float(plane.half_y), ex.ctypes.data_as(_I), len(plane.exclude), int(nbodies))


Oracle.set_plane = _set_plane


class RefHost:
    """The reference's f32 kernels compiled as host C++ (phyz_host_*)."""

    BODY_STRIDE, GEOM_STRIDE, PD_STRIDE = 36, 24, 8

    def __init__(self):
        if not REF_SO.exists():
            build()
        if not REF_SO.exists():
            raise RuntimeError(f"{REF_SO} missing and the reference tree is not available to build it")
        self.lib = C.CDLL(str(REF_SO))
        L = self.lib
        L.phyzref_pack_bodies.argtypes = [C.c_void_p, _F]
        L.phyzref_pack_geometries.argtypes = [C.c_void_p, _D, _D, _F]
        L.phyzref_rollout.argtypes = [C.c_int, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, C.c_float,
                                      C.c_float, C.c_float, _F, _F, C.c_float, C.c_float, C.c_uint32, _F, _F,
                                      _F, _F, _F, C.c_int64, C.c_int32, _F, _F]
        L.phyzref_set_heightfield.argtypes = [C.c_uint32, C.c_uint32, C.c_float, C.c_float, C.c_float, C.c_float,
                                              _F]
        L.phyzref_rollout_impulse.argtypes = [C.c_int, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, C.c_float,
                                              C.c_float, C.c_float, _F, _F, C.c_float, C.c_float, _F, C.c_int32,
                                              C.c_uint32, _F, _F, _F, _F, _F, C.c_int64, C.c_int32, _F, _F, _F]
        u = C.c_uint32
        L.phyz_host_fk.argtypes = [u, u, u, u, _F, _F, _F, _F]
        L.phyz_host_obs.argtypes = [u, u, u, u, u, u, u, _F, _F, _F, _F, _F, _F, _F]
        L.phyz_host_policy.argtypes = [u, u, u, u, u, u, C.c_float, u, C.c_float, u, u, _F, _F, _F, _F, _F, _F,
                                       _F, _F, _F, _F, _F]

    def _bodies(self, model):
        cm, keep = model.to_c()
        bodies = np.zeros(model.nbodies * self.BODY_STRIDE, np.float32)
        self.lib.phyzref_pack_bodies(C.addressof(cm), _f(bodies))
        return bodies

    def kinematics(self, model, q, v):
        """phyz_host_fk: [nworld][nb][18] f32 (world->body rot, origin, w, v)."""
        n, nb = q.shape[0], model.nbodies
        xf = np.zeros((n, nb, 18), np.float32)
        self.lib.phyz_host_fk(n, n, model.nv, nb, _f(self._bodies(model)), _f(np.ascontiguousarray(q, np.float32)),
                              _f(np.ascontiguousarray(v, np.float32)), _f(xf))
        return xf

    def observe(self, model, q, v, table, aux):
        """phyz_host_fk then phyz_host_obs: [nworld][n_in] f32."""
        n, nb, nv = q.shape[0], model.nbodies, model.nv
        qf, vf = np.ascontiguousarray(q, np.float32), np.ascontiguousarray(v, np.float32)
        xf = self.kinematics(model, q, v)
        com = np.array([[b.inertia.mass, *b.inertia.com] for b in model.bodies], np.float32).reshape(-1)
        n_in = table.size // 4
        obs = np.zeros((n, n_in), np.float32)
        aux = np.ascontiguousarray(aux if np.size(aux) else np.zeros(1), np.float32)
        self.lib.phyz_host_obs(n, n, nv, nv, nb, n_in, 0, _f(np.ascontiguousarray(table, np.float32)), _f(aux),
                               _f(com), _f(qf), _f(vf), _f(xf), _f(obs))
        return obs

    def policy(self, spec, weights, std, obs, rng_state, z, base_targets):
        """phyz_host_policy on rows: obs [n][n_in] (noised in place), rng_state
        [n] u64, z [n][n_out], base_targets [n][n_pd]. Returns (targets,
        out [n][n_out + 1], obs, rng_state, z) after one call."""
        n = obs.shape[0]
        npd = base_targets.shape[1]
        obs = np.ascontiguousarray(obs, np.float32).copy()
        words = np.ascontiguousarray(rng_state, np.uint64).view(np.uint32).copy()  # lo, hi per world
        zf = np.ascontiguousarray(z, np.float32).copy()
        clamp = spec.clamp_row().astype(np.float32)
        targets = np.zeros((n, npd), np.float32)
        out = np.zeros((n, spec.n_out + 1), np.float32)
        self.lib.phyz_host_policy(n, n, spec.n_in, spec.hidden, spec.n_out, npd, float(spec.act_clamp),
                                  int(spec.act_clamp_slots is not None), float(spec.noise_rho), 0, 0,
                                  _f(np.ascontiguousarray(weights, np.float32)), _f(np.asarray(std, np.float32)),
                                  _f(np.asarray(spec.input_noise if spec.input_noise is not None
                                                else np.zeros(spec.n_in), np.float32)),
                                  _f(obs), _f(words.view(np.float32)), _f(zf),
                                  _f(np.asarray(spec.act_slots, np.float32)), _f(clamp),
                                  _f(np.ascontiguousarray(base_targets, np.float32)), _f(targets), _f(out))
        return targets, out, obs, words.view(np.uint64).copy(), zf

    def rollout(self, model, q, v, ctrl, nsteps=1, schedule=False, contact=None, pd=None, targets=None,
                nthreads=1):
        cm, keep = model.to_c()
        nb, nv = model.nbodies, model.nv
        bodies = np.zeros(nb * self.BODY_STRIDE, np.float32)
        self.lib.phyzref_pack_bodies(C.addressof(cm), _f(bodies))
        geom = None
        ground = fr = 0.0
        if contact is not None:
            ground, fr, k, d = contact
            k = np.ascontiguousarray(np.broadcast_to(k, (nb,)), np.float64)
            d = np.ascontiguousarray(np.broadcast_to(d, (nb,)), np.float64)
            geom = np.zeros(nb * self.GEOM_STRIDE, np.float32)
            self.lib.phyzref_pack_geometries(C.addressof(cm), _d(k), _d(d), _f(geom))
        n = q.shape[0]
        qf = np.ascontiguousarray(q, np.float32).copy()
        vf = np.ascontiguousarray(v, np.float32).copy()
        cf = np.ascontiguousarray(ctrl, np.float32)
        stride = n * nv if schedule else 0
        npd = 0
        tbl = tg = None
        if pd:
            npd = len(pd)
            tbl = np.zeros(npd * self.PD_STRIDE, np.float32)
            for i, p in enumerate(pd):
                tbl[i * self.PD_STRIDE: i * self.PD_STRIDE + 5] = [p.q_index, p.v_index, p.kp, p.kd, p.max_force]
            tg = np.ascontiguousarray(targets, np.float32)
        qdd = np.zeros((n, nv), np.float32)
        cs = np.zeros((n, nb, 8), np.float32)
        gx, gy, gz = (float(x) for x in model.gravity)
        self.lib.phyzref_rollout(nthreads, n, nv, nb, float(model.dt), gx, gy, gz, _f(bodies), _f(geom),
                                 float(ground), float(fr), npd, _f(tbl), _f(tg), _f(qf), _f(vf), _f(cf), stride,
                                 nsteps, _f(qdd), _f(cs))
        return qf, vf, qdd, cs

    def set_plane(self, plane=None):
        """The body-attached plane of the following host rollouts and
        geometry packs (None: no plane)."""
        self.lib.phyzref_set_plane.argtypes = [C.c_int32, C.c_float, C.c_float, C.c_float, C.c_float, _I,
                                               C.c_int32]
        if plane is None:
            self.lib.phyzref_set_plane(-1, 0.0, 0.0, 0.0, 0.0, None, 0)
            return
        ex = np.ascontiguousarray(list(plane.exclude) or [-1], np.int32)
        self.lib.phyzref_set_plane(int(plane.body), float(plane.offset), float(plane.max_depth),
                                   float(plane.half_x), float(plane.half_y), ex.ctypes.data_as(_I),
                                   len(plane.exclude))

    def set_heightfield(self, hf=None):
        """The terrain the following host rollouts pass to the reference's
        contact kernel (None: the flat plane)."""
        if hf is None:
            self.lib.phyzref_set_heightfield(0, 0, 0.0, 0.0, 0.0, 1.0, None)
            return
        h = np.ascontiguousarray(hf.heights, np.float32).reshape(-1)
        self.lib.phyzref_set_heightfield(hf.nx, hf.ny, *[float(x) for x in hf.origin], float(hf.cell), _f(h))

    def rollout_impulse(self, model, q, v, ctrl, nsteps=1, schedule=False, contact=(0.0, 0.0), sweeps=16,
                        pd=None, targets=None, state=None, nthreads=1):
        """Impulse mode (phyzref_rollout_impulse). state: (ext [n][nb][6],
        cs [n][nb][56]) f32 carried between calls (None: zeros). Returns
        (q, v, qdd, contact_state [n][nb][8], state)."""
        cm, keep = model.to_c()
        nb, nv = model.nbodies, model.nv
        bodies = np.zeros(nb * self.BODY_STRIDE, np.float32)
        self.lib.phyzref_pack_bodies(C.addressof(cm), _f(bodies))
        zeros = np.zeros(nb)
        geom = np.zeros(nb * self.GEOM_STRIDE, np.float32)
        self.lib.phyzref_pack_geometries(C.addressof(cm), _d(zeros), _d(zeros), _f(geom))
        n = q.shape[0]
        qf = np.ascontiguousarray(q, np.float32).copy()
        vf = np.ascontiguousarray(v, np.float32).copy()
        cf = np.ascontiguousarray(ctrl, np.float32)
        stride = n * nv if schedule else 0
        if state is None:
            ext, cs = np.zeros((n, nb, 6), np.float32), np.zeros((n, nb, 56), np.float32)
        else:
            ext, cs = (np.array(a, np.float32, copy=True, order="C") for a in state)
        npd = 0
        tbl = tg = None
        if pd:
            npd = len(pd)
            tbl = np.zeros(npd * self.PD_STRIDE, np.float32)
            for i, p in enumerate(pd):
                tbl[i * self.PD_STRIDE: i * self.PD_STRIDE + 5] = [p.q_index, p.v_index, p.kp, p.kd, p.max_force]
            tg = np.ascontiguousarray(targets, np.float32)
        imp = np.asarray(impulse_material(model.dt), np.float32)
        qdd = np.zeros((n, nv), np.float32)
        gx, gy, gz = (float(x) for x in model.gravity)
        ground, fr = contact
        self.lib.phyzref_rollout_impulse(nthreads, n, nv, nb, float(model.dt), gx, gy, gz, _f(bodies), _f(geom),
                                         float(ground), float(fr), _f(imp), int(sweeps), npd, _f(tbl), _f(tg),
                                         _f(qf), _f(vf), _f(cf), stride, nsteps, _f(ext), _f(cs), _f(qdd))
        return qf, vf, qdd, cs[:, :, :8].copy(), (ext, cs)


REF_CUDA_SO = HERE / "_ref" / "libphyz_ref_cuda.so"


class RefCuda:
    """The reference's own CUDA kernels on this GPU (ref_cuda_driver.cu):
    contact -> aba -> integrate per step, 64-thread blocks, one captured
    graph per rollout. AoS f32 rows, as the reference holds them."""

    def __init__(self, refhost):
        if not REF_CUDA_SO.exists():
            build()
        if not REF_CUDA_SO.exists():
            raise RuntimeError(f"{REF_CUDA_SO} missing and the reference tree is not available to build it")
        self.host = refhost
        self.lib = C.CDLL(str(REF_CUDA_SO))
        u = C.c_uint32
        self.lib.phyzref_cuda_rollout.argtypes = [u, u, u, C.c_float, C.c_float, C.c_float, C.c_float, _F, _F, _F,
                                                  _F, _F, _F, C.c_int64, C.c_int32, C.c_int32, _F, _F, _F]
        self.lib.phyzref_cuda_rollout_sweeps.argtypes = [u, u, u, C.c_float, C.c_float, C.c_float, C.c_float, _F,
                                                         _F, _F, _F, _F, _F, C.c_int64, C.c_int32, C.c_int32,
                                                         C.c_int32, _F, _F, _F]
        refhost.lib.phyzref_pack_cparams.argtypes = [u, u, u, C.c_float, C.c_float, C.c_float, _F]

    def rollout(self, model, q, v, ctrl, nsteps, schedule=False, contact=None, reps=0, sweeps=0):
        """Returns (q, v, qdd, contact_state [n][nb][56], best ms of `reps` replays).
        sweeps > 0: impulse mode with `contact` = (ground, friction) and
        enable_contact_impulse's material."""
        cm, keep = model.to_c()
        nb, nv, n = model.nbodies, model.nv, q.shape[0]
        bodies = np.zeros(nb * RefHost.BODY_STRIDE, np.float32)
        self.host.lib.phyzref_pack_bodies(C.addressof(cm), _f(bodies))
        geom = cp = None
        if contact is not None and sweeps > 0:
            ground, fr = contact
            zeros = np.zeros(nb)
            geom = np.zeros(nb * RefHost.GEOM_STRIDE, np.float32)
            self.host.lib.phyzref_pack_geometries(C.addressof(cm), _d(zeros), _d(zeros), _f(geom))
            cp = np.zeros(32, np.float32)
            self.host.lib.phyzref_pack_cparams(n, nb, nv, float(ground), float(model.dt), float(fr), _f(cp))
            imp = impulse_material(model.dt)
            cp[17] = np.array([1], np.uint32).view(np.float32)[0]  # solve_mode: impulse
            cp[19], cp[20], cp[21], cp[22] = imp[2], imp[3], imp[0], imp[1]
            cp[23:28] = imp[4:9]
        elif contact is not None:
            ground, fr, k, d = contact
            k = np.ascontiguousarray(np.broadcast_to(k, (nb,)), np.float64)
            d = np.ascontiguousarray(np.broadcast_to(d, (nb,)), np.float64)
            geom = np.zeros(nb * RefHost.GEOM_STRIDE, np.float32)
            self.host.lib.phyzref_pack_geometries(C.addressof(cm), _d(k), _d(d), _f(geom))
            cp = np.zeros(32, np.float32)
            self.host.lib.phyzref_pack_cparams(n, nb, nv, float(ground), float(model.dt), float(fr), _f(cp))
        qf = np.ascontiguousarray(q, np.float32).copy()
        vf = np.ascontiguousarray(v, np.float32).copy()
        cf = np.ascontiguousarray(ctrl, np.float32)
        qdd = np.zeros((n, nv), np.float32)
        cs = np.zeros((n, nb, 56), np.float32)
        ms = np.zeros(1, np.float32)
        gx, gy, gz = (float(x) for x in model.gravity)
        rc = self.lib.phyzref_cuda_rollout_sweeps(n, nv, nb, float(model.dt), gx, gy, gz, _f(bodies), _f(geom),
                                                  _f(cp), _f(qf), _f(vf), _f(cf), n * nv if schedule else 0, nsteps,
                                                  int(sweeps), reps, _f(qdd), _f(cs), _f(ms))
        if rc != 0:
            raise RuntimeError(f"reference CUDA rollout failed: cudaError {-rc}")
        return qf, vf, qdd, cs, float(ms[0])


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
