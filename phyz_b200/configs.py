"""The benchmark workloads: BASELINE.json configs 1-4 as models plus seeded
synthetic initial states and per-step controls.

No dataset exists for this path; every input is drawn from the reference's
own per-world stream recipe (rng.py) with fixed seeds. Geometry the configs
leave open is fixed here and stated next to each builder.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .model import (FREE, GRAVITY, REVOLUTE, Geometry, Joint, ModelBuilder, SpatialInertia,
                    Transform)
from .rng import KernelRng

SEED = 0x5EED
CTRL_SEED = 0xC7A1
MODEL_SEED = 0x3D0C

AXES = [np.array([1.0, 0.0, 0.0]), np.array([0.0, 1.0, 0.0]), np.array([0.0, 0.0, 1.0])]

# Passive joint terms of every actuated hinge in configs 2-4. The configs name
# none; phyz's own models give their motors damping and armature (ant
# damping 1 / armature 0.01, half_cheetah 0.5 / 0.1: models/ant.xml:18,
# models/half_cheetah.xml:18). With ant's 0.01 one of the 65536 chain worlds
# still goes non-finite within 1000 steps of N(0,1) torques (a thin rod's
# twist joint has ~1e-4 kg m^2 about its axis); 0.05 keeps every world of
# every config bounded over its horizon (checked in f64 over all worlds, two
# control seeds). Damping enters D implicitly (dt * damping, aba.rs:418-420).
ARMATURE = 0.05
DAMPING = 1.0


def _with_armature(model):
    for b in model.bodies:
        if b.joint.kind == REVOLUTE:
            b.joint.armature = ARMATURE
            b.joint.damping = DAMPING
    return model


def rod(m: float, half_len: float, eps: float = 0.0) -> SpatialInertia:
    """Uniform rod of length 2*half_len hanging along -Y from its joint
    (examples/gpu_batch.rs:31-41): I = diag(mL^2/12, eps, mL^2/12)."""
    L = 2.0 * half_len
    i = m * L * L / 12.0
    return SpatialInertia.new(m, [0.0, -half_len, 0.0], np.diag([i, eps, i]))


def capsule_inertia(m: float, r: float, length: float) -> np.ndarray:
    """Solid-cylinder approximation, axis along local z, about the COM."""
    it = m * (3.0 * r * r + length * length) / 12.0
    return np.diag([it, it, 0.5 * m * r * r])


# ── C1: double pendulum (examples/gpu_batch.rs:43-50) ────────────────────
def double_pendulum(dt: float = 0.002):
    return (ModelBuilder().gravity([0.0, -GRAVITY, 0.0]).dt(dt)
            .add_revolute_body("upper", -1, Transform.identity(), rod(1.0, 0.5))
            .add_revolute_body("lower", 0, Transform.identity(), rod(0.8, 0.4))
            .build())


# ── C2: serial chain of 32 revolute links ─────────────────────────────────
def chain(n: int = 32, dt: float = 0.001, seed: int = MODEL_SEED):
    """m ~ U(0.5, 2), half-length ~ U(0.1, 0.3), axes cycling x, y, z; rods
    hang along -Y with COM (0, -h, 0), each child joint at its parent's tip
    (0, -2 h_parent, 0); the inertia about the rod's own axis is that of a
    2 cm-radius solid rod (0.5 m r^2); every hinge carries ARMATURE and DAMPING."""
    rng = KernelRng(seed, [0])
    b = ModelBuilder().gravity([0.0, -GRAVITY, 0.0]).dt(dt)
    prev_h = 0.0
    for k in range(n):
        m = float(rng.uniform_range(0.5, 2.0)[0])
        h = float(rng.uniform_range(0.1, 0.3)[0])
        ptj = Transform.identity() if k == 0 else Transform.from_translation([0.0, -2.0 * prev_h, 0.0])
        b.add_revolute_body(f"link{k}", k - 1, ptj, rod(m, h, eps=0.5 * m * 0.02 ** 2), axis=AXES[k % 3])
        prev_h = h
    return _with_armature(b.build())


# ── C3: quadruped, Z-up ──────────────────────────────────────────────────
def quadruped(dt: float = 0.002):
    """Free torso (sphere r 0.25, 5 kg) and 4 legs of two hinges about y
    (hips at (+-0.15, +-0.15, -0.15)); thigh and shin capsules r 0.04,
    length 0.2, 0.5 kg, hanging along -Z; a foot sphere r 0.05 at the shin
    tip is the shin's collision shape. Ground z = 0, gravity -Z (the config's
    plane y = 0 restated Z-up). Hinges carry ARMATURE and DAMPING."""
    b = ModelBuilder().gravity([0.0, 0.0, -GRAVITY]).dt(dt)
    b.add_body("torso", -1, Joint.free(), SpatialInertia.sphere(5.0, 0.25))
    cap = SpatialInertia.new(0.5, [0.0, 0.0, -0.1], capsule_inertia(0.5, 0.04, 0.2))
    for leg, (sx, sy) in enumerate([(1, 1), (-1, 1), (-1, -1), (1, -1)]):
        hip = Transform.from_translation([0.15 * sx, 0.15 * sy, -0.15])
        b.add_revolute_body(f"thigh{leg}", 0, hip, cap, axis=AXES[1])
        thigh = len(b._bodies) - 1
        foot = Geometry.sphere(0.05, Transform.from_translation([0.0, 0.0, -0.2]))
        b.add_revolute_body(f"shin{leg}", thigh, Transform.from_translation([0.0, 0.0, -0.2]), cap,
                            axis=AXES[1], geometry=foot)
    return _with_armature(b.build())


# ── C4: humanoid-like tree, Z-up ─────────────────────────────────────────
def humanoid(dt: float = 0.002, seed: int = MODEL_SEED):
    """Free pelvis plus 21 hinges, depth <= 5: spine (abdomen z, y), head
    (neck x, y, z), two arms (shoulder x, y, elbow y) off the chest, two legs
    (hip x, z, y, knee y, ankle y) off the pelvis. Body masses ~ U(0.5, 8).
    Ten contact shapes: pelvis, head, forearms, thighs, shins (capsules /
    spheres) and feet (spheres). Hinges carry ARMATURE and DAMPING."""
    rng = KernelRng(seed + 1, [0])

    def mass():
        return float(rng.uniform_range(0.5, 8.0)[0])

    def link(m, length, r=0.05):
        return SpatialInertia.new(m, [0.0, 0.0, -0.5 * length], capsule_inertia(m, r, length))

    def small(m):
        return SpatialInertia.new(m, [0.0, 0.0, 0.0], np.eye(3) * (0.4 * m * 0.05 ** 2))

    T = Transform.from_translation
    down = lambda length: T([0.0, 0.0, -0.5 * length])  # noqa: E731  capsule centred on the link
    b = ModelBuilder().gravity([0.0, 0.0, -GRAVITY]).dt(dt)
    mp = mass()
    b.add_body("pelvis", -1, Joint.free(),
               SpatialInertia.new(mp, [0.0, 0.0, 0.0], capsule_inertia(mp, 0.1, 0.2)),
               geometry=Geometry.capsule(0.1, 0.2, Transform(np.array([[0.0, 0.0, 1.0], [0.0, 1.0, 0.0],
                                                                       [-1.0, 0.0, 0.0]]), np.zeros(3))))
    # spine
    b.add_revolute_body("abdomen_z", 0, T([0.0, 0.0, 0.1]), small(mass()), axis=AXES[2])
    mc = mass()
    b.add_revolute_body("chest", 1, T([0.0, 0.0, 0.05]),
                        SpatialInertia.new(mc, [0.0, 0.0, 0.15], capsule_inertia(mc, 0.12, 0.3)), axis=AXES[1])
    chest = 2
    b.add_revolute_body("neck_x", chest, T([0.0, 0.0, 0.35]), small(mass()), axis=AXES[0])
    b.add_revolute_body("neck_y", chest + 1, Transform(), small(mass()), axis=AXES[1])
    mh = mass()
    b.add_revolute_body("head", chest + 2, Transform(), SpatialInertia.new(mh, [0.0, 0.0, 0.12],
                                                                           np.eye(3) * 0.4 * mh * 0.1 ** 2),
                        axis=AXES[2], geometry=Geometry.sphere(0.1, T([0.0, 0.0, 0.12])))
    # arms off the chest
    for side, sy in (("r", -1.0), ("l", 1.0)):
        b.add_revolute_body(f"shoulder_x_{side}", chest, T([0.0, 0.2 * sy, 0.3]), small(mass()), axis=AXES[0])
        s = len(b._bodies) - 1
        mu = mass()
        b.add_revolute_body(f"upper_arm_{side}", s, Transform(), link(mu, 0.3, 0.04), axis=AXES[1])
        ua = len(b._bodies) - 1
        mf = mass()
        b.add_revolute_body(f"forearm_{side}", ua, T([0.0, 0.0, -0.3]), link(mf, 0.28, 0.035), axis=AXES[1],
                            geometry=Geometry.capsule(0.035, 0.28, down(0.28)))
    # legs off the pelvis
    for side, sy in (("r", -1.0), ("l", 1.0)):
        b.add_revolute_body(f"hip_x_{side}", 0, T([0.0, 0.1 * sy, -0.1]), small(mass()), axis=AXES[0])
        hx = len(b._bodies) - 1
        b.add_revolute_body(f"hip_z_{side}", hx, Transform(), small(mass()), axis=AXES[2])
        hz = len(b._bodies) - 1
        mt = mass()
        b.add_revolute_body(f"thigh_{side}", hz, Transform(), link(mt, 0.4, 0.06), axis=AXES[1],
                            geometry=Geometry.capsule(0.06, 0.4, down(0.4)))
        th = len(b._bodies) - 1
        ms = mass()
        b.add_revolute_body(f"shin_{side}", th, T([0.0, 0.0, -0.4]), link(ms, 0.4, 0.05), axis=AXES[1],
                            geometry=Geometry.capsule(0.05, 0.4, down(0.4)))
        sh = len(b._bodies) - 1
        mft = mass()
        b.add_revolute_body(f"foot_{side}", sh, T([0.0, 0.0, -0.4]), small(mft), axis=AXES[1],
                            geometry=Geometry.sphere(0.05, T([0.0, 0.0, 0.0])))
    return _with_armature(b.build())


@dataclass
class Config:
    name: str
    builder: object
    nworld: int
    steps: int
    ctrl_sigma: float
    contact: tuple | None  # (ground_height, stiffness, damping, friction)
    precisions: tuple


CONFIGS = {
    "c1_double_pendulum": Config("c1_double_pendulum", double_pendulum, 4096, 500, 0.0, None, ("f64",)),
    "c2_chain32": Config("c2_chain32", chain, 65536, 1000, 1.0, None, ("f32", "f64")),
    "c3_quadruped": Config("c3_quadruped", quadruped, 262144, 1000, 2.0, (0.0, 1e4, 100.0, 1.0), ("f32", "f64")),
    "c4_humanoid": Config("c4_humanoid", humanoid, 131072, 500, 1.0, (0.0, 1e4, 100.0, 1.0), ("f32", "f64")),
}


def actuated(model) -> np.ndarray:
    """DOF mask of the joints a control acts on: every hinge / slide / ball
    DOF; a free base is unactuated."""
    mask = []
    for b in model.bodies:
        mask += [b.joint.kind != FREE] * b.joint.ndof
    return np.array(mask, dtype=bool)


def initial_state(name: str, model, worlds, seed: int = SEED):
    """q0, v0 for the given world indices (one independent stream each)."""
    worlds = np.asarray(worlds)
    n, nv = worlds.size, model.nv
    rng = KernelRng(seed, worlds)
    q = np.zeros((n, nv))
    v = np.zeros((n, nv))
    if name == "c1_double_pendulum":
        for j in range(nv):
            q[:, j] = rng.uniform_range(-np.pi, np.pi)
        for j in range(nv):
            v[:, j] = rng.normal()
    elif name == "c2_chain32":
        for j in range(nv):
            q[:, j] = rng.uniform_range(-0.5, 0.5)
        for j in range(nv):
            v[:, j] = 0.5 * rng.normal()
    elif name == "c3_quadruped":
        q[:, 5] = rng.uniform_range(0.5, 1.0)  # torso height
        for j in range(6, nv):
            q[:, j] = rng.uniform_range(-0.3, 0.3)
    elif name == "c4_humanoid":
        q[:, 5] = 1.0
        for j in range(6, nv):
            q[:, j] = rng.uniform_range(-0.2, 0.2)
    else:
        raise KeyError(name)
    return q, v


def controls(name: str, model, worlds, step: int, seed: int = CTRL_SEED) -> np.ndarray:
    """Controls of one step (nworlds x nv): sigma * N(0,1) on actuated DOFs,
    drawn from the stream of (world, step)."""
    cfg = CONFIGS[name]
    worlds = np.asarray(worlds)
    out = np.zeros((worlds.size, model.nv))
    if cfg.ctrl_sigma == 0.0:
        return out
    rng = KernelRng(seed + 0x10000 * (step + 1), worlds)
    for j in np.flatnonzero(actuated(model)):
        out[:, j] = cfg.ctrl_sigma * rng.normal()
    return out


def control_schedule(name: str, model, worlds, steps: int, seed: int = CTRL_SEED) -> np.ndarray:
    return np.stack([controls(name, model, worlds, t, seed) for t in range(steps)])


# ── C5: the quadruped under an on-device policy ───────────────────────────
C5_HIDDEN = 64
C5_STEPS = 64
C5_SUBSTEPS = 1
C5_PD = (20.0, 1.0, 20.0)  # kp, kd, max force of each hinge servo
C5_SEED = 0xC5C5
C5_STD = 0.3


def c5_pd_dofs(model):
    """A PD servo on every hinge DOF of the quadruped (registration order =
    DOF order), the actions' slots."""
    from .batch_sim import PdDof

    kp, kd, mf = C5_PD
    return [PdDof(j, j, kp, kd, mf) for j in np.flatnonzero(actuated(model))]


def c5_policy_spec(model):
    """Observation 30 -> 64 -> 64 tanh -> 8 actions:
    the 8 hinge angles, the 14 velocities, torso pitch / roll / height / yaw
    error, the centre of mass over the four feet (heading frame, 3 axes) and
    a constant. Actions are PD target offsets of the 8 hinges."""
    from .policy import ObsOp, PolicySpec

    hinges = list(np.flatnonzero(actuated(model)))
    shins = [i for i, b in enumerate(model.bodies) if b.name.startswith("shin")]
    feet = [(b, (0.0, 0.0, -0.2)) for b in shins]
    obs = [ObsOp.q_minus(int(j), 0.0) for j in hinges]
    obs += [ObsOp.v(j) for j in range(model.nv)]
    obs += [ObsOp.body_pitch(0), ObsOp.body_roll(0), ObsOp.body_pos_z(0), ObsOp.body_yaw_error(0, 0.0)]
    obs += [ObsOp.com_over_support(feet, axis, heading_body=0) for axis in range(3)]
    obs += [ObsOp.const(1.0)]
    assert len(obs) == 30
    return PolicySpec(obs=obs, hidden=C5_HIDDEN, act_slots=list(range(len(hinges))), act_clamp=0.5,
                      noise_rho=0.0, input_noise=[0.0] * len(obs), history_steps=C5_STEPS)
