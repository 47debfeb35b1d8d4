"""Articulated-model description, mirroring phyz's ModelBuilder.

A `Model` here is what phyz_model::Model carries for the batched path
(crates/phyz-model/src/model.rs:124-150, body.rs:8-56, joint.rs:28-70):
bodies in topological order, each with the joint that attaches it to its
parent, spatial inertia about the COM, optional primary collision shape,
plus gravity and dt. `Model.to_c()` flattens it into the C ABI's
phyzb_model (include/phyzb.h).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib

GRAVITY = 9.81  # phyz_math::GRAVITY (tang)

REVOLUTE, PRISMATIC, FIXED, BALL, FREE = 0, 1, 2, 3, 4
NDOF = {REVOLUTE: 1, PRISMATIC: 1, FIXED: 0, BALL: 3, FREE: 6}


@dataclass
class Transform:
    """tang::SpatialTransform: `rot` is the parent->child coordinate
    rotation (row-major), `pos` the child origin in parent coordinates."""

    rot: np.ndarray = field(default_factory=lambda: np.eye(3))
    pos: np.ndarray = field(default_factory=lambda: np.zeros(3))

    @staticmethod
    def identity() -> "Transform":
        return Transform()

    @staticmethod
    def from_translation(p) -> "Transform":
        return Transform(np.eye(3), np.asarray(p, dtype=np.float64))


@dataclass
class SpatialInertia:
    """tang::SpatialInertia: mass, COM (body frame), inertia about the COM."""

    mass: float
    com: np.ndarray
    inertia: np.ndarray  # 3x3 about the COM

    @staticmethod
    def new(mass, com, inertia) -> "SpatialInertia":
        return SpatialInertia(float(mass), np.asarray(com, np.float64), np.asarray(inertia, np.float64))

    @staticmethod
    def sphere(mass: float, radius: float) -> "SpatialInertia":
        i = 0.4 * mass * radius * radius
        return SpatialInertia(float(mass), np.zeros(3), np.eye(3) * i)

    @staticmethod
    def point_mass(mass: float, com) -> "SpatialInertia":
        return SpatialInertia(float(mass), np.asarray(com, np.float64), np.zeros((3, 3)))


@dataclass
class Geometry:
    """Primary collision shape with its placement in the body frame
    (layout.rs:38-52): kind is one of the PHYZB_GEOM_* codes."""

    kind: int
    params: tuple = ()
    origin: Transform = field(default_factory=Transform)

    @staticmethod
    def sphere(r, origin=None):
        return Geometry(_lib.GEOM_SPHERE, (r,), origin or Transform())

    @staticmethod
    def box(hx, hy, hz, origin=None):
        return Geometry(_lib.GEOM_BOX, (hx, hy, hz), origin or Transform())

    @staticmethod
    def capsule(r, length, origin=None):
        return Geometry(_lib.GEOM_CAPSULE, (r, length), origin or Transform())

    @staticmethod
    def cylinder(r, height, origin=None):
        return Geometry(_lib.GEOM_CYLINDER, (r, height), origin or Transform())

    @staticmethod
    def mesh_aabb(lo, hi, origin=None):
        return Geometry(_lib.GEOM_MESH_AABB, tuple(lo) + tuple(hi), origin or Transform())


@dataclass
class Heightfield:
    """Terrain as a regular grid of f32 heights: phyz_model::Heightfield
    (crates/phyz-model/src/heightfield.rs:10-37). Node (ix, iy) sits at world
    (origin.x + ix cell, origin.y + iy cell) with height origin.z +
    heights[iy * nx + ix]; sampled bilinearly, clamped to the border outside."""
    origin: tuple = (0.0, 0.0, 0.0)
    cell: float = 1.0
    nx: int = 1
    ny: int = 1
    heights: np.ndarray = field(default_factory=lambda: np.zeros(1, np.float32))

    @staticmethod
    def new(origin, cell: float, nx: int, ny: int) -> "Heightfield":
        return Heightfield(tuple(float(x) for x in origin), float(cell), int(nx), int(ny),
                           np.zeros(nx * ny, np.float32))

    @staticmethod
    def flat(height: float) -> "Heightfield":
        """The infinite plane at z = height (a 1 x 1 field)."""
        return Heightfield.new((0.0, 0.0, height), 1.0, 1, 1)

    def to_c(self):
        h = np.ascontiguousarray(self.heights, np.float32).reshape(-1)
        if h.size != self.nx * self.ny:
            raise ValueError(f"heightfield claims {self.nx}x{self.ny} nodes but carries {h.size} heights")
        c = _lib.PhyzbHeightfield((C.c_double * 3)(*self.origin), float(self.cell), int(self.nx), int(self.ny),
                                  h.ctypes.data_as(C.POINTER(C.c_float)))
        return c, h


@dataclass
class Joint:
    """phyz_model::Joint (joint.rs:28-70)."""

    kind: int
    parent_to_joint: Transform = field(default_factory=Transform)
    axis: np.ndarray = field(default_factory=lambda: np.zeros(3))
    damping: float = 0.0
    limits: tuple | None = None
    limit_stiffness: float = 1000.0  # DEFAULT_LIMIT_STIFFNESS
    limit_damping: float = 60.0  # DEFAULT_LIMIT_DAMPING
    armature: float = 0.0
    stiffness: float = 0.0
    spring_ref: float = 0.0
    friction_loss: float = 0.0

    @staticmethod
    def revolute(ptj=None, axis=(0.0, 0.0, 1.0)) -> "Joint":
        return Joint(REVOLUTE, ptj or Transform(), np.asarray(axis, np.float64))

    @staticmethod
    def prismatic(ptj, axis) -> "Joint":
        return Joint(PRISMATIC, ptj or Transform(), np.asarray(axis, np.float64))

    @staticmethod
    def spherical(ptj=None) -> "Joint":
        return Joint(BALL, ptj or Transform())

    @staticmethod
    def free(ptj=None) -> "Joint":
        return Joint(FREE, ptj or Transform())

    @staticmethod
    def fixed(ptj=None) -> "Joint":
        return Joint(FIXED, ptj or Transform())

    @property
    def ndof(self) -> int:
        return NDOF[self.kind]


@dataclass
class Body:
    name: str
    inertia: SpatialInertia
    parent: int
    joint: Joint
    geometry: Geometry | None = None


@dataclass
class Model:
    bodies: list
    gravity: np.ndarray
    dt: float
    actuators: list = field(default_factory=list)  # MJCF actuators (phyz_b200.mjcf.Actuator)

    @property
    def nbodies(self) -> int:
        return len(self.bodies)

    @property
    def nv(self) -> int:
        return sum(b.joint.ndof for b in self.bodies)

    nq = nv  # exponential coordinates: nq == nv

    @property
    def v_offsets(self) -> list:
        out, o = [], 0
        for b in self.bodies:
            out.append(o)
            o += b.joint.ndof
        return out

    q_offsets = v_offsets

    def to_c(self):
        """(PhyzbModel, body array) — keep both alive while the C side reads them."""
        nb = len(self.bodies)
        arr = (_lib.PhyzbBody * max(nb, 1))()
        for i, b in enumerate(self.bodies):
            c = arr[i]
            j = b.joint
            c.parent = b.parent
            c.joint_type = j.kind
            c.mass = b.inertia.mass
            c.com[:] = list(b.inertia.com)
            I = b.inertia.inertia
            c.inertia[:] = [I[0, 0], I[1, 1], I[2, 2], I[0, 1], I[0, 2], I[1, 2]]
            c.ptj_rot[:] = list(np.asarray(j.parent_to_joint.rot, np.float64).reshape(9))
            c.ptj_pos[:] = list(np.asarray(j.parent_to_joint.pos, np.float64))
            c.axis[:] = list(np.asarray(j.axis, np.float64))
            c.damping = j.damping
            c.stiffness = j.stiffness
            c.spring_ref = j.spring_ref
            c.armature = j.armature
            c.has_limits = 1 if j.limits is not None else 0
            lo, hi = j.limits if j.limits is not None else (0.0, 0.0)
            c.limit_lower, c.limit_upper = lo, hi
            c.limit_stiffness = j.limit_stiffness
            c.limit_damping = j.limit_damping
            c.friction_loss = j.friction_loss
            g = b.geometry
            if g is None:
                c.geom_type = 0
                c.geom_origin_rot[:] = [1, 0, 0, 0, 1, 0, 0, 0, 1]
            else:
                c.geom_type = g.kind
                p = list(g.params) + [0.0] * (6 - len(g.params))
                c.geom_params[:] = p
                c.geom_origin_pos[:] = list(np.asarray(g.origin.pos, np.float64))
                c.geom_origin_rot[:] = list(np.asarray(g.origin.rot, np.float64).reshape(9))
        m = _lib.PhyzbModel()
        m.nbodies = nb
        m.gravity[:] = list(np.asarray(self.gravity, np.float64))
        m.dt = float(self.dt)
        m.bodies = C.cast(arr, C.POINTER(_lib.PhyzbBody))
        return m, arr

    def default_state(self):
        """(q, v, ctrl) zeros, like Model::default_state (model.rs:154)."""
        return np.zeros(self.nv), np.zeros(self.nv), np.zeros(self.nv)


class ModelBuilder:
    """phyz_model::ModelBuilder (model.rs:380-550): gravity (0,0,-g) and dt
    0.001 by default; one joint per body."""

    def __init__(self):
        self._bodies: list = []
        self._gravity = np.array([0.0, 0.0, -GRAVITY])
        self._dt = 0.001

    def gravity(self, g) -> "ModelBuilder":
        self._gravity = np.asarray(g, np.float64)
        return self

    def dt(self, dt: float) -> "ModelBuilder":
        self._dt = float(dt)
        return self

    def add_body(self, name, parent, joint: Joint, inertia: SpatialInertia, geometry=None):
        self._bodies.append(Body(name, inertia, int(parent), joint, geometry))
        return self

    def add_revolute_body(self, name, parent, ptj, inertia, axis=(0.0, 0.0, 1.0), geometry=None):
        return self.add_body(name, parent, Joint.revolute(ptj, axis), inertia, geometry)

    def add_prismatic_body(self, name, parent, ptj, axis, inertia, geometry=None):
        return self.add_body(name, parent, Joint.prismatic(ptj, axis), inertia, geometry)

    def add_spherical_body(self, name, parent, ptj, inertia, geometry=None):
        return self.add_body(name, parent, Joint.spherical(ptj), inertia, geometry)

    def add_free_body(self, name, parent, ptj, inertia, geometry=None):
        return self.add_body(name, parent, Joint.free(ptj), inertia, geometry)

    def add_fixed_body(self, name, parent, ptj, inertia, geometry=None):
        return self.add_body(name, parent, Joint.fixed(ptj), inertia, geometry)

    def build(self) -> Model:
        return Model(list(self._bodies), self._gravity.copy(), self._dt)
