"""MJCF (MuJoCo XML) ingestion into the batched stepper's model table.

The host-side counterpart of phyz's `phyz-mjcf` crate (MjcfLoader,
crates/phyz-mjcf/src/parser.rs), restated in Python because the reference's
host language has no toolchain in this build. Same reading of the format:

  * `<include file>` spliced in before parsing, relative to the model file,
    nested at most 16 deep, cycles rejected (include.rs);
  * `<compiler angle eulerseq meshdir assetdir>`, `<option gravity
    timestep>`; angles in radians unless `angle="degree"` (orientation.rs);
  * `<default>` classes with nesting, `class` / `childclass` resolution
    (defaults.rs), explicit attributes over defaults (attrs.rs);
  * `<body pos>` with any of quat / axisangle / euler / xyaxes / zaxis;
    `<joint>` hinge / slide / ball / free and `<freejoint>`; several joints
    in one body become a chain of links whose all-but-last are massless
    (parser.rs:713-810); `<inertial>` (diaginertia + quat, fullinertia), or
    the inertia of the body's geoms (inertia.rs) when it is absent;
  * `<geom>` sphere / capsule / cylinder / box / mesh (`fromto` included),
    `contype="0" conaffinity="0"` visual-only; the body's first collision
    geom becomes its contact shape with its placement (the GPU path's
    `collisions[0]`, layout.rs:199-218), a mesh as its vertex AABB;
  * `<mesh>` assets from .obj / .stl (ascii or binary) files (assets.rs);
  * `<motor> <position> <velocity> <general>` actuators with MuJoCo's affine
    law gear * (gain ctrl + bias_q q + bias_v v) (parser.rs:638-690);
  * `<sensor>` entries recorded by kind and target; `<tendon>`,
    `<equality>`, `<hfield>` and unloadable meshes reported through
    `unsupported()` instead of dropped silently.
"""
from __future__ import annotations

import math
import os
import re
import struct
import xml.etree.ElementTree as ET
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .model import (BALL, FIXED, FREE, GRAVITY, PRISMATIC, REVOLUTE, Geometry, Joint, Model, SpatialInertia,
                    Transform)

ROOT_CLASS = ""
MAX_INCLUDE_DEPTH = 16


class MjcfError(ValueError):
    """A document phyz's MJCF reader refuses (MjcfError, lib.rs:28-65)."""


@dataclass
class UnsupportedFeature:
    tag: str
    detail: str


@dataclass
class SensorElement:
    name: str
    kind: str
    target: str


@dataclass
class Actuator:
    """phyz_model::Actuator: f = gear * (gain ctrl + bias_q q + bias_v v),
    ctrl clamped to ctrl_range, the force to force_range."""

    name: str
    joint_name: str
    joint_idx: int
    gear: float = 1.0
    ctrl_range: tuple | None = None
    gain: float = 1.0
    bias_q: float = 0.0
    bias_v: float = 0.0
    force_range: tuple | None = None

    def force_at(self, ctrl: float, q: float, v: float) -> float:
        if self.ctrl_range is not None:
            ctrl = min(max(ctrl, self.ctrl_range[0]), self.ctrl_range[1])
        f = self.gear * (self.gain * ctrl + self.bias_q * q + self.bias_v * v)
        if self.force_range is not None:
            lo, hi = self.force_range
            f = min(max(f, min(lo, hi)), max(lo, hi))
        return f


# ── attributes ─────────────────────────────────────────────────────────────
class Attrs:
    """An element's attributes over the defaults resolved for it."""

    def __init__(self, tag: str, own: dict, defaults: dict | None = None):
        self.tag = tag
        self.values = dict(defaults or {})
        self.values.update(own)

    def get(self, key):
        return self.values.get(key)

    def str_or(self, key, dflt):
        v = self.values.get(key)
        return dflt if v is None else v

    def floats(self, key):
        v = self.values.get(key)
        if v is None:
            return None
        try:
            return [float(x) for x in v.split()]
        except ValueError as ex:
            raise MjcfError(f"<{self.tag}> attribute '{key}' has invalid value {v!r}: {ex}") from None

    def f64(self, key):
        f = self.floats(key)
        if f is None:
            return None
        if len(f) != 1:
            raise MjcfError(f"<{self.tag}> attribute '{key}' has invalid value {self.values[key]!r}: "
                            "expected one number")
        return f[0]

    def f64_or(self, key, dflt):
        v = self.f64(key)
        return dflt if v is None else v

    def vec3(self, key):
        f = self.floats(key)
        if f is None:
            return None
        if len(f) != 3:
            raise MjcfError(f"<{self.tag}> attribute '{key}' has invalid value {self.values[key]!r}: "
                            "expected 3 numbers")
        return np.array(f, np.float64)

    def vec3_or(self, key, dflt):
        v = self.vec3(key)
        return np.array(dflt, np.float64) if v is None else v

    def flag(self, key):
        v = self.values.get(key)
        if v is None:
            return None
        if v in ("true", "1"):
            return True
        if v in ("false", "0"):
            return False
        return None  # "auto"

    def range(self, key):
        f = self.floats(key)
        if f is None or len(f) != 2:
            return None
        return (f[0], f[1])


# ── orientation (orientation.rs) ─────────────────────────────────────────
def quat_to_matrix(q):
    w, x, y, z = q
    n = math.sqrt(w * w + x * x + y * y + z * z)
    w, x, y, z = w / n, x / n, y / n, z / n
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])


def quat_axis_angle(axis, angle):
    s = math.sin(0.5 * angle)
    return (math.cos(0.5 * angle), axis[0] * s, axis[1] * s, axis[2] * s)


def quat_mul(a, b):
    aw, ax, ay, az = a
    bw, bx, by, bz = b
    return (aw * bw - ax * bx - ay * by - az * bz, aw * bx + ax * bw + ay * bz - az * by,
            aw * by - ax * bz + ay * bw + az * bx, aw * bz + ax * by - ay * bx + az * bw)


def rotation_z_to(d):
    """The rotation taking +z onto the unit vector d (shortest arc)."""
    dot = float(d[2])
    if dot > 1.0 - 1e-12:
        return np.eye(3)
    if dot < -1.0 + 1e-12:
        return quat_to_matrix(quat_axis_angle((1.0, 0.0, 0.0), math.pi))
    axis = np.cross([0.0, 0.0, 1.0], d)
    axis = axis / np.linalg.norm(axis)
    return quat_to_matrix(quat_axis_angle(axis, math.acos(min(max(dot, -1.0), 1.0))))


@dataclass
class AngleConfig:
    degrees: bool = False
    eulerseq: str = "xyz"

    def rad(self, a):
        return math.radians(a) if self.degrees else a


def parse_orientation(a: Attrs, cfg: AngleConfig):
    """Orientation of an element in its parent frame from quat, axisangle,
    euler, xyaxes or zaxis (first present, in that order); None if none."""

    def expect(key, v, n):
        if len(v) != n:
            raise MjcfError(f"<{a.tag}> attribute '{key}' has invalid value {a.get(key)!r}: "
                            f"expected {n} numbers, found {len(v)}")
        return v

    v = a.floats("quat")
    if v is not None:
        q = expect("quat", v, 4)
        if math.sqrt(sum(x * x for x in q)) < 1e-12:
            raise MjcfError(f"<{a.tag}> attribute 'quat' has invalid value {a.get('quat')!r}: "
                            "quaternion has zero norm")
        return quat_to_matrix(q)
    v = a.floats("axisangle")
    if v is not None:
        aa = expect("axisangle", v, 4)
        n = math.sqrt(aa[0] ** 2 + aa[1] ** 2 + aa[2] ** 2)
        if n < 1e-12:
            raise MjcfError(f"<{a.tag}> attribute 'axisangle': rotation axis is the zero vector")
        return quat_to_matrix(quat_axis_angle((aa[0] / n, aa[1] / n, aa[2] / n), cfg.rad(aa[3])))
    v = a.floats("euler")
    if v is not None:
        e = expect("euler", v, 3)
        q = (1.0, 0.0, 0.0, 0.0)
        for c, ang in zip(cfg.eulerseq, e):
            axis = {"x": (1.0, 0.0, 0.0), "y": (0.0, 1.0, 0.0), "z": (0.0, 0.0, 1.0)}[c.lower()]
            step = quat_axis_angle(axis, cfg.rad(ang))
            # lower case: rotating (intrinsic) axes; upper case: fixed axes
            q = quat_mul(q, step) if c.islower() else quat_mul(step, q)
        return quat_to_matrix(q)
    v = a.floats("xyaxes")
    if v is not None:
        xy = expect("xyaxes", v, 6)
        x = np.array(xy[:3])
        if np.linalg.norm(x) < 1e-12:
            raise MjcfError(f"<{a.tag}> attribute 'xyaxes': x axis is the zero vector")
        x = x / np.linalg.norm(x)
        y = np.array(xy[3:]) - x * float(np.dot(x, xy[3:]))
        if np.linalg.norm(y) < 1e-12:
            raise MjcfError(f"<{a.tag}> attribute 'xyaxes': y axis is parallel to the x axis")
        y = y / np.linalg.norm(y)
        return np.column_stack([x, y, np.cross(x, y)])
    v = a.floats("zaxis")
    if v is not None:
        z = np.array(expect("zaxis", v, 3))
        if np.linalg.norm(z) < 1e-12:
            raise MjcfError(f"<{a.tag}> attribute 'zaxis': z axis is the zero vector")
        return rotation_z_to(z / np.linalg.norm(z))
    return None


# ── mass properties of geoms (inertia.rs) ────────────────────────────────
def shape_volume(kind, s):
    if kind == "sphere":
        return 4.0 / 3.0 * math.pi * s[0] ** 3
    if kind == "capsule":
        return math.pi * s[0] ** 2 * 2.0 * s[1] + 4.0 / 3.0 * math.pi * s[0] ** 3
    if kind == "cylinder":
        return math.pi * s[0] ** 2 * 2.0 * s[1]
    return 8.0 * s[0] * s[1] * s[2]  # box


def principal_inertia(kind, s, m):
    if kind == "sphere":
        i = 0.4 * m * s[0] ** 2
        return np.array([i, i, i])
    if kind == "box":
        x, y, z = s[0], s[1], s[2]
        return np.array([m / 3.0 * (y * y + z * z), m / 3.0 * (x * x + z * z), m / 3.0 * (x * x + y * y)])
    if kind == "cylinder":
        r, h = s[0], 2.0 * s[1]
        ixx = m * (3.0 * r * r + h * h) / 12.0
        return np.array([ixx, ixx, 0.5 * m * r * r])
    # capsule: a cylinder plus two hemispherical caps at density m / volume
    r, hl = s[0], s[1]
    v_cyl = math.pi * r * r * 2.0 * hl
    v_cap = 2.0 / 3.0 * math.pi * r ** 3
    total = v_cyl + 2.0 * v_cap
    if total <= 0.0:
        return np.zeros(3)
    m_cyl, m_cap = m * v_cyl / total, m * v_cap / total
    izz = 0.5 * m_cyl * r * r + 2.0 * (0.4 * m_cap * r * r)
    d = hl + 3.0 / 8.0 * r
    cap_ixx = 83.0 / 320.0 * m_cap * r * r + m_cap * d * d
    ixx = m_cyl * (3.0 * r * r + (2.0 * hl) ** 2) / 12.0 + 2.0 * cap_ixx
    return np.array([ixx, ixx, izz])


def combine_mass(parts):
    """(mass, com, inertia about com) of several (mass, com, inertia) parts."""
    total = sum(p[0] for p in parts)
    if total <= 0.0:
        return None
    com = sum(p[0] * p[1] for p in parts) / total
    inertia = np.zeros((3, 3))
    for m, c, I in parts:
        d = c - com
        inertia += I + m * (np.eye(3) * float(d @ d) - np.outer(d, d))
    return SpatialInertia.new(total, com, inertia)


# ── mesh assets (assets.rs) ───────────────────────────────────────────────
def load_obj(text: str):
    """Vertices and triangles of a Wavefront OBJ (faces fan-triangulated;
    `v/vt/vn` and negative indices accepted)."""
    verts, faces = [], []
    for lineno, line in enumerate(text.splitlines(), 1):
        parts = line.split()
        if not parts:
            continue
        if parts[0] == "v":
            if len(parts) < 4:
                raise MjcfError(f"line {lineno}: vertex needs 3 numbers")
            verts.append([float(x) for x in parts[1:4]])
        elif parts[0] == "f":
            idx = []
            for tok in parts[1:]:
                k = int(tok.split("/")[0])
                k = k - 1 if k > 0 else len(verts) + k
                if not 0 <= k < len(verts):
                    raise MjcfError(f"line {lineno}: face index out of range")
                idx.append(k)
            for t in range(1, len(idx) - 1):
                faces.append((idx[0], idx[t], idx[t + 1]))
    if not verts:
        raise MjcfError("obj has no vertices")
    return np.array(verts, np.float64), faces


def load_stl(data: bytes):
    """Vertices and triangles of an STL, binary or ascii."""
    if len(data) >= 84:
        n = struct.unpack_from("<I", data, 80)[0]
        if 84 + 50 * n == len(data):
            verts = []
            for t in range(n):
                off = 84 + 50 * t + 12
                verts.extend(struct.unpack_from("<9f", data, off))
            v = np.array(verts, np.float64).reshape(-1, 3)
            return v, [(3 * t, 3 * t + 1, 3 * t + 2) for t in range(n)]
    try:
        text = data.decode("ascii")
    except UnicodeDecodeError:
        raise MjcfError("stl is neither binary nor ascii") from None
    verts = []
    for lineno, line in enumerate(text.splitlines(), 1):
        s = line.strip()
        if s.startswith("vertex"):
            nums = s[len("vertex"):].split()
            if len(nums) != 3:
                raise MjcfError(f"line {lineno}: vertex needs 3 numbers")
            verts.append([float(x) for x in nums])
    if not verts or len(verts) % 3:
        raise MjcfError("stl has no whole triangles")
    v = np.array(verts, np.float64)
    return v, [(3 * t, 3 * t + 1, 3 * t + 2) for t in range(len(verts) // 3)]


@dataclass
class MeshAsset:
    name: str
    vertices: np.ndarray | None = None
    faces: list = field(default_factory=list)
    load_error: str | None = None


def parse_mesh(a: Attrs, asset_dir):
    name = a.get("name")
    file = a.get("file")
    if name is None:
        name = Path(file).stem if file else ""
    scale = a.floats("scale") or [1.0, 1.0, 1.0]
    inline = a.floats("vertex")
    try:
        if inline is not None:
            if len(inline) % 3:
                raise MjcfError("inline vertex list is not a multiple of 3")
            v, f = np.array(inline, np.float64).reshape(-1, 3), []
        elif file:
            path = Path(asset_dir) / file if asset_dir is not None else Path(file)
            ext = path.suffix.lower()
            if ext == ".stl":
                v, f = load_stl(path.read_bytes())
            elif ext == ".obj":
                v, f = load_obj(path.read_text())
            else:
                raise MjcfError(f"{path}: unsupported mesh format '{ext}'")
        else:
            raise MjcfError("mesh has neither file nor vertex")
    except (OSError, MjcfError) as ex:
        return MeshAsset(name, load_error=str(ex))
    return MeshAsset(name, v * np.asarray(scale[:3], np.float64), f)


# ── <include> expansion (include.rs) ─────────────────────────────────────
def expand_includes(root: ET.Element, base_dir, depth=0, stack=()):
    """Replace every <include file> by the children of the included file's
    root element, recursively (relative to the including file's directory)."""
    for parent in list(root.iter()):
        children = list(parent)
        for idx, child in enumerate(children):
            if child.tag != "include":
                continue
            file = child.get("file")
            if not file:
                raise MjcfError("<include> is missing required attribute 'file'")
            path = (Path(base_dir) / file) if base_dir is not None else Path(file)
            key = os.path.abspath(path)
            if key in stack:
                raise MjcfError(f"include cycle through {file}")
            if depth + 1 > MAX_INCLUDE_DEPTH:
                raise MjcfError(f"includes nested deeper than {MAX_INCLUDE_DEPTH}")
            try:
                sub = ET.fromstring(path.read_text())
            except OSError as ex:
                raise MjcfError(f"include {file}: {ex}") from None
            except ET.ParseError as ex:
                raise MjcfError(f"XML parse error in {file}: {ex}") from None
            expand_includes(sub, path.parent, depth + 1, stack + (key,))
            pos = list(parent).index(child)
            parent.remove(child)
            for k, sc in enumerate(list(sub)):
                parent.insert(pos + k, sc)
    return root


# ── defaults (defaults.rs) ────────────────────────────────────────────────
class DefaultsManager:
    def __init__(self):
        self.classes = {ROOT_CLASS: {"parent": None, "by_tag": {}}}

    def declare(self, name, parent):
        c = self.classes.setdefault(name, {"parent": None, "by_tag": {}})
        c["parent"] = parent

    def set(self, cls, tag, attrs):
        c = self.classes.setdefault(cls, {"parent": None, "by_tag": {}})
        c["by_tag"].setdefault(tag, {}).update(attrs)

    def resolve(self, tag, cls):
        """The attributes `tag` inherits from class `cls` (None: the root
        class) and its ancestors, nearest winning; an unknown class gives
        nothing."""
        chain, cursor, guard = [], (ROOT_CLASS if cls is None else cls), 0
        while cursor is not None and cursor in self.classes and guard <= 64:
            node = self.classes[cursor]
            chain.append(node)
            cursor = node["parent"]
            guard += 1
        out = {}
        for node in reversed(chain):
            out.update(node["by_tag"].get(tag, {}))
        return out


# ── the loader (parser.rs) ─────────────────────────────────────────────────
@dataclass
class _Joint:
    name: str
    kind: int
    pos: np.ndarray
    axis: np.ndarray
    range: tuple | None
    limited: bool | None
    damping: float
    armature: float
    stiffness: float
    spring_ref: float
    friction_loss: float


@dataclass
class _Geom:
    name: str
    kind: str
    size: list
    pos: np.ndarray
    rot: np.ndarray
    density: float
    mass: float | None
    collides: bool
    mesh: str | None


@dataclass
class _Body:
    name: str
    pos: np.ndarray
    rot: np.ndarray
    parent: int | None
    childclass: str | None
    inertial: SpatialInertia | None = None
    joints: list = field(default_factory=list)
    geoms: list = field(default_factory=list)


class MjcfLoader:
    """phyz_mjcf::MjcfLoader: `from_file` / `from_xml_str`, then
    `build_model()` for the model table; `unsupported()`, `sensors()`,
    `meshes()` report what the document held beyond it."""

    def __init__(self, xml: str, model_dir=None):
        self.defaults = DefaultsManager()
        self.bodies: list = []
        self.actuators_raw: list = []
        self._sensors: list = []
        self._meshes: list = []
        self._unsupported: list = []
        self.gravity = np.array([0.0, 0.0, -GRAVITY])
        self.timestep = 0.002
        self.angles = AngleConfig()
        self.model_dir = Path(model_dir) if model_dir is not None else None
        self.meshdir = None
        try:
            root = ET.fromstring(xml)
        except ET.ParseError as ex:
            raise MjcfError(f"XML parse error: {ex}") from None
        expand_includes(root, self.model_dir)
        self._walk(root)
        if self.angles.degrees:
            for b in self.bodies:
                for j in b.joints:
                    if j.range is not None:
                        j.range = (math.radians(j.range[0]), math.radians(j.range[1]))
            for a in self.actuators_raw:
                if a["ctrl_range"] is not None:
                    a["ctrl_range"] = (math.radians(a["ctrl_range"][0]), math.radians(a["ctrl_range"][1]))

    @staticmethod
    def from_file(path) -> "MjcfLoader":
        path = Path(path)
        return MjcfLoader(path.read_text(), path.parent)

    @staticmethod
    def from_xml_str(xml: str) -> "MjcfLoader":
        """`<include>` resolves against the working directory here."""
        return MjcfLoader(xml, None)

    def unsupported(self):
        return list(self._unsupported)

    def sensors(self):
        return list(self._sensors)

    def meshes(self):
        return list(self._meshes)

    def armature_joints(self):
        return [j.name for b in self.bodies for j in b.joints if j.armature != 0.0]

    def _note(self, tag, detail):
        if not any(u.tag == tag and u.detail == detail for u in self._unsupported):
            self._unsupported.append(UnsupportedFeature(tag, detail))

    # ── document walk ──
    def _walk(self, root):
        for el in root:
            tag = el.tag
            if tag == "compiler":
                self._compiler(Attrs(tag, el.attrib))
            elif tag == "option":
                a = Attrs(tag, el.attrib)
                g = a.vec3("gravity")
                if g is not None:
                    self.gravity = g
                self.timestep = a.f64_or("timestep", self.timestep)
            elif tag == "default":
                self._default(el, None)
            elif tag == "asset":
                for sub in el:
                    if sub.tag == "mesh":
                        m = parse_mesh(Attrs("mesh", sub.attrib), self._asset_dir())
                        if m.load_error is not None:
                            self._note("mesh", f"mesh '{m.name}' not loaded: {m.load_error}")
                        self._meshes.append(m)
                    elif sub.tag == "hfield":
                        self._note("hfield", "heightfields in the document are dropped; load terrain with "
                                             "Heightfield and enable_contact_terrain")
            elif tag == "worldbody":
                for sub in el:
                    if sub.tag == "body":
                        self._body(sub, None)
            elif tag == "actuator":
                for sub in el:
                    if sub.tag in ("motor", "position", "velocity", "general"):
                        self._actuator(sub)
            elif tag == "sensor":
                for sub in el:
                    a = Attrs(sub.tag, sub.attrib)
                    target = a.get("joint") or a.get("site") or a.get("body") or a.get("objname") or ""
                    self._sensors.append(SensorElement(a.str_or("name", f"{sub.tag}_{target}"), sub.tag, target))
            elif tag == "equality":
                self._note("equality", "equality constraints are ignored; closed kinematic loops behave as "
                                       "open chains")
            elif tag == "tendon":
                self._note("tendon", "tendons are ignored; coupled joints move independently")

    def _compiler(self, a):
        angle = a.get("angle")
        if angle is not None:
            self.angles.degrees = angle == "degree"
        seq = a.get("eulerseq")
        if seq is not None:
            if len(seq) != 3 or any(c not in "xyzXYZ" for c in seq):
                raise MjcfError(f"<compiler> attribute 'eulerseq' has invalid value {seq!r}: expected exactly 3 "
                                "characters from x/y/z/X/Y/Z")
            self.angles.eulerseq = seq
        if a.get("assetdir") is not None:
            self.meshdir = a.get("assetdir")
        if a.get("meshdir") is not None:
            self.meshdir = a.get("meshdir")

    def _asset_dir(self):
        if self.model_dir is not None and self.meshdir is not None:
            return self.model_dir / self.meshdir
        if self.model_dir is not None:
            return self.model_dir
        return Path(self.meshdir) if self.meshdir is not None else None

    def _default(self, el, parent):
        name = el.get("class", ROOT_CLASS)
        self.defaults.declare(name, parent)
        for sub in el:
            if sub.tag == "default":
                self._default(sub, name)
            else:
                self.defaults.set(name, sub.tag, dict(sub.attrib))

    def _inherited_class(self, body_idx):
        while body_idx is not None:
            b = self.bodies[body_idx]
            if b.childclass is not None:
                return b.childclass
            body_idx = b.parent
        return None

    def _attrs(self, el, tag, body_idx):
        cls = el.get("class")
        if cls is None and body_idx is not None:
            cls = self._inherited_class(body_idx)
        return Attrs(tag, dict(el.attrib), self.defaults.resolve(tag, cls))

    def _body(self, el, parent):
        a = self._attrs(el, "body", parent)
        idx = len(self.bodies)
        rot = parse_orientation(a, self.angles)
        self.bodies.append(_Body(a.str_or("name", f"body_{idx}"), a.vec3_or("pos", (0.0, 0.0, 0.0)),
                                 np.eye(3) if rot is None else rot, parent, a.get("childclass")))
        for sub in el:
            if sub.tag in ("joint", "freejoint"):
                self._joint(sub, idx)
            elif sub.tag == "inertial":
                self._inertial(sub, idx)
            elif sub.tag == "geom":
                self._geom(sub, idx)
            elif sub.tag == "body":
                self._body(sub, idx)

    def _joint(self, el, body_idx):
        tag = el.tag
        a = self._attrs(el, tag, body_idx)
        if tag == "freejoint":
            kind = FREE
        else:
            t = a.get("type") or "hinge"
            kind = {"hinge": REVOLUTE, "slide": PRISMATIC, "ball": BALL, "free": FREE}.get(t)
            if kind is None:
                self._note("joint", f"joint type '{t}' is unknown; treated as hinge")
                kind = REVOLUTE
        axis = a.vec3("axis")
        if axis is None:
            axis = np.array([0.0, 0.0, 1.0])
        else:
            n = np.linalg.norm(axis)
            axis = axis / n if n > 0 else axis
        limited = a.flag("limited")
        rng = None if limited is False else a.range("range")
        self.bodies[body_idx].joints.append(_Joint(
            a.str_or("name", f"joint_{body_idx}"), kind, a.vec3_or("pos", (0.0, 0.0, 0.0)), axis, rng, limited,
            a.f64_or("damping", 0.0), a.f64_or("armature", 0.0), a.f64_or("stiffness", 0.0),
            a.f64_or("springref", 0.0), a.f64_or("frictionloss", 0.0)))

    def _inertial(self, el, body_idx):
        a = self._attrs(el, "inertial", body_idx)
        pos = a.vec3_or("pos", (0.0, 0.0, 0.0))
        mass = a.f64_or("mass", 1.0)
        full = a.floats("fullinertia")
        if full is not None and len(full) == 6:
            xx, yy, zz, xy, xz, yz = full
            tensor = np.array([[xx, xy, xz], [xy, yy, yz], [xz, yz, zz]])
        else:
            tensor = np.diag(a.vec3_or("diaginertia", (0.001, 0.001, 0.001)))
            q = a.floats("quat")
            if q is not None and len(q) == 4:
                r = quat_to_matrix(q)
                tensor = r @ tensor @ r.T
        self.bodies[body_idx].inertial = SpatialInertia.new(mass, pos, tensor)

    def _geom(self, el, body_idx):
        a = self._attrs(el, "geom", body_idx)
        kind = a.str_or("type", "sphere")
        mesh = a.get("mesh")
        if kind == "mesh" or mesh is not None:
            if not any(m.name == (mesh or "") and m.vertices is not None for m in self._meshes):
                self._note("geom", "mesh geoms whose asset could not be loaded are dropped; the body loses that "
                                   "collision shape and its inertia contribution")
                return
        size = a.floats("size") or [0.05]
        pos = a.vec3_or("pos", (0.0, 0.0, 0.0))
        rot = parse_orientation(a, self.angles)
        rot = np.eye(3) if rot is None else rot
        ft = a.floats("fromto")
        if ft is not None and len(ft) == 6:
            # the two ends of a capsule / cylinder axis: placement and half length
            p0, p1 = np.array(ft[:3]), np.array(ft[3:])
            axis = p1 - p0
            length = float(np.linalg.norm(axis))
            pos = 0.5 * (p0 + p1)
            size = [size[0] if size else 0.05, 0.5 * length]
            if length > 1e-12:
                rot = rotation_z_to(axis / length)
        collides = not (a.f64_or("contype", 1.0) == 0.0 and a.f64_or("conaffinity", 1.0) == 0.0)
        self.bodies[body_idx].geoms.append(_Geom(a.str_or("name", f"geom_{body_idx}"), kind, size, pos, rot,
                                                 a.f64_or("density", 1000.0), a.f64("mass"), collides, mesh))

    def _actuator(self, el):
        tag = el.tag
        a = self._attrs(el, tag, None)
        joint = a.str_or("joint", "")
        if not joint:
            self._note(tag, "actuator without a `joint` target (site/tendon actuators are not supported)")
            return
        gear = (a.floats("gear") or [1.0])[0]
        kp, kv = a.f64_or("kp", 1.0), a.f64_or("kv", 0.0)
        if tag == "position":
            gain, bq, bv = kp, -kp, -kv
        elif tag == "velocity":
            gain, bq, bv = max(kv, 1.0), 0.0, -max(kv, 1.0)
        elif tag == "general":
            gp, bp = a.floats("gainprm") or [], a.floats("biasprm") or []
            if gp or bp:
                gain = gp[0] if gp else 1.0
                bq = bp[1] if len(bp) > 1 else 0.0
                bv = bp[2] if len(bp) > 2 else 0.0
            else:
                gain, bq, bv = 1.0, 0.0, 0.0
        else:
            gain, bq, bv = 1.0, 0.0, 0.0
        self.actuators_raw.append({"name": a.get("name") or f"{tag}_{joint}", "joint": joint, "gear": gear,
                                   "ctrl_range": a.range("ctrlrange"), "force_range": a.range("forcerange"),
                                   "gain": gain, "bias_q": bq, "bias_v": bv})

    # ── the model table ──
    def _body_inertia(self, b: _Body) -> SpatialInertia:
        if b.inertial is not None:
            return b.inertial
        parts = []
        for g in b.geoms:
            if g.kind not in ("sphere", "capsule", "cylinder", "box") or g.mesh is not None:
                continue
            need = 3 if g.kind == "box" else (2 if g.kind in ("capsule", "cylinder") else 1)
            if len(g.size) < need:
                continue
            m = g.mass if g.mass is not None else g.density * shape_volume(g.kind, g.size)
            local = np.diag(principal_inertia(g.kind, g.size, m))
            parts.append((m, np.asarray(g.pos, np.float64), g.rot @ local @ g.rot.T))
        si = combine_mass(parts)
        if si is not None:
            return si
        return SpatialInertia.new(1.0, np.zeros(3), np.diag([0.001, 0.001, 0.001]))

    def _geometry(self, g: _Geom):
        """The contact shape of a geom with its placement (origin rotation
        body -> shape), or None when it cannot collide with the ground."""
        origin = Transform(g.rot.T.copy(), np.asarray(g.pos, np.float64))
        s = g.size
        if g.kind == "mesh" or g.mesh is not None:
            mesh = next((m for m in self._meshes if m.name == g.mesh and m.vertices is not None), None)
            if mesh is None or len(mesh.vertices) == 0:
                return None
            return Geometry.mesh_aabb(mesh.vertices.min(axis=0), mesh.vertices.max(axis=0), origin)
        if g.kind == "sphere":
            return Geometry.sphere(s[0] if s else 0.05, origin)
        if g.kind == "capsule":
            return Geometry.capsule(s[0] if s else 0.05, (s[1] if len(s) > 1 else 0.05) * 2.0, origin)
        if g.kind == "cylinder":
            return Geometry.cylinder(s[0] if s else 0.05, (s[1] if len(s) > 1 else 0.05) * 2.0, origin)
        if g.kind == "box":
            h = s[:3] if len(s) >= 3 else [0.05, 0.05, 0.05]
            return Geometry.box(h[0], h[1], h[2], origin)
        return None  # plane (the ground's own form) and unknown kinds do not collide here

    def build_model(self) -> Model:
        """The model table: one link per joint (a body with several joints
        becomes a chain whose all-but-last links are massless), a jointless
        body a fixed link; each body's first collision geom its contact
        shape; actuators resolved to the link of their joint."""
        bodies, body_map, joint_map = [], {}, {}
        from .model import Body

        for bi, b in enumerate(self.bodies):
            parent = body_map.get(b.parent, -1) if b.parent is not None else -1
            inertia = self._body_inertia(b)
            placement = Transform(np.asarray(b.rot, np.float64), np.asarray(b.pos, np.float64))
            if not b.joints:
                bodies.append(Body(b.name, inertia, parent, Joint(FIXED, placement)))
                body_map[bi] = len(bodies) - 1
                continue
            last = len(b.joints) - 1
            for k, je in enumerate(b.joints):
                name = b.name if len(b.joints) == 1 else f"{b.name}_{k}"
                base = placement if k == 0 else Transform()
                # base composed with a translation by the joint's pos: the
                # rotation stays, the offsets add (tang's compose)
                ptj = Transform(np.asarray(base.rot, np.float64).copy(), np.asarray(base.pos) + je.pos)
                joint = Joint(je.kind, ptj, np.asarray(je.axis, np.float64).copy())
                joint.damping = je.damping
                joint.limits = None if je.limited is False else je.range
                joint.armature = je.armature
                joint.stiffness = je.stiffness
                joint.spring_ref = je.spring_ref
                joint.friction_loss = je.friction_loss
                link_inertia = inertia if k == last else SpatialInertia.new(1e-9, np.zeros(3), np.eye(3) * 1e-9)
                link_parent = parent if k == 0 else len(bodies) - 1
                joint_map[je.name] = len(bodies)
                bodies.append(Body(name, link_inertia, link_parent, joint))
            body_map[bi] = len(bodies) - 1
        for bi, b in enumerate(self.bodies):
            colliding = [g for g in b.geoms if g.collides]
            geom = None
            for g in colliding[:1]:  # the contact shape is the first collision instance
                geom = self._geometry(g)
            bodies[body_map[bi]].geometry = geom
        model = Model(bodies, np.asarray(self.gravity, np.float64), float(self.timestep))
        for a in self.actuators_raw:
            if a["joint"] in joint_map:
                model.actuators.append(Actuator(a["name"], a["joint"], joint_map[a["joint"]], a["gear"],
                                                a["ctrl_range"], a["gain"], a["bias_q"], a["bias_v"],
                                                a["force_range"]))
        return model


def load_mjcf(path) -> Model:
    """The model table of an MJCF file."""
    return MjcfLoader.from_file(path).build_model()
