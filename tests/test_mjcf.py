"""MJCF ingestion (phyz_b200/mjcf.py) against the rules of phyz's MJCF
reader: its parser unit tests (crates/phyz-mjcf/src/parser.rs tests,
tests/parsing.rs, tests/dynamics.rs) restated on documents written here, and
the reference's own benchmark models (models/*.xml, tests/
benchmark_models.rs) where its tree is present. The models then step on the
oracle, so a loaded model is a usable model."""
import math
import os
from pathlib import Path

import numpy as np
import pytest

from phyz_b200.mjcf import MjcfError, MjcfLoader, load_mjcf
from phyz_b200.model import BALL, FIXED, FREE

# the reference tree: $PHYZ_REFERENCE, else a `reference` directory beside the
# repository; the tests that read its models skip when neither exists
REF_MODELS = Path(os.environ.get("PHYZ_REFERENCE", Path(__file__).resolve().parents[2] / "reference")) / "models"


def load(xml):
    return MjcfLoader.from_xml_str(xml)


def body(m, name):
    return next(b for b in m.bodies if b.name == name)


def test_single_hinge_and_multi_joint_bodies():
    m = load("""<mujoco><worldbody><body name="a"><inertial mass="1" diaginertia=".1 .1 .1"/>
        <joint name="j" type="hinge" axis="0 1 0"/></body></worldbody></mujoco>""").build_model()
    assert m.nbodies == 1 and m.nv == 1
    assert np.allclose(m.bodies[0].joint.axis, [0.0, 1.0, 0.0])
    # two joints in one body: a chain of two links, the first massless
    m = load("""<mujoco><worldbody><body name="a" pos="0 0 1"><inertial mass="2" diaginertia=".1 .1 .1"/>
        <joint name="x" type="hinge" axis="1 0 0"/><joint name="y" type="hinge" axis="0 1 0"/>
        </body></worldbody></mujoco>""").build_model()
    assert m.nbodies == 2 and m.nv == 2
    assert [b.name for b in m.bodies] == ["a_0", "a_1"]
    assert m.bodies[0].inertia.mass == 1e-9 and m.bodies[1].inertia.mass == 2.0
    assert m.bodies[1].parent == 0
    assert np.allclose(m.bodies[0].joint.parent_to_joint.pos, [0, 0, 1])
    assert np.allclose(m.bodies[1].joint.parent_to_joint.pos, [0, 0, 0])


def test_every_orientation_spelling_agrees():
    xml = """<mujoco><compiler angle="degree"/><worldbody>
      <body name="by_quat" quat="0.7071067811865476 0 0 0.7071067811865476"><inertial mass="1" diaginertia="1 1 1"/></body>
      <body name="by_euler" euler="0 0 90"><inertial mass="1" diaginertia="1 1 1"/></body>
      <body name="by_axisangle" axisangle="0 0 1 90"><inertial mass="1" diaginertia="1 1 1"/></body>
      <body name="by_xyaxes" xyaxes="0 1 0 -1 0 0"><inertial mass="1" diaginertia="1 1 1"/></body>
      <body name="by_zaxis" zaxis="1 0 0"><inertial mass="1" diaginertia="1 1 1"/></body>
    </worldbody></mujoco>"""
    m = load(xml).build_model()
    q = body(m, "by_quat").joint.parent_to_joint.rot
    for other in ("by_euler", "by_axisangle", "by_xyaxes"):
        assert np.linalg.norm(body(m, other).joint.parent_to_joint.rot - q) < 1e-9, other
    assert np.linalg.norm(q - np.eye(3)) > 1e-6  # not silently identity
    z = body(m, "by_zaxis").joint.parent_to_joint.rot @ [0.0, 0.0, 1.0]
    assert np.allclose(z, [1.0, 0.0, 0.0])


def test_euler_case_selects_intrinsic_or_extrinsic():
    def rot(seq):
        m = load(f"""<mujoco><compiler angle="degree" eulerseq="{seq}"/><worldbody>
            <body name="b" euler="90 90 0"><inertial mass="1" diaginertia="1 1 1"/></body>
            </worldbody></mujoco>""").build_model()
        return m.bodies[0].joint.parent_to_joint.rot

    assert np.allclose(rot("xyz") @ [0, 0, 1], [1.0, 0.0, 0.0])
    assert np.allclose(rot("XYZ") @ [0, 0, 1], [0.0, -1.0, 0.0])
    with pytest.raises(MjcfError):
        load('<mujoco><compiler eulerseq="xy"/></mujoco>')


def test_fromto_sets_capsule_length_centre_and_frame():
    m = load("""<mujoco><worldbody><body name="b"><joint type="hinge"/>
        <geom type="capsule" fromto="0 0 0 0 0 -1" size="0.03"/></body></worldbody></mujoco>""").build_model()
    g = m.bodies[0].geometry
    assert abs(g.params[0] - 0.03) < 1e-12 and abs(g.params[1] - 1.0) < 1e-12  # full length
    assert np.allclose(g.origin.pos, [0, 0, -0.5])
    # the capsule axis (shape z) points along the fromto segment
    axis_in_body = g.origin.rot.T @ [0.0, 0.0, 1.0]
    assert abs(abs(axis_in_body[2]) - 1.0) < 1e-12


def test_defaults_classes_apply_and_inherit():
    xml = """<mujoco><default><joint damping="0.5" limited="true"/>
        <default class="leg"><joint damping="9"/><geom type="capsule" size="0.05 0.2"/></default></default>
      <worldbody>
        <body name="a"><inertial mass="1" diaginertia=".1 .1 .1"/><joint name="ja" range="-1 1"/></body>
        <body name="b" childclass="leg"><joint name="jb"/><geom/></body>
      </worldbody></mujoco>"""
    m = load(xml).build_model()
    assert abs(m.bodies[0].joint.damping - 0.5) < 1e-12 and m.bodies[0].joint.limits == (-1.0, 1.0)
    assert abs(m.bodies[1].joint.damping - 9.0) < 1e-12  # childclass
    g = m.bodies[1].geometry
    assert abs(g.params[0] - 0.05) < 1e-12 and abs(g.params[1] - 0.4) < 1e-12


def test_inertia_from_geoms_and_explicit_mass():
    m = load("""<mujoco><worldbody><body name="b"><joint/><geom type="sphere" size="0.1" density="1000"/>
        </body></worldbody></mujoco>""").build_model()
    expect = 1000.0 * 4.0 / 3.0 * math.pi * 0.1 ** 3
    assert abs(m.bodies[0].inertia.mass - expect) < 1e-9
    assert np.allclose(m.bodies[0].inertia.inertia, np.eye(3) * 0.4 * expect * 0.01)
    m = load("""<mujoco><worldbody><body name="b"><joint/><geom type="box" size=".1 .1 .1" mass="7"
        density="1"/></body></worldbody></mujoco>""").build_model()
    assert abs(m.bodies[0].inertia.mass - 7.0) < 1e-12
    # two geoms: the combined COM and the parallel-axis shift
    m = load("""<mujoco><worldbody><body name="b"><joint/>
        <geom type="sphere" size="0.1" mass="1" pos="1 0 0"/><geom type="sphere" size="0.1" mass="1" pos="-1 0 0"/>
        </body></worldbody></mujoco>""").build_model()
    I = m.bodies[0].inertia
    assert I.mass == 2.0 and np.allclose(I.com, 0.0)
    assert abs(I.inertia[1, 1] - (2 * 0.4 * 0.01 + 2.0)) < 1e-12 and abs(I.inertia[0, 0] - 2 * 0.4 * 0.01) < 1e-12


def test_inertial_forms():
    m = load("""<mujoco><worldbody>
        <body name="a"><joint/><inertial mass="2" pos="0 0 0.1" fullinertia="1 2 3 0.1 0.2 0.3"/></body>
        <body name="b"><joint/><inertial mass="1" diaginertia="1 2 3" quat="0.7071067811865476 0 0 0.7071067811865476"/></body>
        </worldbody></mujoco>""").build_model()
    assert np.allclose(m.bodies[0].inertia.inertia, [[1, 0.1, 0.2], [0.1, 2, 0.3], [0.2, 0.3, 3]])
    assert np.allclose(m.bodies[0].inertia.com, [0, 0, 0.1])
    assert np.allclose(np.diag(m.bodies[1].inertia.inertia), [2, 1, 3])  # rotated 90 deg about z


def test_freejoint_ball_slide_and_fixed():
    m = load("""<mujoco><worldbody>
        <body name="f"><freejoint/><geom type="sphere" size=".1"/>
          <body name="s"><joint type="ball"/><geom type="sphere" size=".05"/>
            <body name="p"><joint type="slide" axis="1 0 0"/><geom type="box" size=".1 .1 .1"/>
              <body name="w"><geom type="sphere" size=".02"/></body></body></body></body>
        </worldbody></mujoco>""").build_model()
    assert [b.joint.kind for b in m.bodies] == [FREE, BALL, 1, FIXED]
    assert m.nv == 6 + 3 + 1 and [b.parent for b in m.bodies] == [-1, 0, 1, 2]


def test_joint_attributes_and_limited_false():
    m = load("""<mujoco><worldbody><body name="b"><inertial mass="1" diaginertia=".1 .1 .1"/>
        <joint range="-0.5 0.5" damping="0.1" armature="0.05" stiffness="3" springref="0.2" frictionloss="0.7"/>
        </body><body name="c"><inertial mass="1" diaginertia=".1 .1 .1"/><joint range="-1 1" limited="false"/>
        </body></worldbody></mujoco>""").build_model()
    j = m.bodies[0].joint
    assert j.limits == (-0.5, 0.5) and (j.damping, j.armature, j.stiffness, j.spring_ref, j.friction_loss) == \
        (0.1, 0.05, 3.0, 0.2, 0.7)
    assert m.bodies[1].joint.limits is None


def test_degree_compiler_converts_ranges():
    L = load("""<mujoco><compiler angle="degree"/><worldbody><body name="b">
        <inertial mass="1" diaginertia=".1 .1 .1"/><joint name="j" range="-90 90"/></body></worldbody>
        <actuator><motor joint="j" ctrlrange="-90 90"/></actuator></mujoco>""")
    m = L.build_model()
    assert abs(m.bodies[0].joint.limits[0] + math.pi / 2) < 1e-12
    assert abs(m.actuators[0].ctrl_range[1] - math.pi / 2) < 1e-12


def test_actuators_use_the_affine_law():
    m = load("""<mujoco><worldbody>
        <body name="a"><inertial mass="1" diaginertia=".1 .1 .1"/><joint name="j1"/></body>
        <body name="b"><inertial mass="1" diaginertia=".1 .1 .1"/><joint name="j2"/></body>
        <body name="c"><inertial mass="1" diaginertia=".1 .1 .1"/><joint name="j3"/></body>
        </worldbody><actuator><motor name="m" joint="j1" gear="100" ctrlrange="-1 1"/>
        <position name="p" joint="j2" kp="10" kv="2"/><velocity name="v" joint="j3" kv="5"/>
        </actuator></mujoco>""").build_model()
    mo, p, v = m.actuators
    assert mo.ctrl_range == (-1.0, 1.0) and abs(mo.force_at(0.5, 1.0, 2.0) - 50.0) < 1e-9
    assert abs(mo.force_at(7.5, 0.0, 0.0) - mo.force_at(1.0, 0.0, 0.0)) < 1e-12  # ctrl clamped
    assert abs(p.force_at(1.0, 0.5, 0.25) - 4.5) < 1e-9  # kp (ctrl - q) - kv v
    assert abs(v.force_at(2.0, 0.0, 0.5) - 7.5) < 1e-9  # kv (ctrl - v)
    assert [a.joint_idx for a in m.actuators] == [0, 1, 2]


def test_unsupported_features_sensors_and_visual_geoms():
    L = load("""<mujoco><asset><mesh name="nope" file="missing.stl"/></asset>
        <worldbody><body name="b"><joint name="j"/><geom type="sphere" size=".1" contype="0" conaffinity="0"/>
        <geom type="mesh" mesh="nope"/></body></worldbody>
        <tendon/><equality/><sensor><jointpos joint="j"/><framepos objname="b"/></sensor></mujoco>""")
    tags = [u.tag for u in L.unsupported()]
    assert "mesh" in tags and "tendon" in tags and "equality" in tags
    assert [(s.kind, s.target) for s in L.sensors()] == [("jointpos", "j"), ("framepos", "b")]
    m = L.build_model()
    assert m.bodies[0].geometry is None  # visual only: no contact shape
    assert m.bodies[0].inertia.mass > 0.0  # but it still carries mass


def test_includes_and_mesh_assets(tmp_path):
    (tmp_path / "parts.xml").write_text("""<mujoco><worldbody><body name="inc"><joint/>
        <geom type="mesh" mesh="tri"/></body></worldbody></mujoco>""")
    (tmp_path / "meshes").mkdir()
    (tmp_path / "meshes" / "tri.obj").write_text("v 0 0 0\nv 1 0 0\nv 0 2 -1\nf 1 2 3\n")
    (tmp_path / "main.xml").write_text("""<mujoco><compiler meshdir="meshes"/>
        <asset><mesh name="tri" file="tri.obj" scale="1 1 1"/></asset><include file="parts.xml"/></mujoco>""")
    m = load_mjcf(tmp_path / "main.xml")
    assert m.nbodies == 1 and m.bodies[0].name == "inc"
    g = m.bodies[0].geometry
    assert np.allclose(g.params, [0, 0, -1, 1, 2, 0])  # the mesh's AABB
    (tmp_path / "a.xml").write_text('<mujoco><include file="b.xml"/></mujoco>')
    (tmp_path / "b.xml").write_text('<mujoco><include file="a.xml"/></mujoco>')
    with pytest.raises(MjcfError, match="cycle"):
        MjcfLoader.from_file(tmp_path / "a.xml")


def test_binary_and_ascii_stl(tmp_path):
    import struct

    tri = [(0, 0, 0), (1, 0, 0), (0, 1, 0)]
    data = b"\0" * 80 + struct.pack("<I", 1) + struct.pack("<3f", 0, 0, 1)
    data += b"".join(struct.pack("<3f", *v) for v in tri) + b"\0\0"
    (tmp_path / "b.stl").write_bytes(data)
    (tmp_path / "a.stl").write_text("solid t\nfacet normal 0 0 1\nouter loop\n vertex 0 0 0\n vertex 2 0 0\n"
                                    " vertex 0 1 0\nendloop\nendfacet\nendsolid t\n")
    for name, hi in (("b.stl", 1.0), ("a.stl", 2.0)):
        (tmp_path / "m.xml").write_text(f"""<mujoco><asset><mesh name="m" file="{name}"/></asset>
            <worldbody><body name="b"><joint/><geom type="mesh" mesh="m"/></body></worldbody></mujoco>""")
        assert abs(load_mjcf(tmp_path / "m.xml").bodies[0].geometry.params[3] - hi) < 1e-6


@pytest.mark.skipif(not REF_MODELS.exists(), reason="the reference tree is not present")
def test_reference_benchmark_models():
    expect = {"ant": (9, 14, 8), "half_cheetah": (None, 12, 6), "humanoid": (None, 23, 17),
              "shadow_hand": (None, 24, 20)}
    for name, (nb, nv, nact) in expect.items():
        L = MjcfLoader.from_file(REF_MODELS / f"{name}.xml")
        m = L.build_model()
        assert m.nv == nv and len(m.actuators) == nact, name
        if nb is not None:
            assert m.nbodies == nb
        assert not L.unsupported(), (name, L.unsupported())
        assert all(b.inertia.mass > 0.0 for b in m.bodies)
    ant = load_mjcf(REF_MODELS / "ant.xml")
    assert sum(b.geometry is not None for b in ant.bodies) >= 9 and abs(ant.gravity[2] + 9.81) < 1e-12
    assert MjcfLoader.from_file(REF_MODELS / "ant.xml").armature_joints()
    cheetah = load_mjcf(REF_MODELS / "half_cheetah.xml")
    assert abs(next(a for a in cheetah.actuators if a.joint_name == "ffoot").gear - 30.0) < 1e-12
    hand = load_mjcf(REF_MODELS / "shadow_hand.xml")
    assert hand.actuators[0].gain > 0.0 and hand.actuators[0].bias_q < 0.0


def test_a_loaded_model_steps_on_the_oracle(oracle):
    """A small legged robot written as MJCF, dropped on the ground on the
    oracle: it stays finite and comes to rest on its feet."""
    m = load_mjcf_string(ROBOT)
    q, v = np.zeros((2, m.nv)), np.zeros((2, m.nv))
    q[:, 5] = 0.5
    q, v, _, cs = oracle.rollout(m, q, v, np.zeros((2, m.nv)), nsteps=800, contact=(0.0, 1.0, 2e4, 400.0))
    assert np.all(np.isfinite(q)) and cs[:, :, 0].sum() > 0
    assert 0.05 < q[0, 5] + 0.0 < 0.6


def load_mjcf_string(xml):
    return MjcfLoader.from_xml_str(xml).build_model()


# A quadruped in MJCF (written for these tests): free torso, four two-hinge
# legs of capsules defined through a default class and fromto.
ROBOT = """<mujoco>
  <option timestep="0.002"/>
  <default><joint damping="1" range="-1 1"/><geom type="capsule" size="0.04" density="500"/>
    <default class="foot"><geom type="sphere" size="0.05"/></default></default>
  <worldbody>
    <body name="torso"><freejoint/><geom type="sphere" size="0.2"/>
      <body name="l0" pos="0.2 0.2 0"><joint axis="0 1 0"/><geom fromto="0 0 0 0 0 -0.2"/>
        <body name="f0" pos="0 0 -0.2"><joint axis="0 1 0"/><geom class="foot"/></body></body>
      <body name="l1" pos="-0.2 0.2 0"><joint axis="0 1 0"/><geom fromto="0 0 0 0 0 -0.2"/>
        <body name="f1" pos="0 0 -0.2"><joint axis="0 1 0"/><geom class="foot"/></body></body>
      <body name="l2" pos="0.2 -0.2 0"><joint axis="0 1 0"/><geom fromto="0 0 0 0 0 -0.2"/>
        <body name="f2" pos="0 0 -0.2"><joint axis="0 1 0"/><geom class="foot"/></body></body>
      <body name="l3" pos="-0.2 -0.2 0"><joint axis="0 1 0"/><geom fromto="0 0 0 0 0 -0.2"/>
        <body name="f3" pos="0 0 -0.2"><joint axis="0 1 0"/><geom class="foot"/></body></body>
    </body>
  </worldbody>
  <actuator><motor joint="joint_1" gear="50"/></actuator>
</mujoco>"""
