"""The reference's own test models and states, restated
(crates/phyz-gpu/tests/cuda_vs_cpu.rs:33-147 models, :199-244 states;
tests/joint_offset_vs_cpu.rs:18-41; phyz-rigid/tests/free_joint.rs)."""
import numpy as np

from phyz_b200.model import GRAVITY, Geometry, Joint, ModelBuilder, SpatialInertia, Transform


def rod(m, half_len):
    L = 2.0 * half_len
    i = m * L * L / 12.0
    return SpatialInertia.new(m, [0.0, -half_len, 0.0], np.diag([i, 0.0, i]))


def iso(mass, i):
    return SpatialInertia.new(mass, np.zeros(3), np.eye(3) * i)


def double_pendulum():
    return (ModelBuilder().gravity([0.0, -GRAVITY, 0.0]).dt(0.001)
            .add_revolute_body("upper", -1, Transform.identity(), rod(1.0, 0.5))
            .add_revolute_body("lower", 0, Transform.from_translation([0.0, -1.0, 0.0]), rod(1.0, 0.5))
            .build())


def arm_6dof():
    length = 0.3
    inertia = SpatialInertia.new(0.5, [0.0, 0.0, -length / 2.0], np.diag([0.00375, 0.00375, 0.001]))
    b = ModelBuilder().gravity([0.0, 0.0, -GRAVITY]).dt(0.001)
    b.add_revolute_body("j1", -1, Transform.identity(), inertia)
    for k in range(1, 6):
        b.add_revolute_body(f"j{k + 1}", k - 1, Transform.from_translation([0.0, 0.0, -length]), inertia)
    return b.build()


def free_base_with_limb():
    return (ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.001)
            .add_body("torso", -1, Joint.free(), iso(5.0, 0.3))
            .add_revolute_body("limb", 0, Transform.from_translation([0.2, 0.0, 0.0]), iso(1.0, 0.05))
            .build())


def ball_joint_model():
    return (ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.001)
            .add_body("ball", -1, Joint.spherical(),
                      SpatialInertia.new(1.0, [0.0, 0.0, -0.3], np.diag([0.05, 0.05, 0.02])))
            .build())


def prismatic_model():
    return (ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.001)
            .add_prismatic_body("slider", -1, Transform.identity(), [0.0, 0.0, 1.0], iso(1.0, 0.1))
            .build())


def free_sphere(mass=1.0, radius=0.1):
    return (ModelBuilder().gravity([0.0, 0.0, -GRAVITY]).dt(0.001)
            .add_free_body("body", -1, Transform.identity(), iso(mass, 0.4 * mass * radius * radius),
                           geometry=Geometry.sphere(radius))
            .build())


def free_box(pos=(0.0, 0.0, 0.5), half=(0.1, 0.1, 0.1), mass=1.0):
    """contact_impulse_parity.rs:48-66: a free box, its joint frame at `pos`."""
    hx, hy, hz = half
    c = mass / 3.0
    inertia = np.diag([c * (hy * hy + hz * hz), c * (hx * hx + hz * hz), c * (hx * hx + hy * hy)])
    return (ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.001)
            .add_free_body("box", -1, Transform.from_translation(list(pos)),
                           SpatialInertia.new(mass, np.zeros(3), inertia), geometry=Geometry.box(hx, hy, hz))
            .build())


def deck_and_riders(nriders=2):
    """A free deck (a thin box resting on the ground) with free riders dropped
    onto its top face: the setting of a body-attached contact plane
    (contact_pipeline.rs:318-355; the deck is body 0)."""
    b = ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.001)
    hx, hy, hz, m = 0.3, 0.15, 0.02, 2.0
    c = m / 3.0
    b.add_free_body("deck", -1, Transform.from_translation([0.0, 0.0, 0.02]),
                    SpatialInertia.new(m, np.zeros(3), np.diag([c * (hy * hy + hz * hz), c * (hx * hx + hz * hz),
                                                                c * (hx * hx + hy * hy)])),
                    geometry=Geometry.box(hx, hy, hz))
    for k in range(nriders):
        x = -0.15 + 0.3 * k / max(nriders - 1, 1)
        if k % 2 == 0:
            b.add_free_body(f"rider{k}", -1, Transform.from_translation([x, 0.0, 0.25]), iso(0.5, 0.4 * 0.5 * 0.05 ** 2),
                            geometry=Geometry.sphere(0.05))
        else:
            r = 0.04
            b.add_free_body(f"rider{k}", -1, Transform.from_translation([x, 0.02, 0.3]),
                            SpatialInertia.new(0.4, np.zeros(3), np.eye(3) * (0.4 * 2 * r * r / 3.0)),
                            geometry=Geometry.box(r, r, r))
    return b.build()


def seesaw_and_riders():
    """A plank on a hinge about y (a body whose frame the kernel relabels)
    carrying a contact plane on its top face, with free riders dropped off
    centre so the plank tips."""
    b = ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.001)
    hx, hy, hz, m = 0.4, 0.1, 0.02, 3.0
    c = m / 3.0
    b.add_revolute_body("plank", -1, Transform.from_translation([0.0, 0.0, 0.3]),
                        SpatialInertia.new(m, np.zeros(3), np.diag([c * (hy * hy + hz * hz), c * (hx * hx + hz * hz),
                                                                    c * (hx * hx + hy * hy)])),
                        axis=(0.0, 1.0, 0.0), geometry=Geometry.box(hx, hy, hz))
    b.add_free_body("ball", -1, Transform.from_translation([0.25, 0.0, 0.5]), iso(0.6, 0.4 * 0.6 * 0.05 ** 2),
                    geometry=Geometry.sphere(0.05))
    r = 0.04
    b.add_free_body("cube", -1, Transform.from_translation([-0.1, 0.03, 0.45]),
                    SpatialInertia.new(0.4, np.zeros(3), np.eye(3) * (0.4 * 2 * r * r / 3.0)),
                    geometry=Geometry.box(r, r, r))
    return b.build()


def single_step_cases():
    """(label, model, q, v, tolerance in the reference's f32 suite)."""
    cases = []
    m = double_pendulum()
    cases.append(("double pendulum", m, [0.3, 0.2], [0.1, -0.1], 5e-3))
    m = arm_6dof()
    cases.append(("6-dof arm", m, [0.1, -0.2, 0.3, -0.1, 0.2, -0.3], [0.0] * 6, 1e-2))
    m = prismatic_model()
    cases.append(("prismatic", m, [0.2], [-0.5], 1e-4))
    m = ball_joint_model()
    cases.append(("ball joint", m, [0.3, -0.2, 0.1], [0.5, -0.4, 0.3], 1e-3))
    m = free_base_with_limb()
    q = [0.2, -0.1, 0.3, 0.1, 0.2, 0.5, 0.4]
    v = [0.3, 0.0, 0.0, -0.2, 0.0, 0.0, 1.0]
    cases.append(("free base with limb", m, q, v, 1e-3))
    return cases


def armature_chain():
    """free_joint.rs:186-206 (crba_and_aba_agree_with_armature)."""
    b = (ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.002)
         .add_revolute_body("l1", -1, Transform.identity(),
                            SpatialInertia.new(1.3, [0.0, 0.0, -0.4], np.eye(3) * 0.2))
         .add_revolute_body("l2", 0, Transform.from_translation([0.0, 0.0, -0.8]),
                            SpatialInertia.new(0.7, [0.0, 0.0, -0.3], np.eye(3) * 0.1)))
    m = b.build()
    m.bodies[0].joint.armature = 0.37
    m.bodies[1].joint.armature = 0.11
    return m


def featureful():
    """A model exercising every per-joint term the CPU applies: a general
    (non-coordinate) hinge axis, a rotated parent->joint frame, damping,
    spring, armature, soft limits, dry friction, a prismatic and a fixed
    joint, a branch point and a ball joint."""
    c, s = np.cos(0.3), np.sin(0.3)
    rot = np.array([[c, -s, 0.0], [s, c, 0.0], [0.0, 0.0, 1.0]])
    b = ModelBuilder().gravity([0.0, 0.0, -9.81]).dt(0.002)
    b.add_body("base", -1, Joint.free(), SpatialInertia.new(3.0, [0.01, 0.0, 0.02], np.diag([0.1, 0.12, 0.08])))
    j = Joint.revolute(Transform(rot, np.array([0.1, 0.05, -0.1])), np.array([0.6, 0.0, 0.8]))
    j.damping, j.stiffness, j.spring_ref, j.armature = 0.3, 2.0, 0.1, 0.02
    j.limits = (-0.2, 0.2)
    j.friction_loss = 0.05
    b.add_body("a1", 0, j, SpatialInertia.new(0.8, [0.0, 0.0, -0.15], np.diag([0.01, 0.012, 0.004])))
    jp = Joint.prismatic(Transform.from_translation([0.0, 0.0, -0.3]), np.array([0.0, 0.0, 1.0]))
    jp.damping = 0.5
    b.add_body("a2", 1, jp, iso(0.4, 0.002))
    b.add_body("tip", 2, Joint.fixed(Transform.from_translation([0.0, 0.05, -0.05])), iso(0.1, 0.0005))
    jb = Joint.revolute(Transform.from_translation([-0.1, 0.0, -0.05]), np.array([1.0, 0.0, 0.0]))
    jb.armature = 0.01
    b.add_body("b1", 0, jb, SpatialInertia.new(0.6, [0.0, 0.0, -0.1], np.diag([0.005, 0.005, 0.002])))
    b.add_body("b2", 4, Joint.spherical(Transform.from_translation([0.0, 0.0, -0.2])),
               SpatialInertia.new(0.3, [0.0, 0.0, -0.05], np.diag([0.002, 0.002, 0.001])))
    return b.build()
