//! `B200BatchSimulator`: phyz-gpu's `BatchSim` surface
//! (`crates/phyz-gpu/src/cuda/mod.rs:430-1377`) over the C ABI, taking
//! phyz_model's `Model` and `State`. Packing follows `layout::pack_bodies`
//! and `layout::pack_geometries` (`crates/phyz-gpu/src/layout.rs:103-279`)
//! in f64: the body record's meaning, and the first collision instance of a
//! body (else its centred `geometry`) as its contact shape.
use crate::{check, phyzb_body, phyzb_body_plane, phyzb_heightfield, phyzb_pd_dof, Error, Precision, Simulator};
use crate::{PHYZB_CONTACT_STRIDE, PHYZB_GEOM_BOX, PHYZB_GEOM_CAPSULE, PHYZB_GEOM_CYLINDER, PHYZB_GEOM_MESH_AABB,
            PHYZB_GEOM_SPHERE};
use phyz_model::{Geometry, Heightfield, JointType, Model, State};

/// phyz-gpu's `PdDof` (pd_pipeline.rs:34-46).
#[derive(Clone, Copy, Debug)]
pub struct PdDof {
    pub q_index: usize,
    pub v_index: usize,
    pub kp: f64,
    pub kd: f64,
    pub max_force: f64,
}

/// phyz-gpu's `BodyContactGains` (contact_pipeline.rs:277-282).
#[derive(Clone, Copy, Debug)]
pub struct BodyContactGains {
    pub stiffness: f64,
    pub damping: f64,
}

/// phyz-gpu's `BodyPlane`: a contact face on one body.
#[derive(Clone, Debug)]
pub struct BodyPlane {
    pub body: usize,
    pub offset: f64,
    pub max_depth: f64,
    pub half_x: f64,
    pub half_y: f64,
    pub exclude: Vec<usize>,
}

/// One body's contact state (layout.rs:81): touching, depth, world point
/// (x, y, z), world force (x, y, z).
#[derive(Clone, Copy, Debug, Default)]
pub struct BodyContactState {
    pub touching: bool,
    pub depth: f64,
    pub point: [f64; 3],
    pub force: [f64; 3],
}

fn joint_code(t: &JointType) -> i32 {
    match t {
        JointType::Revolute | JointType::Hinge => 0,
        JointType::Prismatic | JointType::Slide => 1,
        JointType::Fixed => 2,
        JointType::Spherical | JointType::Ball => 3,
        JointType::Free => 4,
    }
}

/// The model table the C ABI takes.
pub fn pack(model: &Model) -> Vec<phyzb_body> {
    model
        .bodies
        .iter()
        .map(|b| {
            let j = &model.joints[b.joint_idx];
            let mut c = phyzb_body::default();
            c.parent = b.parent;
            c.joint_type = joint_code(&j.joint_type);
            c.mass = b.inertia.mass;
            c.com = [b.inertia.com.x, b.inertia.com.y, b.inertia.com.z];
            let i = &b.inertia.inertia;
            c.inertia = [i[(0, 0)], i[(1, 1)], i[(2, 2)], i[(0, 1)], i[(0, 2)], i[(1, 2)]];
            for r in 0..3 {
                for k in 0..3 {
                    c.ptj_rot[r * 3 + k] = j.parent_to_joint.rot[(r, k)];
                }
            }
            c.ptj_pos = [j.parent_to_joint.pos.x, j.parent_to_joint.pos.y, j.parent_to_joint.pos.z];
            c.axis = [j.axis.x, j.axis.y, j.axis.z];
            c.damping = j.damping;
            c.stiffness = j.stiffness;
            c.spring_ref = j.spring_ref;
            c.armature = j.armature;
            c.friction_loss = j.friction_loss;
            if let Some([lo, hi]) = j.limits {
                c.has_limits = 1;
                c.limit_lower = lo;
                c.limit_upper = hi;
            }
            c.limit_stiffness = j.limit_stiffness;
            c.limit_damping = j.limit_damping;
            c.geom_origin_rot = [1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0];
            let (geom, origin) = match b.collisions.first() {
                Some(inst) => (Some(&inst.geometry), Some(&inst.origin)),
                None => (b.geometry.as_ref(), None),
            };
            if let Some(o) = origin {
                c.geom_origin_pos = [o.pos.x, o.pos.y, o.pos.z];
                for r in 0..3 {
                    for k in 0..3 {
                        c.geom_origin_rot[r * 3 + k] = o.rot[(r, k)];
                    }
                }
            }
            match geom {
                Some(Geometry::Sphere { radius }) => {
                    c.geom_type = PHYZB_GEOM_SPHERE;
                    c.geom_params[0] = *radius;
                }
                Some(Geometry::Box { half_extents }) => {
                    c.geom_type = PHYZB_GEOM_BOX;
                    c.geom_params[..3].copy_from_slice(&[half_extents.x, half_extents.y, half_extents.z]);
                }
                Some(Geometry::Capsule { radius, length }) => {
                    c.geom_type = PHYZB_GEOM_CAPSULE;
                    c.geom_params[0] = *radius;
                    c.geom_params[1] = *length;
                }
                Some(Geometry::Cylinder { radius, height }) => {
                    c.geom_type = PHYZB_GEOM_CYLINDER;
                    c.geom_params[0] = *radius;
                    c.geom_params[1] = *height;
                }
                Some(Geometry::Mesh { vertices, .. }) if !vertices.is_empty() => {
                    c.geom_type = PHYZB_GEOM_MESH_AABB;
                    let mut mn = [f64::INFINITY; 3];
                    let mut mx = [f64::NEG_INFINITY; 3];
                    for v in vertices {
                        for (a, x) in [v.x, v.y, v.z].into_iter().enumerate() {
                            mn[a] = mn[a].min(x);
                            mx[a] = mx[a].max(x);
                        }
                    }
                    c.geom_params[..3].copy_from_slice(&mn);
                    c.geom_params[3..].copy_from_slice(&mx);
                }
                _ => {}
            }
            c
        })
        .collect()
}

fn c_heightfield(h: &Heightfield) -> phyzb_heightfield {
    phyzb_heightfield {
        origin: [h.origin.x, h.origin.y, h.origin.z],
        cell: h.cell,
        nx: h.nx as i32,
        ny: h.ny as i32,
        heights: h.heights.as_ptr(),
    }
}

fn c_plane(p: &BodyPlane, exclude: &[i32]) -> phyzb_body_plane {
    phyzb_body_plane {
        body: p.body as i32,
        offset: p.offset,
        max_depth: p.max_depth,
        half_x: p.half_x,
        half_y: p.half_y,
        exclude: exclude.as_ptr(),
        n_exclude: exclude.len() as i32,
    }
}

fn to_string(e: Error) -> String {
    e.to_string()
}

/// BatchSim's methods over the B200 stepper. Errors are `Result<_, String>`
/// as in the reference; `step` and `load_states` panic on failure as its
/// `step` and `load_states` do (mod.rs:799-827).
pub struct B200BatchSimulator {
    sim: Simulator,
    pub model: Model,
    pub nworld: usize,
}

impl B200BatchSimulator {
    pub fn on_device(model: Model, nworld: usize, ordinal: usize) -> Result<Self, String> {
        Self::with_precision(model, nworld, ordinal, Precision::F32)
    }
    pub fn new(model: Model, nworld: usize) -> Result<Self, String> {
        Self::on_device(model, nworld, 0)
    }
    /// F32 is the reference's precision; F64 runs the same kernels in double.
    pub fn with_precision(model: Model, nworld: usize, ordinal: usize, p: Precision) -> Result<Self, String> {
        let bodies = pack(&model);
        let g = [model.gravity.x, model.gravity.y, model.gravity.z];
        let sim = Simulator::new(&bodies, g, model.dt, nworld, ordinal as i32, p).map_err(to_string)?;
        Ok(Self { sim, model, nworld })
    }
    pub fn simulator(&mut self) -> &mut Simulator {
        &mut self.sim
    }

    pub fn set_model(&mut self, model: Model) -> Result<(), String> {
        let bodies = pack(&model);
        let g = [model.gravity.x, model.gravity.y, model.gravity.z];
        self.sim.set_model(&bodies, g, model.dt).map_err(to_string)?;
        self.model = model;
        Ok(())
    }

    pub fn enable_ground_contact(&mut self, ground_height: f64, stiffness: f64, damping: f64, friction: f64)
                                 -> Result<usize, String> {
        self.sim.enable_ground_contact(ground_height, stiffness, damping, friction).map_err(to_string)
    }
    pub fn enable_ground_contact_per_body(&mut self, ground_height: f64, friction: f64, gains: &[BodyContactGains])
                                          -> Result<usize, String> {
        let k: Vec<f64> = gains.iter().map(|g| g.stiffness).collect();
        let d: Vec<f64> = gains.iter().map(|g| g.damping).collect();
        self.sim.enable_ground_contact_per_body(ground_height, friction, &k, &d).map_err(to_string)
    }
    pub fn enable_contact_terrain(&mut self, ground_height: f64, friction: f64, gains: &[BodyContactGains],
                                  plane: Option<&BodyPlane>, hf: Option<&Heightfield>) -> Result<usize, String> {
        let k: Vec<f64> = gains.iter().map(|g| g.stiffness).collect();
        let d: Vec<f64> = gains.iter().map(|g| g.damping).collect();
        let ex: Vec<i32> = plane.map_or(Vec::new(), |p| p.exclude.iter().map(|&b| b as i32).collect());
        let pl = plane.map(|p| c_plane(p, &ex));
        let h = hf.map(c_heightfield);
        self.sim.enable_contact_terrain(ground_height, friction, &k, &d, pl.as_ref(), h.as_ref()).map_err(to_string)
    }
    pub fn enable_contact_impulse(&mut self, ground_height: f64, friction: f64, gains: Option<&[BodyContactGains]>,
                                  plane: Option<&BodyPlane>, hf: Option<&Heightfield>) -> Result<usize, String> {
        let k: Option<Vec<f64>> = gains.map(|g| g.iter().map(|x| x.stiffness).collect());
        let d: Option<Vec<f64>> = gains.map(|g| g.iter().map(|x| x.damping).collect());
        let ex: Vec<i32> = plane.map_or(Vec::new(), |p| p.exclude.iter().map(|&b| b as i32).collect());
        let pl = plane.map(|p| c_plane(p, &ex));
        let h = hf.map(c_heightfield);
        self.sim
            .enable_contact_impulse(ground_height, friction, k.as_deref(), d.as_deref(), pl.as_ref(), h.as_ref())
            .map_err(to_string)
    }
    pub fn set_heightfield(&mut self, hf: &Heightfield) -> Result<(), String> {
        self.sim.set_heightfield(&c_heightfield(hf)).map_err(to_string)
    }
    /// The reference's public `contact_sweeps` field, as a setter.
    pub fn set_contact_sweeps(&mut self, sweeps: usize) -> Result<(), String> {
        self.sim.set_contact_sweeps(sweeps as i32).map_err(to_string)
    }
    pub fn collidable_bodies(&self) -> usize {
        self.sim.collidable_bodies()
    }

    pub fn enable_pd_control(&mut self, dofs: &[PdDof]) -> Result<(), String> {
        let c: Vec<phyzb_pd_dof> = dofs
            .iter()
            .map(|d| phyzb_pd_dof {
                q_index: d.q_index as i32,
                v_index: d.v_index as i32,
                kp: d.kp,
                kd: d.kd,
                max_force: d.max_force,
            })
            .collect();
        self.sim.enable_pd_control(&c).map_err(to_string)
    }
    /// One row per world, one target per registered PD DOF.
    pub fn set_position_targets(&mut self, targets: &[Vec<f64>]) -> Result<(), String> {
        let flat: Vec<f64> = targets.iter().flat_map(|r| r.iter().copied()).collect();
        self.sim.set_position_targets(&flat).map_err(to_string)
    }

    /// Rows zero-padded or truncated to nv (layout.rs:327-337).
    fn rows<'a>(&self, it: impl Iterator<Item = &'a [f64]>) -> Vec<f64> {
        let nv = self.model.nv;
        let mut out = vec![0.0; self.nworld * nv];
        for (w, r) in it.take(self.nworld).enumerate() {
            let n = r.len().min(nv);
            out[w * nv..w * nv + n].copy_from_slice(&r[..n]);
        }
        out
    }
    pub fn load_states(&mut self, states: &[State]) {
        let q = self.rows(states.iter().map(|s| s.q.as_slice()));
        let v = self.rows(states.iter().map(|s| s.v.as_slice()));
        let c = self.rows(states.iter().map(|s| s.ctrl.as_slice()));
        self.sim.load_states(&q, &v, Some(&c)).expect("load_states");
    }
    pub fn set_controls(&mut self, controls: &[Vec<f64>]) {
        let c = self.rows(controls.iter().map(|r| r.as_slice()));
        self.sim.set_controls(&c).expect("set_controls");
    }

    pub fn try_step(&mut self) -> Result<(), String> {
        self.sim.try_step().map_err(to_string)
    }
    pub fn step(&mut self) {
        self.try_step().expect("B200 step failed")
    }
    /// n steps in one fused launch (the reference replays a cached graph).
    pub fn step_many(&mut self, n: usize) -> Result<(), String> {
        self.sim.step_many(n).map_err(to_string)
    }
    /// 0 generic kernels, 1 compiled for this model at run time, 2 automatic.
    pub fn set_kernel_specialization(&mut self, mode: i32) -> Result<(), String> {
        self.sim.set_kernel_specialization(mode).map_err(to_string)
    }

    pub fn readback_states(&mut self) -> Vec<State> {
        let nv = self.model.nv;
        let (q, v) = self.sim.readback_states().expect("readback_states");
        (0..self.nworld)
            .map(|w| {
                let mut s = self.model.default_state();
                s.q.as_mut_slice()[..nv].copy_from_slice(&q[w * nv..(w + 1) * nv]);
                s.v.as_mut_slice()[..nv].copy_from_slice(&v[w * nv..(w + 1) * nv]);
                s
            })
            .collect()
    }
    pub fn readback_contacts(&mut self) -> Result<Vec<Vec<BodyContactState>>, String> {
        let nb = self.model.bodies.len();
        let cs = self.sim.readback_contacts().map_err(to_string)?;
        Ok((0..self.nworld)
            .map(|w| {
                (0..nb)
                    .map(|b| {
                        let r = &cs[(w * nb + b) * PHYZB_CONTACT_STRIDE..(w * nb + b + 1) * PHYZB_CONTACT_STRIDE];
                        BodyContactState {
                            touching: r[0] != 0.0,
                            depth: r[1],
                            point: [r[2], r[3], r[4]],
                            force: [r[5], r[6], r[7]],
                        }
                    })
                    .collect()
            })
            .collect())
    }

    pub fn enable_state_history(&mut self, slots: usize) -> Result<(), String> {
        self.sim.enable_state_history(slots).map_err(to_string)
    }
    pub fn record_state(&mut self, slot: usize) -> Result<(), String> {
        self.sim.record_state(slot).map_err(to_string)
    }
    pub fn readback_state_history(&mut self, slot0: usize, n: usize) -> Result<Vec<Vec<State>>, String> {
        let nv = self.model.nv;
        let (q, v) = self.sim.readback_state_history(slot0, n).map_err(to_string)?;
        Ok((0..n)
            .map(|k| {
                (0..self.nworld)
                    .map(|w| {
                        let o = (k * self.nworld + w) * nv;
                        let mut s = self.model.default_state();
                        s.q.as_mut_slice()[..nv].copy_from_slice(&q[o..o + nv]);
                        s.v.as_mut_slice()[..nv].copy_from_slice(&v[o..o + nv]);
                        s
                    })
                    .collect()
            })
            .collect())
    }
}

/// Raw status check for callers mixing this wrapper with the raw API.
pub fn status(code: i32) -> Result<(), String> {
    check(code).map_err(to_string)
}
