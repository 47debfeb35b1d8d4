//! Raw bindings to `libphyzb200`, the B200 (sm_100a) batched rigid-body
//! stepper, and a safe flat-array wrapper over them.
//!
//! The C ABI is `include/phyzb.h`; every struct here is `#[repr(C)]` with
//! the header's field order and types (`tests/test_rust_ffi.py` checks each
//! field offset and size against the C compiler's, every constant against
//! its `#define`, and every function against its prototype). Each entry
//! point replaces one method of phyz-gpu's `BatchSim`
//! (`crates/phyz-gpu/src/cuda/mod.rs:430-1377`); the `phyz` feature adds
//! [`phyz::B200BatchSimulator`], which takes phyz_model's `Model` and
//! `State` as `BatchSim` does.
//!
//! Conventions of the C ABI: every call returns 0 or a negative status and
//! leaves a message for [`last_error`]; host arrays are borrowed and copied;
//! one simulator handle is used by one thread at a time.
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_int, c_void, CStr};

#[cfg(feature = "phyz")]
pub mod phyz;

pub const PHYZB_ABI_VERSION: c_int = 1;

pub const PHYZB_OK: c_int = 0;
pub const PHYZB_ERR_INVALID: c_int = -1;
pub const PHYZB_ERR_CUDA: c_int = -2;
pub const PHYZB_ERR_NO_DEVICE: c_int = -3;
pub const PHYZB_ERR_STATE: c_int = -4;
pub const PHYZB_ERR_NONFINITE: c_int = -5;
pub const PHYZB_ERR_TOO_LARGE: c_int = -6;
pub const PHYZB_ERR_UNSUPPORTED: c_int = -7;
pub const PHYZB_ERR_COMM: c_int = -8;

pub const PHYZB_JOINT_REVOLUTE: i32 = 0;
pub const PHYZB_JOINT_PRISMATIC: i32 = 1;
pub const PHYZB_JOINT_FIXED: i32 = 2;
pub const PHYZB_JOINT_BALL: i32 = 3;
pub const PHYZB_JOINT_FREE: i32 = 4;

pub const PHYZB_GEOM_NONE: i32 = 0;
pub const PHYZB_GEOM_SPHERE: i32 = 1;
pub const PHYZB_GEOM_BOX: i32 = 2;
pub const PHYZB_GEOM_CAPSULE: i32 = 3;
pub const PHYZB_GEOM_CYLINDER: i32 = 4;
pub const PHYZB_GEOM_MESH_AABB: i32 = 5;

pub const PHYZB_F32: c_int = 0;
pub const PHYZB_F64: c_int = 1;
pub const PHYZB_HOST_F32: c_int = 0;
pub const PHYZB_HOST_F64: c_int = 1;

pub const PHYZB_MAX_BODIES: usize = 32;
pub const PHYZB_MAX_DOFS: usize = 64;
pub const PHYZB_CONTACT_STRIDE: usize = 8;
pub const PHYZB_DEFAULT_CONTACT_SWEEPS: i32 = 16;
pub const PHYZB_MAX_CONTACT_SWEEPS: i32 = 1024;

pub const PHYZB_OBS_CONST: i32 = 0;
pub const PHYZB_OBS_Q_MINUS: i32 = 1;
pub const PHYZB_OBS_V: i32 = 2;
pub const PHYZB_OBS_BODY_PITCH: i32 = 3;
pub const PHYZB_OBS_BODY_ROLL: i32 = 4;
pub const PHYZB_OBS_BODY_YAW_ERROR: i32 = 5;
pub const PHYZB_OBS_BODY_POS_Z: i32 = 6;
pub const PHYZB_OBS_BODY_POS: i32 = 7;
pub const PHYZB_OBS_COM_OVER_SUPPORT: i32 = 8;
pub const PHYZB_KINEMATICS_STRIDE: usize = 18;

pub const PHYZB_KL_CUMULATIVE: i32 = 0;
pub const PHYZB_KL_MINIBATCH: i32 = 1;

pub const PHYZB_GAE_NOALLOC_MAX_WORLDS: i64 = 1 << 24;
pub const PHYZB_COMM_ID_BYTES: usize = 128;

pub const PHYZB_SPECIALIZE_OFF: i32 = 0;
pub const PHYZB_SPECIALIZE_ON: i32 = 1;
pub const PHYZB_SPECIALIZE_AUTO: i32 = 2;
pub const PHYZB_SPECIALIZE_AUTO_MAX_DEPTH: i32 = 16;
pub const PHYZB_SPECIALIZE_AUTO_MAX_BODIES: i32 = 64;

/// One body and the joint that attaches it to its parent: the meaning of
/// phyz-gpu's packed body record (`crates/phyz-gpu/src/layout.rs:18-37,
/// 103-155`) in f64, plus the limits and friction loss phyz's CPU path
/// applies.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct phyzb_body {
    pub parent: i32,
    pub joint_type: i32,
    pub mass: f64,
    pub com: [f64; 3],
    pub inertia: [f64; 6],
    pub ptj_rot: [f64; 9],
    pub ptj_pos: [f64; 3],
    pub axis: [f64; 3],
    pub damping: f64,
    pub stiffness: f64,
    pub spring_ref: f64,
    pub armature: f64,
    pub has_limits: i32,
    pub limit_lower: f64,
    pub limit_upper: f64,
    pub limit_stiffness: f64,
    pub limit_damping: f64,
    pub friction_loss: f64,
    pub geom_type: i32,
    pub geom_params: [f64; 6],
    pub geom_origin_pos: [f64; 3],
    pub geom_origin_rot: [f64; 9],
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_model {
    pub nbodies: i32,
    pub gravity: [f64; 3],
    pub dt: f64,
    pub bodies: *const phyzb_body,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct phyzb_pd_dof {
    pub q_index: i32,
    pub v_index: i32,
    pub kp: f64,
    pub kd: f64,
    pub max_force: f64,
}

/// Opaque simulator handle.
#[repr(C)]
pub struct phyzb_sim {
    _opaque: [u8; 0],
}

/// Device pointers and shape of a simulator's state (zero-copy access).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_device_view {
    pub q: *mut c_void,
    pub v: *mut c_void,
    pub ctrl: *mut c_void,
    pub qdd: *mut c_void,
    pub nworld: i64,
    pub nv: i32,
    pub nbodies: i32,
    pub precision: i32,
    pub device: i32,
    pub stream: *mut c_void,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_heightfield {
    pub origin: [f64; 3],
    pub cell: f64,
    pub nx: i32,
    pub ny: i32,
    pub heights: *const f32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_body_plane {
    pub body: i32,
    pub offset: f64,
    pub max_depth: f64,
    pub half_x: f64,
    pub half_y: f64,
    pub exclude: *const i32,
    pub n_exclude: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_policy_spec {
    pub n_obs: i32,
    pub obs_ops: *const f32,
    pub n_aux: i32,
    pub obs_aux: *const f32,
    pub hidden: i32,
    pub n_act: i32,
    pub act_slots: *const i32,
    pub act_clamp: f64,
    pub act_clamp_slots: *const f64,
    pub noise_rho: f64,
    pub input_noise: *const f64,
    pub history_steps: i32,
}

/// Opaque PPO trainer handle.
#[repr(C)]
pub struct phyzb_trainer {
    _opaque: [u8; 0],
}

/// Opaque NCCL communicator handle.
#[repr(C)]
pub struct phyzb_comm {
    _opaque: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct phyzb_net_dims {
    pub n_in: i32,
    pub n_h: i32,
    pub n_out: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct phyzb_adam_cfg {
    pub lr: f64,
    pub beta1: f64,
    pub beta2: f64,
    pub eps: f64,
    pub weight_decay: f64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct phyzb_ppo_cfg {
    pub clip: f64,
    pub entropy_coef: f64,
    pub vdelta: f64,
    pub minibatch: i32,
    pub epochs: i32,
    pub target_kl: f64,
    pub kl_scale: f64,
    pub kl_mode: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct phyzb_update_stats {
    pub policy_loss: f64,
    pub value_loss: f64,
    pub kl: f64,
    pub grad_steps: i32,
    pub stopped_early: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_batch_col {
    pub base: *const f32,
    pub block: i64,
    pub features: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_policy_history {
    pub obs: *mut f32,
    pub out: *mut f32,
    pub n_obs: i32,
    pub n_act: i32,
    pub nworld: i64,
    pub steps: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct phyzb_return_cfg {
    pub reward_coef: *const f64,
    pub action_penalty: f64,
    pub gamma: f64,
    pub lambda: f64,
    pub steps: i32,
    pub normalize: i32,
}

#[link(name = "phyzb200")]
extern "C" {
    pub fn phyzb_last_error() -> *const c_char;
    pub fn phyzb_abi_version() -> c_int;
    pub fn phyzb_device_count() -> c_int;

    // lifecycle (BatchSim::new / on_device / set_model, Drop)
    pub fn phyzb_create(model: *const phyzb_model, nworld: i64, device: c_int, precision: c_int,
                        out: *mut *mut phyzb_sim) -> c_int;
    pub fn phyzb_destroy(sim: *mut phyzb_sim) -> c_int;
    pub fn phyzb_set_model(sim: *mut phyzb_sim, model: *const phyzb_model) -> c_int;

    // contact
    pub fn phyzb_enable_ground_contact(sim: *mut phyzb_sim, ground_height: f64, stiffness: f64, damping: f64,
                                       friction: f64, collidable_out: *mut i32) -> c_int;
    pub fn phyzb_enable_ground_contact_per_body(sim: *mut phyzb_sim, ground_height: f64, friction: f64,
                                                stiffness: *const f64, damping: *const f64,
                                                collidable_out: *mut i32) -> c_int;
    pub fn phyzb_enable_contact_terrain(sim: *mut phyzb_sim, ground_height: f64, friction: f64,
                                        stiffness: *const f64, damping: *const f64, plane: *const phyzb_body_plane,
                                        hf: *const phyzb_heightfield, collidable_out: *mut i32) -> c_int;
    pub fn phyzb_set_heightfield(sim: *mut phyzb_sim, hf: *const phyzb_heightfield) -> c_int;
    pub fn phyzb_enable_contact_impulse(sim: *mut phyzb_sim, ground_height: f64, friction: f64,
                                        stiffness: *const f64, damping: *const f64, plane: *const phyzb_body_plane,
                                        hf: *const phyzb_heightfield, collidable_out: *mut i32) -> c_int;
    pub fn phyzb_set_contact_sweeps(sim: *mut phyzb_sim, sweeps: i32) -> c_int;
    pub fn phyzb_disable_contact(sim: *mut phyzb_sim) -> c_int;
    pub fn phyzb_collidable_bodies(sim: *const phyzb_sim) -> c_int;

    // PD servos
    pub fn phyzb_enable_pd(sim: *mut phyzb_sim, dofs: *const phyzb_pd_dof, n: i32) -> c_int;
    pub fn phyzb_set_position_targets(sim: *mut phyzb_sim, targets: *const f64) -> c_int;

    // state and stepping
    pub fn phyzb_load_states(sim: *mut phyzb_sim, q: *const f64, v: *const f64, ctrl: *const f64) -> c_int;
    pub fn phyzb_set_controls(sim: *mut phyzb_sim, ctrl: *const f64) -> c_int;
    pub fn phyzb_step(sim: *mut phyzb_sim, n: i32) -> c_int;
    pub fn phyzb_step_with_controls(sim: *mut phyzb_sim, ctrl: *const c_void, host_dtype: c_int, n: i32) -> c_int;
    pub fn phyzb_sync(sim: *mut phyzb_sim) -> c_int;
    pub fn phyzb_status(sim: *mut phyzb_sim) -> c_int;
    pub fn phyzb_clear_status(sim: *mut phyzb_sim) -> c_int;

    // readback
    pub fn phyzb_readback_states(sim: *mut phyzb_sim, q: *mut f64, v: *mut f64) -> c_int;
    pub fn phyzb_readback_qdd(sim: *mut phyzb_sim, qdd: *mut f64) -> c_int;
    pub fn phyzb_readback_contacts(sim: *mut phyzb_sim, contact_state: *mut f64) -> c_int;
    pub fn phyzb_enable_state_history(sim: *mut phyzb_sim, slots: i32) -> c_int;
    pub fn phyzb_record_state(sim: *mut phyzb_sim, slot: i32) -> c_int;
    pub fn phyzb_readback_state_history(sim: *mut phyzb_sim, slot0: i32, n: i32, q: *mut f64, v: *mut f64)
                                        -> c_int;

    // zero-copy device path
    pub fn phyzb_device_view_get(sim: *mut phyzb_sim, out: *mut phyzb_device_view) -> c_int;
    pub fn phyzb_load_states_device(sim: *mut phyzb_sim, q: *const c_void, v: *const c_void, ctrl: *const c_void)
                                    -> c_int;
    pub fn phyzb_set_stream(sim: *mut phyzb_sim, stream: *mut c_void) -> c_int;
    pub fn phyzb_step_device_controls(sim: *mut phyzb_sim, ctrl_schedule: *const c_void, step_stride: i64,
                                      n: i32) -> c_int;
    pub fn phyzb_objective_device(sim: *mut phyzb_sim, kind: c_int, out_device_scalar: *mut c_void) -> c_int;

    // on-device control loop
    pub fn phyzb_enable_policy(sim: *mut phyzb_sim, spec: *const phyzb_policy_spec) -> c_int;
    pub fn phyzb_set_policy_weights(sim: *mut phyzb_sim, weights: *const f64, n: i64) -> c_int;
    pub fn phyzb_set_policy_std(sim: *mut phyzb_sim, std_dev: *const f64, n: i32) -> c_int;
    pub fn phyzb_set_policy_base_targets(sim: *mut phyzb_sim, rows: *const f64) -> c_int;
    pub fn phyzb_seed_policy(sim: *mut phyzb_sim, seed: u64) -> c_int;
    pub fn phyzb_run_policy(sim: *mut phyzb_sim, step: i32) -> c_int;
    pub fn phyzb_policy_rollout(sim: *mut phyzb_sim, step0: i32, n_control: i32, substeps: i32) -> c_int;
    pub fn phyzb_readback_policy_history(sim: *mut phyzb_sim, step0: i32, n: i32, obs: *mut f32, out: *mut f32)
                                         -> c_int;
    pub fn phyzb_readback_targets(sim: *mut phyzb_sim, rows: *mut f64) -> c_int;
    pub fn phyzb_readback_kinematics(sim: *mut phyzb_sim, xforms: *mut f64) -> c_int;

    // PPO update
    pub fn phyzb_trainer_create(device: i32, actor: phyzb_net_dims, critic: phyzb_net_dims, capacity: i64,
                                max_minibatch: i32, out: *mut *mut phyzb_trainer) -> c_int;
    pub fn phyzb_trainer_destroy(tr: *mut phyzb_trainer) -> c_int;
    pub fn phyzb_trainer_set_adam(tr: *mut phyzb_trainer, actor: *const phyzb_adam_cfg,
                                  critic: *const phyzb_adam_cfg) -> c_int;
    pub fn phyzb_trainer_set_params(tr: *mut phyzb_trainer, which: i32, flat: *const f64, n: i64) -> c_int;
    pub fn phyzb_trainer_params(tr: *mut phyzb_trainer, which: i32, flat: *mut f64, n: i64) -> c_int;
    pub fn phyzb_trainer_upload_batch(tr: *mut phyzb_trainer, n_rows: i64, obs_a: *const f32, obs_c: *const f32,
                                      act: *const f32, logp_old: *const f32, adv: *const f32, ret: *const f32)
                                      -> c_int;
    pub fn phyzb_trainer_update(tr: *mut phyzb_trainer, order: *const u32, n_orders: i32, cfg: *const phyzb_ppo_cfg,
                                out: *mut phyzb_update_stats) -> c_int;
    pub fn phyzb_trainer_set_batch_device(tr: *mut phyzb_trainer, n_rows: i64, cols: *const phyzb_batch_col)
                                          -> c_int;
    pub fn phyzb_trainer_update_shuffled(tr: *mut phyzb_trainer, cfg: *const phyzb_ppo_cfg, seed: u64,
                                         out: *mut phyzb_update_stats) -> c_int;
    pub fn phyzb_trainer_evaluate(tr: *mut phyzb_trainer, which: i32, x: phyzb_batch_col, n_rows: i64,
                                  out: *mut f32) -> c_int;
    pub fn phyzb_trainer_set_comm(tr: *mut phyzb_trainer, comm: *mut phyzb_comm) -> c_int;
    pub fn phyzb_policy_history_view(sim: *mut phyzb_sim, out: *mut phyzb_policy_history) -> c_int;
    pub fn phyzb_policy_advantages(sim: *mut phyzb_sim, tr: *mut phyzb_trainer, comm: *mut phyzb_comm,
                                   cfg: *const phyzb_return_cfg, adv: *mut f32, ret: *mut f32, stats: *mut f64)
                                   -> c_int;
    pub fn phyzb_gae_noalloc(rewards: *const f32, values: *const f32, nworld: i64, steps: i32, gamma: f64,
                             lambda: f64, normalize: i32, device: i32, stream: *mut c_void, adv: *mut f32,
                             ret: *mut f32, stats: *mut f64) -> c_int;
    pub fn phyzb_policy_sync_from_trainer(sim: *mut phyzb_sim, tr: *mut phyzb_trainer) -> c_int;

    // multi-GPU: rank 0 makes the id, every rank joins
    pub fn phyzb_comm_unique_id(id_out: *mut u8) -> c_int;
    pub fn phyzb_comm_init(id: *const u8, nranks: i32, rank: i32, device: i32, timeout_s: f64,
                           out: *mut *mut phyzb_comm) -> c_int;
    pub fn phyzb_comm_destroy(comm: *mut phyzb_comm) -> c_int;
    pub fn phyzb_reduce_objective(sim: *mut phyzb_sim, comm: *mut phyzb_comm, kind: c_int, timeout_s: f64,
                                  out: *mut f64) -> c_int;
    pub fn phyzb_reduce_objective_device(sim: *mut phyzb_sim, comm: *mut phyzb_comm, kind: c_int,
                                         out_device_scalar: *mut c_void) -> c_int;
    pub fn phyzb_comm_sync(comm: *mut phyzb_comm, sim: *mut phyzb_sim, timeout_s: f64) -> c_int;

    // measurement and kernel selection
    pub fn phyzb_flops_per_world_step(sim: *const phyzb_sim, flops: *mut f64, transcendentals: *mut f64) -> c_int;
    pub fn phyzb_flops_executed(sim: *const phyzb_sim, q: *const f64, v: *const f64, ctrl: *const f64, nworld: i64,
                                nsteps: i32, specialized: i32, flops: *mut f64, transcendentals: *mut f64) -> c_int;
    pub fn phyzb_measure_fma_peak(precision: c_int, tflops: *mut f64) -> c_int;
    pub fn phyzb_launch_info(sim: *const phyzb_sim, worlds_per_block: *mut i32, blocks: *mut i32,
                             smem_bytes: *mut i32, scratch_per_world: *mut i32, tmem_cols: *mut i32) -> c_int;
    pub fn phyzb_slice_plan(sim: *const phyzb_sim, nsteps: i32, steps_per_run: *mut i32, worlds_per_block: *mut i32,
                            blocks: *mut i32) -> c_int;
    pub fn phyzb_set_kernel_specialization(sim: *mut phyzb_sim, mode: i32) -> c_int;
    pub fn phyzb_get_kernel_specialization(sim: *const phyzb_sim, mode: *mut i32, active: *mut i32) -> c_int;
    pub fn phyzb_set_world_lanes(sim: *mut phyzb_sim, lanes: i32) -> c_int;
    pub fn phyzb_get_world_lanes(sim: *mut phyzb_sim, lanes: *mut i32, active: *mut i32) -> c_int;
}

/// The message of the calling thread's last failing call.
pub fn last_error() -> String {
    unsafe {
        let p = phyzb_last_error();
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

/// A failing call: its status code and message.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct Error {
    pub code: c_int,
    pub message: String,
}

impl std::fmt::Display for Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "phyzb error {}: {}", self.code, self.message)
    }
}

impl std::error::Error for Error {}

/// 0 -> Ok, otherwise the code with the thread's message.
pub fn check(code: c_int) -> Result<(), Error> {
    if code == PHYZB_OK {
        Ok(())
    } else {
        Err(Error { code, message: last_error() })
    }
}

/// Device precision of a simulator (host arrays are f64 either way).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum Precision {
    F32,
    F64,
}

/// A simulator over flat host arrays: world-major rows `[nworld][nv]` of f64
/// for q, v, controls and accelerations, `[nworld][nbodies][8]` for contact
/// state. The handle owns every device buffer; dropping it frees them.
pub struct Simulator {
    raw: *mut phyzb_sim,
    nworld: usize,
    nv: usize,
    nbodies: usize,
}

// One owner at a time may move the handle to another thread; it is not
// shared between threads (no Sync).
unsafe impl Send for Simulator {}

impl Simulator {
    /// `bodies` in topological order (parents first), as phyz packs them.
    pub fn new(bodies: &[phyzb_body], gravity: [f64; 3], dt: f64, nworld: usize, device: i32,
               precision: Precision) -> Result<Self, Error> {
        let m = phyzb_model { nbodies: bodies.len() as i32, gravity, dt, bodies: bodies.as_ptr() };
        let mut raw = std::ptr::null_mut();
        let prec = match precision {
            Precision::F32 => PHYZB_F32,
            Precision::F64 => PHYZB_F64,
        };
        check(unsafe { phyzb_create(&m, nworld as i64, device, prec, &mut raw) })?;
        let nv = bodies.iter().map(|b| joint_ndof(b.joint_type)).sum();
        Ok(Self { raw, nworld, nv, nbodies: bodies.len() })
    }

    pub fn raw(&self) -> *mut phyzb_sim {
        self.raw
    }
    pub fn nworld(&self) -> usize {
        self.nworld
    }
    pub fn nv(&self) -> usize {
        self.nv
    }

    pub fn set_model(&mut self, bodies: &[phyzb_body], gravity: [f64; 3], dt: f64) -> Result<(), Error> {
        let m = phyzb_model { nbodies: bodies.len() as i32, gravity, dt, bodies: bodies.as_ptr() };
        check(unsafe { phyzb_set_model(self.raw, &m) })?;
        self.nv = bodies.iter().map(|b| joint_ndof(b.joint_type)).sum();
        self.nbodies = bodies.len();
        Ok(())
    }

    /// Uniform penalty gains; returns the number of collidable bodies.
    pub fn enable_ground_contact(&mut self, ground_height: f64, stiffness: f64, damping: f64, friction: f64)
                                 -> Result<usize, Error> {
        let mut n = 0;
        check(unsafe { phyzb_enable_ground_contact(self.raw, ground_height, stiffness, damping, friction, &mut n) })?;
        Ok(n as usize)
    }

    /// Per-body penalty gains (one entry per body).
    pub fn enable_ground_contact_per_body(&mut self, ground_height: f64, friction: f64, stiffness: &[f64],
                                          damping: &[f64]) -> Result<usize, Error> {
        assert!(stiffness.len() == self.nbodies && damping.len() == self.nbodies, "one gain per body");
        let mut n = 0;
        check(unsafe {
            phyzb_enable_ground_contact_per_body(self.raw, ground_height, friction, stiffness.as_ptr(),
                                                 damping.as_ptr(), &mut n)
        })?;
        Ok(n as usize)
    }

    /// Velocity-level impulse contact (16 sweeps per step by default).
    pub fn enable_contact_impulse(&mut self, ground_height: f64, friction: f64, stiffness: Option<&[f64]>,
                                  damping: Option<&[f64]>, plane: Option<&phyzb_body_plane>,
                                  hf: Option<&phyzb_heightfield>) -> Result<usize, Error> {
        let mut n = 0;
        check(unsafe {
            phyzb_enable_contact_impulse(self.raw, ground_height, friction, opt_ptr(stiffness), opt_ptr(damping),
                                         plane.map_or(std::ptr::null(), |p| p as *const _),
                                         hf.map_or(std::ptr::null(), |h| h as *const _), &mut n)
        })?;
        Ok(n as usize)
    }

    /// Penalty contact over a heightfield and/or a body-attached plane.
    pub fn enable_contact_terrain(&mut self, ground_height: f64, friction: f64, stiffness: &[f64], damping: &[f64],
                                  plane: Option<&phyzb_body_plane>, hf: Option<&phyzb_heightfield>)
                                  -> Result<usize, Error> {
        let mut n = 0;
        check(unsafe {
            phyzb_enable_contact_terrain(self.raw, ground_height, friction, stiffness.as_ptr(), damping.as_ptr(),
                                         plane.map_or(std::ptr::null(), |p| p as *const _),
                                         hf.map_or(std::ptr::null(), |h| h as *const _), &mut n)
        })?;
        Ok(n as usize)
    }

    pub fn set_heightfield(&mut self, hf: &phyzb_heightfield) -> Result<(), Error> {
        check(unsafe { phyzb_set_heightfield(self.raw, hf) })
    }
    /// The reference's public `contact_sweeps` field, as a setter (1..=1024).
    pub fn set_contact_sweeps(&mut self, sweeps: i32) -> Result<(), Error> {
        check(unsafe { phyzb_set_contact_sweeps(self.raw, sweeps) })
    }
    pub fn disable_contact(&mut self) -> Result<(), Error> {
        check(unsafe { phyzb_disable_contact(self.raw) })
    }
    pub fn collidable_bodies(&self) -> usize {
        unsafe { phyzb_collidable_bodies(self.raw).max(0) as usize }
    }

    pub fn enable_pd_control(&mut self, dofs: &[phyzb_pd_dof]) -> Result<(), Error> {
        check(unsafe { phyzb_enable_pd(self.raw, dofs.as_ptr(), dofs.len() as i32) })
    }
    /// Rows `[nworld][n_pd]`.
    pub fn set_position_targets(&mut self, targets: &[f64]) -> Result<(), Error> {
        check(unsafe { phyzb_set_position_targets(self.raw, targets.as_ptr()) })
    }

    /// Rows `[nworld][nv]`; `ctrl` None keeps the held controls.
    pub fn load_states(&mut self, q: &[f64], v: &[f64], ctrl: Option<&[f64]>) -> Result<(), Error> {
        let n = self.nworld * self.nv;
        assert!(q.len() == n && v.len() == n && ctrl.map_or(true, |c| c.len() == n), "rows [nworld][nv]");
        check(unsafe { phyzb_load_states(self.raw, q.as_ptr(), v.as_ptr(), opt_ptr(ctrl)) })
    }
    pub fn set_controls(&mut self, ctrl: &[f64]) -> Result<(), Error> {
        assert!(ctrl.len() == self.nworld * self.nv, "rows [nworld][nv]");
        check(unsafe { phyzb_set_controls(self.raw, ctrl.as_ptr()) })
    }

    /// n steps with the held controls (BatchSim::step_many).
    pub fn step_many(&mut self, n: usize) -> Result<(), Error> {
        check(unsafe { phyzb_step(self.raw, n as i32) })
    }
    pub fn try_step(&mut self) -> Result<(), Error> {
        self.step_many(1)
    }
    /// Panics on error, as BatchSim::step does.
    pub fn step(&mut self) {
        self.try_step().expect("phyzb step failed")
    }
    /// len / (nworld nv) steps, each with its own control rows `[step][nworld][nv]`.
    pub fn step_with_controls(&mut self, ctrl: &[f64]) -> Result<(), Error> {
        let row = self.nworld * self.nv;
        assert!(row > 0 && ctrl.len() % row == 0, "rows [step][nworld][nv]");
        check(unsafe {
            phyzb_step_with_controls(self.raw, ctrl.as_ptr() as *const c_void, PHYZB_HOST_F64, (ctrl.len() / row) as i32)
        })
    }
    pub fn sync(&mut self) -> Result<(), Error> {
        check(unsafe { phyzb_sync(self.raw) })
    }

    /// (q, v) rows `[nworld][nv]`.
    pub fn readback_states(&mut self) -> Result<(Vec<f64>, Vec<f64>), Error> {
        let n = self.nworld * self.nv;
        let (mut q, mut v) = (vec![0.0; n], vec![0.0; n]);
        check(unsafe { phyzb_readback_states(self.raw, q.as_mut_ptr(), v.as_mut_ptr()) })?;
        Ok((q, v))
    }
    pub fn readback_qdd(&mut self) -> Result<Vec<f64>, Error> {
        let mut qdd = vec![0.0; self.nworld * self.nv];
        check(unsafe { phyzb_readback_qdd(self.raw, qdd.as_mut_ptr()) })?;
        Ok(qdd)
    }
    /// `[nworld][nbodies][PHYZB_CONTACT_STRIDE]`.
    pub fn readback_contacts(&mut self) -> Result<Vec<f64>, Error> {
        let mut cs = vec![0.0; self.nworld * self.nbodies * PHYZB_CONTACT_STRIDE];
        check(unsafe { phyzb_readback_contacts(self.raw, cs.as_mut_ptr()) })?;
        Ok(cs)
    }

    pub fn enable_state_history(&mut self, slots: usize) -> Result<(), Error> {
        check(unsafe { phyzb_enable_state_history(self.raw, slots as i32) })
    }
    pub fn record_state(&mut self, slot: usize) -> Result<(), Error> {
        check(unsafe { phyzb_record_state(self.raw, slot as i32) })
    }
    /// (q, v) of slots `slot0 .. slot0 + n`, each `[nworld][nv]`.
    pub fn readback_state_history(&mut self, slot0: usize, n: usize) -> Result<(Vec<f64>, Vec<f64>), Error> {
        let len = n * self.nworld * self.nv;
        let (mut q, mut v) = (vec![0.0; len], vec![0.0; len]);
        check(unsafe {
            phyzb_readback_state_history(self.raw, slot0 as i32, n as i32, q.as_mut_ptr(), v.as_mut_ptr())
        })?;
        Ok((q, v))
    }

    /// PHYZB_SPECIALIZE_{OFF, ON, AUTO}.
    pub fn set_kernel_specialization(&mut self, mode: i32) -> Result<(), Error> {
        check(unsafe { phyzb_set_kernel_specialization(self.raw, mode) })
    }
    /// Threads per world for branching trees (2, 4, 8; 0: one thread).
    pub fn set_world_lanes(&mut self, lanes: i32) -> Result<(), Error> {
        check(unsafe { phyzb_set_world_lanes(self.raw, lanes) })
    }
    /// How a rollout launch of `nsteps` steps runs: (steps per run, worlds
    /// per block, blocks); steps per run 0 is tile mode, else slice mode.
    pub fn slice_plan(&self, nsteps: i32) -> Result<(i32, i32, i32), Error> {
        let (mut run, mut wpb, mut blocks) = (0i32, 0i32, 0i32);
        check(unsafe { phyzb_slice_plan(self.raw, nsteps, &mut run, &mut wpb, &mut blocks) })?;
        Ok((run, wpb, blocks))
    }
}

impl Drop for Simulator {
    fn drop(&mut self) {
        unsafe {
            phyzb_destroy(self.raw);
        }
    }
}

/// DOFs of a joint code (layout.rs:23).
pub fn joint_ndof(joint_type: i32) -> usize {
    match joint_type {
        PHYZB_JOINT_REVOLUTE | PHYZB_JOINT_PRISMATIC => 1,
        PHYZB_JOINT_BALL => 3,
        PHYZB_JOINT_FREE => 6,
        _ => 0,
    }
}

fn opt_ptr(x: Option<&[f64]>) -> *const f64 {
    x.map_or(std::ptr::null(), |s| s.as_ptr())
}
