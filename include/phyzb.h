/*
 * phyzb.h — C ABI of the B200 batched rigid-body stepper (libphyzb200.so).
 *
 * This is the drop-in boundary for phyz-gpu's batched-simulation path: one
 * opaque handle owns every device buffer of N independent worlds of one
 * articulated model, exactly as `phyz_gpu::cuda::BatchSim` does
 * (crates/phyz-gpu/src/cuda/mod.rs:430-468), and each entry point below
 * replaces one method of that type. Host arrays are caller-owned and copied
 * in and out; world-major f64 rows, as phyz's `State` packs them
 * (crates/phyz-gpu/src/layout.rs:340-372).
 *
 * Conventions (mirroring the reference's `Result<_, String>`):
 *   - every function returns PHYZB_OK (0) or a negative PHYZB_ERR_* code;
 *   - the message of the last failure on the calling thread is returned by
 *     phyzb_last_error() (thread-local, valid until the next failing call);
 *   - one handle is driven by one host thread at a time;
 *   - nothing here allocates except phyzb_create / phyzb_enable_* (device
 *     buffers) and the staging used by the *_host bulk copies;
 *   - no call ever traps the GPU: device-side failures (non-finite state)
 *     are recorded in a status word that phyzb_status() reads;
 *   - every wait on the device is bounded: stream waits give up after
 *     $PHYZB_SYNC_TIMEOUT seconds (default 600; the kernels hold no spin)
 *     with PHYZB_ERR_CUDA, collectives after the caller's timeout with
 *     PHYZB_ERR_COMM.
 *
 * Joint, geometry and DOF conventions are phyz's:
 *   - joint types use the packed-body-table codes of layout.rs:23;
 *   - free-joint q = [exp-coords(3), pos(3)], v = [angular(3), linear(3)]
 *     (crates/phyz-model/src/joint.rs:278-306); nq == nv;
 *   - bodies are topologically sorted (parent < child), body i owns joint i;
 *   - ground contact is Z-up (phyz_kernels.cu:641-643).
 */
#ifndef PHYZB_H
#define PHYZB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PHYZB_ABI_VERSION 1

/* ── status codes ─────────────────────────────────────────────────────── */
#define PHYZB_OK 0
#define PHYZB_ERR_INVALID (-1)     /* bad argument or model */
#define PHYZB_ERR_CUDA (-2)        /* CUDA runtime call failed */
#define PHYZB_ERR_NO_DEVICE (-3)   /* no CUDA device / driver */
#define PHYZB_ERR_STATE (-4)       /* call not valid in this state (e.g. contact off) */
#define PHYZB_ERR_NONFINITE (-5)   /* a world's state went non-finite on device */
#define PHYZB_ERR_TOO_LARGE (-6)   /* model does not fit the kernel's limits */
#define PHYZB_ERR_UNSUPPORTED (-7) /* feature outside the implemented path */
#define PHYZB_ERR_COMM (-8)        /* NCCL missing, collective failed or timed out */

/* ── enums ────────────────────────────────────────────────────────────── */
/* Joint codes: crates/phyz-gpu/src/layout.rs:23 ([1] joint_type). */
#define PHYZB_JOINT_REVOLUTE 0
#define PHYZB_JOINT_PRISMATIC 1
#define PHYZB_JOINT_FIXED 2
#define PHYZB_JOINT_BALL 3
#define PHYZB_JOINT_FREE 4

/* Geometry codes: crates/phyz-gpu/src/layout.rs:42 ([0] geom_type). */
#define PHYZB_GEOM_NONE 0
#define PHYZB_GEOM_SPHERE 1
#define PHYZB_GEOM_BOX 2
#define PHYZB_GEOM_CAPSULE 3
#define PHYZB_GEOM_CYLINDER 4
#define PHYZB_GEOM_MESH_AABB 5

/* Device precision of a simulator. The host-side arrays stay f64. */
#define PHYZB_F32 0
#define PHYZB_F64 1

/* Element type of a host bulk buffer (phyzb_step_with_controls). */
#define PHYZB_HOST_F32 0
#define PHYZB_HOST_F64 1

/* Maximum bodies per world (layout.rs:100 MAX_BODIES). */
#define PHYZB_MAX_BODIES 32
/* Maximum DOFs per world (every body a free joint would be 192; the
 * kernels bound nv by this). */
#define PHYZB_MAX_DOFS 64

/* Floats per body in phyzb_readback_contacts output: touching, depth,
 * point[3], force[3] — the first 8 slots of layout.rs:68-80. */
#define PHYZB_CONTACT_STRIDE 8

/* ── model description ────────────────────────────────────────────────── */

/* One body and the joint that attaches it to its parent. Field meanings are
 * phyz's: phyz_model::Body (crates/phyz-model/src/body.rs:8-56) with its
 * SpatialInertia about the COM, and phyz_model::Joint
 * (crates/phyz-model/src/joint.rs:28-70). */
typedef struct phyzb_body {
    int32_t parent;     /* -1 for a root attached to the world */
    int32_t joint_type; /* PHYZB_JOINT_* */
    double mass;
    double com[3];      /* centre of mass, body frame */
    double inertia[6];  /* rotational inertia about the COM: xx, yy, zz, xy, xz, yz */
    double ptj_rot[9];  /* parent->joint coordinate rotation, row-major */
    double ptj_pos[3];  /* joint origin in parent coordinates */
    double axis[3];     /* hinge / slide axis, joint frame */
    double damping;     /* viscous: f = -damping * qd, implicit in D */
    double stiffness;   /* passive spring (1-DOF): f = -k (q - spring_ref) */
    double spring_ref;
    double armature;    /* rotor inertia on the D diagonal */
    int32_t has_limits; /* 1-DOF soft limits (joint.rs:184-230) */
    double limit_lower, limit_upper;
    double limit_stiffness, limit_damping;
    double friction_loss; /* smoothed Coulomb: -mu tanh(qd / 1e-3) (joint.rs:240-245) */
    /* primary collision shape (layout.rs:38-52 semantics) */
    int32_t geom_type;          /* PHYZB_GEOM_* */
    double geom_params[6];      /* sphere r | box hx,hy,hz | capsule r,len | cylinder r,h | mesh min[3],max[3] */
    double geom_origin_pos[3];  /* shape origin, body frame */
    double geom_origin_rot[9];  /* body -> shape coordinates, row-major */
} phyzb_body;

/* The model shared by every world: phyz_model::Model
 * (crates/phyz-model/src/model.rs:124-150) restricted to what the batched
 * path reads. */
typedef struct phyzb_model {
    int32_t nbodies;
    double gravity[3];
    double dt;
    const phyzb_body* bodies; /* nbodies entries */
} phyzb_model;

/* One PD-servoed DOF: phyz_gpu::PdDof (crates/phyz-gpu/src/pd_pipeline.rs,
 * packed by layout.rs:300-312). */
typedef struct phyzb_pd_dof {
    int32_t q_index;
    int32_t v_index;
    double kp, kd, max_force;
} phyzb_pd_dof;

typedef struct phyzb_sim phyzb_sim; /* opaque */

/* Device view of a simulator's resident state, for zero-copy callers
 * (torch tensors, other kernels). All arrays are structure-of-arrays:
 * element (world w, dof j) of q lives at q[j * nworld + w]. */
typedef struct phyzb_device_view {
    void* q;        /* nv x nworld */
    void* v;        /* nv x nworld */
    void* ctrl;     /* nv x nworld */
    void* qdd;      /* nv x nworld, accelerations of the last step */
    int64_t nworld;
    int32_t nv;
    int32_t nbodies;
    int32_t precision; /* PHYZB_F32 / PHYZB_F64 */
    int32_t device;
    void* stream;   /* cudaStream_t the simulator launches on */
} phyzb_device_view;

/* ── library ──────────────────────────────────────────────────────────── */

/* Message of the last failing call on this thread ("" if none). */
const char* phyzb_last_error(void);
/* PHYZB_ABI_VERSION. */
int phyzb_abi_version(void);
/* Number of visible CUDA devices (0 without a driver; never fails). */
int phyzb_device_count(void);

/* ── lifecycle ────────────────────────────────────────────────────────── */

/* BatchSim::on_device (cuda/mod.rs:482-485, 497-541): validate the model
 * (nb <= PHYZB_MAX_BODIES, topological order, finite parameters), allocate
 * q/v/ctrl/qdd for `nworld` worlds on `device`, zero them.
 * Errors: PHYZB_ERR_NO_DEVICE without a driver, PHYZB_ERR_TOO_LARGE past
 * the body limit, PHYZB_ERR_INVALID on a malformed model. */
int phyzb_create(const phyzb_model* model, int64_t nworld, int device, int precision,
                 phyzb_sim** out);
/* Drop (frees every device buffer). NULL is a no-op. */
int phyzb_destroy(phyzb_sim* sim);
/* BatchSim::set_model (cuda/mod.rs:573-594): same body count and DOF
 * widths, new parameters. Re-run phyzb_enable_* after it if geometry or
 * gains changed too. */
int phyzb_set_model(phyzb_sim* sim, const phyzb_model* model);

/* ── contact ──────────────────────────────────────────────────────────── */

/* BatchSim::enable_ground_contact (cuda/mod.rs:601-621): penalty ground
 * contact, one global stiffness/damping. Writes the collidable-body count;
 * PHYZB_ERR_INVALID when no body has a supported shape
 * (layout.rs:282-297). */
int phyzb_enable_ground_contact(phyzb_sim* sim, double ground_height, double stiffness,
                                double damping, double friction, int32_t* collidable_out);
/* BatchSim::enable_ground_contact_per_body (cuda/mod.rs:627-634): per-body
 * gains (nbodies entries each). */
int phyzb_enable_ground_contact_per_body(phyzb_sim* sim, double ground_height,
                                         double friction, const double* stiffness,
                                         const double* damping, int32_t* collidable_out);
/* Heightfield terrain: phyz_model::Heightfield
 * (crates/phyz-model/src/heightfield.rs:10-37). Node (ix, iy) at world
 * (origin[0] + ix cell, origin[1] + iy cell), height origin[2] +
 * heights[iy * nx + ix]; bilinear between nodes, clamped to the border
 * outside the grid (phyz_kernels.cu:625-664). Copied in at the call. */
typedef struct phyzb_heightfield {
    double origin[3];
    double cell;          /* > 0 */
    int32_t nx, ny;       /* >= 1 each */
    const float* heights; /* ny rows of nx */
} phyzb_heightfield;
/* A contact plane attached to a body (contact_pipeline.rs:318-355
 * BodyPlane): the face at `offset` along the body's +z, `half_x` x `half_y`
 * in its x/y, contacts deeper than `max_depth` ignored, `exclude` bodies
 * never touch it. */
typedef struct phyzb_body_plane {
    int32_t body;
    double offset, max_depth, half_x, half_y;
    const int32_t* exclude;
    int32_t n_exclude;
} phyzb_body_plane;
/* BatchSim::enable_contact_terrain / enable_ground_contact_with_plane
 * (cuda/mod.rs:642-676): penalty contact with per-body gains (nbodies
 * each) against the heightfield `hf` (NULL: the flat plane at
 * ground_height, which a loaded heightfield overrides) and an optional
 * body-attached plane (NULL: none; phyz_kernels.cu:983-1132). The device
 * node buffer is sized to this first field. */
int phyzb_enable_contact_terrain(phyzb_sim* sim, double ground_height, double friction,
                                 const double* stiffness, const double* damping,
                                 const phyzb_body_plane* plane, const phyzb_heightfield* hf,
                                 int32_t* collidable_out);
/* BatchSim::set_heightfield (cuda/mod.rs:741-759): replace the terrain in
 * place; contact must be enabled and the field fit the node buffer sized at
 * enable time (1 node when enabled without a heightfield). */
int phyzb_set_heightfield(phyzb_sim* sim, const phyzb_heightfield* hf);
/* BatchSim::enable_contact_impulse (cuda/mod.rs:680-701): contact as the
 * velocity-level convex impulse solve -- per step, the backward sweep with
 * the previous step's contact wrenches, then `sweeps` x [one staged Coulomb
 * update per contact point at the free velocity v + dt qdd, backward sweep]
 * (cuda/mod.rs:902-927; phyz_kernels.cu:856-918), warm-started from the
 * previous step's impulses. Material: GroundContactParams::default with
 * solref_erp_from(0.02, 1.0, dt) (contact_pipeline.rs:199-237). The
 * per-body gains (nullable; penalty-only) are kept but do not enter the
 * impulse law. `hf` and `plane` as in phyzb_enable_contact_terrain.
 * Enabling resets the warm start to zero. */
int phyzb_enable_contact_impulse(phyzb_sim* sim, double ground_height, double friction,
                                 const double* stiffness, const double* damping,
                                 const phyzb_body_plane* plane, const phyzb_heightfield* hf,
                                 int32_t* collidable_out);
/* BatchSim::contact_sweeps (cuda/mod.rs:449-451, default 16): contact sweeps
 * per step in impulse mode, 1 .. PHYZB_MAX_CONTACT_SWEEPS. (The reference
 * also accepts 0, which runs one contact pass against the previous step's
 * qdd; that form is not offered.) */
#define PHYZB_DEFAULT_CONTACT_SWEEPS 16
#define PHYZB_MAX_CONTACT_SWEEPS 1024
int phyzb_set_contact_sweeps(phyzb_sim* sim, int32_t sweeps);
/* Turn contact off again (ext forces zero). */
int phyzb_disable_contact(phyzb_sim* sim);
/* BatchSim::collidable_bodies (cuda/mod.rs:999-1001): 0 when disabled. */
int phyzb_collidable_bodies(const phyzb_sim* sim);

/* ── PD servos ────────────────────────────────────────────────────────── */

/* BatchSim::enable_pd_control (cuda/mod.rs:771-790); check_pd_dofs
 * (layout.rs:300-315) rules. */
int phyzb_enable_pd(phyzb_sim* sim, const phyzb_pd_dof* dofs, int32_t n);
/* BatchSim::set_position_targets (cuda/mod.rs:793-801): nworld x n rows. */
int phyzb_set_position_targets(phyzb_sim* sim, const double* targets);

/* ── state ────────────────────────────────────────────────────────────── */

/* BatchSim::load_states (cuda/mod.rs:804-812): world-major q, v (nworld x
 * nv) and ctrl (nworld x nv, NULL = zero). */
int phyzb_load_states(phyzb_sim* sim, const double* q, const double* v, const double* ctrl);
/* BatchSim::set_controls (cuda/mod.rs:815-821): nworld x nv, held across
 * steps until replaced. */
int phyzb_set_controls(phyzb_sim* sim, const double* ctrl);

/* ── stepping ─────────────────────────────────────────────────────────── */

/* BatchSim::step_many(n) (cuda/mod.rs:843-875): n steps of
 * PD -> contact -> ABA -> integrate, run as one fused launch that keeps
 * each world's state on chip across the n steps. Asynchronous on the
 * simulator's stream; n == 0 is a no-op. */
int phyzb_step(phyzb_sim* sim, int32_t n);
/* n steps whose controls change every step: `ctrl` holds n x nworld x nv
 * world-major rows of element type `host_dtype` (PHYZB_HOST_F32/F64) in
 * host memory (pinned memory overlaps the copies with the kernels). Same
 * result as n x (phyzb_set_controls(row t); phyzb_step(1)). On return the
 * ctrl buffer holds the last row, as after that loop. */
int phyzb_step_with_controls(phyzb_sim* sim, const void* ctrl, int host_dtype, int32_t n);
/* Block until every launch on the simulator's stream has finished, then
 * report the device status word (PHYZB_ERR_NONFINITE if any world went
 * non-finite since the last phyzb_clear_status). */
int phyzb_sync(phyzb_sim* sim);
int phyzb_status(phyzb_sim* sim);
int phyzb_clear_status(phyzb_sim* sim);

/* ── readback ─────────────────────────────────────────────────────────── */

/* BatchSim::readback_states (cuda/mod.rs:978-983): world-major q, v. */
int phyzb_readback_states(phyzb_sim* sim, double* q, double* v);
/* Joint accelerations of the last step, world-major (no reference
 * counterpart: the reference keeps qdd on device; needed for qdd parity). */
int phyzb_readback_qdd(phyzb_sim* sim, double* qdd);
/* BatchSim::readback_contacts (cuda/mod.rs:987-996): nworld x nbodies x
 * PHYZB_CONTACT_STRIDE of the last step. PHYZB_ERR_STATE if contact off. */
int phyzb_readback_contacts(phyzb_sim* sim, double* contact_state);

/* State history (mod.rs:1316-1376): `slots` snapshots of q / v kept on the
 * device; record_state copies the current state into a slot after every
 * launch so far (the host does not wait); readback returns rows
 * [n][nworld][nv]. Re-enabling with the same slot count keeps the buffers. */
int phyzb_enable_state_history(phyzb_sim* sim, int32_t slots);
int phyzb_record_state(phyzb_sim* sim, int32_t slot);
int phyzb_readback_state_history(phyzb_sim* sim, int32_t slot0, int32_t n, double* q, double* v);

/* ── device-resident path ─────────────────────────────────────────────── */

/* Device pointers and layout of the resident state (zero-copy). */
int phyzb_device_view_get(phyzb_sim* sim, phyzb_device_view* out);
/* Device-resident form of phyzb_load_states: q, v (and ctrl, NULL = keep)
 * are device arrays in the simulator's precision and SoA layout
 * ([nv][nworld]); copied on the simulator's stream, asynchronously.
 * Device inputs of this and the calls below are read on the simulator's
 * stream (its own non-blocking stream unless phyzb_set_stream named
 * another): work that writes them on another stream must be ordered before
 * the call (an event, a synchronize, or the same stream via
 * phyzb_set_stream). */
int phyzb_load_states_device(phyzb_sim* sim, const void* q, const void* v, const void* ctrl);
/* Launch on a caller-provided stream (a cudaStream_t; NULL = the
 * simulator's own stream). */
int phyzb_set_stream(phyzb_sim* sim, void* stream);
/* n fused steps whose per-step controls are read from a device-resident
 * schedule laid out [n][nv][nworld] (SoA, the simulator's precision,
 * `step_stride` elements between consecutive steps, >= nv*nworld).
 * Asynchronous. The device-side equivalent of phyzb_step_with_controls. */
int phyzb_step_device_controls(phyzb_sim* sim, const void* ctrl_schedule, int64_t step_stride,
                               int32_t n);
/* Sum over worlds of a per-world objective into a device scalar (the
 * simulator's precision): kind 0 = kinetic energy 0.5 v.M(q).v computed
 * body-wise, kind 1 = sum of squared joint positions. The value a
 * multi-GPU job all-reduces at the end of a rollout. */
int phyzb_objective_device(phyzb_sim* sim, int kind, void* out_device_scalar);

/* ── on-device control loop (crates/phyz-gpu/src/policy_pipeline.rs,
 *    cuda/mod.rs:1081-1271, phyz_kernels.cu:1436-1715) ──────────────────── */

/* Observation op kinds, one table row of 4 floats (kind, a, b, c) each, as
 * ObsOp::pack lays them out (policy_pipeline.rs:113-128). */
#define PHYZB_OBS_CONST 0          /* c */
#define PHYZB_OBS_Q_MINUS 1        /* q[a] - c */
#define PHYZB_OBS_V 2              /* v[a] */
#define PHYZB_OBS_BODY_PITCH 3     /* atan2(-r02, r22) of body a */
#define PHYZB_OBS_BODY_ROLL 4      /* atan2(r12, r22) */
#define PHYZB_OBS_BODY_YAW_ERROR 5 /* wrap(c - atan2(r01, r00)) */
#define PHYZB_OBS_BODY_POS_Z 6     /* body a origin, world z */
#define PHYZB_OBS_BODY_POS 7       /* body a origin, world axis b */
#define PHYZB_OBS_COM_OVER_SUPPORT 8 /* aux window (offset a, n_support b), axis c */
#define PHYZB_KINEMATICS_STRIDE 18 /* world->body rot (9), origin (3), body-frame w (3), v (3) */

/* PolicySpec (policy_pipeline.rs:285-320) in flat form. */
typedef struct {
    int32_t n_obs;                 /* observation width = MLP input, 1..128 */
    const float* obs_ops;          /* n_obs x 4 floats */
    int32_t n_aux;                 /* floats in obs_aux */
    const float* obs_aux;          /* ComOverSupport payloads (pack_obs_ops) */
    int32_t hidden;                /* hidden width of both layers, 1..128 */
    int32_t n_act;                 /* actions = MLP output, 1..32 */
    const int32_t* act_slots;      /* PD servo slot (registration order) of each action */
    double act_clamp;              /* applied-action clamp, every slot */
    const double* act_clamp_slots; /* per-action clamp (n_act), or NULL */
    double noise_rho;              /* AR(1) coefficient of the exploration noise */
    const double* input_noise;     /* n_obs input-noise scales (0 = no draw) */
    int32_t history_steps;         /* control steps of obs/action history kept */
} phyzb_policy_spec;

/* enable_policy (mod.rs:1081-1148): needs PD control (the actions are PD
 * targets). PHYZB_ERR_UNSUPPORTED for a hidden width above 128. */
int phyzb_enable_policy(phyzb_sim* sim, const phyzb_policy_spec* spec);
/* set_policy_weights (mod.rs:1151-1162): W1[h][n_obs] b1[h] W2[h][h] b2[h]
 * W3[n_act][h] b3[n_act], row-major, n = their total. */
int phyzb_set_policy_weights(phyzb_sim* sim, const double* weights, int64_t n);
/* set_policy_std (mod.rs:1165-1176): per-action Gaussian standard deviation. */
int phyzb_set_policy_std(phyzb_sim* sim, const double* std_dev, int32_t n);
/* set_policy_base_targets (mod.rs:1180-1186): rows [nworld][n_pd]. */
int phyzb_set_policy_base_targets(phyzb_sim* sim, const double* rows);
/* seed_policy (mod.rs:1191-1205): every world's xorshift64 stream from
 * world_seed(seed, w) (policy_pipeline.rs:420-428); AR(1) state zeroed. */
int phyzb_seed_policy(phyzb_sim* sim, uint64_t seed);
/* run_policy (mod.rs:1209-1271): kinematics, observation row `step`,
 * policy forward + sample into action row `step` and the PD targets. */
int phyzb_run_policy(phyzb_sim* sim, int32_t step);
/* n_control x (phyzb_run_policy(step0 + c); phyzb_step(substeps)) on the
 * device, asynchronously (no host round trip between control steps). */
int phyzb_policy_rollout(phyzb_sim* sim, int32_t step0, int32_t n_control, int32_t substeps);
/* readback_policy_history (mod.rs:1277-1306): obs [n][nworld][n_obs] and
 * out [n][nworld][n_act + 1] (actions, then log-prob), f32. */
int phyzb_readback_policy_history(phyzb_sim* sim, int32_t step0, int32_t n, float* obs, float* out);
/* readback_targets (mod.rs:1309-1313): PD targets, rows [nworld][n_pd]. */
int phyzb_readback_targets(phyzb_sim* sim, double* rows);
/* compute_kinematics + readback (phyz_fk, phyz_kernels.cu:1436-1454):
 * rows [nworld][nbodies][PHYZB_KINEMATICS_STRIDE]. */
int phyzb_readback_kinematics(phyzb_sim* sim, double* xforms);

/* ── PPO update (crates/phyz-gpu/cuda/phyz_train.cu, src/cuda/train.rs) ─ */

/* TrainPipeline (train.rs:474-810): a clipped-surrogate PPO update of a
 * three-layer tanh MLP actor (with a trailing log_std block) and critic,
 * Adam with f64 master parameters and moments, on the device. */
typedef struct phyzb_trainer phyzb_trainer;
typedef struct phyzb_comm phyzb_comm;
typedef struct {
    int32_t n_in, n_h, n_out; /* n_h <= 128, n_out <= 32 */
} phyzb_net_dims;
typedef struct {
    double lr, beta1, beta2, eps, weight_decay; /* tang's ModuleAdam */
} phyzb_adam_cfg;
#define PHYZB_KL_CUMULATIVE 0 /* mean of logp_old - logp over every row so far */
#define PHYZB_KL_MINIBATCH 1  /* Schulman's k3 over the current minibatch */
typedef struct {
    double clip, entropy_coef, vdelta; /* surrogate clip, entropy bonus, value-gradient Huber delta */
    int32_t minibatch, epochs;
    double target_kl, kl_scale; /* the KL brake: stop after the first minibatch above target */
    int32_t kl_mode;
} phyzb_ppo_cfg;
typedef struct {
    double policy_loss, value_loss, kl;
    int32_t grad_steps, stopped_early;
} phyzb_update_stats;

/* TrainPipeline::new (train.rs:523-580): at most `capacity` samples per
 * update and `max_minibatch` per minibatch; the critic has one output. */
int phyzb_trainer_create(int32_t device, phyzb_net_dims actor, phyzb_net_dims critic, int64_t capacity,
                         int32_t max_minibatch, phyzb_trainer** out);
int phyzb_trainer_destroy(phyzb_trainer* tr);
/* set_adam (train.rs:800-806); defaults lr 3e-4, betas 0.9 / 0.999, eps 1e-8. */
int phyzb_trainer_set_adam(phyzb_trainer* tr, const phyzb_adam_cfg* actor, const phyzb_adam_cfg* critic);
/* set_actor_params / set_critic_params (which = 0 / 1): tang's flat order
 * W1 b1 W2 b2 W3 b3 (+ log_std for the actor); params reads them back. */
int phyzb_trainer_set_params(phyzb_trainer* tr, int32_t which, const double* flat, int64_t n);
int phyzb_trainer_params(phyzb_trainer* tr, int32_t which, double* flat, int64_t n);
/* upload_batch (train.rs:602-645): row-major host columns of n_rows rows. */
int phyzb_trainer_upload_batch(phyzb_trainer* tr, int64_t n_rows, const float* obs_a, const float* obs_c,
                               const float* act, const float* logp_old, const float* adv, const float* ret);
/* update (train.rs:655-795): epochs over the uploaded batch in the order
 * given (n_orders permutations of 0..n_rows, one per epoch). */
int phyzb_trainer_update(phyzb_trainer* tr, const uint32_t* order, int32_t n_orders, const phyzb_ppo_cfg* cfg,
                         phyzb_update_stats* out);

/* A column block of per-sample device data: rows r = t * block + w, feature
 * k of row r at base[(r / block) * features * block + k * block + r % block]
 * (the policy history's [step][feature][world]: block = nworld). */
typedef struct {
    const float* base;
    int64_t block;
    int32_t features;
} phyzb_batch_col;
/* The update's batch from device memory instead of upload_batch: columns
 * obs_a, obs_c, act, logp_old, adv, ret, n_rows rows each (not copied). */
int phyzb_trainer_set_batch_device(phyzb_trainer* tr, int64_t n_rows, const phyzb_batch_col* cols /* 6 */);
/* update with one device-generated permutation per epoch (an affine map
 * (a k + c) mod n_rows, a coprime with n_rows, from `seed`). */
int phyzb_trainer_update_shuffled(phyzb_trainer* tr, const phyzb_ppo_cfg* cfg, uint64_t seed,
                                  phyzb_update_stats* out);
/* Network `which` (0 actor, 1 critic) on n_rows rows of x; outputs to the
 * device array out [n_out][n_rows]. */
int phyzb_trainer_evaluate(phyzb_trainer* tr, int32_t which, phyzb_batch_col x, int64_t n_rows, float* out);
/* Data-parallel updates: every gradient and minibatch statistic is summed
 * over the communicator's ranks (NCCL) before Adam and the KL brake, so the
 * ranks' networks stay identical. NULL = one rank. */
int phyzb_trainer_set_comm(phyzb_trainer* tr, struct phyzb_comm* comm);

/* Device pointers of a simulator's policy history: obs [steps][n_obs][nworld],
 * out [steps][n_act + 1][nworld] (actions, then log-prob). */
typedef struct {
    float* obs;
    float* out;
    int32_t n_obs, n_act;
    int64_t nworld;
    int32_t steps;
} phyzb_policy_history;
int phyzb_policy_history_view(phyzb_sim* sim, phyzb_policy_history* out);
/* Returns of a rollout of `steps` control steps (history rows 0..steps):
 * reward r_t = reward_coef . obs_{t+1} - action_penalty |a_t|^2, critic
 * values of rows 0..steps, GAE(gamma, lambda), advantages normalized over
 * every rank when `normalize` (the sums go through `comm`, NULL = one rank).
 * adv, ret: device arrays [steps][nworld]. stats (optional, 3): mean return
 * per world over all ranks, advantage mean and std before normalization. */
typedef struct {
    const double* reward_coef; /* n_obs */
    double action_penalty, gamma, lambda;
    int32_t steps, normalize;
} phyzb_return_cfg;
int phyzb_policy_advantages(phyzb_sim* sim, phyzb_trainer* tr, struct phyzb_comm* comm, const phyzb_return_cfg* cfg,
                            float* adv, float* ret, double* stats);
/* GAE(gamma, lambda) and the advantage normalization of
 * phyzb_policy_advantages (one rank) over caller-owned device buffers --
 * rewards [steps][nworld], values [steps + 1][nworld], adv and ret
 * [steps][nworld], all float on `device` -- that allocates no device memory.
 * It has no counterpart in the reference. It is meant for callers that must
 * not let a library allocate: a host framework that has reserved the GPU's
 * memory for its own allocator or holds the process to a fixed budget, or a
 * latency-bound training loop, where cudaMalloc can fail or stall and
 * cudaFree synchronizes the device. Its only scratch, the GAE kernel's
 * per-block partial sums, lives in a static device array sized for
 * PHYZB_GAE_NOALLOC_MAX_WORLDS worlds (1.5 MiB, held by every device that
 * loads the library until exit); a larger nworld returns
 * PHYZB_ERR_TOO_LARGE. The first call on a device looks that array's address
 * up (cudaGetSymbolAddress), so make the first call on each device before
 * any stream capture. The address is kept for the life of the process: a
 * cudaDeviceReset of a device ends it, so do not call this entry point on a
 * device after resetting that device. All calls on a device share the array: calls whose
 * kernels overlap on the device race, so order them on one stream or with
 * events. Runs on `stream` (a cudaStream_t, NULL = the default stream);
 * asynchronous unless `stats` (optional, host, 3 doubles: mean return per
 * world, advantage mean and std before normalization) is given, in which case
 * it waits for the stream. */
#define PHYZB_GAE_NOALLOC_MAX_WORLDS (1 << 24)
int phyzb_gae_noalloc(const float* rewards, const float* values, int64_t nworld, int32_t steps, double gamma,
                      double lambda, int32_t normalize, int32_t device, void* stream, float* adv, float* ret,
                      double* stats);
/* The trainer's actor (weights, std = exp(log_std)) into the simulator's
 * policy, device to device. */
int phyzb_policy_sync_from_trainer(phyzb_sim* sim, phyzb_trainer* tr);

/* ── multi-GPU: one process per GPU, worlds sharded contiguously ──────── */

/* Worlds are independent, so ranks exchange nothing per step; the one
 * collective is the sum of the per-world objective over every rank's shard
 * at the end of a rollout (NCCL over NVLink; the reduction phyz-gpu's
 * callers do on the host). NCCL is loaded at run time. */
#define PHYZB_COMM_ID_BYTES 128
/* Rank 0 creates the communicator id and hands the bytes to the other
 * ranks (any host channel: a store, an MPI/torch broadcast). */
int phyzb_comm_unique_id(uint8_t* id_out /* PHYZB_COMM_ID_BYTES */);
/* Join the communicator on `device`. Returns PHYZB_ERR_COMM when not every
 * rank joined within timeout_s seconds. */
int phyzb_comm_init(const uint8_t* id, int32_t nranks, int32_t rank, int32_t device, double timeout_s,
                    phyzb_comm** out);
int phyzb_comm_destroy(phyzb_comm* comm);
/* phyzb_objective_device of this rank's shard, summed over all ranks (NCCL
 * all-reduce on the simulator's stream) and returned to the host on every
 * rank. Every rank calls it in the same order. A rank that does not take
 * part makes the others return PHYZB_ERR_COMM after timeout_s seconds; the
 * communicator is then aborted and must be rebuilt. */
int phyzb_reduce_objective(phyzb_sim* sim, phyzb_comm* comm, int kind, double timeout_s, double* out);
/* The same reduction enqueued on the simulator's stream into a device
 * scalar (the simulator's precision), without waiting: a caller closing
 * many rollouts keeps the host from stalling on each one and reads the
 * scalars after one bounded wait (phyzb_comm_sync). A failing or stalled
 * collective is reported by that wait (the communicator is then aborted).
 * No reference counterpart. */
int phyzb_reduce_objective_device(phyzb_sim* sim, phyzb_comm* comm, int kind, void* out_device_scalar);
/* Wait, at most timeout_s, for everything enqueued on the simulator's
 * stream, watching the communicator for errors (PHYZB_ERR_COMM on failure
 * or timeout, the communicator aborted). */
int phyzb_comm_sync(phyzb_comm* comm, phyzb_sim* sim, double timeout_s);

/* ── measurement helpers (no reference counterpart) ───────────────────── */

/* Algorithmic flop count of one world-step of this simulator's model and
 * settings, as executed by the kernel's formulation (add/sub/mul = 1,
 * fma = 2, div = 1), with transcendental calls tallied separately. */
int phyzb_flops_per_world_step(const phyzb_sim* sim, double* flops, double* transcendentals);
/* The flops the kernel executes per world-step on given states, averaged
 * over `nworld` worlds stepped `nsteps` steps on the host by the kernel's
 * own step code with a counting scalar: q, v host rows [nworld][nv] (as
 * phyzb_load_states), ctrl [nsteps][nworld][nv] (NULL: zero controls).
 * Unlike phyzb_flops_per_world_step it counts the contact force law where a
 * body touches the flat ground (penalty or impulse mode, this simulator's
 * settings). specialized = 1 counts as a model-specialized kernel executes
 * (products with zero model-table constants left out), 0 as the generic
 * variants do. Models with a heightfield or body plane return
 * PHYZB_ERR_INVALID. Host work only; nothing touches the device. */
int phyzb_flops_executed(const phyzb_sim* sim, const double* q, const double* v, const double* ctrl, int64_t nworld,
                         int32_t nsteps, int32_t specialized, double* flops, double* transcendentals);
/* FP32 (PHYZB_F32) or FP64 (PHYZB_F64) FMA-pipe throughput of the calling
 * thread's current device in TFLOP/s, measured with independent FMA chains
 * over every SM: the roofline denominator of the stepper's kernels. */
int phyzb_measure_fma_peak(int precision, double* tflops);
/* Launch configuration the fused kernel uses for this simulator; tmem_cols
 * > 0 when its body records live in Tensor Memory (columns per world). With
 * specialization active it is the specialized kernel's once that kernel has
 * been compiled (at the first launch after a table change), the generic
 * variant's before. */
int phyzb_launch_info(const phyzb_sim* sim, int32_t* worlds_per_block, int32_t* blocks,
                      int32_t* smem_bytes, int32_t* scratch_per_world, int32_t* tmem_cols);
/* How a one-thread-per-world rollout launch of `nsteps` steps would run:
 * steps_per_run = 0 in tile mode (each block takes tiles of
 * worlds_per_block worlds for every step), else slice mode (each warp
 * takes jobs of 32 worlds x steps_per_run steps from a device queue, so
 * warps that finish early take the remaining worlds' runs instead of
 * idling through a partial last wave). The library picks slice mode when
 * its wave count says it is faster; PHYZB_SLICES=0 / 1 at creation turns
 * it off / on for every launch of two or more steps. Host work only. */
int phyzb_slice_plan(const phyzb_sim* sim, int32_t nsteps, int32_t* steps_per_run, int32_t* worlds_per_block,
                     int32_t* blocks);

/* ── model-specialized kernels (no reference counterpart) ──────────────── */

/* Kernel specialization mode of a simulator:
 *   PHYZB_SPECIALIZE_OFF  rollouts run the generic kernel variants;
 *   PHYZB_SPECIALIZE_ON   they run a kernel compiled at run time (NVRTC) for
 *                         the simulator's packed model: its body tables
 *                         literal in the code and every body loop unrolled,
 *                         the generic kernel's source and arithmetic (results
 *                         agree to rounding: constant folding may move which
 *                         product of a sum fuses into an FMA);
 *   PHYZB_SPECIALIZE_AUTO ON for models whose longest root-to-leaf chain
 *                         has at most PHYZB_SPECIALIZE_AUTO_MAX_DEPTH bodies
 *                         (and at most PHYZB_SPECIALIZE_AUTO_MAX_BODIES in
 *                         all): branching trees gain from unrolling (their
 *                         limbs interleave), while a long serial chain runs
 *                         faster as the generic loop, whose code stays in the
 *                         instruction cache (measured on B200: a 9-body
 *                         quadruped +68%, a 22-body humanoid +22%, a 32-body
 *                         chain -42%).
 * The compile happens at the first launch after each table change (model,
 * contact or PD settings, world count) and is cached per process and on
 * disk (PHYZB_KERNEL_CACHE: a directory, or "0" for none; default
 * $HOME/.cache/phyzb). A compile or load failure fails that launch with
 * PHYZB_ERR_CUDA and the compiler's log in phyzb_last_error(). A new
 * simulator starts in the mode PHYZB_SPECIALIZE names ("0", "1", "auto"),
 * else OFF. `active` (may be null) tells whether the next launch runs the
 * specialized kernel. PHYZB_SPEC_NVRTC_OPTS appends compiler options
 * (space-separated, for tuning; part of the cache key). */
#define PHYZB_SPECIALIZE_OFF 0
#define PHYZB_SPECIALIZE_ON 1
#define PHYZB_SPECIALIZE_AUTO 2
#define PHYZB_SPECIALIZE_AUTO_MAX_DEPTH 16
#define PHYZB_SPECIALIZE_AUTO_MAX_BODIES 64
int phyzb_set_kernel_specialization(phyzb_sim* sim, int32_t mode);
int phyzb_get_kernel_specialization(const phyzb_sim* sim, int32_t* mode, int32_t* active);

/* One world over several threads: the north star's "one world per warp with
 * per-body parallelism" for branching trees (no reference counterpart; the
 * reference runs one thread per world, phyz_kernels.cu:1175-1369). `lanes`
 * (2, 4, 8; 0 or 1: one thread per world) threads of a warp share a world:
 * each steps the trunk (the bodies with two or more leaves below them) and
 * its share of the limbs (the chains off the trunk), and the backward sweep
 * sums the limbs' articulated inertias and bias forces over the lanes with
 * warp shuffles before the trunk is swept. A world step then takes the
 * trunk's time plus the longest share of limbs instead of every body in
 * turn: for batches too small to fill the GPU with one thread per world,
 * where per-world latency is the bound. Results equal the one-thread
 * kernel's up to the order of those sums. PHYZB_ERR_UNSUPPORTED for a model
 * that does not branch or settings the lanes kernel lacks (PD servos,
 * impulse contact, heightfield / plane); such settings enabled later return
 * the simulator to one thread per world. The last step of every launch runs
 * on one thread per world (it writes qdd and contact state). $PHYZB_LANES
 * sets a new simulator's lanes where its model splits. */
int phyzb_set_world_lanes(phyzb_sim* sim, int32_t lanes);
/* lanes as set; active = 1 when a launch of two or more steps runs the lanes
 * kernel with the current settings (plans and packs the split if needed). */
int phyzb_get_world_lanes(phyzb_sim* sim, int32_t* lanes, int32_t* active);

#ifdef __cplusplus
}
#endif

#endif /* PHYZB_H */
