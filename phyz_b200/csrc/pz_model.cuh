// Device-side model table of the B200 stepper: one record per body, shared
// by every world and staged into shared memory once per thread block.
//
// It carries what phyz's packed body table carries (parent, joint type,
// DOF offset, mass/COM/inertia, parent->joint transform, axis, damping,
// spring, armature: crates/phyz-gpu/src/layout.rs:18-37) plus what the
// reference's CPU path applies and its GPU table drops (soft limits, dry
// friction: crates/phyz-model/src/joint.rs:184-247), the contact geometry
// of layout.rs:38-52, and precomputed quantities of this kernel's
// formulation (inertia about the body origin, m*c, COM inverse inertia,
// armature + dt*damping).
//
// Frames: a hinge about a coordinate axis e_k with an unrotated parent->joint
// frame is stored in its body frame with the coordinates cyclically
// relabelled so that its axis is z (a proper rotation P_k, applied to every
// body-frame constant at pack time). Its parent->child transform is then
// "translate, relabel (a cyclic permutation), rotate about z": one code path
// for all three axes. Joint-space quantities and world-frame outputs do not
// depend on the relabelling.
//
// The integer half names where each body's per-world scratch lives: the
// per-world state is structure-of-arrays in shared memory, slot s of a
// world at smem[s * worlds_per_block + thread].
#pragma once

namespace pz {

enum JointCode { J_REVOLUTE = 0, J_PRISMATIC = 1, J_FIXED = 2, J_BALL = 3, J_FREE = 4 };

enum BodyFlags {
    F_PTJ_ROT = 1 << 0,   // parent->joint rotation is not the identity
    F_PTJ_POS = 1 << 1,   // parent->joint translation is not zero
    F_LIMITS = 1 << 2,    // soft joint limits (1-DOF)
    F_FRICTION = 1 << 3,  // dry friction loss (1-DOF)
    F_SPRING = 1 << 4,    // passive spring (1-DOF)
    F_CONTACT = 1 << 5,   // collidable while contact is enabled (has an F slot)
    F_CHAIN = 1 << 6,     // body i+1 has this body as parent (backward carry)
    F_BRANCH = 1 << 7,    // parent of a child that is not i+1 (stored accumulators)
    F_ZHINGE = 1 << 8,    // hinge about z of its (relabelled) frame; parent->joint rotation
                          // is the cyclic relabelling `qshift` (the kernel's fast path)
    F_PD = 1 << 9,        // a DOF of this body is driven by a PD servo
    F_PLANE = 1 << 10,    // touches the body-attached contact plane
    F_EXTF = 1 << 11,     // receives an external wrench (s_f): collidable, or the plane's body
    F_ROOTQDD = 1 << 12,  // ball/free joint of a root body: its parent acceleration is gravity
                          // alone, so pass 2 solves its qdd outright and W is never formed
};

template <class T>
struct alignas(16) BodyT {
    T mass, mcom[3];          // m, m*c
    T Io[6];                  // rotational inertia about the body origin (xx,yy,zz,xy,xz,yz)
    T com[3];                 // centre of mass
    T ptj_rot[9], ptj_pos[3]; // parent->joint transform (row-major rotation)
    T axis[3];
    T damping, stiffness, spring_ref, d_extra;  // d_extra = armature + dt * damping
    T lim_lo, lim_hi, lim_k, lim_d, fric;
    T Icinv[6];               // inverse of the COM inertia (0 if singular), for contact
    T geom[6], gpos[3], grot[9];
    T gk, gd;                 // penalty gains of this body
    T armature;
};
// A body row is 64 scalars, no padding (the specialized source lists them in order).
constexpr int BODYT_WORDS = 64;
static_assert(sizeof(BodyT<float>) == BODYT_WORDS * sizeof(float), "BodyT<float> layout");
static_assert(sizeof(BodyT<double>) == BODYT_WORDS * sizeof(double), "BodyT<double> layout");

struct alignas(16) BodyI {
    int parent, jtype, off, ndof;
    int axis_k;       // 0/1/2: axis is +e_k exactly (planar fast path); -1 general
    int flags;        // BodyFlags
    int s_xj;         // joint transform data: hinge (c, s); ball/free R_J (9)
    int s_vw;         // body velocity (6) between passes 1 and 2, then W = U D^-1 (6*ndof)
    int s_w0;         // control input of the step (unless s_in is separate), then D^-1 u (ndof)
    int s_in;         // control input of the step (ndof): s_w0, or its own slots in impulse mode
    int s_f;          // external (contact) wrench, body frame (6): F_EXTF bodies
    int s_acc;        // branch: accumulated child inertia (21) + bias force (6)
    int s_vold;       // branch: velocity of the step being finished (6)
    int s_acca;       // branch: acceleration (6)
    int s_wx;         // branch: world frame for contact (up 3, height 1; with a heightfield
                      // rows r0, r1, up and the origin: 12)
    int gtype;        // geometry code (0 none)
    int t_rec;        // Tensor Memory column of the body's record [c, s, v|W] (-1: in s_xj/s_vw)
    int qshift;       // F_ZHINGE: parent->child relabelling (Q v)_a = v_(a+qshift mod 3)
    // impulse-mode contact (-1 otherwise)
    int s_up;         // collidable: world up in the body frame (3) and origin height (1); with
                      // a heightfield the frame of s_wx (12)
    int s_imp;        // collidable: staged impulses [normal, tangent u, tangent w] per point
    int s_vf;         // branch, plane participant: free velocity v + dt qdd of the sweep (6)
    int c_imp;        // collidable: first row of the body's wrench (6) + impulses in the
                      // persistent impulse buffer
    int fshift;       // this body's frame relabelling: stored = P_fshift (original coordinates)
    int s_pimp;       // impulse mode, F_PLANE: staged impulses against the plane per point
    // impulse mode: what the sweeps need to propagate a wrench change alone
    int s_dinv;       // 1-DOF: D^-1 (0: a singular body); ball/free: the Cholesky factor L of D,
                      // row-major lower triangle with 1 / L_aa on the diagonal (first entry 0:
                      // singular)
    int s_w0b;        // D^-1 u of the step's full backward sweep (ndof)
    int s_fp;         // F_EXTF: the wrench that backward sweep applied (6)
    int t_f;          // F_EXTF: Tensor Memory column of the body's external wrench record
                      // [f (6), 0, 0] (-1: in s_f)
};
static_assert(sizeof(BodyI) == 28 * sizeof(int), "BodyI: 28 words");

template <class T>
struct alignas(16) PdT {
    T kp, kd, maxf;
    int qi, vi;
};

// Heightfield terrain (phyz-model/src/heightfield.rs:10-37; the GPU's
// sampling, phyz_kernels.cu:625-664): node (ix, iy) at world
// (ox + ix cell, oy + iy cell) with height oz + h[iy * nx + ix], f32 nodes
// as the reference stores them.
template <class T>
struct Terrain {
    const float* h;
    int nx, ny;
    T ox, oy, oz, cell;
};

// A contact plane attached to a body (contact_pipeline.rs:318-355): the face
// at `offset` along the body's own +z (original, unrelabelled frame),
// half_x x half_y in its x/y, penetrations beyond max_depth ignored.
template <class T>
struct PlaneT {
    int body;  // -1: none
    T offset, max_depth, half_x, half_y;
};

// Impulse-mode contact material (contact_pipeline.rs:85-95): ground height,
// friction, dt, solref error reduction, margin, restitution and its
// threshold, SolImp parameters.
template <class T>
struct ImpMat {
    T ground_h, friction, dt, erp, margin, restitution, rest_thr;
    T dmin, dmax, width, mid, power;
    // derived once per launch (impmat_finish): the SolImp curve's clamped
    // parameters and the reciprocals the per-point law multiplies by
    T c_dmin, c_dmax, c_mid, c_pw, inv_width, mid_scale, omid_scale, inv_margin, inv_dtc, inv_vr;
    bool pw2;  // the curve's power is 2 (the default): x^2 by one multiply
};

// Words of a BodyI before its alignment padding (the model-specialized
// source lists them in this order).
constexpr int BODYI_WORDS = 28;

#ifdef PZ_SPEC
// Model-specialized build: the host emits one packed model's tables as
// literal constants (the definitions below, PZ_SPEC_NB and PZ_SPEC_NV) and
// compiles the kernel for it, so body loops unroll with every table entry
// folded into the instruction stream. The accessors mirror the pointer
// tables of the generic build.
namespace spec {
__device__ __forceinline__ BodyI body(int i);
template <class T>
__device__ __forceinline__ BodyT<T> bodyt(int i);
__device__ __forceinline__ int pd_of(int d);
template <class T>
__device__ __forceinline__ PdT<T> pdt(int k);
}  // namespace spec
struct SpecBodies {
    __device__ __forceinline__ BodyI operator[](int i) const { return spec::body(i); }
};
template <class T>
struct SpecBodyT {
    __device__ __forceinline__ BodyT<T> operator[](int i) const { return spec::bodyt<T>(i); }
};
struct SpecPdOf {
    __device__ __forceinline__ int operator[](int d) const { return spec::pd_of(d); }
};
template <class T>
struct SpecPd {
    __device__ __forceinline__ PdT<T> operator[](int k) const { return spec::pdt<T>(k); }
};
#endif

// Everything a world-step needs besides its own state.
template <class T>
struct ModelView {
#ifdef PZ_SPEC
    SpecBodyT<T> bt;
    SpecBodies bi;
    SpecPd<T> pd;
    SpecPdOf pd_of_dof;
    static constexpr int nb = PZ_SPEC_NB, nv = PZ_SPEC_NV;
    int npd;
#else
    const BodyT<T>* bt;
    const BodyI* bi;
    const PdT<T>* pd;
    const int* pd_of_dof;  // nv entries: PD entry driving this DOF, or -1
    int nb, nv, npd;
#endif
    const BodyT<T>* btp;   // the body table in memory (out-of-line calls take rows by address)
    int contact;           // 0/1
    T dt, gx, gy, gz;
    T ground_h, friction;
    T inv_dt_c;            // 1 / max(dt, 1e-9)   (phyz_kernels.cu:574-578)
    T kstiff_c;            // 4 / max(dt, 1e-9)^2
    ImpMat<T> im;          // impulse-mode contact material
    Terrain<T> ter;        // heightfield (feature bit 32)
    PlaneT<T> plane;       // body-attached plane (contact variants)
};

}  // namespace pz
