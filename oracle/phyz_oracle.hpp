// TEST INFRASTRUCTURE ONLY — the CPU checker for libphyzb200's kernels.
//
// A plain f64 C++ restatement of phyz's CPU rigid-body path, written to be
// read side by side with the reference:
//
//   * spatial algebra with `tang`'s semantics. `tang` (git rev
//     9d28b81067f1a416c73a9e84b7f4f9af29bbfa34, Cargo.toml:148-150) is not
//     vendored in the reference tree; its arithmetic is restated from the
//     reference's own in-tree CUDA C port of it,
//     crates/phyz-gpu/cuda/phyz_kernels.cu:82-359, which the reference pins
//     against its CPU path to 1e-9 (tests/joint_offset_vs_cpu.rs:57-85);
//   * joints: crates/phyz-model/src/joint.rs:164-326;
//   * forward dynamics: crates/phyz-rigid/src/aba.rs:147-420, dense 6x6 as
//     the reference does it (this file does NOT share the kernel's reduced
//     formulation, so it checks the kernel's algebra independently);
//   * generalized forces: crates/phyz-rigid/src/actuation.rs:18-54 and
//     crates/phyz-model/src/model.rs:203-231 (models without actuators:
//     ctrl is a raw per-DOF force);
//   * integrator: crates/phyz-rigid/src/integrate.rs:41-91 with
//     crates/phyz-math/src/lib.rs:43-72 (f64::EPSILON small-angle branches);
//   * kinematics / RNEA / energy: crates/phyz-rigid/src/{kinematics.rs:10-50,
//     rnea.rs:94-169, energy.rs:8-37};
//   * penalty ground contact: the reference has no f64 CPU version of the
//     law its GPU kernels run, so the GPU law itself is restated in f64
//     from phyz_kernels.cu:541-578 (coulomb, eff. mass, gain bounds),
//     :641-643 (flat Z-up terrain), :691-725 (support points), :748-802
//     (FK), :939-965 (penalty branch), :1050-1060 (contact state);
//   * impulse-mode ground contact (enable_contact_impulse, cuda/mod.rs:
//     680-701, 902-927): likewise the GPU's velocity-level staged Coulomb
//     update restated in f64 from phyz_kernels.cu:581-622 (tangents, SolImp
//     impedance, restitution ramp) and :856-918 (the impulse branch), with
//     the sweep sequence of cuda/mod.rs:916-927. The reference's CPU convex
//     solver it is compared with (phyz-contact) needs the unvendored tang
//     crate, so this restatement is pinned against the reference's own
//     contact kernel compiled for the host (oracle/_ref) instead.
//
// Nothing in the product links this file; tests, smoke() and the bench's
// CPU-baseline leg use it through oracle/oracle_capi.cpp.
#pragma once

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../include/phyzb.h"

namespace phyz_oracle {

// ── 3-vectors and 3x3 matrices (row-major), tang::Vec3 / tang::Mat3 ──────

struct Vec3 {
    double x = 0, y = 0, z = 0;
};
inline Vec3 v3(double x, double y, double z) { return Vec3{x, y, z}; }
inline Vec3 operator+(Vec3 a, Vec3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline Vec3 operator-(Vec3 a, Vec3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline Vec3 operator-(Vec3 a) { return {-a.x, -a.y, -a.z}; }
inline Vec3 operator*(Vec3 a, double s) { return {a.x * s, a.y * s, a.z * s}; }
inline double dot(Vec3 a, Vec3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline double norm(Vec3 a) { return std::sqrt(dot(a, a)); }
inline Vec3 cross(Vec3 a, Vec3 b) {
    return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}

struct Mat3 {
    double m[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    static Mat3 identity() {
        Mat3 r;
        r.m[0] = r.m[4] = r.m[8] = 1.0;
        return r;
    }
    double operator()(int r, int c) const { return m[r * 3 + c]; }
    double& operator()(int r, int c) { return m[r * 3 + c]; }
};
inline Vec3 mul(const Mat3& a, Vec3 v) {
    return {a.m[0] * v.x + a.m[1] * v.y + a.m[2] * v.z, a.m[3] * v.x + a.m[4] * v.y + a.m[5] * v.z,
            a.m[6] * v.x + a.m[7] * v.y + a.m[8] * v.z};
}
inline Vec3 tmul(const Mat3& a, Vec3 v) {  // a^T v
    return {a.m[0] * v.x + a.m[3] * v.y + a.m[6] * v.z, a.m[1] * v.x + a.m[4] * v.y + a.m[7] * v.z,
            a.m[2] * v.x + a.m[5] * v.y + a.m[8] * v.z};
}
inline Mat3 mul(const Mat3& a, const Mat3& b) {
    Mat3 r;
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) {
            double s = 0;
            for (int k = 0; k < 3; k++) s += a(i, k) * b(k, j);
            r(i, j) = s;
        }
    return r;
}
inline Mat3 transpose(const Mat3& a) {
    Mat3 t;
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) t(i, j) = a(j, i);
    return t;
}
inline Mat3 add(const Mat3& a, const Mat3& b) {
    Mat3 r;
    for (int i = 0; i < 9; i++) r.m[i] = a.m[i] + b.m[i];
    return r;
}
inline Mat3 sub(const Mat3& a, const Mat3& b) {
    Mat3 r;
    for (int i = 0; i < 9; i++) r.m[i] = a.m[i] - b.m[i];
    return r;
}
inline Mat3 scale(const Mat3& a, double s) {
    Mat3 r;
    for (int i = 0; i < 9; i++) r.m[i] = a.m[i] * s;
    return r;
}
// tang::skew: [[0,-z,y],[z,0,-x],[-y,x,0]]
inline Mat3 skew(Vec3 a) {
    Mat3 r;
    r(0, 1) = -a.z;
    r(0, 2) = a.y;
    r(1, 0) = a.z;
    r(1, 2) = -a.x;
    r(2, 0) = -a.y;
    r(2, 1) = a.x;
    return r;
}
inline Mat3 outer(Vec3 a, Vec3 b) {
    Mat3 r;
    double av[3] = {a.x, a.y, a.z}, bv[3] = {b.x, b.y, b.z};
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) r(i, j) = av[i] * bv[j];
    return r;
}

// ── spatial vectors [angular; linear] and 6x6 block matrices ─────────────

struct SVec {
    Vec3 ang, lin;
};
inline SVec operator+(SVec a, SVec b) { return {a.ang + b.ang, a.lin + b.lin}; }
inline SVec operator-(SVec a, SVec b) { return {a.ang - b.ang, a.lin - b.lin}; }
inline SVec operator*(SVec a, double s) { return {a.ang * s, a.lin * s}; }
inline double dot(SVec a, SVec b) { return dot(a.ang, b.ang) + dot(a.lin, b.lin); }
inline double sv_get(const SVec& a, int i) {
    const double* p = i < 3 ? &a.ang.x : &a.lin.x;
    return p[i % 3];
}
inline void sv_set(SVec& a, int i, double v) {
    double* p = i < 3 ? &a.ang.x : &a.lin.x;
    p[i % 3] = v;
}
// v x w (motion): phyz_kernels.cu:110-116
inline SVec cross_motion(SVec v, SVec w) {
    return {cross(v.ang, w.ang), cross(v.ang, w.lin) + cross(v.lin, w.ang)};
}
// v x* f (force): phyz_kernels.cu:118-124
inline SVec cross_force(SVec v, SVec f) {
    return {cross(v.ang, f.ang) + cross(v.lin, f.lin), cross(v.ang, f.lin)};
}

struct SMat {  // | ul ur ; ll lr |
    Mat3 ul, ur, ll, lr;
};
inline SVec mul(const SMat& a, SVec v) {
    return {mul(a.ul, v.ang) + mul(a.ur, v.lin), mul(a.ll, v.ang) + mul(a.lr, v.lin)};
}
inline SMat mul(const SMat& a, const SMat& b) {
    return {add(mul(a.ul, b.ul), mul(a.ur, b.ll)), add(mul(a.ul, b.ur), mul(a.ur, b.lr)),
            add(mul(a.ll, b.ul), mul(a.lr, b.ll)), add(mul(a.ll, b.ur), mul(a.lr, b.lr))};
}
inline SMat transpose(const SMat& a) {
    return {transpose(a.ul), transpose(a.ll), transpose(a.ur), transpose(a.lr)};
}
inline SMat add(const SMat& a, const SMat& b) {
    return {add(a.ul, b.ul), add(a.ur, b.ur), add(a.ll, b.ll), add(a.lr, b.lr)};
}
inline SMat sub(const SMat& a, const SMat& b) {
    return {sub(a.ul, b.ul), sub(a.ur, b.ur), sub(a.ll, b.ll), sub(a.lr, b.lr)};
}
inline SMat scale(const SMat& a, double s) {
    return {scale(a.ul, s), scale(a.ur, s), scale(a.ll, s), scale(a.lr, s)};
}
inline double sm_get(const SMat& a, int i, int j) {
    const Mat3& b = i < 3 ? (j < 3 ? a.ul : a.ur) : (j < 3 ? a.ll : a.lr);
    return b(i % 3, j % 3);
}
// aba.rs:493-517 outer_product_6
inline SMat outer6(SVec a, SVec b) {
    return {outer(a.ang, b.ang), outer(a.ang, b.lin), outer(a.lin, b.ang), outer(a.lin, b.lin)};
}

// ── Plücker transforms (tang::SpatialTransform) ──────────────────────────

struct SXform {
    Mat3 rot = Mat3::identity();
    Vec3 pos;
    // X v = [R w; R (v - p x w)]  (phyz_kernels.cu:314-320)
    SVec apply_motion(SVec s) const {
        return {mul(rot, s.ang), mul(rot, s.lin - cross(pos, s.ang))};
    }
    // X^{-T} f = [R^T tau + p x R^T f; R^T f]  (phyz_kernels.cu:322-329)
    SVec inv_apply_force(SVec f) const {
        Vec3 rtf = tmul(rot, f.lin);
        return {tmul(rot, f.ang) + cross(pos, rtf), rtf};
    }
    // self.compose(other): rot = self.rot*other.rot, pos = other.pos + other.rot^T self.pos
    // (phyz_kernels.cu:306-312)
    SXform compose(const SXform& other) const {
        SXform r;
        r.rot = mul(rot, other.rot);
        r.pos = other.pos + tmul(other.rot, pos);
        return r;
    }
    // [R 0; -R skew(p) R]  (phyz_kernels.cu:180-200)
    SMat to_motion_matrix() const {
        SMat m;
        m.ul = rot;
        m.lr = rot;
        m.ll = scale(mul(rot, skew(pos)), -1.0);
        return m;
    }
};

// tang::SpatialInertia about the COM -> 6x6 about the body origin
// (phyz_kernels.cu:331-359).
struct SInertia {
    double mass = 0;
    Vec3 com;
    Mat3 inertia;  // about the COM
    SMat to_matrix() const {
        SMat m;
        double cc = dot(com, com);
        m.ul = add(inertia, scale(sub(scale(Mat3::identity(), cc), outer(com, com)), mass));
        m.ur = scale(skew(com), mass);
        m.ll = transpose(m.ur);
        m.lr = scale(Mat3::identity(), mass);
        return m;
    }
};

// ── quaternions (tang::Quat, w + v) and the exp/log maps ──────────────────

struct Quat {
    double w = 1;
    Vec3 v;
};
inline Quat qmul(Quat a, Quat b) {
    return {a.w * b.w - dot(a.v, b.v), b.v * a.w + a.v * b.w + cross(a.v, b.v)};
}
inline Quat qnormalize(Quat q) {
    double n = std::sqrt(q.w * q.w + dot(q.v, q.v));
    return {q.w / n, q.v * (1.0 / n)};
}
// q p q*  (phyz_kernels.cu:298-303)
inline Vec3 qrotate(Quat q, Vec3 p) {
    Vec3 t = cross(q.v, p) * 2.0;
    return p + t * q.w + cross(q.v, t);
}
// row-major rotation matrix of a unit quaternion (phyz_kernels.cu:270-277)
inline Mat3 qto_matrix(Quat q) {
    double w = q.w, x = q.v.x, y = q.v.y, z = q.v.z;
    Mat3 r;
    r.m[0] = 1 - 2 * (y * y + z * z);
    r.m[1] = 2 * (x * y - w * z);
    r.m[2] = 2 * (x * z + w * y);
    r.m[3] = 2 * (x * y + w * z);
    r.m[4] = 1 - 2 * (x * x + z * z);
    r.m[5] = 2 * (y * z - w * x);
    r.m[6] = 2 * (x * z - w * y);
    r.m[7] = 2 * (y * z + w * x);
    r.m[8] = 1 - 2 * (x * x + y * y);
    return r;
}
// crates/phyz-math/src/lib.rs:43-56
inline Quat quat_exp(Vec3 omega) {
    double angle = norm(omega);
    if (angle < DBL_EPSILON) return {1.0, omega * 0.5};
    double s = std::sin(angle * 0.5), c = std::cos(angle * 0.5);
    return {c, omega * (s / angle)};
}
// crates/phyz-math/src/lib.rs:62-70
inline Vec3 quat_log(Quat q) {
    double nv = norm(q.v);
    if (nv < DBL_EPSILON) return q.v * 2.0;
    double angle = 2.0 * std::atan2(nv, q.w);
    return q.v * (angle / nv);
}

// ── model ────────────────────────────────────────────────────────────────

enum JointType { REVOLUTE = 0, PRISMATIC = 1, FIXED = 2, BALL = 3, FREE = 4 };

struct Joint {
    int type = FIXED;
    SXform parent_to_joint;
    Vec3 axis;
    double damping = 0, stiffness = 0, spring_ref = 0, armature = 0;
    bool has_limits = false;
    double lim_lo = 0, lim_hi = 0, lim_k = 1000.0, lim_d = 60.0;
    double friction_loss = 0;

    int ndof() const {  // joint.rs:164-172
        switch (type) {
            case REVOLUTE:
            case PRISMATIC: return 1;
            case BALL: return 3;
            case FREE: return 6;
            default: return 0;
        }
    }
    // joint.rs:254-316
    SXform joint_transform(const double* q) const {
        SXform x;
        switch (type) {
            case REVOLUTE: {
                double s = std::sin(-q[0]), c = std::cos(-q[0]);
                Mat3 k = skew(axis);
                x.rot = add(add(Mat3::identity(), scale(k, s)), scale(mul(k, k), 1.0 - c));
                break;
            }
            case PRISMATIC: x.pos = axis * q[0]; break;
            case BALL: x.rot = transpose(qto_matrix(quat_exp(v3(q[0], q[1], q[2])))); break;
            case FREE:
                x.rot = transpose(qto_matrix(quat_exp(v3(q[0], q[1], q[2]))));
                x.pos = v3(q[3], q[4], q[5]);
                break;
            default: break;
        }
        return x;
    }
    // S qd  (aba.rs:15-30)
    SVec joint_velocity(const double* qd) const {
        switch (type) {
            case REVOLUTE: return {axis * qd[0], Vec3{}};
            case PRISMATIC: return {Vec3{}, axis * qd[0]};
            case BALL: return {v3(qd[0], qd[1], qd[2]), Vec3{}};
            case FREE: return {v3(qd[0], qd[1], qd[2]), v3(qd[3], qd[4], qd[5])};
            default: return {};
        }
    }
    // column k of S (joint.rs:322-362)
    SVec subspace_col(int k) const {
        SVec s{};
        switch (type) {
            case REVOLUTE: s.ang = axis; break;
            case PRISMATIC: s.lin = axis; break;
            case BALL:
            case FREE: sv_set(s, k, 1.0); break;
            default: break;
        }
        return s;
    }
    // joint.rs:184-230
    double limit_force(double q, double qd) const {
        if (ndof() != 1 || !has_limits) return 0.0;
        double depth, sign;
        if (q < lim_lo) {
            depth = lim_lo - q;
            sign = 1.0;
        } else if (q > lim_hi) {
            depth = q - lim_hi;
            sign = -1.0;
        } else {
            return 0.0;
        }
        double inward = std::fmax(-sign * qd, 0.0);
        return sign * (lim_k * depth + lim_d * inward);
    }
    // joint.rs:232-247
    double passive_force(int k, double q, double qd) const {
        double f = -damping * qd;
        if (ndof() == 1 && k == 0) {
            f += -stiffness * (q - spring_ref);
            f += limit_force(q, qd);
            if (friction_loss > 0.0) f += -friction_loss * std::tanh(qd / 1e-3);
        }
        return f;
    }
};

struct Geom {
    int type = 0;
    double p[6] = {0, 0, 0, 0, 0, 0};
    Vec3 opos;
    Mat3 orot = Mat3::identity();
};

struct Body {
    SInertia inertia;
    int parent = -1;
    Geom geom;
};

struct Model {
    std::vector<Body> bodies;
    std::vector<Joint> joints;  // joint i belongs to body i
    Vec3 gravity;
    double dt = 0.001;
    int nq = 0, nv = 0;
    std::vector<int> q_off, v_off;
    int nb() const { return (int)bodies.size(); }
};

inline Vec3 arr3(const double* a) { return v3(a[0], a[1], a[2]); }
inline Mat3 arr9(const double* a) {
    Mat3 m;
    for (int i = 0; i < 9; i++) m.m[i] = a[i];
    return m;
}

// Model from the flat C description; ModelBuilder::build offsets
// (model.rs:530-550).
inline Model from_flat(const phyzb_model* fm) {
    Model m;
    m.gravity = arr3(fm->gravity);
    m.dt = fm->dt;
    for (int i = 0; i < fm->nbodies; i++) {
        const phyzb_body& b = fm->bodies[i];
        Body body;
        body.parent = b.parent;
        body.inertia.mass = b.mass;
        body.inertia.com = arr3(b.com);
        Mat3 I;
        I(0, 0) = b.inertia[0];
        I(1, 1) = b.inertia[1];
        I(2, 2) = b.inertia[2];
        I(0, 1) = I(1, 0) = b.inertia[3];
        I(0, 2) = I(2, 0) = b.inertia[4];
        I(1, 2) = I(2, 1) = b.inertia[5];
        body.inertia.inertia = I;
        body.geom.type = b.geom_type;
        for (int k = 0; k < 6; k++) body.geom.p[k] = b.geom_params[k];
        body.geom.opos = arr3(b.geom_origin_pos);
        body.geom.orot = arr9(b.geom_origin_rot);
        Joint j;
        j.type = b.joint_type;
        j.parent_to_joint.rot = arr9(b.ptj_rot);
        j.parent_to_joint.pos = arr3(b.ptj_pos);
        j.axis = arr3(b.axis);
        j.damping = b.damping;
        j.stiffness = b.stiffness;
        j.spring_ref = b.spring_ref;
        j.armature = b.armature;
        j.has_limits = b.has_limits != 0;
        j.lim_lo = b.limit_lower;
        j.lim_hi = b.limit_upper;
        j.lim_k = b.limit_stiffness;
        j.lim_d = b.limit_damping;
        j.friction_loss = b.friction_loss;
        m.q_off.push_back(m.nq);
        m.v_off.push_back(m.nv);
        m.nq += j.ndof();
        m.nv += j.ndof();
        m.bodies.push_back(body);
        m.joints.push_back(j);
    }
    return m;
}

// ── small dense matrices for the multi-DOF path (tang_la DMat) ────────────

// Inverse by Gauss-Jordan with partial pivoting; false when singular.
inline bool try_inverse(std::vector<double>& a, int n) {
    std::vector<double> inv(n * n, 0.0);
    for (int i = 0; i < n; i++) inv[i * n + i] = 1.0;
    for (int col = 0; col < n; col++) {
        int piv = col;
        double best = std::fabs(a[col * n + col]);
        for (int r = col + 1; r < n; r++)
            if (std::fabs(a[r * n + col]) > best) {
                best = std::fabs(a[r * n + col]);
                piv = r;
            }
        if (best == 0.0) return false;
        if (piv != col)
            for (int c = 0; c < n; c++) {
                std::swap(a[col * n + c], a[piv * n + c]);
                std::swap(inv[col * n + c], inv[piv * n + c]);
            }
        double d = a[col * n + col];
        for (int c = 0; c < n; c++) {
            a[col * n + c] /= d;
            inv[col * n + c] /= d;
        }
        for (int r = 0; r < n; r++) {
            if (r == col) continue;
            double f = a[r * n + col];
            if (f == 0.0) continue;
            for (int c = 0; c < n; c++) {
                a[r * n + c] -= f * a[col * n + c];
                inv[r * n + c] -= f * inv[col * n + c];
            }
        }
    }
    a = inv;
    return true;
}

// ── generalized forces (actuation.rs:18-54) ──────────────────────────────

inline std::vector<double> generalized_forces(const Model& m, const double* q, const double* v,
                                              const double* ctrl) {
    std::vector<double> f(m.nv, 0.0);
    for (int i = 0; i < m.nv; i++) f[i] = ctrl ? ctrl[i] : 0.0;  // model.rs:210-214
    for (int j = 0; j < m.nb(); j++) {
        const Joint& jt = m.joints[j];
        for (int k = 0; k < jt.ndof(); k++)
            f[m.v_off[j] + k] += jt.passive_force(k, q[m.q_off[j] + k], v[m.v_off[j] + k]);
    }
    return f;
}

// ── ABA (aba.rs:152-420) ─────────────────────────────────────────────────

inline std::vector<double> aba(const Model& m, const double* q, const double* v,
                               const double* ctrl, const SVec* ext) {
    const int nb = m.nb();
    std::vector<double> qdd(m.nv, 0.0);
    std::vector<double> qfrc = generalized_forces(m, q, v, ctrl);
    std::vector<SXform> x_tree(nb);
    std::vector<SVec> vel(nb), c_bias(nb), p_a(nb), acc(nb);
    std::vector<SMat> i_a(nb);
    const SVec a0{Vec3{}, -m.gravity};

    // pass 1 (aba.rs:175-213)
    for (int i = 0; i < nb; i++) {
        const Body& body = m.bodies[i];
        const Joint& jt = m.joints[i];
        int ndof = jt.ndof();
        SXform xj = ndof == 0 ? SXform{} : jt.joint_transform(q + m.q_off[i]);
        x_tree[i] = xj.compose(jt.parent_to_joint);
        SVec vj = jt.joint_velocity(v + m.v_off[i]);
        if (body.parent < 0) {
            vel[i] = vj;
            c_bias[i] = SVec{};
        } else {
            vel[i] = x_tree[i].apply_motion(vel[body.parent]) + vj;
            c_bias[i] = cross_motion(vel[i], vj);
        }
        i_a[i] = body.inertia.to_matrix();
        p_a[i] = cross_force(vel[i], mul(i_a[i], vel[i]));
        if (ext) p_a[i] = p_a[i] - ext[i];
    }

    // pass 2 (aba.rs:215-320)
    for (int i = nb - 1; i >= 0; i--) {
        const Body& body = m.bodies[i];
        const Joint& jt = m.joints[i];
        int vi = m.v_off[i];
        int ndof = jt.ndof();
        double imp = m.dt * jt.damping;  // aba.rs:418-420
        if (ndof == 0) {
            if (body.parent >= 0) {
                SMat xm = x_tree[i].to_motion_matrix();
                i_a[body.parent] = add(i_a[body.parent], mul(mul(transpose(xm), i_a[i]), xm));
                p_a[body.parent] = p_a[body.parent] + x_tree[i].inv_apply_force(p_a[i]);
            }
            continue;
        }
        if (ndof == 1) {
            SVec s = jt.subspace_col(0);
            const SMat& ia = i_a[i];
            double u = qfrc[vi] - dot(s, p_a[i]);
            double d = dot(s, mul(ia, s)) + jt.armature + imp;
            if (std::fabs(d) < 1e-20) continue;
            double u_inv_d = u / d;
            SVec ia_s = mul(ia, s);
            if (body.parent >= 0) {
                SMat ia_new = sub(ia, scale(outer6(ia_s, mul(ia, s)), 1.0 / d));
                SVec p_new = p_a[i] + mul(ia_new, c_bias[i]) + ia_s * u_inv_d;
                SMat xm = x_tree[i].to_motion_matrix();
                i_a[body.parent] = add(i_a[body.parent], mul(mul(transpose(xm), ia_new), xm));
                p_a[body.parent] = p_a[body.parent] + x_tree[i].inv_apply_force(p_new);
            }
        } else {
            const SMat& ia = i_a[i];
            // U = I_a S (6 x n), D = S^T U + diag, u = tau - S^T p_a
            std::vector<double> U(6 * ndof), D(ndof * ndof), uvec(ndof);
            for (int k = 0; k < ndof; k++) {
                SVec col = mul(ia, jt.subspace_col(k));
                for (int r = 0; r < 6; r++) U[r * ndof + k] = sv_get(col, r);
                uvec[k] = qfrc[vi + k] - dot(jt.subspace_col(k), p_a[i]);
            }
            for (int r = 0; r < ndof; r++)
                for (int c = 0; c < ndof; c++) {
                    SVec sr = jt.subspace_col(r);
                    double s = 0;
                    for (int t = 0; t < 6; t++) s += sv_get(sr, t) * U[t * ndof + c];
                    D[r * ndof + c] = s;
                }
            for (int k = 0; k < ndof; k++) D[k * ndof + k] += jt.armature + imp;
            if (!try_inverse(D, ndof)) continue;
            if (body.parent >= 0) {
                // U D^-1 (6 x n), I_a^A = I_a - U D^-1 U^T
                std::vector<double> UD(6 * ndof, 0.0);
                for (int r = 0; r < 6; r++)
                    for (int c = 0; c < ndof; c++) {
                        double s = 0;
                        for (int k = 0; k < ndof; k++) s += U[r * ndof + k] * D[k * ndof + c];
                        UD[r * ndof + c] = s;
                    }
                SMat ia_new = ia;
                double dense[36];
                for (int r = 0; r < 6; r++)
                    for (int c = 0; c < 6; c++) {
                        double s = 0;
                        for (int k = 0; k < ndof; k++) s += UD[r * ndof + k] * U[c * ndof + k];
                        dense[r * 6 + c] = sm_get(ia, r, c) - s;
                    }
                for (int r = 0; r < 3; r++)
                    for (int c = 0; c < 3; c++) {
                        ia_new.ul(r, c) = dense[r * 6 + c];
                        ia_new.ur(r, c) = dense[r * 6 + c + 3];
                        ia_new.ll(r, c) = dense[(r + 3) * 6 + c];
                        ia_new.lr(r, c) = dense[(r + 3) * 6 + c + 3];
                    }
                // p_a^A = p_a + I_a^A c + U D^-1 u
                std::vector<double> dinv_u(ndof, 0.0);
                for (int r = 0; r < ndof; r++)
                    for (int c = 0; c < ndof; c++) dinv_u[r] += D[r * ndof + c] * uvec[c];
                SVec udu{};
                for (int r = 0; r < 6; r++) {
                    double s = 0;
                    for (int k = 0; k < ndof; k++) s += U[r * ndof + k] * dinv_u[k];
                    sv_set(udu, r, s);
                }
                SVec p_new = p_a[i] + (mul(ia_new, c_bias[i]) + udu);
                SMat xm = x_tree[i].to_motion_matrix();
                i_a[body.parent] = add(i_a[body.parent], mul(mul(transpose(xm), ia_new), xm));
                p_a[body.parent] = p_a[body.parent] + x_tree[i].inv_apply_force(p_new);
            }
        }
    }

    // pass 3 (aba.rs:322-400)
    for (int i = 0; i < nb; i++) {
        const Body& body = m.bodies[i];
        const Joint& jt = m.joints[i];
        int vi = m.v_off[i];
        int ndof = jt.ndof();
        double imp = m.dt * jt.damping;
        SVec a_parent = body.parent < 0 ? x_tree[i].apply_motion(a0)
                                        : x_tree[i].apply_motion(acc[body.parent]);
        if (ndof == 0) {
            acc[i] = a_parent + c_bias[i];
            continue;
        }
        if (ndof == 1) {
            SVec s = jt.subspace_col(0);
            const SMat& ia = i_a[i];
            double d = dot(s, mul(ia, s)) + jt.armature + imp;
            if (std::fabs(d) < 1e-20) {
                acc[i] = a_parent + c_bias[i];
                continue;
            }
            double u = qfrc[vi] - dot(s, p_a[i]);
            double qdd_i = (u - dot(mul(ia, a_parent + c_bias[i]), s)) / d;
            qdd[vi] = qdd_i;
            acc[i] = a_parent + c_bias[i] + s * qdd_i;
        } else {
            const SMat& ia = i_a[i];
            std::vector<double> U(6 * ndof), D(ndof * ndof), uvec(ndof);
            for (int k = 0; k < ndof; k++) {
                SVec col = mul(ia, jt.subspace_col(k));
                for (int r = 0; r < 6; r++) U[r * ndof + k] = sv_get(col, r);
            }
            for (int r = 0; r < ndof; r++)
                for (int c = 0; c < ndof; c++) {
                    SVec sr = jt.subspace_col(r);
                    double s = 0;
                    for (int t = 0; t < 6; t++) s += sv_get(sr, t) * U[t * ndof + c];
                    D[r * ndof + c] = s;
                }
            for (int k = 0; k < ndof; k++) D[k * ndof + k] += jt.armature + imp;
            if (!try_inverse(D, ndof)) {
                acc[i] = a_parent + c_bias[i];
                continue;
            }
            for (int k = 0; k < ndof; k++) uvec[k] = qfrc[vi + k] - dot(jt.subspace_col(k), p_a[i]);
            SVec a_total = a_parent + c_bias[i];
            SVec ia_a = mul(ia, a_total);
            std::vector<double> rhs(ndof);
            for (int k = 0; k < ndof; k++) rhs[k] = uvec[k] - dot(jt.subspace_col(k), ia_a);
            SVec s_qdd{};
            for (int r = 0; r < ndof; r++) {
                double s = 0;
                for (int c = 0; c < ndof; c++) s += D[r * ndof + c] * rhs[c];
                qdd[vi + r] = s;
            }
            for (int k = 0; k < ndof; k++) s_qdd = s_qdd + jt.subspace_col(k) * qdd[vi + k];
            acc[i] = a_total + s_qdd;
        }
    }
    return qdd;
}

// ── integrator (integrate.rs:41-91) ──────────────────────────────────────

inline void integrate_configuration(const Model& m, double* q, const double* v, double dt) {
    for (int j = 0; j < m.nb(); j++) {
        int qo = m.q_off[j], vo = m.v_off[j];
        switch (m.joints[j].type) {
            case REVOLUTE:
            case PRISMATIC: q[qo] += dt * v[vo]; break;
            case BALL: {
                Vec3 omega = v3(v[vo], v[vo + 1], v[vo + 2]);
                Quat cur = quat_exp(v3(q[qo], q[qo + 1], q[qo + 2]));
                Quat nxt = qnormalize(qmul(cur, quat_exp(omega * dt)));
                Vec3 lg = quat_log(nxt);
                q[qo] = lg.x;
                q[qo + 1] = lg.y;
                q[qo + 2] = lg.z;
                break;
            }
            case FREE: {
                Vec3 omega = v3(v[vo], v[vo + 1], v[vo + 2]);
                Vec3 lin = v3(v[vo + 3], v[vo + 4], v[vo + 5]);
                Quat cur = quat_exp(v3(q[qo], q[qo + 1], q[qo + 2]));
                Vec3 wl = qrotate(cur, lin);
                q[qo + 3] += dt * wl.x;
                q[qo + 4] += dt * wl.y;
                q[qo + 5] += dt * wl.z;
                Quat nxt = qnormalize(qmul(cur, quat_exp(omega * dt)));
                Vec3 lg = quat_log(nxt);
                q[qo] = lg.x;
                q[qo + 1] = lg.y;
                q[qo + 2] = lg.z;
                break;
            }
            default: break;
        }
    }
}

inline void semi_implicit_euler(const Model& m, double* q, double* v, const double* qdd,
                                double dt) {
    for (int i = 0; i < m.nv; i++) v[i] += dt * qdd[i];
    integrate_configuration(m, q, v, dt);
}

// ── kinematics (kinematics.rs:10-50) ─────────────────────────────────────

// World->body transforms and body-frame velocities.
inline void forward_kinematics(const Model& m, const double* q, const double* v,
                               std::vector<SXform>& xw, std::vector<SVec>& vel) {
    int nb = m.nb();
    xw.assign(nb, SXform{});
    vel.assign(nb, SVec{});
    for (int i = 0; i < nb; i++) {
        const Joint& jt = m.joints[i];
        SXform xj = jt.ndof() == 0 ? SXform{} : jt.joint_transform(q + m.q_off[i]);
        SXform xt = xj.compose(jt.parent_to_joint);
        SVec vj = jt.joint_velocity(v + m.v_off[i]);
        int p = m.bodies[i].parent;
        if (p < 0) {
            xw[i] = xt;
            vel[i] = vj;
        } else {
            xw[i] = xt.compose(xw[p]);
            vel[i] = xt.apply_motion(vel[p]) + vj;
        }
    }
}

// ── RNEA (rnea.rs:94-169): tau for given qdd ─────────────────────────────

inline std::vector<double> rnea(const Model& m, const double* q, const double* v,
                                const double* qdd) {
    int nb = m.nb();
    std::vector<SXform> xt(nb);
    std::vector<SVec> vel(nb), acc(nb), f(nb);
    const SVec a0{Vec3{}, -m.gravity};
    for (int i = 0; i < nb; i++) {
        const Joint& jt = m.joints[i];
        SXform xj = jt.ndof() == 0 ? SXform{} : jt.joint_transform(q + m.q_off[i]);
        xt[i] = xj.compose(jt.parent_to_joint);
        SVec vj = jt.joint_velocity(v + m.v_off[i]);
        SVec aj = jt.joint_velocity(qdd + m.v_off[i]);
        int p = m.bodies[i].parent;
        if (p < 0) {
            vel[i] = vj;
            acc[i] = xt[i].apply_motion(a0) + aj;
        } else {
            vel[i] = xt[i].apply_motion(vel[p]) + vj;
            acc[i] = xt[i].apply_motion(acc[p]) + cross_motion(vel[i], vj) + aj;
        }
        SMat I = m.bodies[i].inertia.to_matrix();
        f[i] = mul(I, acc[i]) + cross_force(vel[i], mul(I, vel[i]));
    }
    std::vector<double> tau(m.nv, 0.0);
    for (int i = nb - 1; i >= 0; i--) {
        const Joint& jt = m.joints[i];
        for (int k = 0; k < jt.ndof(); k++) tau[m.v_off[i] + k] = dot(jt.subspace_col(k), f[i]);
        int p = m.bodies[i].parent;
        if (p >= 0) f[p] = f[p] + xt[i].inv_apply_force(f[i]);
    }
    return tau;
}

// ── energy (energy.rs; KE body-wise plus armature, which crba carries) ───

inline double kinetic_energy(const Model& m, const double* q, const double* v) {
    std::vector<SXform> xw;
    std::vector<SVec> vel;
    forward_kinematics(m, q, v, xw, vel);
    double ke = 0;
    for (int i = 0; i < m.nb(); i++) {
        SMat I = m.bodies[i].inertia.to_matrix();
        ke += 0.5 * dot(vel[i], mul(I, vel[i]));
        const Joint& jt = m.joints[i];
        for (int k = 0; k < jt.ndof(); k++) {
            double qd = v[m.v_off[i] + k];
            ke += 0.5 * jt.armature * qd * qd;
        }
    }
    return ke;
}
inline double potential_energy(const Model& m, const double* q) {
    std::vector<double> zero(m.nv, 0.0);
    std::vector<SXform> xw;
    std::vector<SVec> vel;
    forward_kinematics(m, q, zero.data(), xw, vel);
    double pe = 0;
    for (int i = 0; i < m.nb(); i++) {
        Vec3 cw = xw[i].pos + tmul(xw[i].rot, m.bodies[i].inertia.com);
        pe -= m.bodies[i].inertia.mass * dot(m.gravity, cw);
    }
    return pe;
}

// ── penalty ground contact: the GPU law in f64 ───────────────────────────

// Terrain: the flat plane at `ground` or, with nx > 0, a heightfield of
// f32 node heights (phyz-model/src/heightfield.rs:10-37) sampled as the
// GPU samples it (phyz_kernels.cu:625-664).
struct Terrain {
    double ground = 0;
    int nx = 0, ny = 0;
    double ox = 0, oy = 0, oz = 0, cell = 1;
    std::vector<float> h;  // [ny][nx]
    double node(int ix, int iy) const { return oz + (double)h[(size_t)iy * nx + ix]; }
    void locate(double w, double o, int n, int& i, double& t) const {
        if (n < 2) {
            i = 0;
            t = 0.0;
            return;
        }
        double u = std::fmin(std::fmax((w - o) / cell, 0.0), (double)(n - 1));
        int ii = (int)u;
        if (ii > n - 2) ii = n - 2;
        i = ii;
        t = u - ii;
    }
    // height at world (px, py); unit normal out
    double sample(double px, double py, Vec3& n_out) const {
        if (nx == 0) {
            n_out = v3(0, 0, 1);
            return ground;
        }
        int ix, iy;
        double tx, ty;
        locate(px, ox, nx, ix, tx);
        locate(py, oy, ny, iy, ty);
        int ix1 = ix + 1 < nx - 1 ? ix + 1 : nx - 1;
        int iy1 = iy + 1 < ny - 1 ? iy + 1 : ny - 1;
        double h00 = node(ix, iy), h10 = node(ix1, iy), h01 = node(ix, iy1), h11 = node(ix1, iy1);
        double h = (h00 * (1.0 - tx) + h10 * tx) * (1.0 - ty) + (h01 * (1.0 - tx) + h11 * tx) * ty;
        double dhdx = 0.0, dhdy = 0.0;
        double span_x = (nx - 1) * cell, span_y = (ny - 1) * cell;
        if (nx >= 2 && px >= ox && px <= ox + span_x) dhdx = ((h10 - h00) * (1.0 - ty) + (h11 - h01) * ty) / cell;
        if (ny >= 2 && py >= oy && py <= oy + span_y) dhdy = ((h01 - h00) * (1.0 - tx) + (h11 - h10) * tx) / cell;
        Vec3 n = v3(-dhdx, -dhdy, 1.0);
        double l = norm(n);
        n_out = l > 0.0 ? n * (1.0 / l) : n;
        return h;
    }
};

// A contact plane attached to a body (contact_pipeline.rs:318-355
// BodyPlane): the face at `offset` along the body's +z, half_x x half_y in
// its x/y; `no_plane[i]` marks the bodies that never touch it (the plane
// body itself and the exclude list: pack_contact_geometry's geometry[7]).
struct Plane {
    int body = -1;
    double offset = 0, max_depth = 0, half_x = 0, half_y = 0;
    std::vector<char> no_plane;
};

struct ContactParams {
    double ground_height = 0, friction = 0;
    std::vector<double> k, d;  // per body gains (layout.rs:272-278)
    Terrain terrain;           // terrain.ground mirrors ground_height
    Plane plane;
};

// Contact of every body with the body-attached plane, action on the body
// and reaction on the plane's body at one shared point (phyz_kernels.cu:
// 983-1132). `vel`: body-frame velocities (current in penalty mode, free in
// impulse mode); penalty mode uses the gains k, d; impulse mode (imp !=
// null: the material) updates the staged impulses `pimp` [nb][8][3].
struct ImpulseParams;
inline double impedance_at(const ImpulseParams& c, double depth);
inline double effective_restitution(const ImpulseParams& c, double e, double approach);
inline void contact_tangents(Vec3 n, Vec3& u, Vec3& w);
inline double contact_eff_mass(const Body& b, Vec3 r, Vec3 u);
inline Vec3 support_point(const Geom& g, Vec3 n_body);
inline Vec3 box_corner(const Geom& g, int c);
inline double max_damping(double me, double dt);
inline double max_stiffness(double me, double dt);
inline void plane_contact(const Model& m, const Plane& pl, double friction, const double* k, const double* d,
                          const ImpulseParams* imp, const std::vector<Mat3>& wrot, const std::vector<Vec3>& wpos,
                          const std::vector<SVec>& vel, std::vector<SVec>& ext, double* pimp);

inline double fsign(double x) { return x > 0 ? 1.0 : (x < 0 ? -1.0 : 0.0); }

// I^-1 w about the COM, cofactor inverse (phyz_kernels.cu:545-561)
inline Vec3 inertia_solve(const Body& b, Vec3 w) {
    const Mat3& I = b.inertia.inertia;
    double xx = I(0, 0), yy = I(1, 1), zz = I(2, 2), xy = I(0, 1), xz = I(0, 2), yz = I(1, 2);
    double c00 = yy * zz - yz * yz, c01 = xz * yz - xy * zz, c02 = xy * yz - xz * yy;
    double det = xx * c00 + xy * c01 + xz * c02;
    if (std::fabs(det) < 1e-20) return Vec3{};
    double c11 = xx * zz - xz * xz, c12 = xy * xz - xx * yz, c22 = xx * yy - xy * xy;
    double inv = 1.0 / det;
    return v3(inv * (c00 * w.x + c01 * w.y + c02 * w.z), inv * (c01 * w.x + c11 * w.y + c12 * w.z),
              inv * (c02 * w.x + c12 * w.y + c22 * w.z));
}
// phyz_kernels.cu:564-571
inline double contact_eff_mass(const Body& b, Vec3 r, Vec3 u) {
    double m = b.inertia.mass;
    if (m <= 0.0) return 1e30;
    Vec3 a = cross(r - b.inertia.com, u);
    double ang = std::fmax(dot(a, inertia_solve(b, a)), 0.0);
    return 1.0 / (1.0 / m + ang);
}
inline double max_damping(double me, double dt) { return me / std::fmax(dt, 1e-9); }
inline double max_stiffness(double me, double dt) {
    double d = std::fmax(dt, 1e-9);
    return 4.0 * me / (d * d);
}
// support point of the body's shape against body-frame direction n
// (phyz_kernels.cu:691-725) and box corners (:679-689)
inline Vec3 support_point(const Geom& g, Vec3 n_body) {
    Vec3 n = mul(g.orot, n_body);
    Vec3 s{};
    switch (g.type) {
        case 1: s = n * (-g.p[0]); break;
        case 2: s = v3(-g.p[0] * fsign(n.x), -g.p[1] * fsign(n.y), -g.p[2] * fsign(n.z)); break;
        case 3: s = v3(0, 0, -g.p[1] * 0.5 * fsign(n.z)) - n * g.p[0]; break;
        case 4: {
            Vec3 radial = v3(-n.x, -n.y, 0);
            double rl = norm(radial);
            Vec3 rim{};
            if (rl > 1e-6) rim = radial * (g.p[0] / rl);
            s = rim + v3(0, 0, -g.p[1] * 0.5 * fsign(n.z));
            break;
        }
        case 5: {
            Vec3 mn = v3(g.p[0], g.p[1], g.p[2]), mx = v3(g.p[3], g.p[4], g.p[5]);
            Vec3 mc = (mn + mx) * 0.5, mh = (mx - mn) * 0.5;
            s = mc - v3(mh.x * fsign(n.x), mh.y * fsign(n.y), mh.z * fsign(n.z));
            break;
        }
        default: break;
    }
    return g.opos + tmul(g.orot, s);
}
inline Vec3 box_corner(const Geom& g, int c) {
    Vec3 corner = v3(g.p[0] * ((c & 1) ? 1 : -1), g.p[1] * ((c & 2) ? 1 : -1),
                     g.p[2] * ((c & 4) ? 1 : -1));
    return g.opos + tmul(g.orot, corner);
}

// Penalty contact forces (body frame, [torque; force]) for one world from
// (q, v), and the per-body contact state [touching, depth, point(3),
// force(3)] (phyz_kernels.cu:804-1061, penalty mode, flat ground).
inline void penalty_contact(const Model& m, const ContactParams& cp, const double* q,
                            const double* v, std::vector<SVec>& ext, double* cstate) {
    int nb = m.nb();
    ext.assign(nb, SVec{});
    // FK as fk_world does it: body->world rotation, origin, body-frame velocity.
    std::vector<Mat3> wrot(nb);
    std::vector<Vec3> wpos(nb);
    std::vector<SVec> vel(nb);
    for (int i = 0; i < nb; i++) {
        const Joint& jt = m.joints[i];
        SXform xj = jt.ndof() == 0 ? SXform{} : jt.joint_transform(q + m.q_off[i]);
        SXform xt = xj.compose(jt.parent_to_joint);
        SVec vj = jt.joint_velocity(v + m.v_off[i]);
        Mat3 tree_rt = transpose(xt.rot);
        int p = m.bodies[i].parent;
        if (p < 0) {
            wrot[i] = tree_rt;
            wpos[i] = xt.pos;
            vel[i] = vj;
        } else {
            wrot[i] = mul(wrot[p], tree_rt);
            wpos[i] = wpos[p] + mul(wrot[p], xt.pos);
            vel[i] = xt.apply_motion(vel[p]) + vj;
        }
    }
    for (int i = 0; i < nb; i++) {
        const Body& b = m.bodies[i];
        double* cs = cstate ? cstate + i * PHYZB_CONTACT_STRIDE : nullptr;
        if (cs)
            for (int k = 0; k < PHYZB_CONTACT_STRIDE; k++) cs[k] = 0.0;
        if (b.geom.type == 0) continue;
        Vec3 z_body = tmul(wrot[i], v3(0, 0, 1));
        int npts = 1;
        double pt_scale = 1.0;
        if (b.geom.type == 2) {
            npts = 8;
            pt_scale = 0.25;
        }
        Vec3 f_w_total{};
        double deepest = 0;
        Vec3 deepest_w{};
        bool any = false;
        for (int c = 0; c < npts; c++) {
            Vec3 sup = b.geom.type == 2 ? box_corner(b.geom, c) : support_point(b.geom, z_body);
            Vec3 sup_w = wpos[i] + mul(wrot[i], sup);
            Vec3 n_w;
            double terr_h = cp.terrain.nx > 0 ? cp.terrain.sample(sup_w.x, sup_w.y, n_w)
                                              : (n_w = v3(0, 0, 1), cp.ground_height);
            double pen = n_w.z * (terr_h - sup_w.z);
            if (!(pen > 0.0)) continue;
            Vec3 n_body = tmul(wrot[i], n_w);
            Vec3 v_point = vel[i].lin + cross(vel[i].ang, sup);
            double v_n = dot(v_point, n_body);
            double m_n = contact_eff_mass(b, sup, n_body);
            double kb = std::fmin(pt_scale * cp.k[i], max_stiffness(m_n, m.dt));
            double db = std::fmin(pt_scale * cp.d[i], max_damping(m_n, m.dt));
            double f_n = std::fmax(kb * pen - db * v_n, 0.0);
            Vec3 v_tan = v_point - n_body * v_n;
            double vt = norm(v_tan);
            Vec3 f_body = n_body * f_n;
            if (vt > 1e-6) {
                Vec3 t_dir = v_tan * (1.0 / vt);
                double coul = cp.friction * f_n * std::fmin(1.0, vt / 1e-3);
                double f_t = std::fmin(coul, max_damping(contact_eff_mass(b, sup, t_dir), m.dt) * vt);
                f_body = f_body - t_dir * f_t;
            }
            ext[i].ang = ext[i].ang + cross(sup, f_body);
            ext[i].lin = ext[i].lin + f_body;
            f_w_total = f_w_total + mul(wrot[i], f_body);
            any = true;
            if (pen > deepest) {
                deepest = pen;
                deepest_w = v3(sup_w.x, sup_w.y, terr_h);
            }
        }
        if (!any || !cs) continue;
        cs[0] = 1.0;
        cs[1] = deepest;
        cs[2] = deepest_w.x;
        cs[3] = deepest_w.y;
        cs[4] = deepest_w.z;
        cs[5] = f_w_total.x;
        cs[6] = f_w_total.y;
        cs[7] = f_w_total.z;
    }
    plane_contact(m, cp.plane, cp.friction, cp.k.data(), cp.d.data(), nullptr, wrot, wpos, vel, ext, nullptr);
}

// ── impulse-mode ground contact: the velocity-level staged Coulomb update
// of phyz_kernels.cu:804-937 (solve_mode 1, flat ground), in f64 ─────────

// Contact material of the impulse solve: enable_contact_impulse's settings
// (cuda/mod.rs:680-701) over GroundContactParams::default
// (contact_pipeline.rs:199-218).
struct ImpulseParams {
    Terrain terrain;  // nx == 0: the flat plane at ground_height
    Plane plane;
    double ground_height = 0, friction = 0;
    double restitution = 0, restitution_threshold = 0.05;
    double erp = 0;  // solref_erp_from(0.02, 1.0, dt)
    double margin = 0.001;
    double dmin = 0.9, dmax = 0.95, width = 0.001, mid = 0.5, power = 2.0;
    int sweeps = 16;  // DEFAULT_CONTACT_SWEEPS (gpu_batch_simulator.rs:31)
};

// contact_pipeline.rs:229-237
inline double solref_erp_from(double timeconst, double dampratio, double dt) {
    if (dt <= 0.0) return 0.0;
    double tau = std::fmax(timeconst, 0.0), zeta = std::fmax(dampratio, 1e-6);
    double denom = 2.0 * tau * zeta * zeta + dt;
    return denom <= 0.0 ? 1.0 : dt / denom;
}
inline double clampd(double x, double lo, double hi) { return std::fmin(std::fmax(x, lo), hi); }
// phyz_kernels.cu:589-601 (SolImp impedance)
inline double solimp_impedance(const ImpulseParams& c, double r) {
    double dmin = clampd(c.dmin, 1e-4, 1.0 - 1e-9), dmax = clampd(c.dmax, 1e-4, 1.0 - 1e-9);
    if (c.width <= 0.0) return dmax;
    double x = clampd(std::fabs(r) / c.width, 0.0, 1.0);
    double mid = clampd(c.mid, 1e-6, 1.0 - 1e-6);
    double pw = std::fmax(c.power, 1.0);
    double y = x <= mid ? std::pow(x, pw) / std::pow(mid, pw - 1.0)
                        : 1.0 - std::pow(1.0 - x, pw) / std::pow(1.0 - mid, pw - 1.0);
    return dmin + y * (dmax - dmin);
}
// phyz_kernels.cu:604-611
inline double impedance_at(const ImpulseParams& c, double depth) {
    if (depth >= 0.0) return solimp_impedance(c, depth);
    double gap = -depth;
    if (c.margin <= 0.0 || gap >= c.margin) return 0.0;
    double sc = 1.0 - gap / c.margin;
    return sc * sc * (3.0 - 2.0 * sc) * solimp_impedance(c, 0.0);
}
// phyz_kernels.cu:613-622
inline double effective_restitution(const ImpulseParams& c, double e, double approach) {
    double vr = c.restitution_threshold;
    if (vr <= 0.0) return e;
    double sp = std::fabs(approach);
    if (sp <= vr) return 0.0;
    if (sp >= 2.0 * vr) return e;
    double t = (sp - vr) / vr;
    return e * t * t * (3.0 - 2.0 * t);
}
// phyz_kernels.cu:581-586 (tangents around a unit normal)
inline void contact_tangents(Vec3 n, Vec3& u, Vec3& w) {
    Vec3 a = std::fabs(n.x) > 0.9 ? v3(0, 1, 0) : v3(1, 0, 0);
    Vec3 c = cross(n, a);
    double l = norm(c);
    u = l > 0.0 ? c * (1.0 / l) : c;
    w = cross(n, u);
}

// Per-world state the impulse solve carries across sweeps and steps: the
// contact wrench of every body (body frame, the ext_forces buffer) and the
// staged impulse [normal, tangent u, tangent w] of each (body, point) slot
// (contact_state at CS_IMPULSE_OFF).
constexpr int IMPULSE_PTS = 8;
struct ImpulseState {
    std::vector<SVec> ext;
    std::vector<double> imp;   // [nb][IMPULSE_PTS][3]: against the ground
    std::vector<double> pimp;  // [nb][IMPULSE_PTS][3]: against the body-attached plane
    void reset(int nb) {
        ext.assign(nb, SVec{});
        imp.assign((size_t)nb * IMPULSE_PTS * 3, 0.0);
        pimp.assign((size_t)nb * IMPULSE_PTS * 3, 0.0);
    }
};

inline void plane_contact(const Model& m, const Plane& pl, double friction, const double* k, const double* d,
                          const ImpulseParams* imp, const std::vector<Mat3>& wrot, const std::vector<Vec3>& wpos,
                          const std::vector<SVec>& vel, std::vector<SVec>& ext, double* pimp) {
    const int pb = pl.body, nb = m.nb();
    if (pb < 0) return;
    const double dt = m.dt, dtc = std::fmax(dt, 1e-9);
    const Mat3& Rp = wrot[pb];
    const Vec3 n_w = mul(Rp, v3(0, 0, 1));
    const Vec3 p0_w = wpos[pb] + mul(Rp, v3(0, 0, pl.offset));
    const Body& bp = m.bodies[pb];
    for (int i = 0; i < nb; i++) {
        const Body& b = m.bodies[i];
        if (i == pb || b.geom.type == 0 || pl.no_plane[i]) continue;
        const Mat3& Ri = wrot[i];
        const Vec3 n_body = tmul(Ri, n_w);
        const int npts = b.geom.type == 2 ? 8 : 1;
        const double pt_scale = b.geom.type == 2 ? 0.25 : 1.0;
        auto point = [&](int c) { return b.geom.type == 2 ? box_corner(b.geom, c) : support_point(b.geom, n_body); };
        // the shape's footprint in face coordinates, intersected with the face
        double lo_x = 1e30, lo_y = 1e30, hi_x = -1e30, hi_y = -1e30;
        for (int c = 0; c < npts; c++) {
            Vec3 rp = tmul(Rp, wpos[i] + mul(Ri, point(c)) - wpos[pb]);
            lo_x = std::fmin(lo_x, rp.x);
            lo_y = std::fmin(lo_y, rp.y);
            hi_x = std::fmax(hi_x, rp.x);
            hi_y = std::fmax(hi_y, rp.y);
        }
        const double ox0 = std::fmax(lo_x, -pl.half_x), oy0 = std::fmax(lo_y, -pl.half_y);
        const double ox1 = std::fmin(hi_x, pl.half_x), oy1 = std::fmin(hi_y, pl.half_y);
        if (ox0 > ox1 || oy0 > oy1) continue;
        int active = 1;
        if (imp) {
            int cnt = 0;
            for (int c = 0; c < npts; c++) {
                double dd = -dot(wpos[i] + mul(Ri, point(c)) - p0_w, n_w);
                if (dd > 0.0 && dd <= pl.max_depth) cnt++;
            }
            active = cnt > 1 ? cnt : 1;
        }
        for (int c = 0; c < npts; c++) {
            double* slot = pimp ? pimp + ((size_t)i * IMPULSE_PTS + c) * 3 : nullptr;
            const Vec3 sup = point(c);
            const Vec3 sw0 = wpos[i] + mul(Ri, sup);
            const double pen = -dot(sw0 - p0_w, n_w);
            if (pen <= 0.0 || pen > pl.max_depth) {
                if (slot) slot[0] = slot[1] = slot[2] = 0.0;
                continue;
            }
            // the contact point in the face, clamped into the overlap: one
            // world point, a lever on each body
            Vec3 r_p = tmul(Rp, sw0 - wpos[pb]);
            r_p.x = std::fmin(std::fmax(r_p.x, ox0), ox1);
            r_p.y = std::fmin(std::fmax(r_p.y, oy0), oy1);
            const Vec3 sw = wpos[pb] + mul(Rp, r_p);
            const Vec3 sc = tmul(Ri, sw - wpos[i]);
            const Vec3 v_rel = mul(Ri, vel[i].lin + cross(vel[i].ang, sc)) - mul(Rp, vel[pb].lin + cross(vel[pb].ang, r_p));
            const double vn = dot(v_rel, n_w);
            auto pair_mass = [&](Vec3 dir_w) {
                return 1.0 / (1.0 / contact_eff_mass(b, sc, tmul(Ri, dir_w)) +
                              1.0 / contact_eff_mass(bp, r_p, tmul(Rp, dir_w)));
            };
            const double m_n = pair_mass(n_w);
            Vec3 f_w;
            if (imp) {
                Vec3 pu, pw;
                contact_tangents(n_w, pu, pw);
                const double bu = dot(v_rel, pu), bw = dot(v_rel, pw);
                const double ann = active / std::fmax(m_n, 1e-9);
                const double bias = impedance_at(*imp, pen) * imp->erp * std::fmax(pen, 0.0) / dtc;
                const double e = effective_restitution(*imp, imp->restitution, std::fmin(vn, 0.0));
                const double fn = std::fmax((bias - (vn * (1.0 + e) - ann * slot[0])) / ann, 0.0);
                const double auu = active / std::fmax(pair_mass(pu), 1e-9);
                const double aww = active / std::fmax(pair_mass(pw), 1e-9);
                double ju = -(bu - auu * slot[1]) / auu, jw = -(bw - aww * slot[2]) / aww;
                const double lim = friction * fn, jt = std::sqrt(ju * ju + jw * jw);
                if (jt > lim) {
                    const double scl = jt > 0.0 ? lim / jt : 0.0;
                    ju *= scl;
                    jw *= scl;
                }
                slot[0] = fn;
                slot[1] = ju;
                slot[2] = jw;
                f_w = (n_w * fn + pu * ju + pw * jw) * (1.0 / dtc);
            } else {
                const double kb = std::fmin(pt_scale * k[i], max_stiffness(m_n, dt));
                const double db = std::fmin(pt_scale * d[i], max_damping(m_n, dt));
                const double fn = std::fmax(kb * pen - db * vn, 0.0);
                const Vec3 vt3 = v_rel - n_w * vn;
                const double vt = norm(vt3);
                f_w = n_w * fn;
                if (vt > 1e-6) {
                    const Vec3 td = vt3 * (1.0 / vt);
                    const double ft = std::fmin(friction * fn * std::fmin(1.0, vt / 1e-3), max_damping(pair_mass(td), dt) * vt);
                    f_w = f_w - td * ft;
                }
            }
            const Vec3 fi = tmul(Ri, f_w), fp = tmul(Rp, -f_w);
            ext[i].ang = ext[i].ang + cross(sc, fi);
            ext[i].lin = ext[i].lin + fi;
            ext[pb].ang = ext[pb].ang + cross(r_p, fp);
            ext[pb].lin = ext[pb].lin + fp;
        }
    }
}

// One contact sweep of one world: FK with the free velocity v + dt qdd, one
// staged Coulomb update per contact point, the new wrenches into st.ext and
// the contact state [touching, depth, point(3), force(3)] into cstate.
inline void impulse_contact(const Model& m, const ImpulseParams& cp, const double* q, const double* v,
                            const double* qdd, ImpulseState& st, double* cstate) {
    int nb = m.nb();
    const double dt = m.dt, idt = 1.0 / std::fmax(dt, 1e-9);
    std::vector<double> vf(m.nv);
    for (int k = 0; k < m.nv; k++) vf[k] = v[k] + dt * qdd[k];
    std::vector<Mat3> wrot(nb);
    std::vector<Vec3> wpos(nb);
    std::vector<SVec> vel(nb);
    for (int i = 0; i < nb; i++) {
        const Joint& jt = m.joints[i];
        SXform xj = jt.ndof() == 0 ? SXform{} : jt.joint_transform(q + m.q_off[i]);
        SXform xt = xj.compose(jt.parent_to_joint);
        SVec vj = jt.joint_velocity(vf.data() + m.v_off[i]);
        Mat3 tree_rt = transpose(xt.rot);
        int p = m.bodies[i].parent;
        if (p < 0) {
            wrot[i] = tree_rt;
            wpos[i] = xt.pos;
            vel[i] = vj;
        } else {
            wrot[i] = mul(wrot[p], tree_rt);
            wpos[i] = wpos[p] + mul(wrot[p], xt.pos);
            vel[i] = xt.apply_motion(vel[p]) + vj;
        }
    }
    st.ext.assign(nb, SVec{});
    for (int i = 0; i < nb; i++) {
        const Body& b = m.bodies[i];
        double* cs = cstate ? cstate + i * PHYZB_CONTACT_STRIDE : nullptr;
        if (cs)
            for (int k = 0; k < PHYZB_CONTACT_STRIDE; k++) cs[k] = 0.0;
        double* slots = st.imp.data() + (size_t)i * IMPULSE_PTS * 3;
        if (b.geom.type == 0) {
            for (int k = 0; k < IMPULSE_PTS * 3; k++) slots[k] = 0.0;
            continue;
        }
        Vec3 z_body = tmul(wrot[i], v3(0, 0, 1));
        int npts = b.geom.type == 2 ? 8 : 1;
        auto point = [&](int c) { return b.geom.type == 2 ? box_corner(b.geom, c) : support_point(b.geom, z_body); };
        // within-body load sharing: points inside the margin
        int n_active = 0;
        auto terrain = [&](const Vec3& w, Vec3& n) {
            if (cp.terrain.nx > 0) return cp.terrain.sample(w.x, w.y, n);
            n = v3(0, 0, 1);
            return cp.ground_height;
        };
        for (int c = 0; c < npts; c++) {
            Vec3 sw = wpos[i] + mul(wrot[i], point(c));
            Vec3 tn;
            double th = terrain(sw, tn);
            if (tn.z * (th - sw.z) > -cp.margin) n_active++;
        }
        if (n_active < 1) n_active = 1;
        Vec3 f_w_total{};
        double deepest = 0;
        Vec3 deepest_w{};
        bool any = false;
        for (int c = 0; c < npts; c++) {
            double* f_c = slots + 3 * c;
            Vec3 sup = point(c);
            Vec3 sup_w = wpos[i] + mul(wrot[i], sup);
            Vec3 n_w;
            double terr_h = terrain(sup_w, n_w);
            double pen = n_w.z * (terr_h - sup_w.z);
            if (!(pen > -cp.margin)) {
                f_c[0] = f_c[1] = f_c[2] = 0.0;
                continue;
            }
            Vec3 n_body = tmul(wrot[i], n_w);
            Vec3 v_point = vel[i].lin + cross(vel[i].ang, sup);
            Vec3 t_u, t_w;
            contact_tangents(n_body, t_u, t_w);
            double b_n = dot(v_point, n_body), b_u = dot(v_point, t_u), b_w = dot(v_point, t_w);
            double m_n = contact_eff_mass(b, sup, n_body) / n_active;
            double a_nn = 1.0 / std::fmax(m_n, 1e-9);
            double bias = impedance_at(cp, pen) * cp.erp * std::fmax(pen, 0.0) / std::fmax(dt, 1e-9);
            double e = effective_restitution(cp, cp.restitution, std::fmin(b_n, 0.0));
            double r_n = b_n * (1.0 + e) - a_nn * f_c[0];
            double fn = std::fmax((bias - r_n) / a_nn, 0.0);
            double a_uu = n_active / std::fmax(contact_eff_mass(b, sup, t_u), 1e-9);
            double a_ww = n_active / std::fmax(contact_eff_mass(b, sup, t_w), 1e-9);
            double tu = -(b_u - a_uu * f_c[1]) / a_uu;
            double tw = -(b_w - a_ww * f_c[2]) / a_ww;
            double limit = cp.friction * fn;
            double tn = std::sqrt(tu * tu + tw * tw);
            if (tn > limit) {
                double sc = tn > 0.0 ? limit / tn : 0.0;
                tu *= sc;
                tw *= sc;
            }
            f_c[0] = fn;
            f_c[1] = tu;
            f_c[2] = tw;
            Vec3 f_body = (n_body * fn + t_u * tu + t_w * tw) * idt;
            st.ext[i].ang = st.ext[i].ang + cross(sup, f_body);
            st.ext[i].lin = st.ext[i].lin + f_body;
            f_w_total = f_w_total + mul(wrot[i], f_body);
            any = true;
            if (pen > deepest) {
                deepest = pen;
                deepest_w = sup_w;
            }
        }
        if (!any) {
            // the reference clears the body's whole contact-state row here
            // (phyz_kernels.cu:966-969), its plane impulses included: a body
            // off the ground starts every sweep's plane update from zero
            for (int k = 0; k < IMPULSE_PTS * 3; k++) slots[k] = 0.0;
            double* ps = st.pimp.data() + (size_t)i * IMPULSE_PTS * 3;
            for (int k = 0; k < IMPULSE_PTS * 3; k++) ps[k] = 0.0;
            continue;
        }
        if (!cs) continue;
        cs[0] = 1.0;
        cs[1] = deepest;
        cs[2] = deepest_w.x;
        cs[3] = deepest_w.y;
        cs[4] = deepest_w.z;
        cs[5] = f_w_total.x;
        cs[6] = f_w_total.y;
        cs[7] = f_w_total.z;
    }
    plane_contact(m, cp.plane, cp.friction, nullptr, nullptr, &cp, wrot, wpos, vel, st.ext, st.pimp.data());
}

// One step of the batched path for one world: [PD ->] [contact ->] ABA ->
// semi-implicit Euler (cuda/mod.rs:879-945 order), qdd written out.
struct PdEntry {
    int qi, vi;
    double kp, kd, maxf;
};
inline void step_world(const Model& m, const ContactParams* cp, const std::vector<PdEntry>* pd,
                       const double* targets, double* q, double* v, double* ctrl, double* qdd_out,
                       double* cstate) {
    if (pd) {  // phyz_kernels.cu:464-483
        for (size_t d = 0; d < pd->size(); d++) {
            const PdEntry& e = (*pd)[d];
            double tau = e.kp * (targets[d] - q[e.qi]) - e.kd * v[e.vi];
            ctrl[e.vi] = std::fmin(std::fmax(tau, -e.maxf), e.maxf);
        }
    }
    std::vector<SVec> ext;
    if (cp) penalty_contact(m, *cp, q, v, ext, cstate);
    std::vector<double> qdd = aba(m, q, v, ctrl, cp ? ext.data() : nullptr);
    semi_implicit_euler(m, q, v, qdd.data(), m.dt);
    if (qdd_out)
        for (int i = 0; i < m.nv; i++) qdd_out[i] = qdd[i];
}


// One impulse-mode step of one world (cuda/mod.rs:879-945): [PD ->] ABA
// with the wrenches of the previous step's last sweep, `sweeps` x [contact
// at the free velocity v + dt qdd -> ABA], then semi-implicit Euler.
inline void step_world_impulse(const Model& m, const ImpulseParams& cp, const std::vector<PdEntry>* pd,
                               const double* targets, double* q, double* v, double* ctrl, double* qdd_out,
                               double* cstate, ImpulseState& st) {
    if (pd) {
        for (size_t d = 0; d < pd->size(); d++) {
            const PdEntry& e = (*pd)[d];
            double tau = e.kp * (targets[d] - q[e.qi]) - e.kd * v[e.vi];
            ctrl[e.vi] = std::fmin(std::fmax(tau, -e.maxf), e.maxf);
        }
    }
    std::vector<double> qdd = aba(m, q, v, ctrl, st.ext.data());
    for (int s = 0; s < cp.sweeps; s++) {
        impulse_contact(m, cp, q, v, qdd.data(), st, cstate);
        qdd = aba(m, q, v, ctrl, st.ext.data());
    }
    semi_implicit_euler(m, q, v, qdd.data(), m.dt);
    if (qdd_out)
        for (int i = 0; i < m.nv; i++) qdd_out[i] = qdd[i];
}
}  // namespace phyz_oracle
