// One world's fused multi-step rollout: Featherstone's articulated-body
// algorithm with penalty ground contact and the semi-implicit integrator,
// written once for the device kernel and for the host flop counter.
//
// Semantics follow phyz's CPU referee (crates/phyz-rigid/src/aba.rs:147-420,
// integrate.rs:41-91, actuation.rs:18-54, joint.rs:232-316) and the step
// order of phyz-gpu's batched path (cuda/mod.rs:879-945: PD -> contact ->
// ABA -> integrate; contact law phyz_kernels.cu:804-965). The formulation is
// this kernel's own:
//
//   * a step is two sweeps over the bodies instead of the reference's four
//     launches: a backward sweep (ABA pass 2) and a forward sweep that
//     finishes the step (pass 3 + integration) and immediately starts the
//     next one (pass 1 + FK + contact of the new state), so q, v and every
//     per-body intermediate stay on chip for the whole rollout;
//   * articulated inertias are 21-number block forms and transforms are
//     rotate-then-translate (pz_types.cuh); the 1-DOF path is scalar; a hinge
//     about a coordinate axis rotates with a planar formula;
//   * a serial chain passes its recursion state in registers ("carry"); only
//     bodies with a child that is not the next body ("branch" bodies) keep
//     accumulators in scratch.
//
// Per-world scratch is accessed through `Scr`: S(slot) is this world's
// element of a slot, S.prefetch(slot, src) an asynchronous copy of one
// control input into a slot, S.wait() the fence before reading them.
#pragma once

#include "pz_model.cuh"
#include "pz_types.cuh"

// Loops over the bodies (and DOFs) of the model: fully unrolled in a
// model-specialized build, where the table they index is literal.
#ifdef PZ_SPEC
#define PZ_UNROLL_BODIES _Pragma("unroll")
#ifndef PZ_SPEC_INLINE_CONTACT
#define PZ_SPEC_INLINE_CONTACT 1
#endif
#else
#define PZ_UNROLL_BODIES
#endif

namespace pz {

// Compile-time feature mask of a kernel variant: a model without ball/free
// joints (resp. without contact) gets a kernel without that code at all.
// Kernel feature bits: ball/free joints present, ground contact on, some
// hinge frame relabelled by a non-identity cyclic permutation, and (with
// FEAT_PERM) every relabelled hinge relabelled by the same shift 1 -- a chain
// whose axes cycle x, y, z -- so the relabel is a compile-time register
// renaming instead of a run-time branch; and (with FEAT_CONTACT) contact as
// the velocity-level impulse solve instead of the penalty law, and with full
// world frames carried (FEAT_TERRAIN): a heightfield in place of the flat
// ground and/or a body-attached contact plane.
enum Features {
    FEAT_MULTI = 1,
    FEAT_CONTACT = 2,
    FEAT_PERM = 4,
    FEAT_PERM1 = 8,
    FEAT_IMPULSE = 16,
    FEAT_TERRAIN = 32,
    FEAT_LANES = 64  // the world split over lanes (stepper_lanes.cuh): controls through a DOF map
};

// ── quaternions (w, x, y, z), crates/phyz-math/src/lib.rs:43-72 ───────────
template <class T>
struct Q4 {
    T w, x, y, z;
};
template <class T>
PZ_HD Q4<T> qexp(const V3<T>& om) {
    const T ang = pz_sqrt(dot(om, om));
    Q4<T> q;
    if (ang < T(Eps<T>::quat)) {
        q.w = T(1);
        q.x = om.x * T(0.5);
        q.y = om.y * T(0.5);
        q.z = om.z * T(0.5);
        return q;
    }
    T s, c;
    pz_sincos(ang * T(0.5), &s, &c);
    const T k = s / ang;
    q.w = c;
    q.x = om.x * k;
    q.y = om.y * k;
    q.z = om.z * k;
    return q;
}
template <class T>
PZ_HD V3<T> qlog(const Q4<T>& q) {
    const V3<T> v = mk3<T>(q.x, q.y, q.z);
    const T n = pz_sqrt(dot(v, v));
    if (n < T(Eps<T>::quat)) return v * T(2);
    const T ang = T(2) * pz_atan2(n, q.w);
    return v * (ang / n);
}
template <class T>
PZ_HD Q4<T> qmul(const Q4<T>& a, const Q4<T>& b) {
    Q4<T> r;
    r.w = a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z;
    r.x = a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y;
    r.y = a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x;
    r.z = a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w;
    return r;
}
template <class T>
PZ_HD Q4<T> qnormalize(const Q4<T>& q) {
    const T n = pz_sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    const T inv = T(1) / n;
    Q4<T> r;
    r.w = q.w * inv;
    r.x = q.x * inv;
    r.y = q.y * inv;
    r.z = q.z * inv;
    return r;
}
template <class T>
PZ_HD V3<T> qrotate(const Q4<T>& q, const V3<T>& p) {
    const V3<T> u = mk3<T>(q.x, q.y, q.z);
    const V3<T> t = cross(u, p) * T(2);
    return p + t * q.w + cross(u, t);
}
// Joint rotation of a ball / free joint: (to_matrix(exp(w)))^T, joint.rs:276-306.
template <class T>
PZ_HD R3<T> qjoint_rot(const Q4<T>& q) {
    const T w = q.w, x = q.x, y = q.y, z = q.z;
    R3<T> E;  // transpose of the rotation matrix of q
    E.m[0] = T(1) - T(2) * (y * y + z * z);
    E.m[3] = T(2) * (x * y - w * z);
    E.m[6] = T(2) * (x * z + w * y);
    E.m[1] = T(2) * (x * y + w * z);
    E.m[4] = T(1) - T(2) * (x * x + z * z);
    E.m[7] = T(2) * (y * z - w * x);
    E.m[2] = T(2) * (x * z - w * y);
    E.m[5] = T(2) * (y * z + w * x);
    E.m[8] = T(1) - T(2) * (x * x + y * y);
    return E;
}

// Hinge rotation about a general axis a: I + s K + (1 - c) K^2, K = a^x
// (joint.rs:259-266; equal to phyz_kernels.cu:245-256 for a unit axis).
template <class T>
PZ_HD R3<T> hinge_matrix(const V3<T>& a, const T& c, const T& s) {
    const T t = T(1) - c;
    const T aa = dot(a, a);
    R3<T> E;
    E.m[0] = T(1) + t * (a.x * a.x - aa);
    E.m[1] = t * (a.x * a.y) - s * a.z;
    E.m[2] = t * (a.x * a.z) + s * a.y;
    E.m[3] = t * (a.x * a.y) + s * a.z;
    E.m[4] = T(1) + t * (a.y * a.y - aa);
    E.m[5] = t * (a.y * a.z) - s * a.x;
    E.m[6] = t * (a.x * a.z) - s * a.y;
    E.m[7] = t * (a.y * a.z) + s * a.x;
    E.m[8] = T(1) + t * (a.z * a.z - aa);
    return E;
}

template <class T>
PZ_HD V3<T> ld3(const T* p) {
    return mk3<T>(p[0], p[1], p[2]);
}
template <class T>
PZ_HD R3<T> ld9(const T* p) {
    R3<T> E;
#pragma unroll
    for (int k = 0; k < 9; k++) E.m[k] = p[k];
    return E;
}

// ── joint transform of one body, decoded from scratch ─────────────────────
template <class T>
struct JX {
    T c, s;   // hinge: cos, sin of -q
    R3<T> E;  // rotation (ball, free, general-axis hinge)
    V3<T> r;  // translation (prismatic, free)
};

// Body kinds. AX = 2: a hinge about z of its relabelled frame (F_ZHINGE):
// its transform is the joint offset, the cyclic relabelling qshift and a
// planar rotation about z, with the rotation known at compile time. AX = -1:
// any joint, decoded at run time.
PZ_HD int body_kind(const BodyI& bi) { return (bi.flags & F_ZHINGE) ? 2 : -1; }

// Cyclic relabelling Q = P_q of the parent's coordinates into the child's:
// (Q v)_a = v_(a+q mod 3), and Q^T = P_(3-q). q is the same for every world
// (a model constant), so the branches below never diverge.
template <int Q, class T>
PZ_HD V3<T> cperm(const V3<T>& v) {
    if constexpr (Q == 1)
        return mk3<T>(v.y, v.z, v.x);
    else if constexpr (Q == 2)
        return mk3<T>(v.z, v.x, v.y);
    else
        return v;
}
// E^T B E with E = P_Q on each 3x3 block: B'_bd = B_(b-Q)(d-Q)
template <int Q, class T>
PZ_HD void ai_cperm_fixed(AI<T>& I) {
    constexpr int m = (3 - Q) % 3;
    AI<T> o;
#pragma unroll
    for (int b = 0; b < 3; b++)
#pragma unroll
        for (int d = 0; d < 3; d++) {
            o.h[b * 3 + d] = I.h[((b + m) % 3) * 3 + (d + m) % 3];
            if (b <= d) {
                o.a[sidx(b, d)] = I.a[sidx((b + m) % 3, (d + m) % 3)];
                o.m[sidx(b, d)] = I.m[sidx((b + m) % 3, (d + m) % 3)];
            }
        }
    I = o;
}

// The relabelling folded into the planar rotation about e_AX that follows
// (motion: R Q m) or precedes (force: Q^T R^T f; inertia: Q^T R^T I R Q) it:
// one branch per shift, so each branch writes the rotated values straight
// into the permuted slots instead of moving registers after the fact.
template <int AX, int FEAT, class T>
PZ_HD V3<T> rot_fwd3(int q, const T& c, const T& s, const V3<T>& x) {
    if constexpr ((FEAT & FEAT_PERM1) != 0) return prot<AX>(c, s, cperm<1>(x));
    if constexpr ((FEAT & FEAT_PERM) != 0) {
        if (q == 1) return prot<AX>(c, s, cperm<1>(x));
        if (q == 2) return prot<AX>(c, s, cperm<2>(x));
    }
    return prot<AX>(c, s, x);
}
template <int AX, int FEAT, class T>
PZ_HD SV<T> rot_fwd(int q, const T& c, const T& s, const SV<T>& m) {
    if constexpr ((FEAT & FEAT_PERM1) != 0)
        return mksv<T>(prot<AX>(c, s, cperm<1>(m.w)), prot<AX>(c, s, cperm<1>(m.l)));
    if constexpr ((FEAT & FEAT_PERM) != 0) {
        if (q == 1) return mksv<T>(prot<AX>(c, s, cperm<1>(m.w)), prot<AX>(c, s, cperm<1>(m.l)));
        if (q == 2) return mksv<T>(prot<AX>(c, s, cperm<2>(m.w)), prot<AX>(c, s, cperm<2>(m.l)));
    }
    return mksv<T>(prot<AX>(c, s, m.w), prot<AX>(c, s, m.l));
}
template <int AX, int FEAT, class T>
PZ_HD SV<T> rot_bwd(int q, const T& c, const T& s, const SV<T>& f) {
    if constexpr ((FEAT & FEAT_PERM1) != 0)
        return mksv<T>(cperm<2>(prot_t<AX>(c, s, f.w)), cperm<2>(prot_t<AX>(c, s, f.l)));
    if constexpr ((FEAT & FEAT_PERM) != 0) {
        if (q == 1) return mksv<T>(cperm<2>(prot_t<AX>(c, s, f.w)), cperm<2>(prot_t<AX>(c, s, f.l)));
        if (q == 2) return mksv<T>(cperm<1>(prot_t<AX>(c, s, f.w)), cperm<1>(prot_t<AX>(c, s, f.l)));
    }
    return mksv<T>(prot_t<AX>(c, s, f.w), prot_t<AX>(c, s, f.l));
}
template <int AX, int FEAT, class T>
PZ_HD void ai_rot_bwd(int q, const T& c, const T& s, AI<T>& I) {
    if constexpr ((FEAT & FEAT_PERM1) != 0) {
        ai_prot<AX>(c, s, I);
        ai_cperm_fixed<1>(I);
        return;
    }
    if constexpr ((FEAT & FEAT_PERM) != 0) {
        if (q == 1) {
            ai_prot<AX>(c, s, I);
            ai_cperm_fixed<1>(I);
            return;
        }
        if (q == 2) {
            ai_prot<AX>(c, s, I);
            ai_cperm_fixed<2>(I);
            return;
        }
    }
    ai_prot<AX>(c, s, I);
}

// a x (s e_K), with the structurally zero component exact
template <int K, class T>
PZ_HD V3<T> cross_axis(const V3<T>& a, const T& s) {
    if (K == 0) return mk3<T>(T(0), a.z * s, -(a.y * s));
    if (K == 1) return mk3<T>(-(a.z * s), T(0), a.x * s);
    return mk3<T>(a.y * s, -(a.x * s), T(0));
}

// Per-step record of a hinge body: joint cos/sin and the body velocity
// (pass 1 -> pass 2) or W = U/D (pass 2 -> pass 3). The scratch policy
// decides where it lives (shared-memory slots s_xj/s_vw, or Tensor Memory
// columns t_rec).
template <class T>
struct Rec {
    T c, s;
    SV<T> v;
};

template <int AX, int FEAT, class T, class Scr>
PZ_HD JX<T> load_jx(const BodyI& bi, const BodyT<T>& bt, const Scr& S) {
    JX<T> j;
    if constexpr (AX >= 0) {
        j.c = S(bi.s_xj);
        j.s = S(bi.s_xj + 1);
        return j;
    }
    switch (bi.jtype) {
        case J_REVOLUTE:
            j.c = S(bi.s_xj);
            j.s = S(bi.s_xj + 1);
            if (bi.axis_k < 0) j.E = hinge_matrix(ld3(bt.axis), j.c, j.s);
            break;
        case J_PRISMATIC: j.r = ld3(bt.axis) * S(bi.off); break;
        case J_BALL:
            if constexpr ((FEAT & FEAT_MULTI) != 0) {
#pragma unroll
                for (int k = 0; k < 9; k++) j.E.m[k] = S(bi.s_xj + k);
            }
            break;
        case J_FREE:
            if constexpr ((FEAT & FEAT_MULTI) != 0) {
#pragma unroll
                for (int k = 0; k < 9; k++) j.E.m[k] = S(bi.s_xj + k);
                j.r = mk3<T>(S(bi.off + 3), S(bi.off + 4), S(bi.off + 5));
            }
            break;
        default: break;
    }
    return j;
}

// Compute the joint transform data of body i from q and store it.
template <int AX, int FEAT, class T, class Scr>
PZ_HD JX<T> make_jx(const BodyI& bi, const BodyT<T>& bt, const Scr& S) {
    JX<T> j;
    if (AX >= 0 || bi.jtype == J_REVOLUTE) {
        T s, c;
        pz_sincos(-S(bi.off), &s, &c);
        j.c = c;
        j.s = s;
        S(bi.s_xj) = c;
        S(bi.s_xj + 1) = s;
        if constexpr (AX < 0) {
            if (bi.axis_k < 0) j.E = hinge_matrix(ld3(bt.axis), c, s);
        }
        return j;
    }
    if constexpr (AX < 0) {
        switch (bi.jtype) {
            case J_PRISMATIC: j.r = ld3(bt.axis) * S(bi.off); break;
            case J_BALL:
            case J_FREE:
                if constexpr ((FEAT & FEAT_MULTI) != 0) {
                    const Q4<T> q = qexp(mk3<T>(S(bi.off), S(bi.off + 1), S(bi.off + 2)));
                    j.E = qjoint_rot(q);
#pragma unroll
                    for (int k = 0; k < 9; k++) S(bi.s_xj + k) = j.E.m[k];
                    if (bi.jtype == J_FREE) j.r = mk3<T>(S(bi.off + 3), S(bi.off + 4), S(bi.off + 5));
                }
                break;
            default: break;
        }
    }
    return j;
}

// Planar hinge rotation with a runtime axis index (generic path only).
template <class T>
PZ_HD V3<T> hrot(int k, const T& c, const T& s, const V3<T>& x) {
    return k == 0 ? prot<0>(c, s, x) : (k == 1 ? prot<1>(c, s, x) : prot<2>(c, s, x));
}
template <class T>
PZ_HD V3<T> hrot_t(int k, const T& c, const T& s, const V3<T>& x) {
    return k == 0 ? prot_t<0>(c, s, x) : (k == 1 ? prot_t<1>(c, s, x) : prot_t<2>(c, s, x));
}

// The rotation part of X_tree = X_J X_ptj applied to a 3-vector: R_J R_ptj x.
template <int AX, int FEAT, class T>
PZ_HD V3<T> tree_rot(const BodyI& bi, const BodyT<T>& bt, const JX<T>& j, V3<T> x) {
    if constexpr (AX >= 0) return rot_fwd3<AX, FEAT>(bi.qshift, j.c, j.s, x);
    if (bi.flags & F_PTJ_ROT) x = m3v(bt.ptj_rot, x);
    switch (bi.jtype) {
        case J_REVOLUTE: x = bi.axis_k >= 0 ? hrot(bi.axis_k, j.c, j.s, x) : rmul(j.E, x); break;
        case J_BALL:
        case J_FREE:
            if constexpr ((FEAT & FEAT_MULTI) != 0) x = rmul(j.E, x);
            break;
        default: break;
    }
    return x;
}
// Origin of the body in its parent: p_ptj + R_ptj^T p_J (tang compose).
template <int AX, int FEAT, class T>
PZ_HD V3<T> tree_pos(const BodyI& bi, const BodyT<T>& bt, const JX<T>& j) {
    V3<T> p = ld3(bt.ptj_pos);
    if constexpr (AX < 0) {
        if (bi.jtype == J_PRISMATIC || bi.jtype == J_FREE)
            p = p + ((bi.flags & F_PTJ_ROT) ? m3tv(bt.ptj_rot, j.r) : j.r);
    }
    return p;
}

// X_tree m for a motion vector (X_ptj first, then X_J).
template <int AX, int FEAT, class T>
PZ_HD SV<T> mot_X(const BodyI& bi, const BodyT<T>& bt, const JX<T>& j, SV<T> m) {
    // (relabelled hinges translate unconditionally: a zero offset is exact and
    // cheaper than the branch)
    if ((AX >= 0 && !Counting<T>::value) || (bi.flags & F_PTJ_POS)) m = kxm_apply_trans(ld3(bt.ptj_pos), m);
    if constexpr (AX >= 0) {
        return rot_fwd<AX, FEAT>(bi.qshift, j.c, j.s, m);
    } else {
        if (bi.flags & F_PTJ_ROT) {
            const R3<T> P = ld9(bt.ptj_rot);
            m = xm_apply_rot(P, m);
        }
        switch (bi.jtype) {
            case J_REVOLUTE:
                if (bi.axis_k >= 0)
                    m = mksv<T>(hrot(bi.axis_k, j.c, j.s, m.w), hrot(bi.axis_k, j.c, j.s, m.l));
                else
                    m = xm_apply_rot(j.E, m);
                break;
            case J_PRISMATIC: m = xm_apply_trans(j.r, m); break;
            case J_BALL:
                if constexpr ((FEAT & FEAT_MULTI) != 0) m = xm_apply_rot(j.E, m);
                break;
            case J_FREE:
                if constexpr ((FEAT & FEAT_MULTI) != 0) m = xm_apply_rot(j.E, xm_apply_trans(j.r, m));
                break;
            default: break;
        }
        return m;
    }
}

// X_tree^T f for a force vector (phyz's inv_apply_force).
template <int AX, int FEAT, class T>
PZ_HD SV<T> frc_XT(const BodyI& bi, const BodyT<T>& bt, const JX<T>& j, SV<T> f) {
    if constexpr (AX >= 0) {
        f = rot_bwd<AX, FEAT>(bi.qshift, j.c, j.s, f);
    } else {
        switch (bi.jtype) {
            case J_REVOLUTE:
                if (bi.axis_k >= 0)
                    f = mksv<T>(hrot_t(bi.axis_k, j.c, j.s, f.w), hrot_t(bi.axis_k, j.c, j.s, f.l));
                else
                    f = xf_tapply_rot(j.E, f);
                break;
            case J_PRISMATIC: f = xf_tapply_trans(j.r, f); break;
            case J_BALL:
                if constexpr ((FEAT & FEAT_MULTI) != 0) f = xf_tapply_rot(j.E, f);
                break;
            case J_FREE:
                if constexpr ((FEAT & FEAT_MULTI) != 0) f = xf_tapply_trans(j.r, xf_tapply_rot(j.E, f));
                break;
            default: break;
        }
        if (bi.flags & F_PTJ_ROT) {
            const R3<T> P = ld9(bt.ptj_rot);
            f = xf_tapply_rot(P, f);
        }
    }
    if ((AX >= 0 && !Counting<T>::value) || (bi.flags & F_PTJ_POS)) f = kxf_tapply_trans(ld3(bt.ptj_pos), f);
    return f;
}

// X_tree^T I X_tree in place (J part first, then ptj).
template <int AX, int FEAT, class T>
PZ_HD void ai_XtIX(const BodyI& bi, const BodyT<T>& bt, const JX<T>& j, AI<T>& I) {
    if constexpr (AX >= 0) {
        ai_rot_bwd<AX, FEAT>(bi.qshift, j.c, j.s, I);
    } else {
        switch (bi.jtype) {
            case J_REVOLUTE:
                if (bi.axis_k == 0)
                    ai_prot<0>(j.c, j.s, I);
                else if (bi.axis_k == 1)
                    ai_prot<1>(j.c, j.s, I);
                else if (bi.axis_k == 2)
                    ai_prot<2>(j.c, j.s, I);
                else
                    ai_rot(j.E, I);
                break;
            case J_PRISMATIC: ai_trans(j.r, I); break;
            case J_BALL:
                if constexpr ((FEAT & FEAT_MULTI) != 0) ai_rot(j.E, I);
                break;
            case J_FREE:
                if constexpr ((FEAT & FEAT_MULTI) != 0) {
                    ai_rot(j.E, I);
                    ai_trans(j.r, I);
                }
                break;
            default: break;
        }
        if (bi.flags & F_PTJ_ROT) {
            const R3<T> P = ld9(bt.ptj_rot);
            ai_rot(P, I);
        }
    }
    if ((AX >= 0 && !Counting<T>::value) || (bi.flags & F_PTJ_POS)) kai_trans(ld3(bt.ptj_pos), I);
}

// S qd of body i (aba.rs:15-30).
template <int AX, int FEAT, class T, class Scr>
PZ_HD SV<T> joint_vel(const BodyI& bi, const BodyT<T>& bt, const Scr& S, int nv) {
    const int o = nv + bi.off;
    if constexpr (AX >= 0) {
        V3<T> w = zero3<T>();
        at<AX>(w) = S(o);
        return mksv<T>(w, zero3<T>());
    }
    switch (bi.jtype) {
        case J_REVOLUTE: return mksv<T>(ld3(bt.axis) * S(o), zero3<T>());
        case J_PRISMATIC: return mksv<T>(zero3<T>(), ld3(bt.axis) * S(o));
        case J_BALL:
            if constexpr ((FEAT & FEAT_MULTI) != 0) return mksv<T>(mk3<T>(S(o), S(o + 1), S(o + 2)), zero3<T>());
            return zerosv<T>();
        case J_FREE:
            if constexpr ((FEAT & FEAT_MULTI) != 0)
                return mksv<T>(mk3<T>(S(o), S(o + 1), S(o + 2)), mk3<T>(S(o + 3), S(o + 4), S(o + 5)));
            return zerosv<T>();
        default: return zerosv<T>();
    }
}

template <class T, class Scr>
PZ_HD SV<T> ld_sv(const Scr& S, int s) {
    return mksv<T>(mk3<T>(S(s), S(s + 1), S(s + 2)), mk3<T>(S(s + 3), S(s + 4), S(s + 5)));
}
// Velocity (or W) of any body, wherever its record lives.
template <class T, class Scr>
PZ_HD SV<T> ld_vel(const Scr& S, const BodyI& bi) {
    if (bi.t_rec >= 0) return S.rec_get(bi).v;
    return ld_sv<T>(S, bi.s_vw);
}

template <class T, class Scr>
PZ_HD void st_sv(const Scr& S, int s, const SV<T>& v) {
    S(s) = v.w.x;
    S(s + 1) = v.w.y;
    S(s + 2) = v.w.z;
    S(s + 3) = v.l.x;
    S(s + 4) = v.l.y;
    S(s + 5) = v.l.z;
}

// Generalized input force on DOF d: the control (or the PD servo output,
// phyz_kernels.cu:464-483) plus the passive terms of joint.rs:232-247.
// SEP: the control input has slots of its own (impulse mode), else it
// shares the w0 slots (a compile-time choice: no extra table read).
template <bool SEP, class T, class Scr>
PZ_HD T dof_force(const ModelView<T>& M, const BodyI& bi, const BodyT<T>& bt, const Scr& S, int k, bool one_dof) {
    const int d = bi.off + k;
    const T qd = S(M.nv + d);
    T in = S((SEP ? bi.s_in : bi.s_w0) + k);
    if (bi.flags & F_PD) {
        const int pdi = M.pd_of_dof[d];
        if (pdi >= 0) {
            const PdT<T>& e = M.pd[pdi];
            const T tau = e.kp * (in - S(e.qi)) - e.kd * S(M.nv + e.vi);
            in = pz_min(pz_max(tau, -e.maxf), e.maxf);
        }
    }
    T f = in - bt.damping * qd;
    if (one_dof) {
        const T q = S(d);
        // the spring term is exact with stiffness 0, and cheaper than a branch
        if (!Counting<T>::value || (bi.flags & F_SPRING)) f = f - bt.stiffness * (q - bt.spring_ref);
        if (bi.flags & (F_LIMITS | F_FRICTION)) {
            if (bi.flags & F_LIMITS) {
                T depth = T(0), sign = T(0);
                if (q < bt.lim_lo) {
                    depth = bt.lim_lo - q;
                    sign = T(1);
                } else if (q > bt.lim_hi) {
                    depth = q - bt.lim_hi;
                    sign = T(-1);
                }
                const T inward = pz_max(-sign * qd, T(0));
                f = f + sign * (bt.lim_k * depth + bt.lim_d * inward);
            }
            if (bi.flags & F_FRICTION) f = f - bt.fric * pz_tanh(qd / T(1e-3));
        }
    }
    return f;
}

// U = I s for s = e_K in the angular (HINGE) or linear part, and s.U.
template <int K, bool HINGE, class T>
PZ_HD void unit_u(const AI<T>& I, V3<T>& Uw, V3<T>& Ul, T& sU) {
    if (HINGE) {
        Uw = mk3<T>(I.a[sidx(0, K)], I.a[sidx(1, K)], I.a[sidx(2, K)]);
        Ul = mk3<T>(I.h[K * 3 + 0], I.h[K * 3 + 1], I.h[K * 3 + 2]);
        sU = at<K>(Uw);
    } else {
        Uw = mk3<T>(I.h[0 * 3 + K], I.h[1 * 3 + K], I.h[2 * 3 + K]);
        Ul = mk3<T>(I.m[sidx(0, K)], I.m[sidx(1, K)], I.m[sidx(2, K)]);
        sU = at<K>(Ul);
    }
}

// Dense element (r, c) of an articulated inertia.
template <class T>
PZ_HD T ai_el(const AI<T>& I, int r, int c) {
    if (r < 3) return c < 3 ? I.a[sidx(r, c)] : I.h[r * 3 + (c - 3)];
    return c < 3 ? I.h[c * 3 + (r - 3)] : I.m[sidx(r - 3, c - 3)];
}
template <class T>
PZ_HD void ai_sub_el(AI<T>& I, int r, int c, const T& v) {  // only r <= c for symmetric blocks
    if (r < 3) {
        if (c < 3)
            I.a[sidx(r, c)] = I.a[sidx(r, c)] - v;
        else
            I.h[r * 3 + (c - 3)] = I.h[r * 3 + (c - 3)] - v;
    } else {
        I.m[sidx(r - 3, c - 3)] = I.m[sidx(r - 3, c - 3)] - v;
    }
}

// Multi-DOF joint (ball: S = [1;0], free: S = 1, both unit columns e_0..e_{ND-1}):
// U = I S, D = S^T U + d_extra, W = U D^-1, w0 = D^-1 u, stored; when the
// body has a parent, I <- I - W U^T and p <- p + I c + U w0. Returns false
// when D is singular (aba.rs:291-294: the body is skipped).
// A root body (F_ROOTQDD, ag = its parent's acceleration -g in its own
// frame) instead gets w0 = D^-1 (u - U^T ag), its qdd: the step's
// accelerations start from the root as qdd = w0 - W^T a with a = ag (the
// root's bias c = v x S qd vanishes, its v being S qd), and D^-1 U^T =
// W^T, so W is neither solved for nor stored.
template <int ND, bool SEP, class T, class Scr>
PZ_HD bool multi_dof(const ModelView<T>& M, const BodyI& bi, const BodyT<T>& bt, const Scr& S,
                     AI<T>& I, SV<T>& p, const SV<T>& c, bool has_parent, const SV<T>* ag = nullptr) {
    T U[6][ND];
#pragma unroll
    for (int r = 0; r < 6; r++)
#pragma unroll
        for (int k = 0; k < ND; k++) U[r][k] = ai_el(I, r, k);
    // Cholesky of D = U[0..ND) + d_extra 1; the substitutions multiply by
    // the reciprocal diagonal (one division per row instead of one per use)
    T L[ND][ND], Linv[ND];
#pragma unroll
    for (int a = 0; a < ND; a++)
#pragma unroll
        for (int b = 0; b < ND; b++) L[a][b] = T(0);
    T u[ND];
#pragma unroll
    for (int k = 0; k < ND; k++) u[k] = dof_force<SEP>(M, bi, bt, S, k, false) - svget(p, k);
    bool ok = true;
#pragma unroll
    for (int a = 0; a < ND; a++) {
        T d = U[a][a] + bt.d_extra;
#pragma unroll
        for (int k = 0; k < a; k++) d = d - L[a][k] * L[a][k];
        if (!(d > T(0))) {
            ok = false;
            d = T(1);
        }
        const T ld = pz_sqrt(d);
        L[a][a] = ld;
        const T inv = T(1) / ld;
        Linv[a] = inv;
#pragma unroll
        for (int b = a + 1; b < ND; b++) {
            T e = U[b][a];
#pragma unroll
            for (int k = 0; k < a; k++) e = e - L[b][k] * L[a][k];
            L[b][a] = e * inv;
        }
    }
    if (bi.s_dinv >= 0) {  // impulse mode: the factor the sweeps' wrench response solves with
#pragma unroll
        for (int a = 0; a < ND; a++)
#pragma unroll
            for (int b = 0; b <= a; b++)
                S(bi.s_dinv + a * (a + 1) / 2 + b) = ok ? (b == a ? Linv[a] : L[a][b]) : T(0);
    }
    if (!ok) {
#pragma unroll
        for (int k = 0; k < 6 * ND; k++) S(bi.s_vw + k) = T(0);
#pragma unroll
        for (int k = 0; k < ND; k++) S(bi.s_w0 + k) = T(0);
        return false;
    }
    // Solve D X = B for a right-hand side (forward, then backward substitution).
    auto solve = [&](T* x) {
#pragma unroll
        for (int a = 0; a < ND; a++) {
            T e = x[a];
#pragma unroll
            for (int k = 0; k < a; k++) e = e - L[a][k] * x[k];
            x[a] = e * Linv[a];
        }
#pragma unroll
        for (int a = ND - 1; a >= 0; a--) {
            T e = x[a];
#pragma unroll
            for (int k = a + 1; k < ND; k++) e = e - L[k][a] * x[k];
            x[a] = e * Linv[a];
        }
    };
    if (ag) {
#pragma unroll
        for (int k = 0; k < ND; k++) {
            T s = u[k];
#pragma unroll
            for (int r = 0; r < 6; r++) s = s - U[r][k] * svget(*ag, r);
            u[k] = s;
        }
        solve(u);
#pragma unroll
        for (int k = 0; k < ND; k++) S(bi.s_w0 + k) = u[k];
        return true;
    }
    // W row r = D^-1 U row r (D symmetric)
    T W[6][ND];
#pragma unroll
    for (int r = 0; r < 6; r++) {
        T x[ND];
#pragma unroll
        for (int k = 0; k < ND; k++) x[k] = U[r][k];
        solve(x);
#pragma unroll
        for (int k = 0; k < ND; k++) W[r][k] = x[k];
    }
    solve(u);
#pragma unroll
    for (int k = 0; k < ND; k++) {
#pragma unroll
        for (int r = 0; r < 6; r++) S(bi.s_vw + k * 6 + r) = W[r][k];
        S(bi.s_w0 + k) = u[k];
    }
    if (has_parent) {
        // I <- I - W U^T over the upper triangle: covers Ia, H (r < 3 <= c) and M
#pragma unroll
        for (int r = 0; r < 6; r++)
#pragma unroll
            for (int cc = r; cc < 6; cc++) {
                T s = T(0);
#pragma unroll
                for (int k = 0; k < ND; k++) s = s + W[r][k] * U[cc][k];
                ai_sub_el(I, r, cc, s);
            }
        SV<T> uw;
        T tmp[6];
#pragma unroll
        for (int r = 0; r < 6; r++) {
            T s = T(0);
#pragma unroll
            for (int k = 0; k < ND; k++) s = s + U[r][k] * u[k];
            tmp[r] = s;
        }
        uw = mksv<T>(mk3<T>(tmp[0], tmp[1], tmp[2]), mk3<T>(tmp[3], tmp[4], tmp[5]));
        p = p + ai_mul(I, c) + uw;
    }
    return true;
}

// ── penalty ground contact of one body (phyz_kernels.cu:541-578, 691-725, 939-965)
template <class T>
PZ_HD V3<T> ksub3(const V3<T>& x, const T* k) {
    return mk3<T>(ksub(x.x, k[0]), ksub(x.y, k[1]), ksub(x.z, k[2]));
}
template <class T>
PZ_HD T eff_mass(const BodyT<T>& bt, const V3<T>& r, const V3<T>& u) {
    if (!(bt.mass > T(0))) return T(1e30);
    const V3<T> a = cross(ksub3(r, bt.com), u);
    const T ang = pz_max(dot(a, ksymv(bt.Icinv, a)), T(0));
    return T(1) / (T(1) / bt.mass + ang);
}
// Its reciprocal, 1/m + (r x u) . Ic^-1 (r x u), without the division.
template <class T>
PZ_HD T eff_mass_inv(const BodyT<T>& bt, const V3<T>& r, const V3<T>& u) {
    if (!(bt.mass > T(0))) return T(1e-30);
    const V3<T> a = cross(ksub3(r, bt.com), u);
    const T ang = pz_max(dot(a, ksymv(bt.Icinv, a)), T(0));
    return T(1) / bt.mass + ang;
}
template <class T>
PZ_HD T fsign(const T& x) {
    return x > T(0) ? T(1) : (x < T(0) ? T(-1) : T(0));
}
template <class T>
PZ_HD V3<T> support_pt(const BodyI& bi, const BodyT<T>& bt, const V3<T>& n_body, int corner) {
    V3<T> s = zero3<T>();
    if (bi.gtype == 2) {  // box corner (phyz_kernels.cu:679-689)
        s = mk3<T>(bt.geom[0] * ((corner & 1) ? T(1) : T(-1)), bt.geom[1] * ((corner & 2) ? T(1) : T(-1)),
                   bt.geom[2] * ((corner & 4) ? T(1) : T(-1)));
    } else {
        const V3<T> n = km3v(bt.grot, n_body);
        if (bi.gtype == 1) {
            s = n * (-bt.geom[0]);
        } else if (bi.gtype == 3) {
            s = mk3<T>(T(0), T(0), -(bt.geom[1] * T(0.5)) * fsign(n.z)) - n * bt.geom[0];
        } else if (bi.gtype == 4) {
            const V3<T> radial = mk3<T>(-n.x, -n.y, T(0));
            const T rl = pz_sqrt(dot(radial, radial));
            V3<T> rim = zero3<T>();
            if (rl > T(1e-6)) rim = radial * (bt.geom[0] / rl);
            s = rim + mk3<T>(T(0), T(0), -(bt.geom[1] * T(0.5)) * fsign(n.z));
        } else if (bi.gtype == 5) {
            const V3<T> mn = ld3(bt.geom), mx = ld3(bt.geom + 3);
            const V3<T> mc = (mn + mx) * T(0.5), mh = (mx - mn) * T(0.5);
            s = mc - mk3<T>(mh.x * fsign(n.x), mh.y * fsign(n.y), mh.z * fsign(n.z));
        }
    }
    const V3<T> o = km3tv(bt.grot, s);
    return mk3<T>(kadd(o.x, bt.gpos[0]), kadd(o.y, bt.gpos[1]), kadd(o.z, bt.gpos[2]));
}

// World frame of a body for contact: world up seen in the body frame (row 2
// of the body->world rotation) and the height of the body origin. The full
// frame (rows r0, r1 and the origin's x, y) is only built for the contact
// state output (contact_state_pass).
template <class T>
struct WF {
    V3<T> r0, r1, up;
    V3<T> pos;  // pos.z is the height of the origin
};

// A strided output: element k goes to base[k * stride] (null base: dropped).
template <class T>
struct Out {
    T* base;
    long long stride;
    PZ_HD void put(int k, const T& v) const {
        if (base) base[(long long)k * stride] = v;
    }
};

// Heightfield sample at world (px, py) (phyz_kernels.cu:625-664): the
// bilinear height, and the unit normal from the patch's gradient (zero
// slope outside the grid's span, where the clamp extends the border flat).
template <class T>
PZ_HD T terrain_at(const Terrain<T>& t, const T& px, const T& py, V3<T>& n_out) {
    auto locate = [&](const T& w, const T& o, int n, int& i, T& f) {
        if (n < 2) {
            i = 0;
            f = T(0);
            return;
        }
        const T u = pz_min(pz_max((w - o) / t.cell, T(0)), T(n - 1));
        int ii = pz_trunc_int(u);  // u >= 0: truncation is the floor
        if (ii > n - 2) ii = n - 2;
        i = ii;
        f = u - T(ii);
    };
    if (t.nx < 1 || t.ny < 1) {  // no grid loaded (never launched that way): the plane z = 0
        n_out = mk3<T>(T(0), T(0), T(1));
        return T(0);
    }
    int ix, iy;
    T tx, ty;
    locate(px, t.ox, t.nx, ix, tx);
    locate(py, t.oy, t.ny, iy, ty);
    const int ix1 = ix + 1 < t.nx - 1 ? ix + 1 : t.nx - 1;
    const int iy1 = iy + 1 < t.ny - 1 ? iy + 1 : t.ny - 1;
    const T h00 = t.oz + T(t.h[iy * t.nx + ix]), h10 = t.oz + T(t.h[iy * t.nx + ix1]);
    const T h01 = t.oz + T(t.h[iy1 * t.nx + ix]), h11 = t.oz + T(t.h[iy1 * t.nx + ix1]);
    const T h = (h00 * (T(1) - tx) + h10 * tx) * (T(1) - ty) + (h01 * (T(1) - tx) + h11 * tx) * ty;
    T dhdx = T(0), dhdy = T(0);
    const T span_x = T(t.nx - 1) * t.cell, span_y = T(t.ny - 1) * t.cell;
    if (t.nx >= 2 && px >= t.ox && px <= t.ox + span_x)
        dhdx = ((h10 - h00) * (T(1) - ty) + (h11 - h01) * ty) / t.cell;
    if (t.ny >= 2 && py >= t.oy && py <= t.oy + span_y)
        dhdy = ((h01 - h00) * (T(1) - tx) + (h11 - h10) * tx) / t.cell;
    const V3<T> n = mk3<T>(-dhdx, -dhdy, T(1));
    const T l = pz_sqrt(dot(n, n));
    n_out = l > T(0) ? n * (T(1) / l) : n;
    return h;
}

// One contact point against the ground: the penetration along the
// terrain normal (phyz_kernels.cu:916-918), that normal in the body frame,
// and (with a heightfield) the world point and the terrain height there.
// The flat ground only needs the body's world up and origin height.
template <bool TERRAIN, class T>
struct GroundHit {
    T pen, h;
    V3<T> n, w;
};
template <bool TERRAIN, class T>
PZ_HD GroundHit<TERRAIN, T> ground_hit(const Terrain<T>& ter, const T& ground_h, const WF<T>& wf, const V3<T>& sup) {
    GroundHit<TERRAIN, T> g;
    if constexpr (TERRAIN) {
        g.w = mk3<T>(wf.pos.x + dot(wf.r0, sup), wf.pos.y + dot(wf.r1, sup), wf.pos.z + dot(wf.up, sup));
        if (ter.nx < 1) {  // full frames for a body-attached plane, over the flat ground
            g.h = ground_h;
            g.pen = ground_h - g.w.z;
            g.n = wf.up;
            return g;
        }
        V3<T> nw;
        g.h = terrain_at(ter, g.w.x, g.w.y, nw);
        g.pen = nw.z * (g.h - g.w.z);
        g.n = wf.r0 * nw.x + wf.r1 * nw.y + wf.up * nw.z;
    } else {
        g.h = ground_h;
        g.pen = ground_h - (wf.pos.z + dot(wf.up, sup));
        g.n = wf.up;
    }
    return g;
}

// ground_hit on the flat plane with the world point filled in (the contact
// state wants it).
template <class T>
PZ_HD GroundHit<true, T> flat_hit(const T& ground_h, const WF<T>& wf, const V3<T>& sup) {
    GroundHit<true, T> g;
    g.w = mk3<T>(wf.pos.x + dot(wf.r0, sup), wf.pos.y + dot(wf.r1, sup), wf.pos.z + dot(wf.up, sup));
    g.h = ground_h;
    g.pen = ground_h - g.w.z;
    g.n = wf.up;
    return g;
}

// Contact wrench (body frame) of body i at body velocity v, and its state.
// With `full`, the body's contact state [touching, depth, point(3),
// force(3)] (layout.rs:68-80) goes to rows 8*i.. of `cs`.
template <bool TERRAIN, class T>
PZ_HD SV<T> contact_wrench(const ModelView<T>& M, const BodyI& bi, const BodyT<T>& bt, const WF<T>& wf,
                           const SV<T>& v, bool full, int i, const Out<T>& cs) {
    SV<T> f = zerosv<T>();
    V3<T> fw = zero3<T>();
    T deepest = T(0), dx = T(0), dy = T(0), dz = M.ground_h;
    bool any = false;
    const T pt_scale = bi.gtype == 2 ? T(0.25) : T(1);
    const int npts = bi.gtype == 2 ? 8 : 1;
    for (int c = 0; c < npts; c++) {
        const V3<T> sup = support_pt(bi, bt, wf.up, c);
        const GroundHit<TERRAIN, T> g = ground_hit<TERRAIN>(M.ter, M.ground_h, wf, sup);
        const T pen = g.pen;
        if (!(pen > T(0))) continue;
        const V3<T>& n = g.n;
        const V3<T> vp = v.l + cross(v.w, sup);
        const T vn = dot(vp, n);
        // the gains' caps k <= 4 m_eff / dt^2, d <= m_eff / dt and the
        // friction cap m_eff vt / dt, compared through the inverse effective
        // mass: a division only where a cap binds
        const T in = eff_mass_inv(bt, sup, n);
        const T kg = pt_scale * bt.gk, dg = pt_scale * bt.gd;
        const T kb = kg * in <= M.kstiff_c ? kg : M.kstiff_c / in;
        const T db = dg * in <= M.inv_dt_c ? dg : M.inv_dt_c / in;
        const T fn = pz_max(kb * pen - db * vn, T(0));
        const V3<T> vt3 = vp - n * vn;
        const T vt = pz_sqrt(dot(vt3, vt3));
        V3<T> fb = n * fn;
        if (vt > T(1e-6)) {
            const V3<T> td = vt3 * (T(1) / vt);
            const T coul = (M.friction * fn) * pz_min(T(1), vt * T(1e3));
            const T it = eff_mass_inv(bt, sup, td), cap = M.inv_dt_c * vt;
            const T ft = coul * it <= cap ? coul : cap / it;
            fb = fb - td * ft;
        }
        f.w = f.w + cross(sup, fb);
        f.l = f.l + fb;
        any = true;
        if (full) {
            fw = fw + mk3<T>(dot(wf.r0, fb), dot(wf.r1, fb), dot(wf.up, fb));
            if (pen > deepest) {
                deepest = pen;
                if constexpr (TERRAIN) {
                    dx = g.w.x;
                    dy = g.w.y;
                    dz = g.h;
                } else {
                    dx = wf.pos.x + dot(wf.r0, sup);
                    dy = wf.pos.y + dot(wf.r1, sup);
                }
            }
        }
    }
    if (full) {
        cs.put(8 * i + 0, any ? T(1) : T(0));
        cs.put(8 * i + 1, any ? deepest : T(0));
        cs.put(8 * i + 2, any ? dx : T(0));
        cs.put(8 * i + 3, any ? dy : T(0));
        cs.put(8 * i + 4, any ? dz : T(0));
        cs.put(8 * i + 5, any ? fw.x : T(0));
        cs.put(8 * i + 6, any ? fw.y : T(0));
        cs.put(8 * i + 7, any ? fw.z : T(0));
    }
    return f;
}

// Out-of-line entry to contact_wrench: everything by value, so the caller's
// sweep state stays in registers and the contact temporaries do not add to
// the sweep's register pressure.
template <bool TERRAIN, class T>
PZ_OUTLINE SV<T> contact_wrench_call(T ground_h, T friction, T inv_dt_c, T kstiff_c, Terrain<T> ter, BodyI bi,
                                     const BodyT<T>* bt, WF<T> wf, SV<T> v, bool full, int i, Out<T> cs) {
    ModelView<T> M;
    M.ground_h = ground_h;
    M.friction = friction;
    M.inv_dt_c = inv_dt_c;
    M.kstiff_c = kstiff_c;
    M.ter = ter;
    return contact_wrench<TERRAIN>(M, bi, *bt, wf, v, full, i, cs);
}

// ── per-world I/O of a launch ──────────────────────────────────────────────
template <class T>
struct WorldIO {
    const T* ctrl;          // [nv][nworld] held, or [step][nv][nworld] schedule
    long long ctrl_stride;  // elements between steps (0: held)
    const T* targets;       // PD targets [npd][nworld]
    long long nworld;
    long long w;
    const int* gdof = nullptr;  // FEAT_LANES: model DOF of each of the lane's DOFs
};

// Queue the control inputs of `step` for body i into its w0 slots. MAP: the
// world is split over lanes (FEAT_LANES) and a lane's DOF d is the model's
// DOF io.gdof[d] (PD servos do not occur there).
template <bool SEP, class T, class Scr, bool MAP = false>
PZ_HD void prefetch_controls(const ModelView<T>& M, const BodyI& bi, const Scr& S, const WorldIO<T>& io,
                             int step) {
    const int nd = bi.ndof;
    for (int k = 0; k < nd; k++) {
        const int d = bi.off + k;
        const int pdi = (bi.flags & F_PD) ? M.pd_of_dof[d] : -1;
        const long long g = MAP ? (long long)io.gdof[d] : (long long)d;
        const T* src = pdi >= 0 ? io.targets + (long long)pdi * io.nworld + io.w
                                : io.ctrl + (long long)step * io.ctrl_stride + g * io.nworld + io.w;
        S.prefetch((SEP ? bi.s_in : bi.s_w0) + k, src);
    }
}
// One-DOF form for the relabelled-hinge path.
template <bool SEP, class T, class Scr, bool MAP = false>
PZ_HD void prefetch_control1(const ModelView<T>& M, const BodyI& bi, const Scr& S, const WorldIO<T>& io,
                             int step) {
    const int d = bi.off;
    const int pdi = (bi.flags & F_PD) ? M.pd_of_dof[d] : -1;
    const long long g = MAP ? (long long)io.gdof[d] : (long long)d;
    const T* src = pdi >= 0 ? io.targets + (long long)pdi * io.nworld + io.w
                            : io.ctrl + (long long)step * io.ctrl_stride + g * io.nworld + io.w;
    S.prefetch(SEP ? bi.s_in : bi.s_w0, src);
}

// I c for a bias c whose K components are structurally zero (c = v x S qd
// of a hinge about e_K): the products with those zeros are skipped.
template <int K, class T>
PZ_HD SV<T> ai_mul_zk(const AI<T>& I, const SV<T>& c) {
    V3<T> w = zero3<T>(), l = zero3<T>();
#pragma unroll
    for (int r = 0; r < 3; r++) {
        T sw = T(0), sl = T(0);
        bool first_w = true, first_l = true;
#pragma unroll
        for (int k = 0; k < 3; k++) {
            if (k == K) continue;
            const T cw = get(c.w, k), cl = get(c.l, k);
            // [Ia H; H^T M] [cw; cl]
            const T a = I.a[sidx(r, k)] * cw, h = I.h[r * 3 + k] * cl;
            const T ht = I.h[k * 3 + r] * cw, m = I.m[sidx(r, k)] * cl;
            sw = first_w ? a + h : sw + a + h;
            sl = first_l ? ht + m : sl + ht + m;
            first_w = first_l = false;
        }
        if (r == 0) w.x = sw, l.x = sl;
        if (r == 1) w.y = sw, l.y = sl;
        if (r == 2) w.z = sw, l.z = sl;
    }
    return mksv<T>(w, l);
}

// ── pass 1 of body i for the state in scratch: joint transform, velocity,
// world frame and contact wrench. `cv`/`cw` carry body i-1's values.
template <int AX, int FEAT, class T, class Scr>
PZ_HD void pass1_body(const ModelView<T>& M, const Scr& S, int i, const BodyI& bi, SV<T>& cv, WF<T>& cw) {
    const BodyT<T>& bt = M.bt[i];
    const int p = bi.parent;
    SV<T> vpar;
    if (p < 0)
        vpar = zerosv<T>();
    else if (p == i - 1)
        vpar = cv;
    else {
        S.fence_st();  // the parent's record was stored earlier in this sweep
        vpar = ld_vel<T>(S, M.bi[p]);
    }
    JX<T> j;
    SV<T> v;
    if constexpr (AX >= 0) {
        T sn, cs;
        pz_sincos(-S(bi.off), &sn, &cs);
        j.c = cs;
        j.s = sn;
        v = mot_X<AX, FEAT>(bi, bt, j, vpar);
        at<AX>(v.w) = at<AX>(v.w) + S(M.nv + bi.off);
        Rec<T> r;
        r.c = cs;
        r.s = sn;
        r.v = v;
        S.rec_put(bi, r);
    } else {
        j = make_jx<AX, FEAT>(bi, bt, S);
        v = mot_X<AX, FEAT>(bi, bt, j, vpar) + joint_vel<AX, FEAT>(bi, bt, S, M.nv);
        st_sv(S, bi.s_vw, v);
    }
    cv = v;
    if constexpr ((FEAT & FEAT_CONTACT) != 0) {
        constexpr bool TERRAIN = (FEAT & FEAT_TERRAIN) != 0;
        constexpr int NW = TERRAIN ? 12 : 4;  // frame words kept per body
        // the parent's world frame: up and origin height, or with a
        // heightfield the rows r0, r1, up of its body->world rotation and its
        // origin (a row transforms into the child frame like a vector)
        WF<T> pf;
        if (p < 0) {
            pf.r0 = mk3<T>(T(1), T(0), T(0));
            pf.r1 = mk3<T>(T(0), T(1), T(0));
            pf.up = mk3<T>(T(0), T(0), T(1));
            pf.pos = zero3<T>();
        } else if (p == i - 1) {
            pf = cw;
        } else {
            const int s = M.bi[p].s_wx;
            if constexpr (TERRAIN) {
                pf.r0 = mk3<T>(S(s), S(s + 1), S(s + 2));
                pf.r1 = mk3<T>(S(s + 3), S(s + 4), S(s + 5));
                pf.up = mk3<T>(S(s + 6), S(s + 7), S(s + 8));
                pf.pos = mk3<T>(S(s + 9), S(s + 10), S(s + 11));
            } else {
                pf.up = mk3<T>(S(s), S(s + 1), S(s + 2));
                pf.pos.z = S(s + 3);
            }
        }
        WF<T> wf;
        const V3<T> tp = tree_pos<AX, FEAT>(bi, bt, j);
        wf.up = tree_rot<AX, FEAT>(bi, bt, j, pf.up);
        wf.pos.z = pf.pos.z + dot(pf.up, tp);
        if constexpr (TERRAIN) {
            wf.r0 = tree_rot<AX, FEAT>(bi, bt, j, pf.r0);
            wf.r1 = tree_rot<AX, FEAT>(bi, bt, j, pf.r1);
            wf.pos.x = pf.pos.x + dot(pf.r0, tp);
            wf.pos.y = pf.pos.y + dot(pf.r1, tp);
        }
        cw = wf;
        auto store = [&](int s) {
            if constexpr (TERRAIN) {
                S(s) = wf.r0.x;
                S(s + 1) = wf.r0.y;
                S(s + 2) = wf.r0.z;
                S(s + 3) = wf.r1.x;
                S(s + 4) = wf.r1.y;
                S(s + 5) = wf.r1.z;
                S(s + 6) = wf.up.x;
                S(s + 7) = wf.up.y;
                S(s + 8) = wf.up.z;
                S(s + 9) = wf.pos.x;
                S(s + 10) = wf.pos.y;
                S(s + 11) = wf.pos.z;
            } else {
                S(s) = wf.up.x;
                S(s + 1) = wf.up.y;
                S(s + 2) = wf.up.z;
                S(s + 3) = wf.pos.z;
            }
        };
        static_assert(NW == 4 || NW == 12, "frame words");
        if (bi.flags & F_BRANCH) store(bi.s_wx);
        if (bi.flags & F_CONTACT) {
            if constexpr ((FEAT & FEAT_IMPULSE) != 0) {
                store(bi.s_up);  // the impulse sweeps read the body's frame
            } else {
#if defined(PZ_SPEC) && PZ_SPEC_INLINE_CONTACT
                // specialized: inline, the body's shape and gains literal
                const SV<T> f = contact_wrench<TERRAIN>(M, bi, M.bt[i], wf, v, false, i, Out<T>{nullptr, 0});
#else
                const SV<T> f = contact_wrench_call<TERRAIN>(M.ground_h, M.friction, M.inv_dt_c, M.kstiff_c, M.ter,
                                                             bi, M.btp + i, wf, v, false, i, Out<T>{nullptr, 0});
#endif
                S.ext_put(bi, f);
            }
        }
    }
}

// Full world frame of body i for the state in scratch (joint transforms of
// pass 1 in place), built by walking its ancestor chain: a body-frame vector
// d maps into its parent as E_tree^T d (plus tree_pos for points).
template <int FEAT, class T, class Scr>
PZ_HD WF<T> world_frame(const ModelView<T>& M, const Scr& S, int i) {
    // columns of the body->world rotation and the origin, built upwards
    V3<T> cx = mk3<T>(T(1), T(0), T(0)), cy = mk3<T>(T(0), T(1), T(0)), cz = mk3<T>(T(0), T(0), T(1));
    V3<T> o = zero3<T>();
    // (at most nb ancestors: the bound lets a specialized build unroll the
    // walk with every ancestor's table entry folded)
    int b = i;
    PZ_UNROLL_BODIES
    for (int k = 0; k < M.nb && b >= 0; k++) {
        const BodyI bb = M.bi[b];
        const BodyT<T>& tb = M.bt[b];
        b = bb.parent;
        JX<T> j;
        if (bb.t_rec >= 0) {
            const Rec<T> r = S.rec_get(bb);
            j.c = r.c;
            j.s = r.s;
        } else {
            j = load_jx<-1, FEAT>(bb, tb, S);
        }
        // E_tree^T d = R_ptj^T R_J^T d
        auto up_dir = [&](V3<T> d) {
            switch (bb.jtype) {
                case J_REVOLUTE: d = bb.axis_k >= 0 ? hrot_t(bb.axis_k, j.c, j.s, d) : rtmul(j.E, d); break;
                case J_BALL:
                case J_FREE:
                    if constexpr ((FEAT & FEAT_MULTI) != 0) d = rtmul(j.E, d);
                    break;
                default: break;
            }
            if (bb.flags & F_PTJ_ROT) d = m3tv(tb.ptj_rot, d);
            return d;
        };
        cx = up_dir(cx);
        cy = up_dir(cy);
        cz = up_dir(cz);
        o = up_dir(o) + tree_pos<-1, FEAT>(bb, tb, j);
    }
    WF<T> wf;  // rows of the body->world rotation = components of the columns
    wf.r0 = mk3<T>(cx.x, cy.x, cz.x);
    wf.r1 = mk3<T>(cx.y, cy.y, cz.y);
    wf.up = mk3<T>(cx.z, cy.z, cz.z);
    wf.pos = o;
    return wf;
}

// Contact state [touching, depth, point(3), force(3)] of every body for the
// state in scratch (joint transforms and velocities of pass 1 in place),
// written to rows 8*i.. of `cs` (layout.rs:68-80).
template <int FEAT, class T, class Scr>
PZ_HD void contact_state_pass(const ModelView<T>& M, const Scr& S, const Out<T>& cs) {
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
        if (!(bi.flags & F_CONTACT)) {
            for (int k = 0; k < 8; k++) cs.put(8 * i + k, T(0));
            continue;
        }
        const WF<T> wf = world_frame<FEAT>(M, S, i);
        contact_wrench<(FEAT & FEAT_TERRAIN) != 0>(M, bi, M.bt[i], wf, ld_vel<T>(S, bi), true, i, cs);
    }
}

// ── impulse-mode ground contact (phyz_kernels.cu:581-622 helpers, :856-918
// the impulse branch of contact_thread; flat ground) ───────────────────────
// The per-launch constants of the impulse law: the SolImp curve's clamped
// parameters (phyz_kernels.cu:589-601 clamps them at every call) and the
// reciprocals of the divisors that do not change within a launch.
template <class T>
PZ_HD void impmat_finish(ImpMat<T>& m) {
    m.c_dmin = pz_min(pz_max(m.dmin, T(1e-4)), T(1) - T(1e-9));
    m.c_dmax = pz_min(pz_max(m.dmax, T(1e-4)), T(1) - T(1e-9));
    m.c_mid = pz_min(pz_max(m.mid, T(1e-6)), T(1) - T(1e-6));
    m.c_pw = pz_max(m.power, T(1));
    m.pw2 = !(m.c_pw < T(2)) && !(m.c_pw > T(2));
    m.inv_width = m.width > T(0) ? T(1) / m.width : T(0);
    m.mid_scale = T(1) / pz_pow(m.c_mid, m.c_pw - T(1));
    m.omid_scale = T(1) / pz_pow(T(1) - m.c_mid, m.c_pw - T(1));
    m.inv_margin = m.margin > T(0) ? T(1) / m.margin : T(0);
    m.inv_dtc = T(1) / pz_max(m.dt, T(1e-9));
    m.inv_vr = m.rest_thr > T(0) ? T(1) / m.rest_thr : T(0);
}
// SolImp impedance at depth r (phyz_kernels.cu:589-601):
// y = x^p / mid^(p-1) below mid, 1 - (1-x)^p / (1-mid)^(p-1) above.
template <class T>
PZ_HD T solimp_impedance(const ImpMat<T>& m, const T& r) {
    if (!(m.width > T(0))) return m.c_dmax;
    const T x = pz_min(pz_max(pz_abs(r) * m.inv_width, T(0)), T(1));
    const bool lo = x <= m.c_mid;
    const T z = lo ? x : T(1) - x;
    const T zp = m.pw2 ? z * z : pz_pow(z, m.c_pw);
    const T y = lo ? zp * m.mid_scale : T(1) - zp * m.omid_scale;
    return m.c_dmin + y * (m.c_dmax - m.c_dmin);
}
// solimp when penetrating, smoothstep to zero across the margin (:604-611)
template <class T>
PZ_HD T impedance_at(const ImpMat<T>& m, const T& depth) {
    if (depth >= T(0)) return solimp_impedance(m, depth);
    const T gap = -depth;
    if (!(m.margin > T(0)) || gap >= m.margin) return T(0);
    const T sc = T(1) - gap * m.inv_margin;
    return sc * sc * (T(3) - T(2) * sc) * solimp_impedance(m, T(0));
}
// restitution ramp between v_rest and 2 v_rest (:613-622); no restitution
// (the default material) is zero throughout the ramp
template <class T>
PZ_HD T effective_restitution(const ImpMat<T>& m, const T& e, const T& approach) {
    const T vr = m.rest_thr;
    if (!(vr > T(0))) return e;
    if (!(pz_abs(e) > T(0))) return T(0);
    const T sp = pz_abs(approach);
    if (sp <= vr) return T(0);
    if (sp >= T(2) * vr) return e;
    const T t = (sp - vr) * m.inv_vr;
    return e * t * t * (T(3) - T(2) * t);
}
// orthonormal tangents around a unit normal (:581-586)
template <class T>
PZ_HD void contact_tangents(const V3<T>& n, V3<T>& u, V3<T>& w) {
    const V3<T> a = pz_abs(n.x) > T(0.9) ? mk3<T>(T(0), T(1), T(0)) : mk3<T>(T(1), T(0), T(0));
    const V3<T> c = cross(n, a);
    const T l = pz_sqrt(dot(c, c));
    u = l > T(0) ? c * (T(1) / l) : c;
    w = cross(n, u);
}

// The tangents of contact_tangents taken in the body's original frame and
// expressed in its stored (relabelled) one: the staged update treats the two
// tangent directions separately, so its result depends on the basis, which
// has to be the reference's.
template <class T>
PZ_HD void body_tangents(const BodyI& bi, const V3<T>& n, V3<T>& u, V3<T>& w) {
    if (bi.fshift == 1) {
        contact_tangents(cperm<2>(n), u, w);
        u = cperm<1>(u);
        w = cperm<1>(w);
    } else if (bi.fshift == 2) {
        contact_tangents(cperm<1>(n), u, w);
        u = cperm<2>(u);
        w = cperm<2>(w);
    } else {
        contact_tangents(n, u, w);
    }
}

// One staged Coulomb update of every contact point of body i (normal
// impulse first, then the tangential impulse clamped into the friction disc
// that normal admits), at the body's free velocity `vf` (body frame), with
// the body's world frame `wf` (up and origin height; all of it with a
// heightfield). The impulses of the previous sweep are read from and the new
// ones written to the body's impulse slots; returns the wrench (body frame)
// they apply over one step.
template <bool TERRAIN, class T, class Scr>
PZ_HD SV<T> impulse_wrench(const ImpMat<T>& m, const Terrain<T>& ter, const BodyI& bi, const BodyT<T>& bt,
                           const WF<T>& wf, const SV<T>& vf, const Scr& S) {
    const int npts = bi.gtype == 2 ? 8 : 1;
    // within-body load sharing: points inside the margin
    int n_active = 0;
    for (int c = 0; c < npts; c++) {
        const V3<T> sup = support_pt(bi, bt, wf.up, c);
        if (ground_hit<TERRAIN>(ter, m.ground_h, wf, sup).pen > -m.margin) n_active++;
    }
    const T na = T(n_active < 1 ? 1 : n_active);
    SV<T> f = zerosv<T>();
    bool any = false;
    for (int c = 0; c < npts; c++) {
        const int slot = bi.s_imp + 3 * c;
        const V3<T> sup = support_pt(bi, bt, wf.up, c);
        const GroundHit<TERRAIN, T> g = ground_hit<TERRAIN>(ter, m.ground_h, wf, sup);
        const T pen = g.pen;
        if (!(pen > -m.margin)) {
            S(slot) = T(0);
            S(slot + 1) = T(0);
            S(slot + 2) = T(0);
            continue;
        }
        const V3<T>& n = g.n;
        const V3<T> vp = vf.l + cross(vf.w, sup);
        V3<T> tu, tw;
        body_tangents(bi, n, tu, tw);
        const T bn = dot(vp, n), bu = dot(vp, tu), bw = dot(vp, tw);
        // the reference's A = 1 / max(m_eff / n_active, 1e-9) along the
        // normal and n_active / max(m_eff, 1e-9) along each tangent, taken
        // from the inverse effective mass (no division)
        const T ann = pz_min(na * eff_mass_inv(bt, sup, n), T(1e9));
        const T bias = impedance_at(m, pen) * m.erp * pz_max(pen, T(0)) * m.inv_dtc;
        const T e = effective_restitution(m, m.restitution, pz_min(bn, T(0)));
        const T rn = bn * (T(1) + e) - ann * S(slot);
        const T fn = pz_max((bias - rn) / ann, T(0));
        const T auu = pz_min(na * eff_mass_inv(bt, sup, tu), na * T(1e9));
        const T aww = pz_min(na * eff_mass_inv(bt, sup, tw), na * T(1e9));
        T ju = -(bu - auu * S(slot + 1)) / auu;
        T jw = -(bw - aww * S(slot + 2)) / aww;
        const T limit = m.friction * fn;
        const T jt = pz_sqrt(ju * ju + jw * jw);
        if (jt > limit) {
            const T sc = jt > T(0) ? limit / jt : T(0);
            ju = ju * sc;
            jw = jw * sc;
        }
        S(slot) = fn;
        S(slot + 1) = ju;
        S(slot + 2) = jw;
        const V3<T> fb = (n * fn + tu * ju + tw * jw) * m.inv_dtc;
        f.w = f.w + cross(sup, fb);
        f.l = f.l + fb;
        any = true;
    }
    if (!any) {
        for (int k = 0; k < 3 * npts; k++) S(bi.s_imp + k) = T(0);
        // the reference clears the body's whole contact-state row here
        // (phyz_kernels.cu:966-969), its plane impulses included: a body off
        // the ground starts every sweep's plane update from zero
        if (bi.s_pimp >= 0)
            for (int k = 0; k < 3 * npts; k++) S(bi.s_pimp + k) = T(0);
    }
    return f;
}

// Contact state of every body in impulse mode, from the impulses the last
// sweep left in the slots (phyz_kernels.cu:964-980 with the impulse
// branch's point and force): [touching, depth, point(3), force(3)].
template <int FEAT, class T, class Scr>
PZ_HD void contact_state_impulse_pass(const ModelView<T>& M, const Scr& S, const Out<T>& cs) {
    const T idt = T(1) / pz_max(M.im.dt, T(1e-9));
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
        if (!(bi.flags & F_CONTACT)) {
            for (int k = 0; k < 8; k++) cs.put(8 * i + k, T(0));
            continue;
        }
        const BodyT<T>& bt = M.bt[i];
        const WF<T> wf = world_frame<FEAT>(M, S, i);
        const int npts = bi.gtype == 2 ? 8 : 1;
        V3<T> fw = zero3<T>(), dp = zero3<T>();
        T deepest = T(0);
        bool any = false;
        for (int c = 0; c < npts; c++) {
            const V3<T> sup = support_pt(bi, bt, wf.up, c);
            // the world frame is complete here: the world point is at hand
            GroundHit<true, T> g;
            if constexpr ((FEAT & FEAT_TERRAIN) != 0)
                g = ground_hit<true>(M.ter, M.im.ground_h, wf, sup);
            else
                g = flat_hit(M.im.ground_h, wf, sup);
            const T pen = g.pen;
            if (!(pen > -M.im.margin)) continue;
            V3<T> tu, tw;
            body_tangents(bi, g.n, tu, tw);
            const int slot = bi.s_imp + 3 * c;
            const V3<T> fb = (g.n * S(slot) + tu * S(slot + 1) + tw * S(slot + 2)) * idt;
            fw = fw + mk3<T>(dot(wf.r0, fb), dot(wf.r1, fb), dot(wf.up, fb));
            any = true;
            if (pen > deepest) {
                deepest = pen;
                dp = g.w;
            }
        }
        cs.put(8 * i + 0, any ? T(1) : T(0));
        cs.put(8 * i + 1, any ? deepest : T(0));
        cs.put(8 * i + 2, any ? dp.x : T(0));
        cs.put(8 * i + 3, any ? dp.y : T(0));
        cs.put(8 * i + 4, any ? dp.z : T(0));
        cs.put(8 * i + 5, any ? fw.x : T(0));
        cs.put(8 * i + 6, any ? fw.y : T(0));
        cs.put(8 * i + 7, any ? fw.z : T(0));
    }
}

// ── body-attached contact plane (phyz_kernels.cu:983-1132) ───────────────
// R x and R^T y for a body->world rotation held as its rows.
template <class T>
PZ_HD V3<T> wf_mul(const WF<T>& f, const V3<T>& x) {
    return mk3<T>(dot(f.r0, x), dot(f.r1, x), dot(f.up, x));
}
template <class T>
PZ_HD V3<T> wf_tmul(const WF<T>& f, const V3<T>& y) {
    return f.r0 * y.x + f.r1 * y.y + f.up * y.z;
}
// A body-frame vector between the stored (relabelled) and the original
// coordinates of a body with frame shift s.
template <class T>
PZ_HD V3<T> to_stored(int s, const V3<T>& v) {
    return s == 1 ? cperm<1>(v) : (s == 2 ? cperm<2>(v) : v);
}
template <class T>
PZ_HD V3<T> to_original(int s, const V3<T>& v) {
    return s == 1 ? cperm<2>(v) : (s == 2 ? cperm<1>(v) : v);
}

// Every F_PLANE body against the plane: the action on the body and the
// reaction on the plane's body at one shared point, added to both wrench
// slots (the plane body's slot is cleared first unless its own ground
// contact has just written it). Penalty mode (the gains of the touching
// body, the pair's series effective mass bounding them) reads the body
// velocities of pass 1; impulse mode the sweep's free velocities and the
// staged impulses of the plane slots. Every lane runs every body (record
// loads are warp-wide); per-world tests only skip arithmetic.
template <bool IMPULSE, int FEAT, class T, class Scr>
PZ_HD void plane_pass(const ModelView<T>& M, const Scr& S) {
    const int pb = M.plane.body;
    const BodyI bp = M.bi[pb];
    const BodyT<T>& tp = M.bt[pb];
    if (!(bp.flags & F_CONTACT))
        for (int k = 0; k < 6; k++) S(bp.s_f + k) = T(0);
    const WF<T> fp = world_frame<FEAT>(M, S, pb);
    SV<T> vpb;
    if constexpr (IMPULSE)
        vpb = ld_sv<T>(S, bp.s_vf);
    else
        vpb = ld_vel<T>(S, bp);
    const V3<T> ez = to_stored<T>(bp.fshift, mk3<T>(T(0), T(0), T(1)));  // the body's own +z
    const V3<T> n_w = wf_mul(fp, ez);
    const V3<T> p0_w = fp.pos + wf_mul(fp, ez * M.plane.offset);
    const V3<T> n_p = wf_tmul(fp, n_w);
    SV<T> fpb = zerosv<T>();
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
        if (!(bi.flags & F_PLANE)) continue;  // a model constant: uniform over the warp
        const BodyT<T>& bt = M.bt[i];
        const WF<T> fi = world_frame<FEAT>(M, S, i);
        SV<T> vi;
        if constexpr (IMPULSE)
            vi = ld_sv<T>(S, bi.s_vf);
        else
            vi = ld_vel<T>(S, bi);
        const V3<T> n_i = wf_tmul(fi, n_w);
        const int npts = bi.gtype == 2 ? 8 : 1;
        const T pt_scale = bi.gtype == 2 ? T(0.25) : T(1);
        // the shape's footprint in face coordinates (the plane body's original
        // x, y), intersected with the face
        T lo_x = T(1e30), lo_y = T(1e30), hi_x = T(-1e30), hi_y = T(-1e30);
        int active = 0;
        for (int c = 0; c < npts; c++) {
            const V3<T> sw = fi.pos + wf_mul(fi, support_pt(bi, bt, n_i, c));
            const V3<T> rp = to_original(bp.fshift, wf_tmul(fp, sw - fp.pos));
            lo_x = pz_min(lo_x, rp.x);
            lo_y = pz_min(lo_y, rp.y);
            hi_x = pz_max(hi_x, rp.x);
            hi_y = pz_max(hi_y, rp.y);
            const T d = -dot(sw - p0_w, n_w);
            if (d > T(0) && d <= M.plane.max_depth) active++;
        }
        const T ox0 = pz_max(lo_x, -M.plane.half_x), oy0 = pz_max(lo_y, -M.plane.half_y);
        const T ox1 = pz_min(hi_x, M.plane.half_x), oy1 = pz_min(hi_y, M.plane.half_y);
        // no overlap: no contact (a per-world test, so the loop below is
        // skipped rather than the body: the next body's record loads stay
        // converged)
        const bool overlap = !(ox0 > ox1 || oy0 > oy1);
        const T na = T(active > 1 ? active : 1);
        SV<T> f = zerosv<T>();
        for (int c = 0; c < (overlap ? npts : 0); c++) {
            const V3<T> sup = support_pt(bi, bt, n_i, c);
            const V3<T> sw0 = fi.pos + wf_mul(fi, sup);
            const T pen = -dot(sw0 - p0_w, n_w);
            if (!(pen > T(0)) || pen > M.plane.max_depth) {
                if constexpr (IMPULSE) {
                    S(bi.s_pimp + 3 * c) = T(0);
                    S(bi.s_pimp + 3 * c + 1) = T(0);
                    S(bi.s_pimp + 3 * c + 2) = T(0);
                }
                continue;
            }
            // the point in the face, clamped into the overlap: one world
            // point, a lever on each body
            V3<T> ro = to_original(bp.fshift, wf_tmul(fp, sw0 - fp.pos));
            ro.x = pz_min(pz_max(ro.x, ox0), ox1);
            ro.y = pz_min(pz_max(ro.y, oy0), oy1);
            const V3<T> r_p = to_stored(bp.fshift, ro);
            const V3<T> sw = fp.pos + wf_mul(fp, r_p);
            const V3<T> sc = wf_tmul(fi, sw - fi.pos);
            const V3<T> v_rel = wf_mul(fi, vi.l + cross(vi.w, sc)) - wf_mul(fp, vpb.l + cross(vpb.w, r_p));
            const T vn = dot(v_rel, n_w);
            auto pair_mass = [&](const V3<T>& dir_w) {
                return T(1) / (T(1) / eff_mass(bt, sc, wf_tmul(fi, dir_w)) + T(1) / eff_mass(tp, r_p, wf_tmul(fp, dir_w)));
            };
            const T m_n = T(1) / (T(1) / eff_mass(bt, sc, n_i) + T(1) / eff_mass(tp, r_p, n_p));
            V3<T> f_w;
            if constexpr (IMPULSE) {
                const int slot = bi.s_pimp + 3 * c;
                V3<T> pu, pw;
                contact_tangents(n_w, pu, pw);  // world frame: no relabelling enters
                const T bu = dot(v_rel, pu), bw = dot(v_rel, pw);
                const T ann = na / pz_max(m_n, T(1e-9));
                const T bias = impedance_at(M.im, pen) * M.im.erp * pz_max(pen, T(0)) * M.im.inv_dtc;
                const T e = effective_restitution(M.im, M.im.restitution, pz_min(vn, T(0)));
                const T fn = pz_max((bias - (vn * (T(1) + e) - ann * S(slot))) / ann, T(0));
                const T auu = na / pz_max(pair_mass(pu), T(1e-9));
                const T aww = na / pz_max(pair_mass(pw), T(1e-9));
                T ju = -(bu - auu * S(slot + 1)) / auu;
                T jw = -(bw - aww * S(slot + 2)) / aww;
                const T lim = M.friction * fn;
                const T jt = pz_sqrt(ju * ju + jw * jw);
                if (jt > lim) {
                    const T scl = jt > T(0) ? lim / jt : T(0);
                    ju = ju * scl;
                    jw = jw * scl;
                }
                S(slot) = fn;
                S(slot + 1) = ju;
                S(slot + 2) = jw;
                f_w = (n_w * fn + pu * ju + pw * jw) * M.im.inv_dtc;
            } else {
                const T kb = pz_min(pt_scale * bt.gk, M.kstiff_c * m_n);
                const T db = pz_min(pt_scale * bt.gd, M.inv_dt_c * m_n);
                const T fn = pz_max(kb * pen - db * vn, T(0));
                const V3<T> vt3 = v_rel - n_w * vn;
                const T vt = pz_sqrt(dot(vt3, vt3));
                f_w = n_w * fn;
                if (vt > T(1e-6)) {
                    const V3<T> td = vt3 * (T(1) / vt);
                    const T coul = (M.friction * fn) * pz_min(T(1), vt / T(1e-3));
                    f_w = f_w - td * pz_min(coul, (M.inv_dt_c * pair_mass(td)) * vt);
                }
            }
            const V3<T> fib = wf_tmul(fi, f_w), fpbb = wf_tmul(fp, f_w * T(-1));
            f.w = f.w + cross(sc, fib);
            f.l = f.l + fib;
            fpb.w = fpb.w + cross(r_p, fpbb);
            fpb.l = fpb.l + fpbb;
        }
        st_sv(S, bi.s_f, ld_sv<T>(S, bi.s_f) + f);
    }
    st_sv(S, bp.s_f, ld_sv<T>(S, bp.s_f) + fpb);
}

// Run f<AX>() for the body's kind.
#define PZ_BY_KIND(kind, CALL) \
    if ((kind) == 2) {         \
        CALL(2);               \
    } else {                   \
        CALL(-1);              \
    }

// ── pass 2 of body i (aba.rs:215-320). I, pA carry the child's contribution
// in from the next body (when it is this body's child) and this body's
// contribution out to its parent.
template <int AX, int FEAT, class T, class Scr>
PZ_HD void pass2_body(const ModelView<T>& M, const Scr& S, int i, const BodyI& bi, AI<T>& I, SV<T>& pA) {
    const BodyT<T>& bt = M.bt[i];
    const int p = bi.parent;
    Rec<T> rec;
    SV<T> v;
    if constexpr (AX >= 0) {
        rec = S.rec_get(bi);
        v = rec.v;
    } else {
        v = ld_sv<T>(S, bi.s_vw);
    }
    if (!(bi.flags & F_CHAIN)) {
        ai_zero(I);
        pA = zerosv<T>();
    }
    // rigid inertia about the origin [Io, (mc)^x; -(mc)^x, m 1] and the
    // bias force v x* (I v) - f_ext
#pragma unroll
    for (int k = 0; k < 6; k++) I.a[k] = kadd(I.a[k], bt.Io[k]);
    I.h[1] = ksub(I.h[1], bt.mcom[2]);
    I.h[2] = kadd(I.h[2], bt.mcom[1]);
    I.h[3] = kadd(I.h[3], bt.mcom[2]);
    I.h[5] = ksub(I.h[5], bt.mcom[0]);
    I.h[6] = ksub(I.h[6], bt.mcom[1]);
    I.h[7] = kadd(I.h[7], bt.mcom[0]);
    I.m[0] = I.m[0] + bt.mass;
    I.m[1] = I.m[1] + bt.mass;
    I.m[2] = I.m[2] + bt.mass;
    const V3<T> mc = ld3(bt.mcom);
    const SV<T> hv = mksv<T>(ksymv(bt.Io, v.w) + kcross(mc, v.l), v.l * bt.mass + crossk(v.w, mc));
    SV<T> bias = crf(v, hv);
    if constexpr ((FEAT & FEAT_CONTACT) != 0) {
        if (bi.flags & F_EXTF) bias = bias - S.ext_get(bi);
    }
    pA = pA + bias;
    if (bi.flags & F_BRANCH) {
        const int s = bi.s_acc;
#pragma unroll
        for (int k = 0; k < 6; k++) I.a[k] = I.a[k] + S(s + k);
#pragma unroll
        for (int k = 0; k < 9; k++) I.h[k] = I.h[k] + S(s + 6 + k);
#pragma unroll
        for (int k = 0; k < 6; k++) I.m[k] = I.m[k] + S(s + 15 + k);
        pA = pA + ld_sv<T>(S, s + 21);
    }
    SV<T> c;
    if constexpr (AX >= 0) {
        const T qd = S(M.nv + bi.off);
        c = mksv<T>(cross_axis<AX>(v.w, qd), cross_axis<AX>(v.l, qd));
    } else {
        c = crm(v, joint_vel<AX, FEAT>(bi, bt, S, M.nv));
    }
    bool live = true;
    if (AX >= 0 || bi.ndof == 1) {
        V3<T> Uw, Ul;
        T sU, sp;
        if constexpr (AX >= 0) {
            unit_u<AX, true>(I, Uw, Ul, sU);
            sp = at<AX>(pA.w);
        } else {
            const V3<T> a = ld3(bt.axis);
            const bool hinge = bi.jtype == J_REVOLUTE;
            // U = I s: a column of the blocks for a coordinate axis (indices are
            // compile-time in every branch, so I stays in registers)
            switch (hinge ? bi.axis_k : bi.axis_k + 3) {
                case 0: unit_u<0, true>(I, Uw, Ul, sU); break;
                case 1: unit_u<1, true>(I, Uw, Ul, sU); break;
                case 2: unit_u<2, true>(I, Uw, Ul, sU); break;
                case 3: unit_u<0, false>(I, Uw, Ul, sU); break;
                case 4: unit_u<1, false>(I, Uw, Ul, sU); break;
                case 5: unit_u<2, false>(I, Uw, Ul, sU); break;
                default:
                    if (hinge) {
                        Uw = symv(I.a, a);
                        Ul = m3tv(I.h, a);
                        sU = dot(a, Uw);
                    } else {
                        Uw = m3v(I.h, a);
                        Ul = symv(I.m, a);
                        sU = dot(a, Ul);
                    }
                    break;
            }
            sp = hinge ? dot(a, pA.w) : dot(a, pA.l);
        }
        const T D = sU + bt.d_extra;
        const T u = dof_force<(FEAT & FEAT_IMPULSE) != 0>(M, bi, bt, S, 0, AX >= 0 || bi.ndof == 1) - sp;
        // aba.rs:240-242: a singular D skips the body (W = 0, w0 = 0). The
        // record store happens once, outside any per-world branch, because
        // a Tensor-Memory store is warp-wide.
        live = !(pz_abs(D) < T(1e-20));
        const T invD = live ? T(1) / D : T(0);
        if constexpr ((FEAT & FEAT_IMPULSE) != 0) S(bi.s_dinv) = invD;  // the sweeps' wrench response
        const V3<T> Ww = Uw * invD, Wl = Ul * invD;
        const T w0 = u * invD;
        if constexpr (AX >= 0)
            S.rec_put_vw(bi, mksv<T>(Ww, Wl));
        else
            st_sv(S, bi.s_vw, mksv<T>(Ww, Wl));
        S(bi.s_w0) = w0;
        {  // (a skipped body's contribution is dropped below; W = 0 keeps this exact)
            if (p >= 0) {
                // I <- I - W U^T (rank-1, symmetric)
#pragma unroll
                for (int r = 0; r < 3; r++)
#pragma unroll
                    for (int q = r; q < 3; q++) {
                        I.a[sidx(r, q)] = I.a[sidx(r, q)] - get(Ww, r) * get(Uw, q);
                        I.m[sidx(r, q)] = I.m[sidx(r, q)] - get(Wl, r) * get(Ul, q);
                    }
#pragma unroll
                for (int r = 0; r < 3; r++)
#pragma unroll
                    for (int q = 0; q < 3; q++) I.h[r * 3 + q] = I.h[r * 3 + q] - get(Ww, r) * get(Ul, q);
                SV<T> Ic;
                if constexpr (AX >= 0)
                    Ic = ai_mul_zk<AX>(I, c);
                else
                    Ic = ai_mul(I, c);
                pA = pA + Ic + mksv<T>(Uw * w0, Ul * w0);
            }
        }
    } else if constexpr (AX < 0) {
        if (bi.ndof > 1) {
            if constexpr ((FEAT & FEAT_MULTI) != 0) {
                SV<T> ag;
                const bool root = (bi.flags & F_ROOTQDD) != 0;
                if (root) {
                    const JX<T> jr = load_jx<AX, FEAT>(bi, bt, S);
                    ag = mot_X<AX, FEAT>(bi, bt, jr, mksv<T>(zero3<T>(), mk3<T>(-M.gx, -M.gy, -M.gz)));
                }
                if (bi.ndof == 3)
                    live = multi_dof<3, (FEAT & FEAT_IMPULSE) != 0>(M, bi, bt, S, I, pA, c, p >= 0,
                                                                    root ? &ag : nullptr);
                else
                    live = multi_dof<6, (FEAT & FEAT_IMPULSE) != 0>(M, bi, bt, S, I, pA, c, p >= 0,
                                                                    root ? &ag : nullptr);
            }
        }
    }
    if (p < 0) return;
    if (!live) {  // a skipped body passes nothing to its parent
        ai_zero(I);
        pA = zerosv<T>();
        return;
    }
    JX<T> j;
    if constexpr (AX >= 0) {
        j.c = rec.c;
        j.s = rec.s;
    } else {
        j = load_jx<AX, FEAT>(bi, bt, S);
    }
    ai_XtIX<AX, FEAT>(bi, bt, j, I);
    pA = frc_XT<AX, FEAT>(bi, bt, j, pA);
    if (p != i - 1) {
        const int s = M.bi[p].s_acc;
#pragma unroll
        for (int k = 0; k < 6; k++) S(s + k) = S(s + k) + I.a[k];
#pragma unroll
        for (int k = 0; k < 9; k++) S(s + 6 + k) = S(s + 6 + k) + I.h[k];
#pragma unroll
        for (int k = 0; k < 6; k++) S(s + 15 + k) = S(s + 15 + k) + I.m[k];
        const SV<T> old = ld_sv<T>(S, s + 21);
        st_sv(S, s + 21, old + pA);
    }
}

// ── pass 2: backward sweep ─────────────────────────────────────────────────
template <int FEAT, class T, class Scr>
PZ_HD void pass2(const ModelView<T>& M, const Scr& S) {
    // zero the stored accumulators of branch bodies
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
        if (bi.flags & F_BRANCH)
            for (int k = 0; k < 27; k++) S(bi.s_acc + k) = T(0);
    }
    AI<T> I;
    SV<T> pA = zerosv<T>();
    ai_zero(I);
    PZ_UNROLL_BODIES
    for (int i = M.nb - 1; i >= 0; i--) {
        const BodyI bi = M.bi[i];
#define PZ_P2(AX) pass2_body<AX, FEAT>(M, S, i, bi, I, pA)
        PZ_BY_KIND(body_kind(bi), PZ_P2)
#undef PZ_P2
    }
    S.fence_st();
}

// ── integrator of body i (integrate.rs:41-91), v first then q ─────────────
template <class T, class Scr>
PZ_HD void integrate_1dof(const ModelView<T>& M, const BodyI& bi, const Scr& S, const T& qdd) {
    const int o = bi.off, ov = M.nv + bi.off;
    const T vn = S(ov) + M.dt * qdd;
    S(ov) = vn;
    S(o) = S(o) + M.dt * vn;
}

// Multi-DOF accelerations qdd = w0 - W^T a, written into the w0 slots (the
// integrator reads them back), and a += S qdd. A root's w0 is its qdd
// already (F_ROOTQDD).
template <class T, class Scr>
PZ_HD void multi_qdd(const BodyI& bi, const Scr& S, SV<T>& a) {
    const int nd = bi.ndof;
    const bool root = (bi.flags & F_ROOTQDD) != 0;
    T q[6];
#pragma unroll
    for (int k = 0; k < 6; k++)
        q[k] = k < nd ? (root ? S(bi.s_w0 + k) : S(bi.s_w0 + k) - dot(ld_sv<T>(S, bi.s_vw + 6 * k), a)) : T(0);
#pragma unroll
    for (int k = 0; k < 6; k++)
        if (k < nd) S(bi.s_w0 + k) = q[k];
    a.w = a.w + mk3<T>(q[0], q[1], q[2]);
    if (nd == 6) a.l = a.l + mk3<T>(q[3], q[4], q[5]);
}

// Ball / free joint: exponential-map step of the rotation, body-frame linear
// velocity rotated into the parent for the free joint's position.
template <class T, class Scr>
PZ_HD void integrate_multi(const ModelView<T>& M, const BodyI& bi, const Scr& S, const Out<T>& qdd_out) {
    const int o = bi.off, ov = M.nv + bi.off;
    const T dt = M.dt;
    for (int k = 0; k < bi.ndof; k++) {
        const T qk = S(bi.s_w0 + k);
        qdd_out.put(bi.off + k, qk);
        S(ov + k) = S(ov + k) + dt * qk;
    }
    const V3<T> om = mk3<T>(S(ov), S(ov + 1), S(ov + 2));
    const Q4<T> cur = qexp(mk3<T>(S(o), S(o + 1), S(o + 2)));
    if (bi.jtype == J_FREE) {
        const V3<T> wl = qrotate(cur, mk3<T>(S(ov + 3), S(ov + 4), S(ov + 5)));
        S(o + 3) = S(o + 3) + dt * wl.x;
        S(o + 4) = S(o + 4) + dt * wl.y;
        S(o + 5) = S(o + 5) + dt * wl.z;
    }
    const Q4<T> nxt = qnormalize(qmul(cur, qexp(om * dt)));
    const V3<T> lg = qlog(nxt);
    S(o) = lg.x;
    S(o + 1) = lg.y;
    S(o + 2) = lg.z;
}

// ── pass 3 + integration of body i for the current step, fused with pass 1
// of the next (aba.rs:322-400, then integrate.rs, then aba.rs:175-213 and
// the contact pass). `next_step` < 0: the last step of the launch.
template <int AX, int FEAT, bool LAST, class T, class Scr>
PZ_HD void pass3_body(const ModelView<T>& M, const Scr& S, const WorldIO<T>& io, int i, const BodyI& bi,
                      int next_step, const Out<T>& qdd_out, SV<T>& cvo, SV<T>& ca, SV<T>& cvn, WF<T>& cw) {
    const BodyT<T>& bt = M.bt[i];
    const int p = bi.parent;
    JX<T> j;
    SV<T> Wv;
    if constexpr (AX >= 0) {
        const Rec<T> rec = S.rec_get(bi);
        j.c = rec.c;
        j.s = rec.s;
        Wv = rec.v;
    } else {
        j = load_jx<AX, FEAT>(bi, bt, S);
    }
    SV<T> vpo, apar;
    if (p < 0) {
        vpo = zerosv<T>();
        apar = mksv<T>(zero3<T>(), mk3<T>(-M.gx, -M.gy, -M.gz));
    } else if (p == i - 1) {
        vpo = cvo;
        apar = ca;
    } else {
        vpo = ld_sv<T>(S, M.bi[p].s_vold);
        apar = ld_sv<T>(S, M.bi[p].s_acca);
    }
    SV<T> vo, c;
    if constexpr (AX >= 0) {
        const T qd = S(M.nv + bi.off);
        vo = mot_X<AX, FEAT>(bi, bt, j, vpo);
        at<AX>(vo.w) = at<AX>(vo.w) + qd;
        c = mksv<T>(cross_axis<AX>(vo.w, qd), cross_axis<AX>(vo.l, qd));
    } else {
        const SV<T> vj = joint_vel<AX, FEAT>(bi, bt, S, M.nv);
        vo = mot_X<AX, FEAT>(bi, bt, j, vpo) + vj;
        c = crm(vo, vj);
    }
    SV<T> a = mot_X<AX, FEAT>(bi, bt, j, apar) + c;
    T qdd0 = T(0);
    if (AX >= 0 || bi.ndof == 1) {
        if constexpr (AX >= 0)
            qdd0 = S(bi.s_w0) - dot(Wv, a);
        else
            qdd0 = S(bi.s_w0) - dot(ld_sv<T>(S, bi.s_vw), a);
        if constexpr (AX >= 0) {
            at<AX>(a.w) = at<AX>(a.w) + qdd0;
        } else {
            const V3<T> ax = ld3(bt.axis);
            if (bi.jtype == J_REVOLUTE)
                a.w = a.w + ax * qdd0;
            else
                a.l = a.l + ax * qdd0;
        }
    } else if constexpr (AX < 0 && (FEAT & FEAT_MULTI) != 0) {
        if (bi.ndof > 1) multi_qdd(bi, S, a);
    }
    if (bi.flags & F_BRANCH) {
        st_sv(S, bi.s_vold, vo);
        st_sv(S, bi.s_acca, a);
    }
    cvo = vo;
    ca = a;
    if (AX >= 0 || bi.ndof == 1) {
        integrate_1dof(M, bi, S, qdd0);
        if constexpr (LAST) qdd_out.put(bi.off, qdd0);
    } else if constexpr (AX < 0 && (FEAT & FEAT_MULTI) != 0) {
        if (bi.ndof > 1) integrate_multi(M, bi, S, qdd_out);
    }
    if constexpr (!LAST) {
        if constexpr (AX >= 0)
            prefetch_control1<(FEAT & FEAT_IMPULSE) != 0, T, Scr, (FEAT & FEAT_LANES) != 0>(M, bi, S, io, next_step);
        else
            prefetch_controls<(FEAT & FEAT_IMPULSE) != 0, T, Scr, (FEAT & FEAT_LANES) != 0>(M, bi, S, io, next_step);
        pass1_body<AX, FEAT>(M, S, i, bi, cvn, cw);
    }
}

// LAST: the launch's final step (qdd written out, no next step); otherwise
// `next_step` is the step whose controls are prefetched and whose pass 1 runs.
template <int FEAT, bool LAST, class T, class Scr>
PZ_HD void pass3_next(const ModelView<T>& M, const Scr& S, const WorldIO<T>& io, int next_step,
                      const Out<T>& qdd_out) {
    SV<T> cvo = zerosv<T>(), ca = zerosv<T>(), cvn = zerosv<T>();
    WF<T> cw;
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
#define PZ_P3(AX) pass3_body<AX, FEAT, LAST>(M, S, io, i, bi, next_step, qdd_out, cvo, ca, cvn, cw)
        PZ_BY_KIND(body_kind(bi), PZ_P3)
#undef PZ_P3
    }
    S.fence_st();
}

// ── one impulse sweep, forward half (cuda/mod.rs:916-927; phyz_kernels.cu
// :1322-1368 then :804-918): body i's accelerations from the backward
// quantities in place (W of the step's backward sweep, w0 of the last
// wrench response), its free velocity X v_f,parent + S (qd + dt qdd), and --
// if collidable -- one staged impulse update whose wrench the next wrench
// response applies. The free velocity carries every impulse written so far
// through the whole articulated chain, which is what makes the iteration
// matrix-free.
template <int AX, int FEAT, class T, class Scr>
PZ_HD void sweep_body(const ModelView<T>& M, const Scr& S, int i, const BodyI& bi, SV<T>& cvo, SV<T>& ca,
                      SV<T>& cvf) {
    const BodyT<T>& bt = M.bt[i];
    const int p = bi.parent;
    JX<T> j;
    SV<T> Wv;
    if constexpr (AX >= 0) {
        const Rec<T> rec = S.rec_get(bi);
        j.c = rec.c;
        j.s = rec.s;
        Wv = rec.v;
    } else {
        j = load_jx<AX, FEAT>(bi, bt, S);
    }
    SV<T> vpo, apar, vfp;
    if (p < 0) {
        vpo = zerosv<T>();
        vfp = zerosv<T>();
        apar = mksv<T>(zero3<T>(), mk3<T>(-M.gx, -M.gy, -M.gz));
    } else if (p == i - 1) {
        vpo = cvo;
        apar = ca;
        vfp = cvf;
    } else {
        vpo = ld_sv<T>(S, M.bi[p].s_vold);
        apar = ld_sv<T>(S, M.bi[p].s_acca);
        vfp = ld_sv<T>(S, M.bi[p].s_vf);
    }
    SV<T> vo, c;
    if constexpr (AX >= 0) {
        const T qd = S(M.nv + bi.off);
        vo = mot_X<AX, FEAT>(bi, bt, j, vpo);
        at<AX>(vo.w) = at<AX>(vo.w) + qd;
        c = mksv<T>(cross_axis<AX>(vo.w, qd), cross_axis<AX>(vo.l, qd));
    } else {
        const SV<T> vj = joint_vel<AX, FEAT>(bi, bt, S, M.nv);
        vo = mot_X<AX, FEAT>(bi, bt, j, vpo) + vj;
        c = crm(vo, vj);
    }
    SV<T> a = mot_X<AX, FEAT>(bi, bt, j, apar) + c;
    SV<T> vf = mot_X<AX, FEAT>(bi, bt, j, vfp);
    if (AX >= 0 || bi.ndof == 1) {
        T qdd0;
        if constexpr (AX >= 0)
            qdd0 = S(bi.s_w0) - dot(Wv, a);
        else
            qdd0 = S(bi.s_w0) - dot(ld_sv<T>(S, bi.s_vw), a);
        const T u = S(M.nv + bi.off) + M.dt * qdd0;
        if constexpr (AX >= 0) {
            at<AX>(a.w) = at<AX>(a.w) + qdd0;
            at<AX>(vf.w) = at<AX>(vf.w) + u;
        } else {
            const V3<T> ax = ld3(bt.axis);
            if (bi.jtype == J_REVOLUTE) {
                a.w = a.w + ax * qdd0;
                vf.w = vf.w + ax * u;
            } else {
                a.l = a.l + ax * qdd0;
                vf.l = vf.l + ax * u;
            }
        }
    } else if constexpr (AX < 0 && (FEAT & FEAT_MULTI) != 0) {
        if (bi.ndof > 1) {
            multi_qdd(bi, S, a);  // qdd into the w0 slots
            const int o = M.nv + bi.off;
            vf.w = vf.w + mk3<T>(S(o) + M.dt * S(bi.s_w0), S(o + 1) + M.dt * S(bi.s_w0 + 1),
                                 S(o + 2) + M.dt * S(bi.s_w0 + 2));
            if (bi.ndof == 6)
                vf.l = vf.l + mk3<T>(S(o + 3) + M.dt * S(bi.s_w0 + 3), S(o + 4) + M.dt * S(bi.s_w0 + 4),
                                     S(o + 5) + M.dt * S(bi.s_w0 + 5));
        }
    }
    if (bi.flags & F_BRANCH) {
        st_sv(S, bi.s_vold, vo);
        st_sv(S, bi.s_acca, a);
    }
    if (bi.s_vf >= 0) st_sv(S, bi.s_vf, vf);  // a branch, or a body the plane pass reads
    cvo = vo;
    ca = a;
    cvf = vf;
    if (bi.flags & F_CONTACT) {
        constexpr bool TERRAIN = (FEAT & FEAT_TERRAIN) != 0;
        const int s = bi.s_up;
        WF<T> wf;
        if constexpr (TERRAIN) {
            wf.r0 = mk3<T>(S(s), S(s + 1), S(s + 2));
            wf.r1 = mk3<T>(S(s + 3), S(s + 4), S(s + 5));
            wf.up = mk3<T>(S(s + 6), S(s + 7), S(s + 8));
            wf.pos = mk3<T>(S(s + 9), S(s + 10), S(s + 11));
        } else {
            wf.up = mk3<T>(S(s), S(s + 1), S(s + 2));
            wf.pos.z = S(s + 3);
        }
        const SV<T> f = impulse_wrench<TERRAIN>(M.im, M.ter, bi, bt, wf, vf, S);
        st_sv(S, bi.s_f, f);
    }
}

// ── one impulse sweep, wrench response (replaces a full backward sweep) ──
// Between sweeps only the contact wrenches change, and the articulated-body
// recursion is linear in them: with the step's backward quantities kept
// (W = U D^-1 per body, D^-1 or the factor of D, w0 of the step), the change
// dF of the external wrenches moves the bias forces by dp = -dF plus the
// children's share, each joint's w0 by D^-1 (-S^T dp), and passes
// X^T (dp + W (-S^T dp)) to the parent. This is exactly the difference
// between the backward sweeps the reference reruns per sweep (aba.rs:215-320)
// with the old and the new wrenches, without their inertia work.
// The wrench response of a ball (ND 3) or free (ND 6) joint: D dw0 = du with
// D = L L^T (the factor kept by the backward sweep), w0 = w0_step + dw0, and
// dp += W du. Returns false for a body the backward sweep skipped.
template <int ND, class T, class Scr>
PZ_HD bool wrench_multi(const BodyI& bi, const Scr& S, SV<T>& dp) {
    T du[ND], x[ND];
#pragma unroll
    for (int k = 0; k < ND; k++) du[k] = -svget(dp, k);
    const bool live = pz_abs(S(bi.s_dinv)) > T(0);
    if (live) {
#pragma unroll
        for (int a = 0; a < ND; a++) {
            T e = du[a];
#pragma unroll
            for (int k = 0; k < a; k++) e = e - S(bi.s_dinv + a * (a + 1) / 2 + k) * x[k];
            x[a] = e * S(bi.s_dinv + a * (a + 1) / 2 + a);  // the stored diagonal is 1 / L_aa
        }
#pragma unroll
        for (int a = ND - 1; a >= 0; a--) {
            T e = x[a];
#pragma unroll
            for (int k = a + 1; k < ND; k++) e = e - S(bi.s_dinv + k * (k + 1) / 2 + a) * x[k];
            x[a] = e * S(bi.s_dinv + a * (a + 1) / 2 + a);
        }
    }
#pragma unroll
    for (int k = 0; k < ND; k++) {
        S(bi.s_w0 + k) = S(bi.s_w0b + k) + (live ? x[k] : T(0));
        if (!(bi.flags & F_ROOTQDD)) {  // a root passes nothing on (and has no W)
            const SV<T> wk = ld_sv<T>(S, bi.s_vw + 6 * k);
            dp = dp + mksv<T>(wk.w * du[k], wk.l * du[k]);
        }
    }
    return live;
}

template <int AX, int FEAT, class T, class Scr>
PZ_HD void wrench_body(const ModelView<T>& M, const Scr& S, int i, const BodyI& bi, SV<T>& dp) {
    const BodyT<T>& bt = M.bt[i];
    const int p = bi.parent;
    if (!(bi.flags & F_CHAIN)) dp = zerosv<T>();
    if (bi.flags & F_EXTF) dp = dp - (ld_sv<T>(S, bi.s_f) - ld_sv<T>(S, bi.s_fp));
    if (bi.flags & F_BRANCH) dp = dp + ld_sv<T>(S, bi.s_acc + 21);
    JX<T> j;
    SV<T> Wv;
    if constexpr (AX >= 0) {
        const Rec<T> rec = S.rec_get(bi);
        j.c = rec.c;
        j.s = rec.s;
        Wv = rec.v;
    } else {
        j = load_jx<AX, FEAT>(bi, bt, S);
    }
    bool live = true;
    if (AX >= 0 || bi.ndof == 1) {
        T du;
        if constexpr (AX >= 0) {
            du = -at<AX>(dp.w);
        } else {
            Wv = ld_sv<T>(S, bi.s_vw);
            const V3<T> a = ld3(bt.axis);
            du = -(bi.jtype == J_REVOLUTE ? dot(a, dp.w) : dot(a, dp.l));
        }
        const T invD = S(bi.s_dinv);
        S(bi.s_w0) = S(bi.s_w0b) + invD * du;
        live = pz_abs(invD) > T(0);
        dp = dp + mksv<T>(Wv.w * du, Wv.l * du);
    } else if constexpr (AX < 0 && (FEAT & FEAT_MULTI) != 0) {
        if (bi.ndof == 3)
            live = wrench_multi<3>(bi, S, dp);
        else if (bi.ndof == 6)
            live = wrench_multi<6>(bi, S, dp);
    }
    if (p < 0) return;
    dp = live ? frc_XT<AX, FEAT>(bi, bt, j, dp) : zerosv<T>();  // a skipped body passes nothing
    if (p != i - 1) {
        const int s = M.bi[p].s_acc + 21;
        st_sv(S, s, ld_sv<T>(S, s) + dp);
    }
}

template <int FEAT, class T, class Scr>
PZ_HD void wrench_response(const ModelView<T>& M, const Scr& S) {
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
        if (bi.flags & F_BRANCH)
            for (int k = 0; k < 6; k++) S(bi.s_acc + 21 + k) = T(0);
    }
    SV<T> dp = zerosv<T>();
    PZ_UNROLL_BODIES
    for (int i = M.nb - 1; i >= 0; i--) {
        const BodyI bi = M.bi[i];
#define PZ_WR(AX) wrench_body<AX, FEAT>(M, S, i, bi, dp)
        PZ_BY_KIND(body_kind(bi), PZ_WR)
#undef PZ_WR
    }
}

// The step's backward quantities the wrench responses start from: w0 and
// the wrenches it applied.
template <class T, class Scr>
PZ_HD void keep_backward_state(const ModelView<T>& M, const Scr& S) {
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
        for (int k = 0; k < bi.ndof; k++) S(bi.s_w0b + k) = S(bi.s_w0 + k);
        if (bi.flags & F_EXTF)
            for (int k = 0; k < 6; k++) S(bi.s_fp + k) = S(bi.s_f + k);
    }
}

template <int FEAT, class T, class Scr>
PZ_HD void sweep_forward(const ModelView<T>& M, const Scr& S) {
    SV<T> cvo = zerosv<T>(), ca = zerosv<T>(), cvf = zerosv<T>();
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
#define PZ_SW(AX) sweep_body<AX, FEAT>(M, S, i, bi, cvo, ca, cvf)
        PZ_BY_KIND(body_kind(bi), PZ_SW)
#undef PZ_SW
    }
    S.fence_st();
}

// The initial pass 1 over the state loaded at the start of a launch.
template <int FEAT, class T, class Scr>
PZ_HD void pass1_all(const ModelView<T>& M, const Scr& S) {
    SV<T> cv = zerosv<T>();
    WF<T> cw;
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
#define PZ_P1(AX) pass1_body<AX, FEAT>(M, S, i, bi, cv, cw)
        PZ_BY_KIND(body_kind(bi), PZ_P1)
#undef PZ_P1
    }
    S.fence_st();
}

}  // namespace pz
