// Host-side packing of a phyzb_model into the device model table
// (pz_model.cuh), including the per-world scratch layout. Host C++ only.
//
// The field semantics are those of phyz's pack_bodies / pack_geometries
// (crates/phyz-gpu/src/layout.rs:103-279); values are kept in the
// simulator's precision (f32 or f64) instead of always f32.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/phyzb.h"
#include "pz_model.cuh"

namespace pz {

inline int ndof_of(int jt) {
    switch (jt) {
        case J_REVOLUTE:
        case J_PRISMATIC: return 1;
        case J_BALL: return 3;
        case J_FREE: return 6;
        default: return 0;
    }
}

inline bool finite_all(const double* p, int n) {
    for (int k = 0; k < n; k++)
        if (!std::isfinite(p[k])) return false;
    return true;
}

// Checks the reference applies at construction (cuda/mod.rs:499-510: body
// limit, nq == nv) plus what this kernel relies on: topological order,
// known codes, finite parameters. Returns "" when the model is usable.
inline std::string validate_model(const phyzb_model* m, int* nv_out) {
    if (!m || !m->bodies) return "model is null";
    if (m->nbodies < 1) return "model has no bodies";
    if (m->nbodies > PHYZB_MAX_BODIES)
        return "model has " + std::to_string(m->nbodies) + " bodies but the kernels hold at most " +
               std::to_string(PHYZB_MAX_BODIES) + " per world";
    if (!finite_all(m->gravity, 3) || !std::isfinite(m->dt) || !(m->dt > 0.0))
        return "gravity and dt must be finite, dt > 0";
    int nv = 0;
    for (int i = 0; i < m->nbodies; i++) {
        const phyzb_body& b = m->bodies[i];
        const std::string at = "body " + std::to_string(i) + ": ";
        if (b.parent < -1 || b.parent >= i) return at + "parent must be -1 or an earlier body (topological order)";
        if (b.joint_type < 0 || b.joint_type > 4) return at + "unknown joint type " + std::to_string(b.joint_type);
        if (b.geom_type < 0 || b.geom_type > 5) return at + "unknown geometry type " + std::to_string(b.geom_type);
        const double* groups[] = {b.com, b.inertia, b.ptj_rot, b.ptj_pos, b.axis, b.geom_params, b.geom_origin_pos,
                                  b.geom_origin_rot};
        const int sizes[] = {3, 6, 9, 3, 3, 6, 3, 9};
        for (int g = 0; g < 8; g++)
            if (!finite_all(groups[g], sizes[g])) return at + "non-finite parameter";
        const double sc[] = {b.mass, b.damping, b.stiffness, b.spring_ref, b.armature, b.friction_loss};
        if (!finite_all(sc, 6)) return at + "non-finite parameter";
        if (b.has_limits &&
            !(std::isfinite(b.limit_lower) && std::isfinite(b.limit_upper) && std::isfinite(b.limit_stiffness) &&
              std::isfinite(b.limit_damping)))
            return at + "non-finite joint limit";
        nv += ndof_of(b.joint_type);
    }
    if (nv > PHYZB_MAX_DOFS)
        return "model has " + std::to_string(nv) + " DOFs; at most " + std::to_string(PHYZB_MAX_DOFS) + " supported";
    if (nv_out) *nv_out = nv;
    return "";
}

struct PackInfo {
    int off_bi = 0, off_pd = 0, off_pdmap = 0, bytes = 0;
    int scratch = 0;     // scratch slots per world
    int collidable = 0;  // bodies with a contact shape
    int feat = 0;        // kernel variant: 1 = ball/free joints, 2 = contact on, 4 = relabelled hinges,
                         // 8 = (with 4) every relabel is the shift-1 cycle, 16 = (with 2) impulse contact,
                         // 32 = (with 2) full world frames (heightfield / body plane)
    int tmem_cols = 0;   // Tensor Memory columns per world holding body records (0: none)
    int imp_slots = 0;   // impulse mode: rows per world of the persistent wrench + impulse buffer
};

inline int pad16(int b) { return (b + 15) & ~15; }

// Contact and PD settings that change the table.
struct PackCfg {
    bool contact = false;
    bool impulse = false;                // contact as the velocity-level impulse solve
    bool terrain = false;                // full world frames: a heightfield and/or a body plane
    int plane_body = -1;                 // body carrying a contact plane (-1: none)
    std::vector<int> plane_exclude;      // bodies that never touch the plane
    std::vector<double> gk, gd;          // per-body penalty gains (contact)
    std::vector<phyzb_pd_dof> pd;        // PD servos
    // one lane's part of a model split over several threads per world
    // (pz_lanes.h): bodies that keep branch slots whatever their children,
    // and a body whose chain flag is set whatever its next body
    std::vector<int> force_branch;
    int force_chain = -1;
};

// A body whose per-step record [cos, sin, velocity | W] can live in Tensor
// Memory: a hinge about exactly +e_k with an unrotated parent->joint frame
// (the kernel's compile-time body kinds).
inline bool tmem_kind(const phyzb_body& b) {
    if (b.joint_type != J_REVOLUTE) return false;
    const double* R = b.ptj_rot;
    if (!(R[0] == 1.0 && R[1] == 0.0 && R[2] == 0.0 && R[3] == 0.0 && R[4] == 1.0 && R[5] == 0.0 && R[6] == 0.0 &&
          R[7] == 0.0 && R[8] == 1.0))
        return false;
    for (int k = 0; k < 3; k++) {
        bool unit = true;
        for (int q = 0; q < 3; q++) unit = unit && (b.axis[q] == (q == k ? 1.0 : 0.0));
        if (unit) return true;
    }
    return false;
}

// Coordinate relabelling of each body frame (pz_model.cuh): shift s with
// (P_s v)_a = v_(a+s mod 3). A hinge about e_x gets s = 1, about e_y s = 2
// (both map the axis to e_z); every other body keeps s = 0.
inline int frame_shift(const phyzb_body& b) {
    if (!tmem_kind(b)) return 0;
    return b.axis[0] == 1.0 ? 1 : (b.axis[1] == 1.0 ? 2 : 0);
}

// The model with every body-frame constant expressed in the relabelled
// frames: com, COM inertia, axis, geometry origin (P_i), the parent->joint
// offset in the parent's frame (P_p), and the parent->joint rotation
// P_i R P_p^T (for a relabelled hinge the cyclic permutation P_(s_i - s_p)).
inline std::vector<phyzb_body> relabel_frames(const phyzb_model* m, std::vector<int>& shift) {
    const int nb = m->nbodies;
    std::vector<phyzb_body> out(m->bodies, m->bodies + nb);
    shift.assign(nb, 0);
    for (int i = 0; i < nb; i++) shift[i] = frame_shift(m->bodies[i]);
    auto pv = [](const double* v, int s, double* o) {
        double t[3];
        for (int a = 0; a < 3; a++) t[a] = v[(a + s) % 3];
        for (int a = 0; a < 3; a++) o[a] = t[a];
    };
    for (int i = 0; i < nb; i++) {
        const phyzb_body& b = m->bodies[i];
        phyzb_body& o = out[i];
        const int si = shift[i], sp = b.parent >= 0 ? shift[b.parent] : 0;
        pv(b.com, si, o.com);
        pv(b.axis, si, o.axis);
        pv(b.geom_origin_pos, si, o.geom_origin_pos);
        pv(b.ptj_pos, sp, o.ptj_pos);
        // COM inertia P I P^T: I'_rc = I_(r+s)(c+s)
        const double* J = b.inertia;
        const double full[9] = {J[0], J[3], J[4], J[3], J[1], J[5], J[4], J[5], J[2]};
        auto f = [&](int r, int c) { return full[((r + si) % 3) * 3 + (c + si) % 3]; };
        o.inertia[0] = f(0, 0);
        o.inertia[1] = f(1, 1);
        o.inertia[2] = f(2, 2);
        o.inertia[3] = f(0, 1);
        o.inertia[4] = f(0, 2);
        o.inertia[5] = f(1, 2);
        // parent->joint rotation P_i R P_p^T: R'_rc = R_(r+si)(c+sp)
        for (int r = 0; r < 3; r++)
            for (int c = 0; c < 3; c++) o.ptj_rot[r * 3 + c] = b.ptj_rot[((r + si) % 3) * 3 + (c + sp) % 3];
        // geometry rotation (body -> geometry) O P_i^T: O'_rc = O_r(c+si)
        for (int r = 0; r < 3; r++)
            for (int c = 0; c < 3; c++)
                o.geom_origin_rot[r * 3 + c] = b.geom_origin_rot[r * 3 + (c + si) % 3];
    }
    return out;
}

// `tmem_budget` > 0: place the records of all tmem_kind bodies in Tensor
// Memory columns (8 words per record in f32, 16 in f64) if they all fit the
// budget (else none: info.tmem_cols = 0); their s_xj / s_vw slots are then
// not allocated in shared memory. The collidable bodies' contact wrenches
// follow them there when all of them fit too (penalty contact, no body
// plane), and then have no s_f slot.
template <class T>
inline PackInfo pack_model(const phyzb_model* m, int nv, const PackCfg& cfg, std::vector<unsigned char>& blob,
                           int tmem_budget = 0) {
    const int nb = m->nbodies;
    const int npd = (int)cfg.pd.size();
    PackInfo info;
    const int szT = pad16((int)sizeof(BodyT<T>) * nb);
    const int szI = pad16((int)sizeof(BodyI) * nb);
    const int szP = pad16((int)sizeof(PdT<T>) * (npd > 0 ? npd : 1));
    const int szM = pad16((int)sizeof(int) * (nv > 0 ? nv : 1));
    info.off_bi = szT;
    info.off_pd = szT + szI;
    info.off_pdmap = szT + szI + szP;
    info.bytes = szT + szI + szP + szM;
    blob.assign(info.bytes, 0);
    BodyT<T>* bt = reinterpret_cast<BodyT<T>*>(blob.data());
    BodyI* bi = reinterpret_cast<BodyI*>(blob.data() + info.off_bi);
    PdT<T>* pd = reinterpret_cast<PdT<T>*>(blob.data() + info.off_pd);
    int* pdmap = reinterpret_cast<int*>(blob.data() + info.off_pdmap);

    std::vector<int> shift;
    const std::vector<phyzb_body> rb = relabel_frames(m, shift);
    // a Tensor-Memory layout holds the records of every relabelled hinge
    // (the kernel then accesses them without a per-body test) or none
    // and, when they fit beside those, the external wrenches of the
    // collidable bodies (penalty contact without a body plane: each wrench is
    // stored once per step by the forward sweep and read once by the
    // backward sweep), all of them or none
    bool tmem_wrench = false;
    {
        const int rec = 8 * (int)(sizeof(T) / 4);
        int need = 0, wneed = 0;
        for (int i = 0; i < nb; i++) {
            if (tmem_kind(m->bodies[i])) need += rec;
            if (m->bodies[i].geom_type != 0) wneed += rec;
        }
        if (need > tmem_budget) tmem_budget = 0;
        tmem_wrench = tmem_budget > 0 && cfg.contact && !cfg.impulse && cfg.plane_body < 0 && wneed > 0 &&
                      need + wneed <= tmem_budget;
    }
    int next = 2 * nv;  // q, v
    int off = 0;
    for (int i = 0; i < nb; i++) {
        const phyzb_body& b = rb[i];
        BodyT<T>& t = bt[i];
        BodyI& d = bi[i];
        const int nd = ndof_of(b.joint_type);
        d.parent = b.parent;
        d.jtype = b.joint_type;
        d.off = off;
        d.ndof = nd;
        off += nd;
        // mass properties: I_o = I_c + m (|c|^2 1 - c c^T)  (phyz_kernels.cu:332-359)
        const double mass = b.mass, cx = b.com[0], cy = b.com[1], cz = b.com[2];
        t.mass = T(mass);
        t.mcom[0] = T(mass * cx);
        t.mcom[1] = T(mass * cy);
        t.mcom[2] = T(mass * cz);
        t.Io[0] = T(b.inertia[0] + mass * (cy * cy + cz * cz));
        t.Io[1] = T(b.inertia[1] + mass * (cx * cx + cz * cz));
        t.Io[2] = T(b.inertia[2] + mass * (cx * cx + cy * cy));
        t.Io[3] = T(b.inertia[3] - mass * cx * cy);
        t.Io[4] = T(b.inertia[4] - mass * cx * cz);
        t.Io[5] = T(b.inertia[5] - mass * cy * cz);
        for (int k = 0; k < 3; k++) t.com[k] = T(b.com[k]);
        for (int k = 0; k < 9; k++) t.ptj_rot[k] = T(b.ptj_rot[k]);
        for (int k = 0; k < 3; k++) t.ptj_pos[k] = T(b.ptj_pos[k]);
        for (int k = 0; k < 3; k++) t.axis[k] = T(b.axis[k]);
        t.damping = T(b.damping);
        t.stiffness = T(b.stiffness);
        t.spring_ref = T(b.spring_ref);
        t.armature = T(b.armature);
        t.d_extra = T(b.armature + m->dt * b.damping);
        t.lim_lo = T(b.limit_lower);
        t.lim_hi = T(b.limit_upper);
        t.lim_k = T(b.limit_stiffness);
        t.lim_d = T(b.limit_damping);
        t.fric = T(b.friction_loss);
        // COM inverse inertia by cofactors (phyz_kernels.cu:545-561)
        {
            const double xx = b.inertia[0], yy = b.inertia[1], zz = b.inertia[2];
            const double xy = b.inertia[3], xz = b.inertia[4], yz = b.inertia[5];
            const double c00 = yy * zz - yz * yz, c01 = xz * yz - xy * zz, c02 = xy * yz - xz * yy;
            const double det = xx * c00 + xy * c01 + xz * c02;
            double inv[6] = {0, 0, 0, 0, 0, 0};
            if (std::fabs(det) >= 1e-20) {
                const double c11 = xx * zz - xz * xz, c12 = xy * xz - xx * yz, c22 = xx * yy - xy * xy;
                const double r = 1.0 / det;
                inv[0] = c00 * r;
                inv[1] = c11 * r;
                inv[2] = c22 * r;
                inv[3] = c01 * r;
                inv[4] = c02 * r;
                inv[5] = c12 * r;
            }
            for (int k = 0; k < 6; k++) t.Icinv[k] = T(inv[k]);
        }
        for (int k = 0; k < 6; k++) t.geom[k] = T(b.geom_params[k]);
        for (int k = 0; k < 3; k++) t.gpos[k] = T(b.geom_origin_pos[k]);
        for (int k = 0; k < 9; k++) t.grot[k] = T(b.geom_origin_rot[k]);
        t.gk = T(cfg.contact && (int)cfg.gk.size() > i ? cfg.gk[i] : 0.0);
        t.gd = T(cfg.contact && (int)cfg.gd.size() > i ? cfg.gd[i] : 0.0);

        // structure flags
        int flags = 0;
        const double* R = b.ptj_rot;
        const bool rot_id = R[0] == 1.0 && R[1] == 0.0 && R[2] == 0.0 && R[3] == 0.0 && R[4] == 1.0 &&
                            R[5] == 0.0 && R[6] == 0.0 && R[7] == 0.0 && R[8] == 1.0;
        if (!rot_id) flags |= F_PTJ_ROT;
        if (b.ptj_pos[0] != 0.0 || b.ptj_pos[1] != 0.0 || b.ptj_pos[2] != 0.0) flags |= F_PTJ_POS;
        if (nd == 1 && b.has_limits) flags |= F_LIMITS;
        if (nd == 1 && b.friction_loss > 0.0) flags |= F_FRICTION;
        if (nd == 1 && b.stiffness != 0.0) flags |= F_SPRING;
        d.axis_k = -1;
        if (nd == 1)
            for (int k = 0; k < 3; k++) {
                bool unit = true;
                for (int q = 0; q < 3; q++) unit = unit && (b.axis[q] == (q == k ? 1.0 : 0.0));
                if (unit) d.axis_k = k;
            }
        d.qshift = 0;
        d.fshift = shift[i];
        if (tmem_kind(m->bodies[i])) {
            flags |= F_ZHINGE;
            d.qshift = (shift[i] - (b.parent >= 0 ? shift[b.parent] : 0) + 3) % 3;
        }
        if (i + 1 < nb && m->bodies[i + 1].parent == i) flags |= F_CHAIN;
        if (i == cfg.force_chain) flags |= F_CHAIN;
        if (nd > 1 && b.parent < 0) flags |= F_ROOTQDD;
        for (int j = i + 2; j < nb; j++)
            if (m->bodies[j].parent == i) flags |= F_BRANCH;
        if (std::find(cfg.force_branch.begin(), cfg.force_branch.end(), i) != cfg.force_branch.end())
            flags |= F_BRANCH;
        d.gtype = b.geom_type;
        if (b.geom_type != 0) info.collidable++;

        // scratch layout of this body
        const int rec_cols = 8 * (int)(sizeof(T) / 4);
        d.t_rec = -1;
        if (tmem_budget > 0 && (flags & F_ZHINGE) && info.tmem_cols + rec_cols <= tmem_budget) {
            d.t_rec = info.tmem_cols;
            info.tmem_cols += rec_cols;
            d.s_xj = d.s_vw = -1;
        } else {
            d.s_xj = next;
            next += b.joint_type == J_REVOLUTE ? 2 : ((b.joint_type == J_BALL || b.joint_type == J_FREE) ? 9 : 0);
            d.s_vw = next;
            next += nd > 1 ? 6 * nd : 6;
        }
        d.s_w0 = next;
        next += nd;
        const bool impulse = cfg.contact && cfg.impulse;
        d.s_in = d.s_w0;
        d.s_dinv = d.s_w0b = d.s_fp = -1;
        if (impulse) {
            // the sweeps rewrite w0 from the step's own (s_w0b) plus the
            // response to the wrench change, through D^-1 (s_dinv)
            d.s_w0b = next;
            next += nd;
            d.s_dinv = next;
            next += nd > 1 ? nd * (nd + 1) / 2 : 1;
        }
        d.s_f = d.s_up = d.s_imp = d.s_vf = d.c_imp = d.s_pimp = -1;
        const bool plane = cfg.contact && cfg.plane_body >= 0;
        const bool on_plane = plane && b.geom_type != 0 && i != cfg.plane_body &&
                              std::find(cfg.plane_exclude.begin(), cfg.plane_exclude.end(), i) ==
                                  cfg.plane_exclude.end();
        const bool is_pb = plane && i == cfg.plane_body;
        const int npts = b.geom_type == 2 ? 8 : 1;
        d.t_f = -1;
        if (cfg.contact && b.geom_type != 0) {
            flags |= F_CONTACT | F_EXTF;
            if (tmem_wrench) {
                d.t_f = info.tmem_cols;
                info.tmem_cols += rec_cols;
            } else {
                d.s_f = next;
                next += 6;
            }
            if (impulse) {
                d.s_fp = next;
                next += 6;
            }
            if (impulse) {
                d.s_up = next;
                next += cfg.terrain ? 12 : 4;
                d.s_imp = next;
                next += 3 * npts;
                d.c_imp = info.imp_slots;
                info.imp_slots += 6 + 3 * npts;
            }
        } else if (is_pb) {  // the plane's body takes the reaction even without a shape
            flags |= F_EXTF;
            d.s_f = next;
            next += 6;
            if (impulse) {
                d.s_fp = next;
                next += 6;
            }
            if (impulse) {
                d.c_imp = info.imp_slots;
                info.imp_slots += 6;
            }
        }
        if (on_plane) {
            flags |= F_PLANE;
            if (impulse) {
                d.s_pimp = next;
                next += 3 * npts;
                info.imp_slots += 3 * npts;  // after the ground impulses in the persistent rows
            }
        }
        if (impulse && (on_plane || is_pb)) {
            d.s_vf = next;  // the plane pass reads both bodies' free velocities
            next += 6;
        }
        d.s_acc = d.s_vold = d.s_acca = d.s_wx = -1;
        if (flags & F_BRANCH) {
            d.s_acc = next;
            next += 27;
            d.s_vold = next;
            next += 6;
            d.s_acca = next;
            next += 6;
            if (cfg.contact) {
                d.s_wx = next;  // world up (3) and origin height (1), or the full frame (12)
                next += cfg.terrain ? 12 : 4;
            }
            if (impulse && d.s_vf < 0) {
                d.s_vf = next;
                next += 6;
            }
        }
        d.flags = flags;
    }
    for (int j = 0; j < nv; j++) pdmap[j] = -1;
    for (int k = 0; k < npd; k++) {
        pd[k].kp = T(cfg.pd[k].kp);
        pd[k].kd = T(cfg.pd[k].kd);
        pd[k].maxf = T(cfg.pd[k].max_force);
        pd[k].qi = cfg.pd[k].q_index;
        pd[k].vi = cfg.pd[k].v_index;
        pdmap[cfg.pd[k].v_index] = k;
    }
    for (int i = 0; i < nb; i++)
        for (int k = 0; k < bi[i].ndof; k++)
            if (pdmap[bi[i].off + k] >= 0) bi[i].flags |= F_PD;
    info.scratch = next;
    for (int i = 0; i < nb; i++)
        if (m->bodies[i].joint_type == J_BALL || m->bodies[i].joint_type == J_FREE) info.feat |= 1;
    if (cfg.contact) info.feat |= 2;
    if (cfg.contact && cfg.impulse) info.feat |= 16;
    if (cfg.contact && cfg.terrain) info.feat |= 32;
    bool all_one = true;
    for (int i = 0; i < nb; i++)
        if (bi[i].flags & F_ZHINGE) {
            if (bi[i].qshift != 0) info.feat |= 4;
            all_one = all_one && bi[i].qshift == 1;
        }
    if ((info.feat & 4) && all_one) info.feat |= 8;  // every relabel is the shift-1 cycle
    return info;
}

// Algorithmic flop count of one steady-state world-step (flops.cpp).
struct FlopCount {
    double flops = 0, transcendentals = 0;
};
// `sweeps`: contact sweeps per step when cfg.impulse.
FlopCount count_world_step(const phyzb_model* m, int nv, const PackCfg& cfg, int sweeps = 0);
// The flops a rollout executes per world-step, averaged over `nworld`
// worlds (host rows q, v [nworld][nv]; ctrl [nsteps][nworld][nv] or null)
// stepped `nsteps` steps on the flat ground at `ground_h` (the contact force
// law counted where a body touches); `specialized`: products with zero
// table constants left out as a model-specialized kernel leaves them out.
FlopCount count_rollout(const phyzb_model* m, int nv, const PackCfg& cfg, int sweeps, double ground_h,
                        double friction, double erp, const double* q, const double* v, const double* ctrl,
                        long long nworld, int nsteps, bool specialized);

}  // namespace pz
