// TEST INFRASTRUCTURE ONLY — extern "C" face of the f64 CPU oracle
// (phyz_oracle.hpp), loaded by tests/ through ctypes. Batched over worlds,
// world-major rows as phyz's State packs them (layout.rs:340-372), with the
// worlds split across std::threads when asked.
#include <algorithm>
#include <thread>
#include <vector>

#include "phyz_oracle.hpp"

using namespace phyz_oracle;

namespace {

template <class F>
void parallel_worlds(int64_t nworld, int nthreads, F f) {
    if (nthreads <= 1 || nworld < 2) {
        f((int64_t)0, nworld);
        return;
    }
    int nt = (int)std::min<int64_t>(nthreads, nworld);
    std::vector<std::thread> pool;
    int64_t chunk = (nworld + nt - 1) / nt;
    for (int t = 0; t < nt; t++) {
        int64_t a = t * chunk, b = std::min(nworld, a + chunk);
        if (a >= b) break;
        pool.emplace_back([=] { f(a, b); });
    }
    for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

int oracle_abi_version(void) { return 1; }

// Forward dynamics only: qdd[w] = ABA(q[w], v[w], ctrl[w], ext[w]).
// ext: nworld x nb x 6 body-frame [torque; force] or NULL.
int oracle_aba(const phyzb_model* fm, int64_t nworld, const double* q, const double* v,
               const double* ctrl, const double* ext, double* qdd) {
    Model m = from_flat(fm);
    int nb = m.nb();
    for (int64_t w = 0; w < nworld; w++) {
        std::vector<SVec> e;
        if (ext) {
            e.resize(nb);
            for (int i = 0; i < nb; i++) {
                const double* p = ext + (w * nb + i) * 6;
                e[i] = SVec{v3(p[0], p[1], p[2]), v3(p[3], p[4], p[5])};
            }
        }
        std::vector<double> r = aba(m, q + w * m.nv, v + w * m.nv, ctrl ? ctrl + w * m.nv : nullptr,
                                    ext ? e.data() : nullptr);
        std::copy(r.begin(), r.end(), qdd + w * m.nv);
    }
    return 0;
}

// Inverse dynamics: tau[w] = RNEA(q[w], v[w], qdd[w]).
int oracle_rnea(const phyzb_model* fm, int64_t nworld, const double* q, const double* v,
                const double* qdd, double* tau) {
    Model m = from_flat(fm);
    for (int64_t w = 0; w < nworld; w++) {
        std::vector<double> r = rnea(m, q + w * m.nv, v + w * m.nv, qdd + w * m.nv);
        std::copy(r.begin(), r.end(), tau + w * m.nv);
    }
    return 0;
}

// integrate_configuration over worlds (q updated in place).
int oracle_integrate_configuration(const phyzb_model* fm, int64_t nworld, double* q,
                                   const double* v, double dt) {
    Model m = from_flat(fm);
    for (int64_t w = 0; w < nworld; w++) integrate_configuration(m, q + w * m.nq, v + w * m.nv, dt);
    return 0;
}

// Body world poses: xw = nworld x nb x 12 (world->body rot row-major, origin).
int oracle_forward_kinematics(const phyzb_model* fm, int64_t nworld, const double* q,
                              const double* v, double* xw_out, double* vel_out) {
    Model m = from_flat(fm);
    int nb = m.nb();
    for (int64_t w = 0; w < nworld; w++) {
        std::vector<SXform> xw;
        std::vector<SVec> vel;
        forward_kinematics(m, q + w * m.nq, v + w * m.nv, xw, vel);
        for (int i = 0; i < nb; i++) {
            double* o = xw_out + (w * nb + i) * 12;
            for (int k = 0; k < 9; k++) o[k] = xw[i].rot.m[k];
            o[9] = xw[i].pos.x;
            o[10] = xw[i].pos.y;
            o[11] = xw[i].pos.z;
            if (vel_out) {
                double* vo = vel_out + (w * nb + i) * 6;
                vo[0] = vel[i].ang.x;
                vo[1] = vel[i].ang.y;
                vo[2] = vel[i].ang.z;
                vo[3] = vel[i].lin.x;
                vo[4] = vel[i].lin.y;
                vo[5] = vel[i].lin.z;
            }
        }
    }
    return 0;
}

// Kinetic and potential energy per world.
int oracle_energy(const phyzb_model* fm, int64_t nworld, const double* q, const double* v,
                  double* ke, double* pe) {
    Model m = from_flat(fm);
    for (int64_t w = 0; w < nworld; w++) {
        if (ke) ke[w] = kinetic_energy(m, q + w * m.nq, v + w * m.nv);
        if (pe) pe[w] = potential_energy(m, q + w * m.nq);
    }
    return 0;
}

// Penalty contact forces only: ext = nworld x nb x 6, cstate = nworld x nb x 8.
// The heightfield the following contact rollouts sample (nx == 0: none, the
// flat plane at their ground height). Test-only process state.
static Terrain g_terrain;
static Plane g_plane;

// The body-attached plane of the following contact rollouts (body < 0:
// none); `exclude` lists bodies that never touch it.
int oracle_set_plane(int32_t body, double offset, double max_depth, double half_x, double half_y,
                     const int32_t* exclude, int32_t n_exclude, int32_t nb) {
    g_plane = Plane{};
    g_plane.body = body;
    g_plane.offset = offset;
    g_plane.max_depth = max_depth;
    g_plane.half_x = half_x;
    g_plane.half_y = half_y;
    g_plane.no_plane.assign(nb > 0 ? nb : 0, 0);
    for (int k = 0; k < n_exclude; k++)
        if (exclude[k] >= 0 && exclude[k] < nb) g_plane.no_plane[exclude[k]] = 1;
    if (body >= 0 && body < nb) g_plane.no_plane[body] = 1;
    return 0;
}

int oracle_set_heightfield(int32_t nx, int32_t ny, double ox, double oy, double oz, double cell,
                           const float* heights) {
    g_terrain = Terrain{};
    if (nx > 0) {
        g_terrain.nx = nx;
        g_terrain.ny = ny;
        g_terrain.ox = ox;
        g_terrain.oy = oy;
        g_terrain.oz = oz;
        g_terrain.cell = cell;
        g_terrain.h.assign(heights, heights + (size_t)nx * ny);
    }
    return 0;
}

// Height and unit normal of the current terrain at world (x, y).
double oracle_terrain_at(double x, double y, double* n_out) {
    Vec3 n;
    const double h = g_terrain.sample(x, y, n);
    n_out[0] = n.x;
    n_out[1] = n.y;
    n_out[2] = n.z;
    return h;
}

int oracle_penalty_contact(const phyzb_model* fm, int64_t nworld, const double* q,
                           const double* v, double ground_height, double friction,
                           const double* k, const double* d, double* ext_out,
                           double* cstate_out) {
    Model m = from_flat(fm);
    int nb = m.nb();
    ContactParams cp;
    cp.ground_height = ground_height;
    cp.friction = friction;
    cp.k.assign(k, k + nb);
    cp.d.assign(d, d + nb);
    cp.terrain = g_terrain;
    cp.plane = g_plane;
    for (int64_t w = 0; w < nworld; w++) {
        std::vector<SVec> ext;
        penalty_contact(m, cp, q + w * m.nq, v + w * m.nv, ext,
                        cstate_out ? cstate_out + w * nb * PHYZB_CONTACT_STRIDE : nullptr);
        for (int i = 0; i < nb; i++) {
            double* o = ext_out + (w * nb + i) * 6;
            o[0] = ext[i].ang.x;
            o[1] = ext[i].ang.y;
            o[2] = ext[i].ang.z;
            o[3] = ext[i].lin.x;
            o[4] = ext[i].lin.y;
            o[5] = ext[i].lin.z;
        }
    }
    return 0;
}

// The batched step sequence, nsteps times, worlds in parallel on `nthreads`.
//   q, v:   nworld x nv (in/out)
//   ctrl:   nworld x nv held (ctrl_step_stride == 0) or a schedule with
//           ctrl_step_stride elements between steps (world-major rows)
//   contact (has_contact != 0): ground_height, friction, per-body k, d
//   pd (npd > 0): entries (qi, vi as int32; kp, kd, maxf), targets nworld x npd
//   qdd_out (nworld x nv) and cstate_out (nworld x nb x 8) of the last step
int oracle_rollout(const phyzb_model* fm, int64_t nworld, double* q, double* v,
                   const double* ctrl, int64_t ctrl_step_stride, int32_t nsteps,
                   int32_t has_contact, double ground_height, double friction, const double* k,
                   const double* d, int32_t npd, const int32_t* pd_idx, const double* pd_gains,
                   const double* targets, double* qdd_out, double* cstate_out, int32_t nthreads) {
    Model m = from_flat(fm);
    int nb = m.nb(), nv = m.nv;
    ContactParams cp;
    if (has_contact) {
        cp.ground_height = ground_height;
        cp.friction = friction;
        cp.k.assign(k, k + nb);
        cp.d.assign(d, d + nb);
        cp.terrain = g_terrain;
        cp.plane = g_plane;
    }
    std::vector<PdEntry> pd;
    for (int i = 0; i < npd; i++)
        pd.push_back(PdEntry{pd_idx[2 * i], pd_idx[2 * i + 1], pd_gains[3 * i],
                             pd_gains[3 * i + 1], pd_gains[3 * i + 2]});
    parallel_worlds(nworld, nthreads, [&](int64_t a, int64_t b) {
        std::vector<double> c(nv), qdd(nv);
        for (int64_t w = a; w < b; w++) {
            double* qw = q + w * nv;
            double* vw = v + w * nv;
            for (int s = 0; s < nsteps; s++) {
                const double* src = ctrl ? ctrl + s * ctrl_step_stride + w * nv : nullptr;
                for (int j = 0; j < nv; j++) c[j] = src ? src[j] : 0.0;
                double* cs = (cstate_out && s == nsteps - 1) ? cstate_out + w * nb * PHYZB_CONTACT_STRIDE
                                                             : nullptr;
                step_world(m, has_contact ? &cp : nullptr, npd > 0 ? &pd : nullptr,
                           targets ? targets + w * npd : nullptr, qw, vw, c.data(), qdd.data(), cs);
            }
            if (qdd_out)
                for (int j = 0; j < nv; j++) qdd_out[w * nv + j] = qdd[j];
        }
    });
    return 0;
}

// Impulse-mode rollout (step_world_impulse), nsteps times. `state` carries
// the per-world impulse state across calls: per world, nb x 6 wrenches then
// nb x 8 x 3 staged impulses against the ground, then as many against the
// body-attached plane (in/out; zeros to start).
int oracle_rollout_impulse(const phyzb_model* fm, int64_t nworld, double* q, double* v,
                           const double* ctrl, int64_t ctrl_step_stride, int32_t nsteps,
                           const double* params /* ground, friction, erp, margin, restitution,
                                                    restitution_threshold, dmin, dmax, width, mid,
                                                    power */,
                           int32_t sweeps, int32_t npd, const int32_t* pd_idx, const double* pd_gains,
                           const double* targets, double* state, double* qdd_out, double* cstate_out,
                           int32_t nthreads) {
    Model m = from_flat(fm);
    int nb = m.nb(), nv = m.nv;
    ImpulseParams cp;
    cp.ground_height = params[0];
    cp.friction = params[1];
    cp.erp = params[2];
    cp.margin = params[3];
    cp.restitution = params[4];
    cp.restitution_threshold = params[5];
    cp.dmin = params[6];
    cp.dmax = params[7];
    cp.width = params[8];
    cp.mid = params[9];
    cp.power = params[10];
    cp.sweeps = sweeps;
    cp.terrain = g_terrain;
    cp.plane = g_plane;
    std::vector<PdEntry> pd;
    for (int i = 0; i < npd; i++)
        pd.push_back(PdEntry{pd_idx[2 * i], pd_idx[2 * i + 1], pd_gains[3 * i], pd_gains[3 * i + 1],
                             pd_gains[3 * i + 2]});
    const int64_t per = (int64_t)nb * 6 + 2 * (int64_t)nb * IMPULSE_PTS * 3;
    parallel_worlds(nworld, nthreads, [&](int64_t a, int64_t b) {
        std::vector<double> c(nv), qdd(nv);
        ImpulseState st;
        for (int64_t w = a; w < b; w++) {
            double* qw = q + w * nv;
            double* vw = v + w * nv;
            double* sw = state + w * per;
            st.reset(nb);
            for (int i = 0; i < nb; i++) {
                st.ext[i].ang = v3(sw[6 * i], sw[6 * i + 1], sw[6 * i + 2]);
                st.ext[i].lin = v3(sw[6 * i + 3], sw[6 * i + 4], sw[6 * i + 5]);
            }
            for (int k = 0; k < nb * IMPULSE_PTS * 3; k++) st.imp[k] = sw[nb * 6 + k];
            for (int k = 0; k < nb * IMPULSE_PTS * 3; k++) st.pimp[k] = sw[nb * 6 + nb * IMPULSE_PTS * 3 + k];
            for (int s = 0; s < nsteps; s++) {
                const double* src = ctrl ? ctrl + s * ctrl_step_stride + w * nv : nullptr;
                for (int j = 0; j < nv; j++) c[j] = src ? src[j] : 0.0;
                double* cs = (cstate_out && s == nsteps - 1) ? cstate_out + w * nb * PHYZB_CONTACT_STRIDE
                                                             : nullptr;
                step_world_impulse(m, cp, npd > 0 ? &pd : nullptr, targets ? targets + w * npd : nullptr, qw, vw,
                                   c.data(), qdd.data(), cs, st);
            }
            for (int i = 0; i < nb; i++) {
                const SVec& e = st.ext[i];
                const double vals[6] = {e.ang.x, e.ang.y, e.ang.z, e.lin.x, e.lin.y, e.lin.z};
                for (int k = 0; k < 6; k++) sw[6 * i + k] = vals[k];
            }
            for (int k = 0; k < nb * IMPULSE_PTS * 3; k++) sw[nb * 6 + k] = st.imp[k];
            for (int k = 0; k < nb * IMPULSE_PTS * 3; k++) sw[nb * 6 + nb * IMPULSE_PTS * 3 + k] = st.pimp[k];
            if (qdd_out)
                for (int j = 0; j < nv; j++) qdd_out[w * nv + j] = qdd[j];
        }
    });
    return 0;
}

}  // extern "C"
