// TEST INFRASTRUCTURE / CPU BASELINE ONLY — a driver around the reference's
// own kernels compiled as host C++.
//
// oracle/Makefile compiles crates/phyz-gpu/cuda/phyz_kernels.cu from the
// reference tree as plain C++ (exactly as the reference's build.rs does for
// its `cuda-host` feature, crates/phyz-gpu/build.rs:8-19) and links it with
// this file into oracle/_ref/libphyz_ref_host.so. This file adds only what
// the reference's HostBatchSimulator adds around those loops
// (crates/phyz-gpu/src/cuda/host.rs, cuda/mod.rs:879-945): the packed body
// and geometry tables (layout.rs:103-155, 185-279), the ContactParams
// header (contact_pipeline.rs:60-98), and the step sequence
// contact -> aba -> integrate. Worlds are split across std::threads by
// pointer offsets; the reference itself is single-threaded.
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../include/phyzb.h"

typedef unsigned int u32;

extern "C" {
void phyz_host_contact(u32 n_threads, const float* cparams, const float* bodies,
                       const float* geometry, const float* q, const float* v, float* ext_forces,
                       float* contact_state, const float* hf_heights, const float* qdd);
void phyz_host_aba(u32 n_threads, u32 nworld, u32 nv, float dt, u32 nbodies, float gx, float gy,
                   float gz, const float* bodies, const float* q, const float* v, const float* ctrl,
                   float* qdd, const float* ext_forces);
void phyz_host_integrate(u32 n_threads, u32 nworld, u32 nv, float dt, u32 nbodies, float* q,
                         float* v, const float* qdd, const float* bodies);
void phyz_host_pd(u32 n_threads, u32 nworld, u32 nq, u32 nv, u32 n_dofs, const float* dofs,
                  const float* q, const float* v, const float* targets, float* ctrl);
}

namespace {

const int BODY_STRIDE = 36, GEOM_STRIDE = 24, CP_STRIDE = 32, CS_STRIDE = 56, PD_STRIDE = 8;

float bits_i(int32_t i) {
    float f;
    std::memcpy(&f, &i, 4);
    return f;
}
float bits_u(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

int ndof_of(int jt) { return jt == 2 ? 0 : jt == 3 ? 3 : jt == 4 ? 6 : 1; }

}  // namespace

extern "C" {

int phyzref_abi_version(void) { return 1; }

// layout.rs:103-155 pack_bodies
int phyzref_pack_bodies(const phyzb_model* m, float* out) {
    int off = 0;
    for (int i = 0; i < m->nbodies; i++) {
        const phyzb_body& b = m->bodies[i];
        float* d = out + i * BODY_STRIDE;
        std::memset(d, 0, sizeof(float) * BODY_STRIDE);
        d[0] = bits_i(b.parent);
        d[1] = bits_u((uint32_t)b.joint_type);
        d[2] = bits_u((uint32_t)off);
        d[3] = bits_u((uint32_t)off);
        d[4] = (float)b.mass;
        for (int k = 0; k < 3; k++) d[5 + k] = (float)b.com[k];
        for (int k = 0; k < 6; k++) d[8 + k] = (float)b.inertia[k];
        for (int k = 0; k < 9; k++) d[14 + k] = (float)b.ptj_rot[k];
        for (int k = 0; k < 3; k++) d[23 + k] = (float)b.ptj_pos[k];
        for (int k = 0; k < 3; k++) d[26 + k] = (float)b.axis[k];
        d[29] = (float)b.damping;
        d[30] = (float)b.stiffness;
        d[31] = (float)b.spring_ref;
        d[32] = (float)b.armature;
        off += ndof_of(b.joint_type);
    }
    return off;
}

// The body-attached plane of the following host rollouts (body < 0: none):
// ContactParams fields 6-10 (contact_pipeline.rs:74-78) and the exclusion
// flag geometry[7] that pack_contact_geometry sets (contact_pipeline.rs:
// 637-641). Test-only process state.
static int32_t g_plane_body = -1;
static float g_plane[4] = {0, 0, 0, 0};  // offset, max_depth, half_x, half_y
static std::vector<int32_t> g_plane_excl;

// layout.rs:185-279 pack_geometries (primary shape, per-body gains)
int phyzref_pack_geometries(const phyzb_model* m, const double* k, const double* dmp, float* out) {
    int collidable = 0;
    for (int i = 0; i < m->nbodies; i++) {
        const phyzb_body& b = m->bodies[i];
        float* d = out + i * GEOM_STRIDE;
        std::memset(d, 0, sizeof(float) * GEOM_STRIDE);
        for (int r = 0; r < 9; r++) d[13 + r] = (float)b.geom_origin_rot[r];
        for (int r = 0; r < 3; r++) d[10 + r] = (float)b.geom_origin_pos[r];
        d[0] = (float)b.geom_type;
        for (int r = 0; r < 6; r++) d[1 + r] = (float)b.geom_params[r];
        if (b.geom_type != 0) collidable++;
        d[8] = (float)k[i];
        d[9] = (float)dmp[i];
    }
    if (g_plane_body >= 0 && g_plane_body < m->nbodies) {
        out[g_plane_body * GEOM_STRIDE + 7] = 1.0f;
        for (int32_t b : g_plane_excl)
            if (b >= 0 && b < m->nbodies) out[b * GEOM_STRIDE + 7] = 1.0f;
    }
    return collidable;
}

// The heightfield the following rollouts pass to the contact kernel
// (contact_pipeline.rs:79-84 header fields, node buffer as the reference
// uploads it); nx == 0: none. Test-only process state.
static uint32_t g_hf_nx = 0, g_hf_ny = 0;
static float g_hf_o[3] = {0, 0, 0}, g_hf_cell = 1.0f;
static std::vector<float> g_hf(1, 0.0f);


void phyzref_set_plane(int32_t body, float offset, float max_depth, float half_x, float half_y,
                       const int32_t* exclude, int32_t n_exclude) {
    g_plane_body = body;
    g_plane[0] = offset;
    g_plane[1] = max_depth;
    g_plane[2] = half_x;
    g_plane[3] = half_y;
    g_plane_excl.assign(exclude, exclude + (n_exclude > 0 ? n_exclude : 0));
}

void phyzref_set_heightfield(uint32_t nx, uint32_t ny, float ox, float oy, float oz, float cell,
                             const float* heights) {
    g_hf_nx = nx;
    g_hf_ny = ny;
    g_hf_o[0] = ox;
    g_hf_o[1] = oy;
    g_hf_o[2] = oz;
    g_hf_cell = nx ? cell : 1.0f;
    if (nx)
        g_hf.assign(heights, heights + (size_t)nx * ny);
    else
        g_hf.assign(1, 0.0f);
}

// contact_pipeline.rs:60-98 ContactParams::pack (penalty, flat ground, no plane)
void phyzref_pack_cparams(uint32_t nworld, uint32_t nb, uint32_t nv, float ground, float dt,
                          float friction, float* out) {
    std::memset(out, 0, sizeof(float) * CP_STRIDE);
    out[0] = bits_u(nworld);
    out[1] = bits_u(nb);
    out[2] = bits_u(nv);
    out[3] = ground;
    out[4] = dt;
    out[5] = friction;
    out[6] = bits_i(-1);
    out[16] = 1.0f;  // hf_cell default
}

// The host rollouts' header of the heightfield set by phyzref_set_heightfield
// (ContactParams::set_heightfield, contact_pipeline.rs:101-108).
static void apply_heightfield(float* cp) {
    cp[6] = bits_i(g_plane_body);
    if (g_plane_body >= 0)
        for (int k = 0; k < 4; k++) cp[7 + k] = g_plane[k];
    cp[11] = bits_u(g_hf_nx);
    cp[12] = bits_u(g_hf_ny);
    cp[13] = g_hf_o[0];
    cp[14] = g_hf_o[1];
    cp[15] = g_hf_o[2];
    cp[16] = g_hf_cell;
}

// n steps of the reference sequence over nworld worlds (AoS f32, as
// layout.rs:340-355 packs them), worlds split over nthreads.
//   ctrl: nworld x nv, or a schedule (ctrl_step_stride floats between steps)
//   geometry == NULL: no contact pass
//   pd_table (npd rows of PD_STRIDE, layout.rs:300-312) + targets (nworld x npd) or NULL
int phyzref_rollout(int nthreads, uint32_t nworld, uint32_t nv, uint32_t nb, float dt, float gx,
                    float gy, float gz, const float* bodies, const float* geometry, float ground,
                    float friction, uint32_t npd, const float* pd_table, const float* targets,
                    float* q, float* v, const float* ctrl, int64_t ctrl_step_stride, int32_t nsteps,
                    float* qdd_out, float* cstate_out) {
    if (nthreads < 1) nthreads = 1;
    if ((uint32_t)nthreads > nworld) nthreads = (int)(nworld ? nworld : 1);
    uint32_t chunk = (nworld + nthreads - 1) / nthreads;
    auto work = [&](uint32_t a, uint32_t b) {
        uint32_t n = b - a;
        std::vector<float> ext((size_t)n * nb * 6, 0.0f), cs((size_t)n * nb * CS_STRIDE, 0.0f);
        std::vector<float> qdd((size_t)n * nv, 0.0f), c((size_t)n * nv, 0.0f);
        float cp[CP_STRIDE];
        phyzref_pack_cparams(n, nb, nv, ground, dt, friction, cp);
        apply_heightfield(cp);
        float* qa = q + (size_t)a * nv;
        float* va = v + (size_t)a * nv;
        for (int s = 0; s < nsteps; s++) {
            const float* src = ctrl + (size_t)s * ctrl_step_stride + (size_t)a * nv;
            std::memcpy(c.data(), src, sizeof(float) * n * nv);
            if (npd)
                phyz_host_pd(n * npd, n, nv, nv, npd, pd_table, qa, va, targets + (size_t)a * npd,
                             c.data());
            if (geometry)
                phyz_host_contact(n, cp, bodies, geometry, qa, va, ext.data(), cs.data(), g_hf.data(),
                                  qdd.data());
            phyz_host_aba(n, n, nv, dt, nb, gx, gy, gz, bodies, qa, va, c.data(), qdd.data(),
                          ext.data());
            phyz_host_integrate(n * nb, n, nv, dt, nb, qa, va, qdd.data(), bodies);
        }
        if (qdd_out) std::memcpy(qdd_out + (size_t)a * nv, qdd.data(), sizeof(float) * n * nv);
        if (cstate_out)
            for (uint32_t w = 0; w < n; w++)
                for (uint32_t i = 0; i < nb; i++)
                    for (int k = 0; k < PHYZB_CONTACT_STRIDE; k++)
                        cstate_out[((size_t)(a + w) * nb + i) * PHYZB_CONTACT_STRIDE + k] =
                            cs[((size_t)w * nb + i) * CS_STRIDE + k];
    };
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; t++) {
        uint32_t a = t * chunk, b = a + chunk < nworld ? a + chunk : nworld;
        if (a >= b) break;
        if (nthreads == 1)
            work(a, b);
        else
            pool.emplace_back(work, a, b);
    }
    for (auto& th : pool) th.join();
    return 0;
}

// Impulse mode (cuda/mod.rs:902-927): cparams with solve_mode 1 and the
// impulse material (contact_pipeline.rs:85-95), then per step [PD ->] ABA,
// `sweeps` x [contact -> ABA], integrate. ext (nworld x nb x 6) and cs
// (nworld x nb x CS_STRIDE, the warm-start impulses at CS_IMPULSE_OFF) carry
// over between calls, as the reference's device buffers do between steps.
//   imp: erp, margin, restitution, restitution_threshold, dmin, dmax, width, mid, power
int phyzref_rollout_impulse(int nthreads, uint32_t nworld, uint32_t nv, uint32_t nb, float dt, float gx,
                            float gy, float gz, const float* bodies, const float* geometry, float ground,
                            float friction, const float* imp, int32_t sweeps, uint32_t npd,
                            const float* pd_table, const float* targets, float* q, float* v, const float* ctrl,
                            int64_t ctrl_step_stride, int32_t nsteps, float* ext_io, float* cs_io,
                            float* qdd_out) {
    if (nthreads < 1) nthreads = 1;
    if ((uint32_t)nthreads > nworld) nthreads = (int)(nworld ? nworld : 1);
    uint32_t chunk = (nworld + nthreads - 1) / nthreads;
    auto work = [&](uint32_t a, uint32_t b) {
        uint32_t n = b - a;
        float* ext = ext_io + (size_t)a * nb * 6;
        float* cs = cs_io + (size_t)a * nb * CS_STRIDE;
        std::vector<float> qdd((size_t)n * nv, 0.0f), c((size_t)n * nv, 0.0f);
        float cp[CP_STRIDE];
        phyzref_pack_cparams(n, nb, nv, ground, dt, friction, cp);
        apply_heightfield(cp);
        cp[17] = bits_u(1u);  // solve_mode: impulse
        cp[19] = imp[2];      // restitution
        cp[20] = imp[3];      // restitution_threshold
        cp[21] = imp[0];      // solref_erp
        cp[22] = imp[1];      // margin
        for (int k = 0; k < 5; k++) cp[23 + k] = imp[4 + k];  // solimp dmin, dmax, width, mid, power
        float* qa = q + (size_t)a * nv;
        float* va = v + (size_t)a * nv;
        for (int s = 0; s < nsteps; s++) {
            const float* src = ctrl + (size_t)s * ctrl_step_stride + (size_t)a * nv;
            std::memcpy(c.data(), src, sizeof(float) * n * nv);
            if (npd)
                phyz_host_pd(n * npd, n, nv, nv, npd, pd_table, qa, va, targets + (size_t)a * npd,
                             c.data());
            phyz_host_aba(n, n, nv, dt, nb, gx, gy, gz, bodies, qa, va, c.data(), qdd.data(), ext);
            for (int k = 0; k < sweeps; k++) {
                phyz_host_contact(n, cp, bodies, geometry, qa, va, ext, cs, g_hf.data(), qdd.data());
                phyz_host_aba(n, n, nv, dt, nb, gx, gy, gz, bodies, qa, va, c.data(), qdd.data(), ext);
            }
            phyz_host_integrate(n * nb, n, nv, dt, nb, qa, va, qdd.data(), bodies);
        }
        if (qdd_out) std::memcpy(qdd_out + (size_t)a * nv, qdd.data(), sizeof(float) * n * nv);
    };
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; t++) {
        uint32_t a = t * chunk, b = a + chunk < nworld ? a + chunk : nworld;
        if (a >= b) break;
        if (nthreads == 1)
            work(a, b);
        else
            pool.emplace_back(work, a, b);
    }
    for (auto& th : pool) th.join();
    return 0;
}

}  // extern "C"
