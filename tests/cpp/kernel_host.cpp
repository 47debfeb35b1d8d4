// The rollout kernel's own step functions (pz_world.cuh: pass 1, the
// backward sweep, the fused finish / next-step sweep, penalty ground
// contact) compiled for the host in f64 and run one world at a time, so the
// kernel source's arithmetic can be checked against the oracle without a
// GPU. Built twice by tests/test_kernel_host.py: as the generic kernel
// evaluates it, and with PZ_KSKIP, where every product with a zero
// model-table constant is left out exactly as a model-specialized kernel
// leaves it out at compile time.
#include <cmath>
#include "pz_pack.h"
// host versions of the device scalar shims of pz_types.cuh
namespace pz {
inline void pz_sincos(double x, double* s, double* c) { *s = std::sin(x); *c = std::cos(x); }
inline double pz_sqrt(double x) { return std::sqrt(x); }
inline double pz_atan2(double y, double x) { return std::atan2(y, x); }
inline double pz_tanh(double x) { return std::tanh(x); }
inline double pz_pow(double x, double y) { return std::pow(x, y); }
inline double pz_abs(double x) { return std::fabs(x); }
inline double pz_min(double a, double b) { return std::fmin(a, b); }
inline double pz_max(double a, double b) { return std::fmax(a, b); }
inline bool pz_finite(double x) { return std::isfinite(x); }
inline int pz_trunc_int(double x) { return (int)x; }
}
#include "pz_world.cuh"
using namespace pz;
// scratch of one world (the kernel's shared-memory layout, stride 1)
struct HS {
    double* base;
    double& operator()(int s) const { return base[s]; }
    void prefetch(int s, const double* g) const { base[s] = *g; }
    void commit() const {}
    void wait() const {}
    void fence_st() const {}
    Rec<double> rec_get(const BodyI& bi) const {
        Rec<double> r; r.c = base[bi.s_xj]; r.s = base[bi.s_xj + 1];
        r.v = mksv<double>(mk3<double>(base[bi.s_vw], base[bi.s_vw + 1], base[bi.s_vw + 2]),
                           mk3<double>(base[bi.s_vw + 3], base[bi.s_vw + 4], base[bi.s_vw + 5]));
        return r;
    }
    void rec_put(const BodyI& bi, const Rec<double>& r) const { base[bi.s_xj] = r.c; base[bi.s_xj + 1] = r.s; rec_put_vw(bi, r.v); }
    SV<double> ext_get(const BodyI& bi) const { return ld_sv<double>(*this, bi.s_f); }
    void ext_put(const BodyI& bi, const SV<double>& f) const { st_sv(*this, bi.s_f, f); }
    void rec_put_vw(const BodyI& bi, const SV<double>& v) const {
        base[bi.s_vw] = v.w.x; base[bi.s_vw + 1] = v.w.y; base[bi.s_vw + 2] = v.w.z;
        base[bi.s_vw + 3] = v.l.x; base[bi.s_vw + 4] = v.l.y; base[bi.s_vw + 5] = v.l.z;
    }
};
// One world, nsteps steps, the kernel's sequence: pass 1 once, then per step
// the backward sweep, (impulse mode) the kept backward state and `sweeps` x
// [forward sweep with the staged impulse update, wrench response], and the
// fused finish / next-step sweep. Impulse state starts at zero.
template <int F>
void run(const ModelView<double>& M, const PackInfo& info, double* q, double* v, const double* ctrl, int nsteps,
         int sweeps) {
    constexpr bool IMP = (F & FEAT_IMPULSE) != 0;
    std::vector<double> scr(info.scratch + 1, 0.0);
    HS S{scr.data()};
    const int nv = M.nv;
    for (int j = 0; j < nv; j++) { S(j) = q[j]; S(nv + j) = v[j]; }
    const WorldIO<double> io{ctrl, 0, nullptr, 1, 0};
    for (int i = 0; i < M.nb; i++) prefetch_controls<IMP>(M, M.bi[i], S, io, 0);
    const Out<double> none{nullptr, 0};
    pass1_all<F>(M, S);
    for (int s = 0; s < nsteps; s++) {
        pass2<F>(M, S);
        if constexpr (IMP) {
            keep_backward_state(M, S);
            for (int k = 0; k < sweeps; k++) {
                sweep_forward<F>(M, S);
                wrench_response<F>(M, S);
            }
        }
        if (s == nsteps - 1) pass3_next<F, true>(M, S, io, -1, none);
        else pass3_next<F, false>(M, S, io, s + 1, none);
    }
    for (int j = 0; j < nv; j++) { q[j] = S(j); v[j] = S(nv + j); }
}
template <int F = 0>
bool dispatch(int feat, const ModelView<double>& M, const PackInfo& info, double* q, double* v, const double* c, int n,
              int sweeps) {
    if constexpr (F < 64) {
        if constexpr (!((F & 8) && !(F & 4)) && !((F & 16) && !(F & 2)) && !((F & 32) && !(F & 2)))
            if (feat == F) { run<F>(M, info, q, v, c, n, sweeps); return true; }
        return dispatch<F + 1>(feat, M, info, q, v, c, n, sweeps);
    }
    return false;
}
// The heightfield of the following rollouts with contact (nx = 0: the flat
// ground): f32 nodes [ny][nx], node (ix, iy) at (ox + ix cell, oy + iy cell).
static std::vector<float> g_hf;
static int g_nx = 0, g_ny = 0;
static double g_ho[3] = {0, 0, 0}, g_cell = 1.0;
extern "C" void host_set_heightfield(int nx, int ny, double ox, double oy, double oz, double cell, const float* h) {
    g_nx = nx;
    g_ny = ny;
    g_ho[0] = ox;
    g_ho[1] = oy;
    g_ho[2] = oz;
    g_cell = cell;
    g_hf.assign(h, h + (size_t)(nx > 0 ? nx * ny : 0));
}

// contact: 0 none, 1 penalty (gains k, d), 2 impulse (`sweeps` per step,
// enable_contact_impulse's material)
extern "C" int host_rollout(const phyzb_model* m, int nworld, double* q, double* v, const double* ctrl, int nsteps,
                            int contact, double ground, double friction, double k, double d, int sweeps) {
    const int nv = [&] { int s = 0; for (int i = 0; i < m->nbodies; i++) { int t = m->bodies[i].joint_type;
        s += t == 3 ? 3 : (t == 4 ? 6 : (t == 2 ? 0 : 1)); } return s; }();
    PackCfg cfg; cfg.contact = contact != 0; cfg.impulse = contact == 2; cfg.terrain = contact != 0 && g_nx > 0;
    cfg.gk.assign(m->nbodies, k); cfg.gd.assign(m->nbodies, d);
    std::vector<unsigned char> blob;
    PackInfo info = pack_model<double>(m, nv, cfg, blob, 0);
    ModelView<double> M{};
    M.bt = M.btp = reinterpret_cast<const BodyT<double>*>(blob.data());
    M.bi = reinterpret_cast<const BodyI*>(blob.data() + info.off_bi);
    M.pd = reinterpret_cast<const PdT<double>*>(blob.data() + info.off_pd);
    M.pd_of_dof = reinterpret_cast<const int*>(blob.data() + info.off_pdmap);
    M.nb = m->nbodies; M.nv = nv; M.npd = 0; M.contact = cfg.contact ? 1 : 0;
    M.dt = m->dt; M.gx = m->gravity[0]; M.gy = m->gravity[1]; M.gz = m->gravity[2];
    M.ground_h = ground; M.friction = friction;
    const double dtc = m->dt > 1e-9 ? m->dt : 1e-9;
    M.inv_dt_c = 1.0 / dtc; M.kstiff_c = 4.0 / (dtc * dtc);
    // GroundContactParams::default with solref_erp_from(0.02, 1.0, dt)
    const double erp = m->dt > 0.0 ? m->dt / (2.0 * 0.02 + m->dt) : 0.0;
    M.im = ImpMat<double>{ground, friction, m->dt, erp, 0.001, 0.0, 0.05, 0.9, 0.95, 0.001, 0.5, 2.0};
    impmat_finish(M.im);
    M.ter = cfg.terrain ? Terrain<double>{g_hf.data(), g_nx, g_ny, g_ho[0], g_ho[1], g_ho[2], g_cell}
                        : Terrain<double>{nullptr, 0, 0, 0, 0, 0, 1};
    M.plane = PlaneT<double>{-1, 0, 0, 0, 0};
    for (int w = 0; w < nworld; w++)
        if (!dispatch(info.feat, M, info, q + (size_t)w * nv, v + (size_t)w * nv, ctrl + (size_t)w * nv, nsteps,
                      sweeps))
            return -1;
    return info.feat;
}
