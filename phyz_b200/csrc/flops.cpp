// Algorithmic flop count of one world-step, taken by running the kernel's
// own world-step code (pz_world.cuh) on the host with a counting scalar.
// This is a measurement helper only: the counting scalar carries values
// so branches follow a real state, but nothing here is a way to step a
// simulation on the CPU (no float/double host instantiation exists).
//
// Convention: +, -, *, / count one flop each (a fused multiply-add is the
// two flops it replaces); sqrt, sin/cos, atan2 and tanh are tallied
// separately as transcendental calls; min/max/abs/compares count nothing.
#include <vector>

#include "pz_pack.h"
#include "pz_types.cuh"

namespace pz {

struct Tally {
    double flops = 0, trans = 0;
};
static thread_local Tally g_tally;
// count as a model-specialized kernel executes: products with zero table
// constants left out (pz_types.cuh kzero)
static thread_local bool g_kskip = false;

struct Cnt {
    double v;
    Cnt() = default;
    Cnt(double x) : v(x) {}
};
inline Cnt operator+(Cnt a, Cnt b) {
    g_tally.flops += 1;
    return Cnt(a.v + b.v);
}
inline Cnt operator-(Cnt a, Cnt b) {
    g_tally.flops += 1;
    return Cnt(a.v - b.v);
}
inline Cnt operator*(Cnt a, Cnt b) {
    g_tally.flops += 1;
    return Cnt(a.v * b.v);
}
inline Cnt operator/(Cnt a, Cnt b) {
    g_tally.flops += 1;
    return Cnt(a.v / b.v);
}
inline Cnt operator-(Cnt a) { return Cnt(-a.v); }
inline Cnt& operator+=(Cnt& a, Cnt b) { return a = a + b; }
inline bool operator<(Cnt a, Cnt b) { return a.v < b.v; }
inline bool operator>(Cnt a, Cnt b) { return a.v > b.v; }
inline bool operator<=(Cnt a, Cnt b) { return a.v <= b.v; }
inline bool operator>=(Cnt a, Cnt b) { return a.v >= b.v; }
inline void pz_sincos(Cnt x, Cnt* s, Cnt* c) {
    g_tally.trans += 1;
    *s = Cnt(std::sin(x.v));
    *c = Cnt(std::cos(x.v));
}
inline Cnt pz_sqrt(Cnt x) {
    g_tally.trans += 1;
    return Cnt(std::sqrt(x.v));
}
inline Cnt pz_atan2(Cnt y, Cnt x) {
    g_tally.trans += 1;
    return Cnt(std::atan2(y.v, x.v));
}
inline Cnt pz_tanh(Cnt x) {
    g_tally.trans += 1;
    return Cnt(std::tanh(x.v));
}
inline Cnt pz_pow(Cnt x, Cnt y) {
    g_tally.trans += 1;
    return Cnt(std::pow(x.v, y.v));
}
inline Cnt pz_abs(Cnt x) { return Cnt(std::fabs(x.v)); }
inline int pz_trunc_int(Cnt x) { return (int)x.v; }
inline Cnt pz_min(Cnt a, Cnt b) { return Cnt(std::fmin(a.v, b.v)); }
inline Cnt pz_max(Cnt a, Cnt b) { return Cnt(std::fmax(a.v, b.v)); }

template <>
struct Eps<Cnt> {
    static constexpr double quat = 2.220446049250313e-16;
};
template <>
struct Counting<Cnt> {
    static constexpr bool value = true;
    static bool kskip_on() { return g_kskip; }
};

}  // namespace pz

#include "pz_world.cuh"

namespace pz {

namespace {
struct HostScr {
    Cnt* base;
    Cnt& operator()(int s) const { return base[s]; }
    void prefetch(int s, const Cnt* g) const { base[s] = *g; }
    void commit() const {}
    void wait() const {}
    void fence_st() const {}
    Rec<Cnt> rec_get(const BodyI& bi) const {
        Rec<Cnt> r;
        r.c = base[bi.s_xj];
        r.s = base[bi.s_xj + 1];
        r.v = mksv<Cnt>(mk3<Cnt>(base[bi.s_vw], base[bi.s_vw + 1], base[bi.s_vw + 2]),
                        mk3<Cnt>(base[bi.s_vw + 3], base[bi.s_vw + 4], base[bi.s_vw + 5]));
        return r;
    }
    void rec_put(const BodyI& bi, const Rec<Cnt>& r) const {
        base[bi.s_xj] = r.c;
        base[bi.s_xj + 1] = r.s;
        rec_put_vw(bi, r.v);
    }
    SV<Cnt> ext_get(const BodyI& bi) const { return ld_sv<Cnt>(*this, bi.s_f); }
    void ext_put(const BodyI& bi, const SV<Cnt>& f) const { st_sv(*this, bi.s_f, f); }
    void rec_put_vw(const BodyI& bi, const SV<Cnt>& v) const {
        base[bi.s_vw] = v.w.x;
        base[bi.s_vw + 1] = v.w.y;
        base[bi.s_vw + 2] = v.w.z;
        base[bi.s_vw + 3] = v.l.x;
        base[bi.s_vw + 4] = v.l.y;
        base[bi.s_vw + 5] = v.l.z;
    }
};
}  // namespace

namespace {
// The packed model in the counting scalar, and a view of it whose ground
// sits at `ground_h` (far below: detection is counted, the force law is not).
struct CountModel {
    std::vector<unsigned char> blob;
    PackInfo info;
    std::vector<BodyT<Cnt>> bt;
    std::vector<PdT<Cnt>> pd;
    ModelView<Cnt> M;
};

void make_count_model(const phyzb_model* m, int nv, const PackCfg& cfg, double ground_h, double friction, double erp,
                      CountModel* cm) {
    std::vector<unsigned char>& blob = cm->blob;
    cm->info = pack_model<double>(m, nv, cfg, blob);
    const PackInfo& info = cm->info;
    const int nb = m->nbodies, npd = (int)cfg.pd.size();
    std::vector<BodyT<Cnt>>& bt = cm->bt;
    bt.resize(nb);
    const BodyT<double>* src = reinterpret_cast<const BodyT<double>*>(blob.data());
    static_assert(sizeof(BodyT<double>) == sizeof(BodyT<Cnt>), "layout");
    std::memcpy((void*)bt.data(), src, sizeof(BodyT<double>) * nb);
    std::vector<PdT<Cnt>>& pd = cm->pd;
    pd.resize(npd > 0 ? npd : 1);
    const PdT<double>* psrc = reinterpret_cast<const PdT<double>*>(blob.data() + info.off_pd);
    for (int k = 0; k < npd; k++) {
        pd[k].kp = psrc[k].kp;
        pd[k].kd = psrc[k].kd;
        pd[k].maxf = psrc[k].maxf;
        pd[k].qi = psrc[k].qi;
        pd[k].vi = psrc[k].vi;
    }
    ModelView<Cnt>& M = cm->M;
    M.bt = M.btp = bt.data();
    M.bi = reinterpret_cast<const BodyI*>(blob.data() + info.off_bi);
    M.pd = pd.data();
    M.pd_of_dof = reinterpret_cast<const int*>(blob.data() + info.off_pdmap);
    M.nb = nb;
    M.nv = nv;
    M.npd = npd;
    M.contact = cfg.contact ? 1 : 0;
    M.dt = Cnt(m->dt);
    M.gx = Cnt(m->gravity[0]);
    M.gy = Cnt(m->gravity[1]);
    M.gz = Cnt(m->gravity[2]);
    M.ground_h = Cnt(ground_h);
    M.friction = Cnt(friction);
    const double dtc = m->dt > 1e-9 ? m->dt : 1e-9;
    M.inv_dt_c = Cnt(1.0 / dtc);
    M.kstiff_c = Cnt(4.0 / (dtc * dtc));
    // the impulse material of enable_contact_impulse (capi.cu rollout_args)
    M.im = ImpMat<Cnt>{M.ground_h, M.friction, M.dt, Cnt(erp), Cnt(0.001), Cnt(0.0), Cnt(0.05),
                       Cnt(0.9),   Cnt(0.95),  Cnt(0.001), Cnt(0.5), Cnt(2.0)};
    impmat_finish(M.im);  // per-launch constants, outside the counted step
    // a 2 x 2 heightfield far below: terrain sampling is counted like
    // detection, the force law is not
    static const float hf_nodes[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    M.ter = Terrain<Cnt>{hf_nodes, 2, 2, Cnt(-1.0), Cnt(-1.0), Cnt(-1e9), Cnt(1.0)};
    M.plane = PlaneT<Cnt>{-1, Cnt(0.0), Cnt(0.0), Cnt(0.0), Cnt(0.0)};  // plane contacts are not counted
}
}  // namespace

FlopCount count_world_step(const phyzb_model* m, int nv, const PackCfg& cfg, int sweeps) {
    g_kskip = false;
    CountModel cm;
    // Ground far below: contact detection is counted, the force law is not
    // (a lower bound on the work of a contact step).
    make_count_model(m, nv, cfg, -1e9, 1.0, 0.0, &cm);
    const PackInfo& info = cm.info;
    const ModelView<Cnt>& M = cm.M;
    const int nb = m->nbodies, npd = (int)cfg.pd.size();
    std::vector<Cnt> scratch(info.scratch > 0 ? info.scratch : 1, Cnt(0.0));
    HostScr S{scratch.data()};
    // a generic state, away from the exp/log small-angle branches
    for (int j = 0; j < nv; j++) {
        scratch[j] = Cnt(0.1 + 0.01 * j);
        scratch[nv + j] = Cnt(0.2 - 0.03 * j);
    }
    std::vector<Cnt> ctrl(nv > 0 ? nv : 1, Cnt(0.5)), targets(npd > 0 ? npd : 1, Cnt(0.0));
    const WorldIO<Cnt> io{ctrl.data(), 0, targets.data(), 1, 0};
    const Out<Cnt> none{nullptr, 0};
    for (int i = 0; i < nb; i++) {
        if (cfg.contact && cfg.impulse)
            prefetch_controls<true>(M, M.bi[i], S, io, 0);
        else
            prefetch_controls<false>(M, M.bi[i], S, io, 0);
    }
    constexpr int ALL = FEAT_MULTI | FEAT_CONTACT;  // runtime flags select the paths taken
    constexpr int ALLI = ALL | FEAT_IMPULSE;
    if (cfg.contact && cfg.terrain) {
        constexpr int AT = ALL | FEAT_TERRAIN, ATI = ALLI | FEAT_TERRAIN;
        if (cfg.impulse) {
            pass1_all<ATI>(M, S);
            g_tally = Tally{};
            pass2<ATI>(M, S);
            keep_backward_state(M, S);
            for (int k = 0; k < sweeps; k++) {
                sweep_forward<ATI>(M, S);
                wrench_response<ATI>(M, S);
            }
            pass3_next<ATI, false>(M, S, io, 1, none);
        } else {
            pass1_all<AT>(M, S);
            g_tally = Tally{};
            pass2<AT>(M, S);
            pass3_next<AT, false>(M, S, io, 1, none);
        }
    } else if (cfg.contact && cfg.impulse) {
        pass1_all<ALLI>(M, S);
        // steady state: the leading backward sweep, `sweeps` x [forward
        // sweep with contact, backward sweep], the fused finish/start sweep
        g_tally = Tally{};
        pass2<ALLI>(M, S);
        keep_backward_state(M, S);
        for (int k = 0; k < sweeps; k++) {
            sweep_forward<ALLI>(M, S);
            wrench_response<ALLI>(M, S);
        }
        pass3_next<ALLI, false>(M, S, io, 1, none);
    } else {
        pass1_all<ALL>(M, S);
        // steady state: one backward sweep + one fused finish/start sweep
        g_tally = Tally{};
        pass2<ALL>(M, S);
        pass3_next<ALL, false>(M, S, io, 1, none);
    }
    FlopCount fc;
    fc.flops = g_tally.flops;
    fc.transcendentals = g_tally.trans;
    return fc;
}

FlopCount count_rollout(const phyzb_model* m, int nv, const PackCfg& cfg, int sweeps, double ground_h,
                        double friction, double erp, const double* q, const double* v, const double* ctrl,
                        long long nworld, int nsteps, bool specialized) {
    CountModel cm;
    make_count_model(m, nv, cfg, ground_h, friction, erp, &cm);
    const ModelView<Cnt>& M = cm.M;
    const int npd = (int)cfg.pd.size();
    std::vector<Cnt> scratch(cm.info.scratch > 0 ? cm.info.scratch : 1, Cnt(0.0));
    // one world's schedule [step][nv], its last row repeated for the
    // prefetch of the step after the last
    std::vector<Cnt> sched((size_t)(nsteps + 1) * (nv > 0 ? nv : 1), Cnt(0.0)), targets(npd > 0 ? npd : 1, Cnt(0.0));
    g_kskip = specialized;
    Tally total{};
    for (long long w = 0; w < nworld; w++) {
        std::fill(scratch.begin(), scratch.end(), Cnt(0.0));
        for (int j = 0; j < nv; j++) {
            scratch[j] = Cnt(q[w * nv + j]);
            scratch[nv + j] = Cnt(v[w * nv + j]);
        }
        for (int s = 0; s <= nsteps; s++)
            for (int j = 0; j < nv; j++) {
                const int t = s < nsteps ? s : nsteps - 1;
                sched[(size_t)s * nv + j] = Cnt(ctrl ? ctrl[((size_t)t * nworld + w) * nv + j] : 0.0);
            }
        const WorldIO<Cnt> io{sched.data(), nv, targets.data(), 1, 0};
        HostScr S{scratch.data()};
        // the relabelling of frames (FEAT_PERM) places the contact shapes
        constexpr int ALL = FEAT_MULTI | FEAT_CONTACT | FEAT_PERM;
        // the counted steps only: pass 1 of the launch's first step is not one
        Tally base;
        g_tally = Tally{};
        if (cfg.contact && cfg.impulse) {
            for (int i = 0; i < M.nb; i++) prefetch_controls<true>(M, M.bi[i], S, io, 0);
            pass1_all<ALL | FEAT_IMPULSE>(M, S);
            base = g_tally;
            for (int s = 0; s < nsteps; s++) {
                pass2<ALL | FEAT_IMPULSE>(M, S);
                keep_backward_state(M, S);
                for (int k = 0; k < sweeps; k++) {
                    sweep_forward<ALL | FEAT_IMPULSE>(M, S);
                    wrench_response<ALL | FEAT_IMPULSE>(M, S);
                }
                pass3_next<ALL | FEAT_IMPULSE, false>(M, S, io, s + 1, Out<Cnt>{nullptr, 0});
            }
        } else {
            for (int i = 0; i < M.nb; i++) prefetch_controls<false>(M, M.bi[i], S, io, 0);
            pass1_all<ALL>(M, S);
            base = g_tally;
            for (int s = 0; s < nsteps; s++) {
                pass2<ALL>(M, S);
                pass3_next<ALL, false>(M, S, io, s + 1, Out<Cnt>{nullptr, 0});
            }
        }
        total.flops += g_tally.flops - base.flops;
        total.trans += g_tally.trans - base.trans;
    }
    g_kskip = false;
    const double n = (double)nworld * (double)nsteps;
    FlopCount fc;
    fc.flops = n > 0 ? total.flops / n : 0.0;
    fc.transcendentals = n > 0 ? total.trans / n : 0.0;
    return fc;
}

}  // namespace pz
