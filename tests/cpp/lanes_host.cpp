// The split of one world over lanes (pz_lanes.h: the plan and the lanes'
// sub-model tables; pz_lanes_sweep.cuh: the two halves of a lane's backward
// sweep) run on the host in f64: every lane's sub-model is stepped by the
// kernel's own sweep functions, and where the device sums over a warp's
// lanes with shuffles this sums over the lanes in C++. tests/test_lanes_host.py
// compares the result with the f64 oracle.
#include "kernel_host.cpp"

#include "pz_lanes.h"
#include "pz_lanes_sweep.cuh"

namespace {

struct Lane {
    std::vector<unsigned char> blob;
    PackInfo info;
    ModelView<double> M{};
    std::vector<double> scr;
    std::vector<int> gdof;
};

template <int F>
void run_lanes(std::vector<Lane>& lanes, int nt, int trunk_nv, double* q, double* v, const double* ctrl,
               int nsteps) {
    const int L = (int)lanes.size();
    std::vector<HS> S;
    std::vector<WorldIO<double>> io;
    for (auto& ln : lanes) {
        std::fill(ln.scr.begin(), ln.scr.end(), 0.0);
        S.push_back(HS{ln.scr.data()});
        const int nv = ln.M.nv;
        for (int j = 0; j < nv; j++) {
            S.back()(j) = q[ln.gdof[j]];
            S.back()(nv + j) = v[ln.gdof[j]];
        }
        WorldIO<double> w{ctrl, 0, nullptr, 1, 0};
        w.gdof = ln.gdof.data();
        io.push_back(w);
    }
    const Out<double> none{nullptr, 0};
    for (int l = 0; l < L; l++) {
        for (int i = 0; i < lanes[l].M.nb; i++)
            prefetch_controls<false, double, HS, true>(lanes[l].M, lanes[l].M.bi[i], S[l], io[l], 0);
        pass1_all<F>(lanes[l].M, S[l]);
    }
    std::vector<AI<double>> I(L);
    std::vector<SV<double>> pA(L);
    for (int s = 0; s < nsteps; s++) {
        for (int l = 0; l < L; l++) pass2_limbs<F>(lanes[l].M, S[l], nt, I[l], pA[l]);
        // the sums the device forms with warp shuffles
        AI<double> Is;
        ai_zero(Is);
        SV<double> ps = zerosv<double>();
        for (int l = 0; l < L; l++) {
            for (int k = 0; k < 6; k++) Is.a[k] += I[l].a[k];
            for (int k = 0; k < 9; k++) Is.h[k] += I[l].h[k];
            for (int k = 0; k < 6; k++) Is.m[k] += I[l].m[k];
            ps = ps + pA[l];
        }
        for (int t = 0; t < nt; t++) {
            const BodyI bi = lanes[0].M.bi[t];
            if (!(bi.flags & F_BRANCH)) continue;
            for (int k = 0; k < 27; k++) {
                double sum = 0.0;
                for (int l = 0; l < L; l++) sum += S[l](lanes[l].M.bi[t].s_acc + k);
                for (int l = 0; l < L; l++) S[l](lanes[l].M.bi[t].s_acc + k) = sum;
            }
        }
        for (int l = 0; l < L; l++) {
            I[l] = Is;
            pA[l] = ps;
            pass2_trunk<F>(lanes[l].M, S[l], nt, I[l], pA[l]);
            pass3_next<F, false>(lanes[l].M, S[l], io[l], s + 1, none);
        }
    }
    for (int l = 0; l < L; l++) {
        const int nv = lanes[l].M.nv;
        for (int j = l == 0 ? 0 : trunk_nv; j < nv; j++) {
            q[lanes[l].gdof[j]] = S[l](j);
            v[lanes[l].gdof[j]] = S[l](nv + j);
        }
    }
}

template <int F = 0>
bool dispatch_lanes(int feat, std::vector<Lane>& lanes, int nt, int tnv, double* q, double* v, const double* c,
                    int n) {
    if constexpr (F < 16) {
        if constexpr (!((F & 8) && !(F & 4)))
            if (feat == F) {
                run_lanes<F | FEAT_LANES>(lanes, nt, tnv, q, v, c, n);
                return true;
            }
        return dispatch_lanes<F + 1>(feat, lanes, nt, tnv, q, v, c, n);
    }
    return false;
}

}  // namespace

// nworld worlds of `m`, each over `nlanes` lanes, held controls [nworld][nv],
// penalty contact when `contact` (gains k, d on every body). Returns the
// trunk size, or -1 when the model does not split.
extern "C" int host_rollout_lanes(const phyzb_model* m, int nworld, double* q, double* v, const double* ctrl,
                                  int nsteps, int contact, double ground, double friction, double k, double d,
                                  int nlanes) {
    LanePlan plan;
    if (!plan_lanes(m, nlanes, &plan).empty()) return -1;
    int nv_all = 0;
    for (int i = 0; i < m->nbodies; i++) nv_all += ndof_of(m->bodies[i].joint_type);
    std::vector<Lane> lanes(nlanes);
    int feat_or = 0;
    bool perm1 = true;
    int trunk_nv = 0;
    for (int t = 0; t < plan.nt; t++) trunk_nv += ndof_of(plan.sub[0][t].joint_type);
    for (int l = 0; l < nlanes; l++) {
        phyzb_model sub{};
        sub.nbodies = (int)plan.sub[l].size();
        for (int a = 0; a < 3; a++) sub.gravity[a] = m->gravity[a];
        sub.dt = m->dt;
        sub.bodies = plan.sub[l].data();
        PackCfg cfg;
        cfg.contact = contact != 0;
        cfg.gk.assign(sub.nbodies, k);
        cfg.gd.assign(sub.nbodies, d);
        cfg.force_branch = plan.force_branch;
        cfg.force_chain = plan.force_chain;
        Lane& ln = lanes[l];
        const int nv = (int)plan.dof[l].size();
        ln.info = pack_model<double>(&sub, nv, cfg, ln.blob, 0);
        ln.gdof = plan.dof[l];
        ln.scr.assign(ln.info.scratch + 1, 0.0);
        ModelView<double>& M = ln.M;
        M.bt = M.btp = reinterpret_cast<const BodyT<double>*>(ln.blob.data());
        M.bi = reinterpret_cast<const BodyI*>(ln.blob.data() + ln.info.off_bi);
        M.pd = reinterpret_cast<const PdT<double>*>(ln.blob.data() + ln.info.off_pd);
        M.pd_of_dof = reinterpret_cast<const int*>(ln.blob.data() + ln.info.off_pdmap);
        M.nb = sub.nbodies;
        M.nv = nv;
        M.npd = 0;
        M.contact = cfg.contact ? 1 : 0;
        M.dt = m->dt;
        M.gx = m->gravity[0];
        M.gy = m->gravity[1];
        M.gz = m->gravity[2];
        M.ground_h = ground;
        M.friction = friction;
        const double dtc = m->dt > 1e-9 ? m->dt : 1e-9;
        M.inv_dt_c = 1.0 / dtc;
        M.kstiff_c = 4.0 / (dtc * dtc);
        M.ter = Terrain<double>{nullptr, 0, 0, 0, 0, 0, 1};
        M.plane = PlaneT<double>{-1, 0, 0, 0, 0};
        feat_or |= ln.info.feat & ~8;
        perm1 = perm1 && (ln.info.feat & 8) != 0;
    }
    const int feat = feat_or | ((perm1 && (feat_or & 4)) ? 8 : 0);
    for (int w = 0; w < nworld; w++)
        if (!dispatch_lanes(feat, lanes, plan.nt, trunk_nv, q + (size_t)w * nv_all, v + (size_t)w * nv_all,
                            ctrl + (size_t)w * nv_all, nsteps))
            return -2;
    return plan.nt;
}
