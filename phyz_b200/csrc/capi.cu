// C ABI of libphyzb200 (include/phyzb.h): the BatchSim of phyz-gpu
// (crates/phyz-gpu/src/cuda/mod.rs:430-1377) re-designed around one fused
// multi-step kernel per launch. The handle owns every device buffer; host
// arrays are copied in and out through a device staging buffer and
// converted on the device between phyz's world-major f64 rows and the
// simulator's structure-of-arrays state (f32 or f64).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <thread>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/phyzb.h"
#include "capi_internal.h"
#include "pz_launch.h"
#include "pz_lanes.h"
#include "pz_pack.h"

namespace pzc {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}
const char* last_error() { return g_err.c_str(); }

int bounded_sync(cudaStream_t stream) {
    static const double limit = [] {
        const char* e = getenv("PHYZB_SYNC_TIMEOUT");
        const double v = e ? atof(e) : 0.0;
        return v > 0.0 ? v : 600.0;
    }();
    const auto t0 = std::chrono::steady_clock::now();
    for (long k = 0;; k++) {
        const cudaError_t q = cudaStreamQuery(stream);
        if (q == cudaSuccess) return PHYZB_OK;
        if (q != cudaErrorNotReady)
            return fail(PHYZB_ERR_CUDA, std::string("stream wait: ") + cudaGetErrorString(q));
        const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (waited > limit)
            return fail(PHYZB_ERR_CUDA, "stream wait: nothing finished within " + std::to_string(limit) + " s");
        // poll for the first millisecond, then back off
        if (waited > 1e-3) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

}  // namespace pzc

using namespace pzc;

namespace pzc {

bool is_f64(const phyzb_sim* s) { return s->precision == PHYZB_F64; }

int upload_layout(phyzb_sim* s, phyzb_sim::Layout& L, const std::vector<unsigned char>& blob) {
    if ((size_t)L.info.bytes > L.cap) {
        if (L.blob) cudaFree(L.blob);
        L.blob = nullptr;
        L.cap = 0;
        PZ_CUDA(cudaMalloc(&L.blob, L.info.bytes));
        L.cap = L.info.bytes;
    }
    PZ_CUDA(cudaMemcpy(L.blob, blob.data(), L.info.bytes, cudaMemcpyHostToDevice));
    L.host = blob;
    return PHYZB_OK;
}

template <class T>
int repack_t(phyzb_sim* s) {
    // kernels already queued may read the tables: drain the stream first
    PZ_TRY(bounded_sync(s->stream));
    pz::spec_release(s->spec);
    pz::spec_release(s->spec_sliced);
    s->spec = s->spec_sliced = nullptr;  // the tables change: specialize again at the next launch
    s->lanes_built = false;  // and split over lanes again
    std::vector<unsigned char> blob;
    phyzb_sim::Layout& L0 = s->lay[0];
    L0.info = pz::pack_model<T>(&s->model, s->nv, s->cfg, blob, 0);
    s->collidable = L0.info.collidable;
    PZ_TRY(upload_layout(s, L0, blob));
    cudaError_t e = pz::rollout_config<T>(L0.info.scratch, L0.info.bytes, s->nworld, L0.info.feat, 0, &L0.launch);
    if (e == cudaErrorInvalidConfiguration)
        return fail(PHYZB_ERR_TOO_LARGE, "per-world scratch (" + std::to_string(L0.info.scratch) +
                                             " slots) does not fit shared memory at 32 worlds per block");
    PZ_CUDA(e);
    s->use = 0;
    // PHYZB_TMEM=0: shared memory only; =1: a Tensor-Memory layout whenever
    // one configures (tests use it to cover both layouts at small sizes).
    const char* env = getenv("PHYZB_TMEM");
    if (env && env[0] == '0') return PHYZB_OK;
    const bool force = env && env[0] == '1';
    // Tensor-Memory layouts: records of up to 512 or 256 columns per world
    // (one or two warps per TMEM lane quarter); keep the best if it beats
    // the shared-memory layout clearly.
    double best = force ? -1.0 : L0.launch.score;
    for (int budget : {512, 256}) {
        std::vector<unsigned char> tb;
        pz::PackInfo ti = pz::pack_model<T>(&s->model, s->nv, s->cfg, tb, budget);
        if (ti.tmem_cols == 0) break;
        pz::LaunchCfg tc{};
        e = pz::rollout_config<T>(ti.scratch, ti.bytes, s->nworld, ti.feat, ti.tmem_cols, &tc);
        if (e != cudaSuccess) {  // not launchable here: keep the shared-memory layout
            cudaGetLastError();
            continue;
        }
        if (force ? tc.score > best : tc.score > best * 1.05) {
            best = tc.score;
            s->lay[1].info = ti;
            s->lay[1].launch = tc;
            PZ_TRY(upload_layout(s, s->lay[1], tb));
            s->use = 1;
        }
    }
    return PHYZB_OK;
}

int repack(phyzb_sim* s) { return is_f64(s) ? repack_t<double>(s) : repack_t<float>(s); }

void set_model_copy(phyzb_sim* s, const phyzb_model* m) {
    s->bodies.assign(m->bodies, m->bodies + m->nbodies);
    s->model = *m;
    s->model.bodies = s->bodies.data();
    // bodies on the longest root-to-leaf path (parents precede children)
    std::vector<int> d(s->bodies.size(), 1);
    s->depth = 0;
    for (size_t i = 0; i < s->bodies.size(); i++) {
        const int p = s->bodies[i].parent;
        if (p >= 0 && (size_t)p < i) d[i] = d[p] + 1;
        s->depth = std::max(s->depth, d[i]);
    }
}

template <class T>
pz::RolloutArgs<T> rollout_args(const phyzb_sim* s, const phyzb_sim::Layout& L, const void* ctrl, long long stride,
                                int nsteps) {
    pz::RolloutArgs<T> a;
    a.model_blob = L.blob;
    a.model_bytes = L.info.bytes;
    a.off_bi = L.info.off_bi;
    a.off_pd = L.info.off_pd;
    a.off_pdmap = L.info.off_pdmap;
    a.nb = s->nb;
    a.nv = s->nv;
    a.npd = (int)s->cfg.pd.size();
    a.contact = s->cfg.contact ? 1 : 0;
    a.feat = L.info.feat;
    a.dt = s->model.dt;
    a.gx = s->model.gravity[0];
    a.gy = s->model.gravity[1];
    a.gz = s->model.gravity[2];
    a.ground_h = s->ground_h;
    a.friction = s->friction;
    a.q = (T*)s->q;
    a.v = (T*)s->v;
    a.ctrl = (const T*)ctrl;
    a.ctrl_stride = stride;
    a.targets = (const T*)s->targets;
    a.qdd = (T*)s->qdd;
    a.cstate = s->cfg.contact ? (T*)s->cstate : nullptr;
    a.status = s->status;
    a.nworld = s->nworld;
    a.nsteps = nsteps;
    a.scratch = L.info.scratch;
    // impulse material: enable_contact_impulse over GroundContactParams::default
    // (cuda/mod.rs:680-701, contact_pipeline.rs:199-218)
    a.imp = (T*)s->imp;
    a.imp_slots = L.info.imp_slots;
    a.sweeps = s->sweeps;
    a.erp = s->erp;
    a.margin = 0.001;
    a.restitution = 0.0;
    a.rest_thr = 0.05;
    a.si_dmin = 0.9;
    a.si_dmax = 0.95;
    a.si_width = 0.001;
    a.si_mid = 0.5;
    a.si_power = 2.0;
    a.hf = (const float*)s->hf;
    a.hf_nx = s->cfg.terrain ? s->hf_nx : 0;
    a.hf_ny = s->cfg.terrain ? s->hf_ny : 0;
    a.hf_ox = s->hf_o[0];
    a.hf_oy = s->hf_o[1];
    a.hf_oz = s->hf_o[2];
    a.hf_cell = s->hf_cell;
    a.plane_body = s->cfg.contact ? s->cfg.plane_body : -1;
    a.plane_offset = s->plane[0];
    a.plane_max_depth = s->plane[1];
    a.plane_half_x = s->plane[2];
    a.plane_half_y = s->plane[3];
    return a;
}

bool specialized(const phyzb_sim* s) {
    return s->specialize == PHYZB_SPECIALIZE_ON ||
           (s->specialize == PHYZB_SPECIALIZE_AUTO && s->depth <= PHYZB_SPECIALIZE_AUTO_MAX_DEPTH &&
            s->nb <= PHYZB_SPECIALIZE_AUTO_MAX_BODIES);
}

pz::SpecLayout spec_layout(const pz::PackInfo& i, const std::vector<unsigned char>& blob, bool tm, int w0) {
    return pz::SpecLayout{blob.data(), i.bytes, i.off_bi, i.off_pd, i.off_pdmap, i.scratch, i.feat, i.tmem_cols, tm, w0};
}

// Time each compiled candidate on scratch copies of the simulator's state
// (one untimed launch of kTrialSteps steps, then the faster of two timed
// ones) and return the fastest, a later candidate replacing an earlier one
// only when 3 % faster (the shared-memory table comes first): whether more
// resident worlds beat the cheaper shared-memory record access depends on
// the model, so the choice is measured, not modelled. The launches are long
// enough that the per-tile load and store of the state do not decide it.
// Without device memory for the scratch copies the first candidate is kept
// untimed.
constexpr int kTrialSteps = 16;

template <class T>
int time_spec_choices(phyzb_sim* s, const std::vector<pz::PackInfo>& infos,
                      const std::vector<const std::vector<unsigned char>*>& hosts,
                      const std::vector<pz::SpecChoice>& ch, size_t* best) {
    struct Scratch {
        std::vector<void*> p;
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        ~Scratch() {
            for (void* x : p) cudaFree(x);
            if (e0) cudaEventDestroy(e0);
            if (e1) cudaEventDestroy(e1);
        }
        void* alloc(size_t bytes) {
            void* x = nullptr;
            if (cudaMalloc(&x, bytes > 0 ? bytes : 16) != cudaSuccess) return nullptr;
            p.push_back(x);
            return x;
        }
    } sc;
    const size_t sb = s->state_bytes();
    void* q = sc.alloc(sb);
    void* v = sc.alloc(sb);
    void* qdd = sc.alloc(sb);
    void* status = sc.alloc(2 * sizeof(int));
    void* cs = s->cstate ? sc.alloc((size_t)s->nworld * s->nb * PHYZB_CONTACT_STRIDE * s->esz()) : nullptr;
    void* imp = s->imp ? sc.alloc(s->imp_bytes) : nullptr;
    std::vector<void*> blobs;
    for (size_t i = 0; i < infos.size(); i++) blobs.push_back(sc.alloc(infos[i].bytes));
    bool room = q && v && qdd && status && (!s->cstate || cs) && (!s->imp || imp);
    for (void* b : blobs) room = room && b;
    if (!room) {  // no device memory to time the candidates on: keep the first
        cudaGetLastError();
        *best = 0;
        return PHYZB_OK;
    }
    PZ_CUDA(cudaMemcpyAsync(q, s->q, sb, cudaMemcpyDeviceToDevice, s->stream));
    PZ_CUDA(cudaMemcpyAsync(v, s->v, sb, cudaMemcpyDeviceToDevice, s->stream));
    if (imp) PZ_CUDA(cudaMemcpyAsync(imp, s->imp, s->imp_bytes, cudaMemcpyDeviceToDevice, s->stream));
    PZ_CUDA(cudaMemsetAsync(status, 0, 2 * sizeof(int), s->stream));
    for (size_t i = 0; i < infos.size(); i++)
        PZ_CUDA(cudaMemcpyAsync(blobs[i], hosts[i]->data(), infos[i].bytes, cudaMemcpyHostToDevice, s->stream));
    PZ_CUDA(cudaEventCreate(&sc.e0));
    PZ_CUDA(cudaEventCreate(&sc.e1));
    float best_ms = -1.0f;
    for (size_t c = 0; c < ch.size(); c++) {
        phyzb_sim::Layout L;
        L.info = infos[ch[c].layout];
        L.blob = blobs[ch[c].layout];
        pz::RolloutArgs<T> a = rollout_args<T>(s, L, s->ctrl, 0, kTrialSteps);
        a.q = (T*)q;
        a.v = (T*)v;
        a.qdd = (T*)qdd;
        a.cstate = (T*)cs;
        a.imp = (T*)imp;
        a.status = (int*)status;
        L.blob = nullptr;  // owned by the scratch
        if (pz::spec_launch<T>(ch[c].k, a, ch[c].cfg, s->stream) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        float ms = -1.0f;
        for (int rep = 0; rep < 2; rep++) {
            PZ_CUDA(cudaEventRecord(sc.e0, s->stream));
            PZ_CUDA(pz::spec_launch<T>(ch[c].k, a, ch[c].cfg, s->stream));
            PZ_CUDA(cudaEventRecord(sc.e1, s->stream));
            PZ_CUDA(cudaEventSynchronize(sc.e1));
            float t = 0.0f;
            PZ_CUDA(cudaEventElapsedTime(&t, sc.e0, sc.e1));
            if (ms < 0.0f || t < ms) ms = t;
        }
        if (best_ms < 0.0f || ms < 0.97f * best_ms) {
            best_ms = ms;
            *best = c;
        }
    }
    PZ_TRY(bounded_sync(s->stream));
    if (best_ms < 0.0f) return fail(PHYZB_ERR_CUDA, "no specialized kernel candidate launched");
    return PHYZB_OK;
}

// Compile the model-specialized kernel of the current tables: candidates
// are the shared-memory layout and (unless PHYZB_TMEM=0; only it with
// PHYZB_TMEM=1) a Tensor-Memory layout, each at two widths; the fastest on
// this simulator's state is kept and its table uploaded into spec_lay.
template <class T>
int prepare_spec(phyzb_sim* s) {
    const phyzb_sim::Layout& L0 = s->lay[0];
    std::vector<pz::SpecLayout> cands;
    std::vector<pz::PackInfo> infos;
    std::vector<const std::vector<unsigned char>*> hosts;
    const char* env = getenv("PHYZB_TMEM");
    auto add = [&](const pz::PackInfo& i, const std::vector<unsigned char>& b, bool tm, int w0) {
        cands.push_back(spec_layout(i, b, tm, w0));
        infos.push_back(i);
        hosts.push_back(&b);
    };
    if (!(env && env[0] == '1')) add(L0.info, L0.host, false, L0.launch.W);
    std::vector<unsigned char> tb;
    pz::PackInfo ti{};
    if (!(env && env[0] == '0')) {
        for (int budget : {512, 256}) {
            std::vector<unsigned char> b;
            const pz::PackInfo i = pz::pack_model<T>(&s->model, s->nv, s->cfg, b, budget);
            if (i.tmem_cols == 0) break;
            pz::LaunchCfg c{};
            if (pz::rollout_config<T>(i.scratch, i.bytes, s->nworld, i.feat, i.tmem_cols, &c) != cudaSuccess) {
                cudaGetLastError();  // not launchable as a generic variant: try the smaller budget
                continue;
            }
            tb.swap(b);
            ti = i;
            add(ti, tb, true, c.W);
            break;
        }
    }
    if (cands.empty()) add(L0.info, L0.host, false, L0.launch.W);
    const pz::RolloutArgs<T> a = rollout_args<T>(s, L0, nullptr, 0, 1);
    std::vector<pz::SpecChoice> ch;
    std::string err;
    if (pz::spec_candidates<T>(cands.data(), (int)cands.size(), a, &ch, &err) != cudaSuccess) {
        cudaGetLastError();
        return fail(PHYZB_ERR_CUDA, err);
    }
    size_t pick = 0;
    if (ch.size() > 1) PZ_TRY(time_spec_choices<T>(s, infos, hosts, ch, &pick));
    const int li = ch[pick].layout;
    s->spec_lay.info = infos[li];
    PZ_TRY(upload_layout(s, s->spec_lay, *hosts[li]));
    s->spec_lay.launch = ch[pick].cfg;
    s->spec = ch[pick].k;
    pz::spec_retain(s->spec);  // the candidates not picked may now be unloaded
    return PHYZB_OK;
}

// Why this simulator's settings keep one thread per world ("" when the
// model may split over lanes).
std::string lanes_unsupported(const phyzb_sim* s) {
    if (!s->cfg.pd.empty()) return "PD servos are enabled";
    if (s->cfg.contact && s->cfg.impulse) return "impulse contact is enabled";
    if (s->cfg.contact && s->cfg.terrain) return "heightfield / plane contact is enabled";
    return "";
}

// Plan and pack the lanes' sub-model tables (pz_lanes.h) and configure the
// lanes kernel; on a model or settings that do not split, lanes_ok stays
// false with the reason.
template <class T>
int build_lanes(phyzb_sim* s) {
    s->lanes_built = true;
    s->lanes_ok = false;
    s->lanes_why = lanes_unsupported(s);
    if (!s->lanes_why.empty()) return PHYZB_OK;
    pz::LanePlan plan;
    s->lanes_why = pz::plan_lanes(&s->model, s->lanes, &plan);
    if (!s->lanes_why.empty()) return PHYZB_OK;
    const int L = s->lanes;
    std::vector<std::vector<unsigned char>> blobs(L);
    std::vector<pz::PackInfo> infos(L);
    int bytes = 0, scratch = 0, nv_max = 1, feat_or = 0;
    bool perm1 = true;
    pz::LanesArgs la{};
    la.lanes = L;
    la.nt = plan.nt;
    la.trunk_nv = 0;
    for (int t = 0; t < plan.nt; t++) la.trunk_nv += pz::ndof_of(plan.sub[0][t].joint_type);
    for (int l = 0; l < L; l++) {
        phyzb_model sub{};
        sub.nbodies = (int)plan.sub[l].size();
        for (int k = 0; k < 3; k++) sub.gravity[k] = s->model.gravity[k];
        sub.dt = s->model.dt;
        sub.bodies = plan.sub[l].data();
        pz::PackCfg c = s->cfg;
        c.gk.clear();
        c.gd.clear();
        for (int b : plan.bodies[l]) {
            c.gk.push_back((int)s->cfg.gk.size() > b ? s->cfg.gk[b] : 0.0);
            c.gd.push_back((int)s->cfg.gd.size() > b ? s->cfg.gd[b] : 0.0);
        }
        c.force_branch = plan.force_branch;
        c.force_chain = plan.force_chain;
        const int nv = (int)plan.dof[l].size();
        infos[l] = pz::pack_model<T>(&sub, nv, c, blobs[l], 0);
        bytes = std::max(bytes, infos[l].bytes);
        scratch = std::max(scratch, infos[l].scratch);
        nv_max = std::max(nv_max, nv);
        feat_or |= infos[l].feat & ~8;
        perm1 = perm1 && (infos[l].feat & 8) != 0;
        la.nb[l] = sub.nbodies;
        la.nv[l] = nv;
        la.off_bi[l] = infos[l].off_bi;
        la.off_pd[l] = infos[l].off_pd;
        la.off_pdmap[l] = infos[l].off_pdmap;
    }
    const int feat = feat_or | ((perm1 && (feat_or & 4)) ? 8 : 0);
    bytes = (bytes + 15) & ~15;
    la.lane_bytes = bytes;
    la.off_gdof = bytes * L;
    la.nv_max = nv_max;
    const int total = la.off_gdof + (((int)sizeof(int) * L * nv_max + 15) & ~15);
    std::vector<unsigned char> host(total, 0);
    for (int l = 0; l < L; l++) {
        std::memcpy(host.data() + l * bytes, blobs[l].data(), blobs[l].size());
        int* g = reinterpret_cast<int*>(host.data() + la.off_gdof) + l * nv_max;
        for (int j = 0; j < (int)plan.dof[l].size(); j++) g[j] = plan.dof[l][j];
    }
    if ((size_t)total > s->lanes_cap) {
        free_ptr(s->lanes_blob);
        s->lanes_cap = 0;
        PZ_CUDA(cudaMalloc(&s->lanes_blob, total));
        s->lanes_cap = total;
    }
    PZ_CUDA(cudaMemcpy(s->lanes_blob, host.data(), total, cudaMemcpyHostToDevice));
    cudaError_t e = pz::lanes_config<T>(feat, L, scratch, total, s->nworld, &s->lanes_launch);
    if (e == cudaErrorInvalidConfiguration) {
        cudaGetLastError();
        s->lanes_why = "the sub-models' scratch does not fit shared memory";
        return PHYZB_OK;
    }
    PZ_CUDA(e);
    s->la = la;
    s->lanes_bytes = total;
    s->lanes_scratch = scratch;
    s->lanes_feat = feat;
    s->lanes_ok = true;
    return PHYZB_OK;
}

template <class T>
int launch_t(phyzb_sim* s, const void* ctrl, long long stride, int nsteps) {
    if (s->lanes >= 2 && nsteps >= 2) {
        if (!s->lanes_built) PZ_TRY(build_lanes<T>(s));
        if (s->lanes_ok) {
            // every step but the last on the lanes kernel; the last on the
            // one-thread kernel, which writes its accelerations and contact state
            pz::RolloutArgs<T> a = rollout_args<T>(s, s->lay[0], ctrl, stride, nsteps - 1);
            a.model_blob = s->lanes_blob;
            a.model_bytes = s->lanes_bytes;
            a.feat = s->lanes_feat;
            a.scratch = s->lanes_scratch;
            PZ_CUDA(pz::launch_lanes<T>(a, s->la, s->lanes_launch, s->stream));
            ctrl = (const char*)ctrl + (size_t)(nsteps - 1) * (size_t)stride * sizeof(T);
            nsteps = 1;
        }
    }
    const bool spec = specialized(s);
    if (spec && !s->spec) PZ_TRY(prepare_spec<T>(s));
    const phyzb_sim::Layout& L = spec ? s->spec_lay : s->lay[s->use];
    pz::RolloutArgs<T> a = rollout_args<T>(s, L, ctrl, stride, nsteps);
    // tile or slice mode (pz::plan_slices)
    pz::LaunchCfg cfg = L.launch;
    const int chunk = s->slices ? pz::plan_slices(L.launch, s->nworld, nsteps, s->slice_force, &cfg) : 0;
    if (chunk > 0) {
        PZ_CUDA(cudaMemsetAsync(s->slices, 0, s->slices_bytes(), s->stream));
        if (s->slice_stall) {
            s->slice_stall_start = (unsigned)((s->nworld + 31) / 32);
            PZ_CUDA(cudaMemcpyAsync(s->slices, &s->slice_stall_start, sizeof(unsigned), cudaMemcpyHostToDevice,
                                    s->stream));
        }
        a.chunk = chunk;
        a.slices = s->slices;
    } else {
        cfg = L.launch;
    }
    if (spec) {
        if (chunk > 0 && !s->spec_sliced) {
            // the slice-mode twin of the chosen kernel: same table and width
            const phyzb_sim::Layout& SL = s->spec_lay;
            std::string err;
            if (pz::spec_sliced<T>(spec_layout(SL.info, SL.host, SL.launch.tm != 0, SL.launch.W),
                                   rollout_args<T>(s, SL, nullptr, 0, 1), SL.launch.slice_W, &s->spec_sliced,
                                   &err) != cudaSuccess) {
                cudaGetLastError();
                s->spec_sliced = nullptr;
                return fail(PHYZB_ERR_CUDA, err);
            }
            pz::spec_retain(s->spec_sliced);
        }
        PZ_CUDA(pz::spec_launch<T>(chunk > 0 ? s->spec_sliced : s->spec, a, cfg, s->stream));
    } else {
        PZ_CUDA(pz::launch_rollout<T>(a, cfg, s->stream));
    }
    return PHYZB_OK;
}

int launch(phyzb_sim* s, const void* ctrl, long long stride, int nsteps) {
    return is_f64(s) ? launch_t<double>(s, ctrl, stride, nsteps) : launch_t<float>(s, ctrl, stride, nsteps);
}

// host rows [nworld][width] f64 -> device SoA [width][nworld] in the sim precision
int upload_rows(phyzb_sim* s, const double* host, int width, void* dst) {
    const size_t bytes = (size_t)s->nworld * width * sizeof(double);
    if (bytes == 0) return PHYZB_OK;
    if (bytes > s->staging_bytes) return fail(PHYZB_ERR_INVALID, "internal: staging too small");
    PZ_CUDA(cudaMemcpyAsync(s->staging, host, bytes, cudaMemcpyHostToDevice, s->stream));
    cudaError_t e = is_f64(s) ? pz::launch_aos_to_soa<double, double>((const double*)s->staging, (double*)dst,
                                                                      s->nworld, width, 1, s->stream)
                              : pz::launch_aos_to_soa<double, float>((const double*)s->staging, (float*)dst,
                                                                     s->nworld, width, 1, s->stream);
    PZ_CUDA(e);
    // the caller may reuse `host` as soon as this returns
    PZ_TRY(bounded_sync(s->stream));
    return PHYZB_OK;
}

// device SoA [width][nworld] -> host rows [nworld][width] f64
int download_rows(phyzb_sim* s, const void* src, int width, double* host) {
    const size_t bytes = (size_t)s->nworld * width * sizeof(double);
    if (bytes == 0) return PHYZB_OK;
    cudaError_t e = is_f64(s) ? pz::launch_soa_to_aos<double, double>((const double*)src, (double*)s->staging,
                                                                      s->nworld, width, s->stream)
                              : pz::launch_soa_to_aos<float, double>((const float*)src, (double*)s->staging,
                                                                     s->nworld, width, s->stream);
    PZ_CUDA(e);
    PZ_CUDA(cudaMemcpyAsync(host, s->staging, bytes, cudaMemcpyDeviceToHost, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    return PHYZB_OK;
}

void free_ptr(void*& p) {
    if (p) cudaFree(p);
    p = nullptr;
}

int check_sim(const phyzb_sim* s) {
    if (!s) return fail(PHYZB_ERR_INVALID, "simulator handle is null");
    return PHYZB_OK;
}

int read_status(phyzb_sim* s) {
    int st[2] = {0, 0};
    PZ_CUDA(cudaMemcpyAsync(st, s->status, sizeof(st), cudaMemcpyDeviceToHost, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    if (st[0] & 1)
        return fail(PHYZB_ERR_NONFINITE, "state went non-finite on device (first world " + std::to_string(st[1]) + ")");
    if (st[0] & 2) return fail(PHYZB_ERR_CUDA, "a slice-mode run waited past its bound for the run before it");
    return PHYZB_OK;
}

// contact_pipeline.rs:229-237 (SolRef error reduction at dt)
double solref_erp_from(double timeconst, double dampratio, double dt) {
    if (dt <= 0.0) return 0.0;
    const double tau = std::max(timeconst, 0.0), zeta = std::max(dampratio, 1e-6);
    const double denom = 2.0 * tau * zeta * zeta + dt;
    return denom <= 0.0 ? 1.0 : dt / denom;
}

// The impulse buffer sized for the current layout, zeroed (a fresh warm start).
int reset_impulse_state(phyzb_sim* s) {
    const size_t bytes = (size_t)s->lay[0].info.imp_slots * s->nworld * s->esz();
    if (bytes > s->imp_bytes) {
        free_ptr(s->imp);
        s->imp_bytes = 0;
        PZ_CUDA(cudaMalloc(&s->imp, bytes));
        s->imp_bytes = bytes;
    }
    if (bytes) PZ_CUDA(cudaMemsetAsync(s->imp, 0, bytes, s->stream));
    return PHYZB_OK;
}

// contact_pipeline.rs:651-672 validate_heightfield (plus finite values)
int check_heightfield(const phyzb_heightfield* hf) {
    if (hf->nx < 1 || hf->ny < 1) return fail(PHYZB_ERR_INVALID, "heightfield needs at least one node per axis");
    if (!hf->heights) return fail(PHYZB_ERR_INVALID, "heightfield heights are null");
    if (!(std::isfinite(hf->cell) && hf->cell > 0.0))
        return fail(PHYZB_ERR_INVALID, "heightfield cell must be positive, got " + std::to_string(hf->cell));
    for (int k = 0; k < 3; k++)
        if (!std::isfinite(hf->origin[k])) return fail(PHYZB_ERR_INVALID, "heightfield origin must be finite");
    const size_t n = (size_t)hf->nx * hf->ny;
    for (size_t i = 0; i < n; i++)
        if (!std::isfinite(hf->heights[i])) return fail(PHYZB_ERR_INVALID, "heightfield heights must be finite");
    return PHYZB_OK;
}

// Heightfield nodes into the device buffer (already large enough) and the
// grid header into the simulator; kernels already queued finish first.
int upload_heightfield(phyzb_sim* s, const phyzb_heightfield* hf) {
    PZ_TRY(bounded_sync(s->stream));
    PZ_CUDA(cudaMemcpy(s->hf, hf->heights, (size_t)hf->nx * hf->ny * sizeof(float), cudaMemcpyHostToDevice));
    s->hf_nx = hf->nx;
    s->hf_ny = hf->ny;
    for (int k = 0; k < 3; k++) s->hf_o[k] = hf->origin[k];
    s->hf_cell = hf->cell;
    return PHYZB_OK;
}

int set_contact(phyzb_sim* s, double ground, double friction, const double* k, const double* d, bool impulse,
                const phyzb_body_plane* plane = nullptr, const phyzb_heightfield* hf = nullptr) {
    if (plane) {  // contact_pipeline.rs:614-627
        if (plane->body < 0 || plane->body >= s->nb)
            return fail(PHYZB_ERR_INVALID, "plane body " + std::to_string(plane->body) +
                                               " out of range for a model with " + std::to_string(s->nb) + " bodies");
        if (plane->n_exclude < 0 || (plane->n_exclude > 0 && !plane->exclude))
            return fail(PHYZB_ERR_INVALID, "plane exclude list is null");
        for (int k = 0; k < plane->n_exclude; k++)
            if (plane->exclude[k] < 0 || plane->exclude[k] >= s->nb)
                return fail(PHYZB_ERR_INVALID, "plane exclude body " + std::to_string(plane->exclude[k]) +
                                                   " out of range");
        const double pv[4] = {plane->offset, plane->max_depth, plane->half_x, plane->half_y};
        for (double x : pv)
            if (!std::isfinite(x)) return fail(PHYZB_ERR_INVALID, "plane parameters must be finite");
    }
    if (hf) PZ_TRY(check_heightfield(hf));
    int collidable = 0;
    for (int i = 0; i < s->nb; i++)
        if (s->bodies[i].geom_type != PHYZB_GEOM_NONE) collidable++;
    if (collidable == 0) {
        // layout.rs:282-297 no_collidable_geometry_error
        std::string names;
        for (int i = 0; i < s->nb; i++) names += (i ? ", body " : "body ") + std::to_string(i);
        return fail(PHYZB_ERR_INVALID,
                    "ground contact enabled but no body has GPU-collidable geometry (supported: sphere, box, "
                    "capsule, cylinder, mesh); bodies without a supported shape: [" + names + "]");
    }
    if (!std::isfinite(ground) || !std::isfinite(friction))
        return fail(PHYZB_ERR_INVALID, "contact parameters must be finite");
    for (int i = 0; i < s->nb; i++)
        if (!std::isfinite(k[i]) || !std::isfinite(d[i]))
            return fail(PHYZB_ERR_INVALID, "contact gains must be finite");
    if (!s->cstate) {
        const size_t bytes = (size_t)s->nworld * s->nb * PHYZB_CONTACT_STRIDE * s->esz();
        PZ_CUDA(cudaMalloc(&s->cstate, bytes > 0 ? bytes : 16));
        PZ_CUDA(cudaMemsetAsync(s->cstate, 0, bytes, s->stream));
    }
    // the node buffer is sized to this first field (1 node without one)
    const size_t nodes = hf ? (size_t)hf->nx * hf->ny : 1;
    if (nodes > s->hf_cap) {
        free_ptr(s->hf);
        s->hf_cap = 0;
        PZ_CUDA(cudaMalloc(&s->hf, nodes * sizeof(float)));
        s->hf_cap = nodes;
    }
    if (hf) {
        PZ_TRY(upload_heightfield(s, hf));
    } else {  // no terrain: the flat ground (a plane alone also runs the full-frame kernel)
        s->hf_nx = s->hf_ny = 0;
    }
    s->cfg.contact = true;
    s->cfg.impulse = impulse;
    // full world frames (kernel feature bit 32) serve both the heightfield
    // and the body-attached plane
    s->cfg.terrain = hf != nullptr || plane != nullptr;
    s->cfg.plane_body = plane ? plane->body : -1;
    s->cfg.plane_exclude.clear();
    if (plane) {
        s->cfg.plane_exclude.assign(plane->exclude, plane->exclude + plane->n_exclude);
        s->plane[0] = plane->offset;
        s->plane[1] = plane->max_depth;
        s->plane[2] = plane->half_x;
        s->plane[3] = plane->half_y;
    }
    s->cfg.gk.assign(k, k + s->nb);
    s->cfg.gd.assign(d, d + s->nb);
    s->ground_h = ground;
    s->friction = friction;
    s->erp = solref_erp_from(0.02, 1.0, s->model.dt);
    PZ_TRY(repack(s));
    if (impulse) PZ_TRY(reset_impulse_state(s));
    return PHYZB_OK;
}

int ensure_pipeline(phyzb_sim* s, size_t raw_bytes, size_t soa_bytes) {
    if (raw_bytes > s->pipe_raw_bytes) {
        for (int b = 0; b < 2; b++) {
            free_ptr(s->pipe_raw[b]);
            PZ_CUDA(cudaMalloc(&s->pipe_raw[b], raw_bytes));
        }
        s->pipe_raw_bytes = raw_bytes;
    }
    if (soa_bytes > s->pipe_soa_bytes) {
        for (int b = 0; b < 2; b++) {
            free_ptr(s->pipe_soa[b]);
            PZ_CUDA(cudaMalloc(&s->pipe_soa[b], soa_bytes));
        }
        s->pipe_soa_bytes = soa_bytes;
    }
    for (int b = 0; b < 2; b++) {
        if (!s->ev_copied[b]) PZ_CUDA(cudaEventCreateWithFlags(&s->ev_copied[b], cudaEventDisableTiming));
        if (!s->ev_converted[b]) PZ_CUDA(cudaEventCreateWithFlags(&s->ev_converted[b], cudaEventDisableTiming));
    }
    if (!s->copy_stream) PZ_CUDA(cudaStreamCreateWithFlags(&s->copy_stream, cudaStreamNonBlocking));
    return PHYZB_OK;
}

void destroy_sim(phyzb_sim* s) {
    if (!s) return;
    DeviceGuard g(s->device);
    destroy_policy(s);
    if (s->stream) bounded_sync(s->stream);
    if (s->copy_stream) bounded_sync(s->copy_stream);
    pz::spec_release(s->spec);
    pz::spec_release(s->spec_sliced);
    s->spec = s->spec_sliced = nullptr;
    free_ptr(s->lanes_blob);
    free_ptr(s->q);
    free_ptr(s->v);
    free_ptr(s->ctrl);
    free_ptr(s->qdd);
    free_ptr(s->targets);
    free_ptr(s->cstate);
    free_ptr(s->imp);
    free_ptr(s->hf);
    void* st = s->status;
    free_ptr(st);
    void* sl = s->slices;
    free_ptr(sl);
    free_ptr(s->lay[0].blob);
    free_ptr(s->lay[1].blob);
    free_ptr(s->spec_lay.blob);
    free_ptr(s->staging);
    free_ptr(s->hist_q);
    free_ptr(s->hist_v);
    for (int b = 0; b < 2; b++) {
        free_ptr(s->pipe_raw[b]);
        free_ptr(s->pipe_soa[b]);
        if (s->ev_copied[b]) cudaEventDestroy(s->ev_copied[b]);
        if (s->ev_converted[b]) cudaEventDestroy(s->ev_converted[b]);
    }
    free_ptr(s->obj);
    if (s->obj_host) cudaFreeHost(s->obj_host);
    if (s->ev_obj) cudaEventDestroy(s->ev_obj);
    if (s->copy_stream) cudaStreamDestroy(s->copy_stream);
    if (s->own_stream) cudaStreamDestroy(s->own_stream);
    delete s;
}

}  // namespace pzc

extern "C" {

const char* phyzb_last_error(void) { return pzc::last_error(); }

int phyzb_abi_version(void) { return PHYZB_ABI_VERSION; }

int phyzb_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int phyzb_create(const phyzb_model* model, int64_t nworld, int device, int precision, phyzb_sim** out) {
    if (!out) return fail(PHYZB_ERR_INVALID, "out pointer is null");
    *out = nullptr;
    int nv = 0;
    const std::string why = pz::validate_model(model, &nv);
    if (!why.empty()) {
        const bool too_large = model && model->nbodies > PHYZB_MAX_BODIES;
        return fail(too_large ? PHYZB_ERR_TOO_LARGE : PHYZB_ERR_INVALID, why);
    }
    if (nworld < 1) return fail(PHYZB_ERR_INVALID, "nworld must be >= 1");
    if (precision != PHYZB_F32 && precision != PHYZB_F64) return fail(PHYZB_ERR_INVALID, "precision must be F32 or F64");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(PHYZB_ERR_NO_DEVICE, "no CUDA device is available");
    }
    if (device < 0 || device >= ndev)
        return fail(PHYZB_ERR_NO_DEVICE, "device " + std::to_string(device) + " out of range (" + std::to_string(ndev) +
                                             " visible)");
    DeviceGuard g(device);
    phyzb_sim* s = new phyzb_sim();
    s->device = device;
    s->precision = precision;
    s->nworld = nworld;
    s->nb = model->nbodies;
    s->nv = nv;
    if (const char* env = getenv("PHYZB_SPECIALIZE"))
        s->specialize = env[0] == '1' ? PHYZB_SPECIALIZE_ON : (env[0] == 'a' ? PHYZB_SPECIALIZE_AUTO : PHYZB_SPECIALIZE_OFF);
    set_model_copy(s, model);
    if (const char* env = getenv("PHYZB_LANES")) {
        // a new simulator's lanes per world, where its model splits (the test
        // suite runs with it to cover the lanes kernel everywhere it applies;
        // settings that keep one thread per world are checked at each launch)
        const int l = atoi(env);
        pz::LanePlan plan;
        if ((l == 2 || l == 4 || l == 8) && pz::plan_lanes(&s->model, l, &plan).empty()) s->lanes = l;
    }
    auto bail = [&](int code) {
        destroy_sim(s);
        return code;
    };
    if (cudaStreamCreateWithFlags(&s->own_stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(PHYZB_ERR_CUDA, "cudaStreamCreate failed"));
    s->stream = s->own_stream;
    const size_t sb = s->state_bytes() > 0 ? s->state_bytes() : 16;
    void** bufs[] = {&s->q, &s->v, &s->ctrl, &s->qdd};
    for (void** b : bufs) {
        cudaError_t e = cudaMalloc(b, sb);
        if (e != cudaSuccess) return bail(fail(PHYZB_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e)));
        cudaMemsetAsync(*b, 0, sb, s->stream);
    }
    void* st = nullptr;
    if (cudaMalloc(&st, 2 * sizeof(int)) != cudaSuccess) return bail(fail(PHYZB_ERR_CUDA, "cudaMalloc status"));
    s->status = (int*)st;
    const int init[2] = {0, 0x7fffffff};
    cudaMemcpy(s->status, init, sizeof(init), cudaMemcpyHostToDevice);
    if (const char* env = getenv("PHYZB_SLICES")) s->slice_force = env[0] == '0' ? 0 : (env[0] == '1' ? 1 : -1);
    if (const char* env = getenv("PHYZB_SLICES_STALL")) s->slice_stall = env[0] == '1';
    if (cudaMalloc(&s->slices, s->slices_bytes()) != cudaSuccess) return bail(fail(PHYZB_ERR_CUDA, "cudaMalloc slices"));
    s->staging_bytes = (size_t)nworld * std::max(nv, s->nb * PHYZB_CONTACT_STRIDE) * sizeof(double);
    if (cudaMalloc(&s->staging, s->staging_bytes > 0 ? s->staging_bytes : 16) != cudaSuccess)
        return bail(fail(PHYZB_ERR_CUDA, "cudaMalloc staging"));
    int r = repack(s);
    if (r != PHYZB_OK) {
        std::string msg = pzc::last_error();
        destroy_sim(s);
        return fail(r, msg);
    }
    if (bounded_sync(s->stream) != PHYZB_OK) return bail(PHYZB_ERR_CUDA);
    *out = s;
    return PHYZB_OK;
}

int phyzb_destroy(phyzb_sim* sim) {
    destroy_sim(sim);
    return PHYZB_OK;
}

int phyzb_set_model(phyzb_sim* s, const phyzb_model* model) {
    PZ_TRY(check_sim(s));
    int nv = 0;
    const std::string why = pz::validate_model(model, &nv);
    if (!why.empty()) return fail(PHYZB_ERR_INVALID, why);
    if (model->nbodies != s->nb || nv != s->nv)
        return fail(PHYZB_ERR_INVALID, "set_model: shape changed (" + std::to_string(model->nbodies) + " bodies, nv " +
                                           std::to_string(nv) + " vs " + std::to_string(s->nb) + " bodies, nv " +
                                           std::to_string(s->nv) + "); build a new simulator");
    for (int i = 0; i < s->nb; i++)
        if (model->bodies[i].joint_type != s->bodies[i].joint_type || model->bodies[i].parent != s->bodies[i].parent)
            return fail(PHYZB_ERR_INVALID, "set_model: topology or joint types changed; build a new simulator");
    DeviceGuard g(s->device);
    set_model_copy(s, model);
    PZ_TRY(repack(s));
    // a geometry change can add impulse slots: those start from zero
    if (s->cfg.contact && s->cfg.impulse &&
        (size_t)s->lay[0].info.imp_slots * s->nworld * s->esz() > s->imp_bytes)
        PZ_TRY(reset_impulse_state(s));
    return PHYZB_OK;
}

int phyzb_enable_ground_contact(phyzb_sim* s, double ground_height, double stiffness, double damping, double friction,
                                int32_t* collidable_out) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    std::vector<double> k(s->nb, stiffness), d(s->nb, damping);
    PZ_TRY(set_contact(s, ground_height, friction, k.data(), d.data(), false));
    if (collidable_out) *collidable_out = s->collidable;
    return PHYZB_OK;
}

int phyzb_enable_ground_contact_per_body(phyzb_sim* s, double ground_height, double friction,
                                         const double* stiffness, const double* damping, int32_t* collidable_out) {
    PZ_TRY(check_sim(s));
    if (!stiffness || !damping) return fail(PHYZB_ERR_INVALID, "per-body gains are null");
    DeviceGuard g(s->device);
    PZ_TRY(set_contact(s, ground_height, friction, stiffness, damping, false));
    if (collidable_out) *collidable_out = s->collidable;
    return PHYZB_OK;
}

int phyzb_enable_contact_terrain(phyzb_sim* s, double ground_height, double friction, const double* stiffness,
                                 const double* damping, const phyzb_body_plane* plane, const phyzb_heightfield* hf,
                                 int32_t* collidable_out) {
    PZ_TRY(check_sim(s));
    if (!stiffness || !damping) return fail(PHYZB_ERR_INVALID, "per-body gains are null");
    DeviceGuard g(s->device);
    PZ_TRY(set_contact(s, ground_height, friction, stiffness, damping, false, plane, hf));
    if (collidable_out) *collidable_out = s->collidable;
    return PHYZB_OK;
}

int phyzb_set_heightfield(phyzb_sim* s, const phyzb_heightfield* hf) {
    PZ_TRY(check_sim(s));
    if (!hf) return fail(PHYZB_ERR_INVALID, "heightfield is null");
    if (!s->cfg.contact)
        return fail(PHYZB_ERR_STATE, "contact not enabled — call enable_contact_terrain first");
    PZ_TRY(check_heightfield(hf));
    const size_t nodes = (size_t)hf->nx * hf->ny;
    if (nodes > s->hf_cap)
        return fail(PHYZB_ERR_INVALID, "heightfield has " + std::to_string(nodes) +
                                           " nodes but the buffer was sized for " + std::to_string(s->hf_cap) +
                                           "; enable contact with the largest grid first");
    DeviceGuard g(s->device);
    PZ_TRY(upload_heightfield(s, hf));
    if (!s->cfg.terrain) {  // the kernel variant changes
        s->cfg.terrain = true;
        PZ_TRY(repack(s));
    }
    return PHYZB_OK;
}

int phyzb_enable_contact_impulse(phyzb_sim* s, double ground_height, double friction, const double* stiffness,
                                 const double* damping, const phyzb_body_plane* plane, const phyzb_heightfield* hf,
                                 int32_t* collidable_out) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    // the per-body gains only enter the penalty law; they are kept (and
    // checked) so a later penalty enable sees the same table
    std::vector<double> k(s->nb, 0.0), d(s->nb, 0.0);
    if (stiffness) k.assign(stiffness, stiffness + s->nb);
    if (damping) d.assign(damping, damping + s->nb);
    PZ_TRY(set_contact(s, ground_height, friction, k.data(), d.data(), true, plane, hf));
    if (collidable_out) *collidable_out = s->collidable;
    return PHYZB_OK;
}

int phyzb_set_contact_sweeps(phyzb_sim* s, int32_t sweeps) {
    PZ_TRY(check_sim(s));
    if (sweeps < 1 || sweeps > PHYZB_MAX_CONTACT_SWEEPS)
        return fail(PHYZB_ERR_INVALID, "contact sweeps must be in [1, " + std::to_string(PHYZB_MAX_CONTACT_SWEEPS) +
                                           "], got " + std::to_string(sweeps));
    s->sweeps = sweeps;
    return PHYZB_OK;
}

int phyzb_disable_contact(phyzb_sim* s) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    s->cfg.contact = false;
    s->cfg.impulse = false;
    s->cfg.terrain = false;
    return repack(s);
}

int phyzb_collidable_bodies(const phyzb_sim* s) { return (s && s->cfg.contact) ? s->collidable : 0; }

int phyzb_enable_pd(phyzb_sim* s, const phyzb_pd_dof* dofs, int32_t n) {
    PZ_TRY(check_sim(s));
    // layout.rs:300-315 check_pd_dofs
    if (!dofs || n <= 0) return fail(PHYZB_ERR_INVALID, "PD pipeline needs at least one servoed DOF");
    for (int k = 0; k < n; k++)
        if (dofs[k].q_index < 0 || dofs[k].q_index >= s->nv || dofs[k].v_index < 0 || dofs[k].v_index >= s->nv)
            return fail(PHYZB_ERR_INVALID, "PD DOF out of range: q_index " + std::to_string(dofs[k].q_index) +
                                               " (nq " + std::to_string(s->nv) + "), v_index " +
                                               std::to_string(dofs[k].v_index) + " (nv " + std::to_string(s->nv) +
                                               ")");
    DeviceGuard g(s->device);
    const bool same = (int)s->cfg.pd.size() == n && s->targets;
    s->cfg.pd.assign(dofs, dofs + n);
    if (!same) {
        free_ptr(s->targets);
        const size_t bytes = (size_t)n * s->nworld * s->esz();
        PZ_CUDA(cudaMalloc(&s->targets, bytes));
        PZ_CUDA(cudaMemsetAsync(s->targets, 0, bytes, s->stream));
    }
    return repack(s);
}

int phyzb_set_position_targets(phyzb_sim* s, const double* targets) {
    PZ_TRY(check_sim(s));
    if (s->cfg.pd.empty()) return fail(PHYZB_ERR_STATE, "PD control not enabled — call enable_pd_control first");
    if (!targets) return fail(PHYZB_ERR_INVALID, "targets is null");
    DeviceGuard g(s->device);
    return upload_rows(s, targets, (int)s->cfg.pd.size(), s->targets);
}

int phyzb_load_states(phyzb_sim* s, const double* q, const double* v, const double* ctrl) {
    PZ_TRY(check_sim(s));
    if (!q || !v) return fail(PHYZB_ERR_INVALID, "q and v must not be null");
    DeviceGuard g(s->device);
    PZ_TRY(upload_rows(s, q, s->nv, s->q));
    PZ_TRY(upload_rows(s, v, s->nv, s->v));
    if (ctrl) return upload_rows(s, ctrl, s->nv, s->ctrl);
    PZ_CUDA(cudaMemsetAsync(s->ctrl, 0, s->state_bytes(), s->stream));
    PZ_TRY(bounded_sync(s->stream));
    return PHYZB_OK;
}

int phyzb_set_controls(phyzb_sim* s, const double* ctrl) {
    PZ_TRY(check_sim(s));
    if (!ctrl) return fail(PHYZB_ERR_INVALID, "ctrl is null");
    DeviceGuard g(s->device);
    return upload_rows(s, ctrl, s->nv, s->ctrl);
}

int phyzb_step(phyzb_sim* s, int32_t n) {
    PZ_TRY(check_sim(s));
    if (n < 0) return fail(PHYZB_ERR_INVALID, "step count must be >= 0");
    if (n == 0) return PHYZB_OK;
    DeviceGuard g(s->device);
    return launch(s, s->ctrl, 0, n);
}

int phyzb_step_device_controls(phyzb_sim* s, const void* sched, int64_t step_stride, int32_t n) {
    PZ_TRY(check_sim(s));
    if (n < 0) return fail(PHYZB_ERR_INVALID, "step count must be >= 0");
    if (n == 0) return PHYZB_OK;
    if (!sched) return fail(PHYZB_ERR_INVALID, "control schedule is null");
    if (step_stride < (int64_t)s->nv * s->nworld)
        return fail(PHYZB_ERR_INVALID, "step_stride must be >= nv * nworld");
    DeviceGuard g(s->device);
    PZ_TRY(launch(s, sched, step_stride, n));
    // leave the held controls equal to the last row, as n x (set_controls; step)
    const char* last = (const char*)sched + (size_t)(n - 1) * step_stride * s->esz();
    PZ_CUDA(cudaMemcpyAsync(s->ctrl, last, s->state_bytes(), cudaMemcpyDeviceToDevice, s->stream));
    return PHYZB_OK;
}

int phyzb_step_with_controls(phyzb_sim* s, const void* ctrl, int host_dtype, int32_t n) {
    PZ_TRY(check_sim(s));
    if (n < 0) return fail(PHYZB_ERR_INVALID, "step count must be >= 0");
    if (n == 0) return PHYZB_OK;
    if (!ctrl) return fail(PHYZB_ERR_INVALID, "ctrl is null");
    if (host_dtype != PHYZB_HOST_F32 && host_dtype != PHYZB_HOST_F64)
        return fail(PHYZB_ERR_INVALID, "host_dtype must be PHYZB_HOST_F32 or PHYZB_HOST_F64");
    DeviceGuard g(s->device);
    const size_t hsz = host_dtype == PHYZB_HOST_F64 ? 8 : 4;
    const size_t row = (size_t)s->nworld * s->nv;  // elements per step
    // chunk: about 128 MB of host rows per copy, at least one step
    size_t chunk = row ? std::max<size_t>(1, (128u << 20) / (row * hsz)) : 1;
    chunk = std::min<size_t>(chunk, (size_t)n);
    PZ_TRY(ensure_pipeline(s, chunk * row * hsz, chunk * row * s->esz()));
    const char* host = (const char*)ctrl;
    int done = 0, c = 0;
    while (done < n) {
        const int len = (int)std::min<size_t>(chunk, (size_t)(n - done));
        const int b = c & 1;
        if (c >= 2) PZ_CUDA(cudaStreamWaitEvent(s->copy_stream, s->ev_converted[b], 0));
        PZ_CUDA(cudaMemcpyAsync(s->pipe_raw[b], host + (size_t)done * row * hsz, (size_t)len * row * hsz,
                                cudaMemcpyHostToDevice, s->copy_stream));
        PZ_CUDA(cudaEventRecord(s->ev_copied[b], s->copy_stream));
        PZ_CUDA(cudaStreamWaitEvent(s->stream, s->ev_copied[b], 0));
        cudaError_t e;
        if (is_f64(s))
            e = host_dtype == PHYZB_HOST_F64
                    ? pz::launch_aos_to_soa<double, double>((const double*)s->pipe_raw[b], (double*)s->pipe_soa[b],
                                                            s->nworld, s->nv, len, s->stream)
                    : pz::launch_aos_to_soa<float, double>((const float*)s->pipe_raw[b], (double*)s->pipe_soa[b],
                                                           s->nworld, s->nv, len, s->stream);
        else
            e = host_dtype == PHYZB_HOST_F64
                    ? pz::launch_aos_to_soa<double, float>((const double*)s->pipe_raw[b], (float*)s->pipe_soa[b],
                                                           s->nworld, s->nv, len, s->stream)
                    : pz::launch_aos_to_soa<float, float>((const float*)s->pipe_raw[b], (float*)s->pipe_soa[b],
                                                          s->nworld, s->nv, len, s->stream);
        PZ_CUDA(e);
        PZ_CUDA(cudaEventRecord(s->ev_converted[b], s->stream));
        PZ_TRY(launch(s, s->pipe_soa[b], (long long)row, len));
        if (done + len == n) {
            const char* last = (const char*)s->pipe_soa[b] + (size_t)(len - 1) * row * s->esz();
            PZ_CUDA(cudaMemcpyAsync(s->ctrl, last, row * s->esz(), cudaMemcpyDeviceToDevice, s->stream));
        }
        done += len;
        c++;
    }
    // every host row has been read once the copy stream drains
    PZ_TRY(bounded_sync(s->copy_stream));
    return PHYZB_OK;
}

int phyzb_sync(phyzb_sim* s) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    PZ_TRY(bounded_sync(s->stream));
    return read_status(s);
}

int phyzb_status(phyzb_sim* s) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    return read_status(s);
}

int phyzb_clear_status(phyzb_sim* s) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    const int init[2] = {0, 0x7fffffff};
    PZ_CUDA(cudaMemcpyAsync(s->status, init, sizeof(init), cudaMemcpyHostToDevice, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    return PHYZB_OK;
}

int phyzb_readback_states(phyzb_sim* s, double* q, double* v) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    if (q) PZ_TRY(download_rows(s, s->q, s->nv, q));
    if (v) PZ_TRY(download_rows(s, s->v, s->nv, v));
    return PHYZB_OK;
}

int phyzb_enable_state_history(phyzb_sim* s, int32_t slots) {
    PZ_TRY(check_sim(s));
    if (slots < 1) return fail(PHYZB_ERR_INVALID, "state history needs at least one slot");
    if (s->hist_slots == slots) return PHYZB_OK;  // re-enabling keeps the buffers (mod.rs:1324-1326)
    DeviceGuard g(s->device);
    free_ptr(s->hist_q);
    free_ptr(s->hist_v);
    s->hist_slots = 0;
    PZ_CUDA(cudaMalloc(&s->hist_q, (size_t)slots * s->state_bytes()));
    PZ_CUDA(cudaMalloc(&s->hist_v, (size_t)slots * s->state_bytes()));
    s->hist_slots = slots;
    return PHYZB_OK;
}

int phyzb_record_state(phyzb_sim* s, int32_t slot) {
    PZ_TRY(check_sim(s));
    if (!s->hist_slots) return fail(PHYZB_ERR_STATE, "state history not enabled — call enable_state_history first");
    if (slot < 0 || slot >= s->hist_slots)
        return fail(PHYZB_ERR_INVALID, "history slot " + std::to_string(slot) + " exceeds " +
                                           std::to_string(s->hist_slots) + " slots");
    DeviceGuard g(s->device);
    const size_t b = s->state_bytes();
    PZ_CUDA(cudaMemcpyAsync((char*)s->hist_q + (size_t)slot * b, s->q, b, cudaMemcpyDeviceToDevice, s->stream));
    PZ_CUDA(cudaMemcpyAsync((char*)s->hist_v + (size_t)slot * b, s->v, b, cudaMemcpyDeviceToDevice, s->stream));
    return PHYZB_OK;
}

int phyzb_readback_state_history(phyzb_sim* s, int32_t slot0, int32_t n, double* q, double* v) {
    PZ_TRY(check_sim(s));
    if (!s->hist_slots) return fail(PHYZB_ERR_STATE, "state history not enabled");
    if (slot0 < 0 || n < 0 || (int64_t)slot0 + n > s->hist_slots)
        return fail(PHYZB_ERR_INVALID, "history range outside 0.." + std::to_string(s->hist_slots));
    DeviceGuard g(s->device);
    const size_t b = s->state_bytes(), rows = (size_t)s->nworld * s->nv;
    for (int k = 0; k < n; k++) {
        if (q) PZ_TRY(download_rows(s, (char*)s->hist_q + (size_t)(slot0 + k) * b, s->nv, q + k * rows));
        if (v) PZ_TRY(download_rows(s, (char*)s->hist_v + (size_t)(slot0 + k) * b, s->nv, v + k * rows));
    }
    return PHYZB_OK;
}

int phyzb_readback_qdd(phyzb_sim* s, double* qdd) {
    PZ_TRY(check_sim(s));
    if (!qdd) return fail(PHYZB_ERR_INVALID, "qdd is null");
    DeviceGuard g(s->device);
    return download_rows(s, s->qdd, s->nv, qdd);
}

int phyzb_readback_contacts(phyzb_sim* s, double* cs) {
    PZ_TRY(check_sim(s));
    if (!s->cfg.contact || !s->cstate)
        return fail(PHYZB_ERR_STATE, "ground contact not enabled — call enable_ground_contact first");
    if (!cs) return fail(PHYZB_ERR_INVALID, "output is null");
    DeviceGuard g(s->device);
    return download_rows(s, s->cstate, s->nb * PHYZB_CONTACT_STRIDE, cs);
}

int phyzb_device_view_get(phyzb_sim* s, phyzb_device_view* out) {
    PZ_TRY(check_sim(s));
    if (!out) return fail(PHYZB_ERR_INVALID, "out is null");
    out->q = s->q;
    out->v = s->v;
    out->ctrl = s->ctrl;
    out->qdd = s->qdd;
    out->nworld = s->nworld;
    out->nv = s->nv;
    out->nbodies = s->nb;
    out->precision = s->precision;
    out->device = s->device;
    out->stream = (void*)s->stream;
    return PHYZB_OK;
}

int phyzb_load_states_device(phyzb_sim* s, const void* q, const void* v, const void* ctrl) {
    PZ_TRY(check_sim(s));
    if (!q || !v) return fail(PHYZB_ERR_INVALID, "q and v must not be null");
    DeviceGuard g(s->device);
    PZ_CUDA(cudaMemcpyAsync(s->q, q, s->state_bytes(), cudaMemcpyDeviceToDevice, s->stream));
    PZ_CUDA(cudaMemcpyAsync(s->v, v, s->state_bytes(), cudaMemcpyDeviceToDevice, s->stream));
    if (ctrl) PZ_CUDA(cudaMemcpyAsync(s->ctrl, ctrl, s->state_bytes(), cudaMemcpyDeviceToDevice, s->stream));
    return PHYZB_OK;
}

int phyzb_set_stream(phyzb_sim* s, void* stream) {
    PZ_TRY(check_sim(s));
    DeviceGuard g(s->device);
    PZ_TRY(bounded_sync(s->stream));
    s->stream = stream ? (cudaStream_t)stream : s->own_stream;
    return PHYZB_OK;
}

int phyzb_objective_device(phyzb_sim* s, int kind, void* out) {
    PZ_TRY(check_sim(s));
    if (kind != 0 && kind != 1) return fail(PHYZB_ERR_INVALID, "objective kind must be 0 or 1");
    if (!out) return fail(PHYZB_ERR_INVALID, "output is null");
    DeviceGuard g(s->device);
    cudaError_t e = is_f64(s) ? pz::launch_objective<double>(rollout_args<double>(s, s->lay[0], s->ctrl, 0, 1),
                                                             s->lay[0].launch, kind, (double*)out, s->stream)
                              : pz::launch_objective<float>(rollout_args<float>(s, s->lay[0], s->ctrl, 0, 1),
                                                            s->lay[0].launch, kind, (float*)out, s->stream);
    PZ_CUDA(e);
    return PHYZB_OK;
}

int phyzb_flops_per_world_step(const phyzb_sim* s, double* flops, double* transcendentals) {
    PZ_TRY(check_sim(s));
    const pz::FlopCount fc = pz::count_world_step(&s->model, s->nv, s->cfg, s->sweeps);
    if (flops) *flops = fc.flops;
    if (transcendentals) *transcendentals = fc.transcendentals;
    return PHYZB_OK;
}

int phyzb_flops_executed(const phyzb_sim* s, const double* q, const double* v, const double* ctrl, int64_t nworld,
                         int32_t nsteps, int32_t specialized, double* flops, double* transcendentals) {
    PZ_TRY(check_sim(s));
    if (!q || !v) return fail(PHYZB_ERR_INVALID, "null state rows");
    if (nworld < 1 || nsteps < 1) return fail(PHYZB_ERR_INVALID, "nworld and nsteps must be >= 1");
    if (s->cfg.terrain) return fail(PHYZB_ERR_INVALID, "executed flops are counted on the flat ground only");
    const pz::FlopCount fc = pz::count_rollout(&s->model, s->nv, s->cfg, s->sweeps, s->ground_h, s->friction,
                                               s->erp, q, v, ctrl, nworld, nsteps, specialized != 0);
    if (flops) *flops = fc.flops;
    if (transcendentals) *transcendentals = fc.transcendentals;
    return PHYZB_OK;
}

int phyzb_set_world_lanes(phyzb_sim* s, int32_t lanes) {
    PZ_TRY(check_sim(s));
    if (lanes != 0 && lanes != 1 && lanes != 2 && lanes != 4 && lanes != 8)
        return fail(PHYZB_ERR_INVALID, "lanes per world must be 0, 1, 2, 4 or 8, not " + std::to_string(lanes));
    if (lanes >= 2) {
        std::string why = lanes_unsupported(s);
        if (why.empty()) {
            pz::LanePlan plan;
            why = pz::plan_lanes(&s->model, lanes, &plan);
        }
        if (!why.empty()) return fail(PHYZB_ERR_UNSUPPORTED, "cannot split a world over lanes: " + why);
    }
    s->lanes = lanes >= 2 ? lanes : 0;
    s->lanes_built = false;
    return PHYZB_OK;
}

int phyzb_get_world_lanes(phyzb_sim* s, int32_t* lanes, int32_t* active) {
    PZ_TRY(check_sim(s));
    if (lanes) *lanes = s->lanes;
    if (active) {
        *active = 0;
        if (s->lanes >= 2) {
            DeviceGuard g(s->device);
            if (!s->lanes_built) PZ_TRY(is_f64(s) ? build_lanes<double>(s) : build_lanes<float>(s));
            *active = s->lanes_ok ? 1 : 0;
        }
    }
    return PHYZB_OK;
}

int phyzb_set_kernel_specialization(phyzb_sim* s, int32_t mode) {
    PZ_TRY(check_sim(s));
    if (mode != PHYZB_SPECIALIZE_OFF && mode != PHYZB_SPECIALIZE_ON && mode != PHYZB_SPECIALIZE_AUTO)
        return fail(PHYZB_ERR_INVALID, "specialization mode " + std::to_string(mode) + " is not 0, 1 or 2");
    s->specialize = mode;
    return PHYZB_OK;
}

int phyzb_get_kernel_specialization(const phyzb_sim* s, int32_t* mode, int32_t* active) {
    PZ_TRY(check_sim(s));
    if (!mode) return fail(PHYZB_ERR_INVALID, "null output");
    *mode = s->specialize;
    if (active) *active = specialized(s) ? 1 : 0;
    return PHYZB_OK;
}

int phyzb_launch_info(const phyzb_sim* s, int32_t* wpb, int32_t* blocks, int32_t* smem, int32_t* scratch,
                      int32_t* tmem_cols) {
    PZ_TRY(check_sim(s));
    const phyzb_sim::Layout& L = specialized(s) && s->spec ? s->spec_lay : s->lay[s->use];
    if (wpb) *wpb = L.launch.W;
    if (blocks) *blocks = L.launch.grid;
    if (smem) *smem = L.launch.smem;
    if (scratch) *scratch = L.info.scratch;
    if (tmem_cols) *tmem_cols = L.launch.tm ? L.info.tmem_cols : 0;
    return PHYZB_OK;
}

int phyzb_slice_plan(const phyzb_sim* s, int32_t nsteps, int32_t* steps_per_run, int32_t* wpb, int32_t* blocks) {
    PZ_TRY(check_sim(s));
    const phyzb_sim::Layout& L = specialized(s) && s->spec ? s->spec_lay : s->lay[s->use];
    pz::LaunchCfg cfg = L.launch;
    int chunk = s->slices ? pz::plan_slices(L.launch, s->nworld, nsteps, s->slice_force, &cfg) : 0;
    if (chunk <= 0) {
        chunk = 0;
        cfg = L.launch;
    }
    if (steps_per_run) *steps_per_run = chunk;
    if (wpb) *wpb = cfg.W;
    if (blocks) *blocks = cfg.grid;
    return PHYZB_OK;
}

}  // extern "C"

// ── multi-GPU: NCCL communicator and the all-reduced objective ────────────
//
// NCCL is loaded at run time (libnccl.so.2; in a process that already holds
// one -- e.g. torch's -- that copy is reused), so the library itself keeps no
// link-time dependency on it. Communicators are created non-blocking and
// every wait on one is bounded: a rank that never joins or a collective that
// never completes ends in PHYZB_ERR_COMM after the caller's timeout, with the
// communicator aborted.

namespace {

struct NcclApi {
    bool tried = false, ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
    static NcclApi api;
    if (api.tried) return api;
    api.tried = true;
    void* h = nullptr;
    for (const char* name : {"libnccl.so.2", "libnccl.so"})
        if ((h = dlopen(name, RTLD_NOW | RTLD_GLOBAL)) != nullptr) break;
    if (!h) {
        api.why = std::string("NCCL not found (dlopen libnccl.so.2): ") + dlerror();
        return api;
    }
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.GetUniqueId = (decltype(api.GetUniqueId))sym("ncclGetUniqueId");
    api.CommInitRankConfig = (decltype(api.CommInitRankConfig))sym("ncclCommInitRankConfig");
    api.CommGetAsyncError = (decltype(api.CommGetAsyncError))sym("ncclCommGetAsyncError");
    api.CommAbort = (decltype(api.CommAbort))sym("ncclCommAbort");
    api.CommDestroy = (decltype(api.CommDestroy))sym("ncclCommDestroy");
    api.AllReduce = (decltype(api.AllReduce))sym("ncclAllReduce");
    api.GetErrorString = (decltype(api.GetErrorString))sym("ncclGetErrorString");
    api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.CommAbort &&
             api.CommDestroy && api.AllReduce && api.GetErrorString;
    if (!api.ok) api.why = "NCCL library lacks a required entry point (needs NCCL >= 2.14)";
    return api;
}

std::string nccl_msg(ncclResult_t r) {
    NcclApi& n = nccl();
    return n.GetErrorString ? n.GetErrorString(r) : ("NCCL error " + std::to_string((int)r));
}

double seconds_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

struct phyzb_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0;
    bool broken = false;
    cudaEvent_t ev = nullptr;  // comm_wait
};

namespace {

// Wait (bounded) until a non-blocking communicator has no operation in
// progress. On error or timeout the communicator is aborted.
int comm_settle(phyzb_comm* c, double timeout_s, const char* what) {
    NcclApi& n = nccl();
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = n.CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return PHYZB_OK;
        if (st != ncclInProgress) {
            n.CommAbort(c->comm);
            c->broken = true;
            return fail(PHYZB_ERR_COMM, std::string(what) + ": " + nccl_msg(st));
        }
        if (seconds_since(t0) > timeout_s) {
            n.CommAbort(c->comm);
            c->broken = true;
            return fail(PHYZB_ERR_COMM, std::string(what) + ": timed out after " + std::to_string(timeout_s) +
                                            " s (a rank did not take part)");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}


}  // namespace

namespace pzc {

int comm_nranks(const phyzb_comm* c) { return c ? c->nranks : 1; }

int comm_allreduce_sum(phyzb_comm* c, void* buf, size_t count, bool f64, cudaStream_t stream) {
    if (!c) return PHYZB_OK;
    if (c->broken) return fail(PHYZB_ERR_COMM, "communicator was aborted by an earlier failure");
    NcclApi& n = nccl();
    const ncclResult_t r = n.AllReduce(buf, buf, count, f64 ? ncclFloat64 : ncclFloat32, ncclSum, c->comm, stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        n.CommAbort(c->comm);
        c->broken = true;
        return fail(PHYZB_ERR_COMM, "ncclAllReduce: " + nccl_msg(r));
    }
    return comm_settle(c, 60.0, "all-reduce (enqueue)");
}

int comm_wait(phyzb_comm* c, cudaStream_t stream, double timeout_s) {
    if (!c) {
        PZ_TRY(bounded_sync(stream));
        return PHYZB_OK;
    }
    NcclApi& n = nccl();
    if (!c->ev) PZ_CUDA(cudaEventCreateWithFlags(&c->ev, cudaEventDisableTiming));
    PZ_CUDA(cudaEventRecord(c->ev, stream));
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaEventQuery(c->ev);
        if (q == cudaSuccess) return PHYZB_OK;
        if (q != cudaErrorNotReady) PZ_CUDA(q);
        ncclResult_t st = ncclSuccess;
        n.CommGetAsyncError(c->comm, &st);
        if (st != ncclSuccess && st != ncclInProgress) {
            n.CommAbort(c->comm);
            c->broken = true;
            return fail(PHYZB_ERR_COMM, "collective failed: " + nccl_msg(st));
        }
        if (seconds_since(t0) > timeout_s) {
            n.CommAbort(c->comm);
            c->broken = true;
            return fail(PHYZB_ERR_COMM, "collective timed out after " + std::to_string(timeout_s) +
                                            " s (a rank did not take part)");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

}  // namespace pzc

namespace {
}  // namespace

extern "C" {

int phyzb_comm_unique_id(uint8_t* id_out) {
    if (!id_out) return fail(PHYZB_ERR_INVALID, "id buffer is null");
    NcclApi& n = nccl();
    if (!n.ok) return fail(PHYZB_ERR_COMM, n.why);
    ncclUniqueId id;
    const ncclResult_t r = n.GetUniqueId(&id);
    if (r != ncclSuccess) return fail(PHYZB_ERR_COMM, "ncclGetUniqueId: " + nccl_msg(r));
    static_assert(sizeof(ncclUniqueId) == PHYZB_COMM_ID_BYTES, "NCCL unique id size");
    std::memcpy(id_out, &id, sizeof(id));
    return PHYZB_OK;
}

int phyzb_comm_init(const uint8_t* id, int32_t nranks, int32_t rank, int32_t device, double timeout_s,
                    phyzb_comm** out) {
    if (!id || !out) return fail(PHYZB_ERR_INVALID, "id or output is null");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(PHYZB_ERR_INVALID, "rank must be in [0, nranks)");
    if (!(timeout_s > 0.0)) return fail(PHYZB_ERR_INVALID, "timeout must be > 0");
    NcclApi& n = nccl();
    if (!n.ok) return fail(PHYZB_ERR_COMM, n.why);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(PHYZB_ERR_NO_DEVICE, "no CUDA device");
    }
    if (device < 0 || device >= ndev) return fail(PHYZB_ERR_INVALID, "device ordinal out of range");
    DeviceGuard g(device);
    phyzb_comm* c = new phyzb_comm;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = n.CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return fail(PHYZB_ERR_COMM, "ncclCommInitRankConfig: " + nccl_msg(r));
    }
    const int rc = comm_settle(c, timeout_s, "communicator init");
    if (rc != PHYZB_OK) {
        delete c;
        return rc;
    }
    *out = c;
    return PHYZB_OK;
}

int phyzb_comm_destroy(phyzb_comm* c) {
    if (!c) return PHYZB_OK;
    NcclApi& n = nccl();
    if (c->comm && n.ok) {
        DeviceGuard g(c->device);
        if (c->broken)
            n.CommAbort(c->comm);
        else
            n.CommDestroy(c->comm);
    }
    if (c->ev) cudaEventDestroy(c->ev);
    delete c;
    return PHYZB_OK;
}

int phyzb_reduce_objective_device(phyzb_sim* s, phyzb_comm* c, int kind, void* out) {
    PZ_TRY(check_sim(s));
    if (!c || !out) return fail(PHYZB_ERR_INVALID, "communicator or output is null");
    if (c->broken) return fail(PHYZB_ERR_COMM, "communicator was aborted by an earlier failure");
    if (c->device != s->device) return fail(PHYZB_ERR_INVALID, "communicator and simulator are on different devices");
    NcclApi& n = nccl();
    DeviceGuard g(s->device);
    PZ_CUDA(cudaMemsetAsync(out, 0, s->esz(), s->stream));
    PZ_TRY(phyzb_objective_device(s, kind, out));
    const ncclResult_t r = n.AllReduce(out, out, 1, is_f64(s) ? ncclFloat64 : ncclFloat32, ncclSum, c->comm, s->stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        n.CommAbort(c->comm);
        c->broken = true;
        return fail(PHYZB_ERR_COMM, "ncclAllReduce: " + nccl_msg(r));
    }
    return comm_settle(c, 60.0, "objective all-reduce (enqueue)");
}

int phyzb_comm_sync(phyzb_comm* c, phyzb_sim* s, double timeout_s) {
    PZ_TRY(check_sim(s));
    if (!c) return fail(PHYZB_ERR_INVALID, "communicator is null");
    if (c->broken) return fail(PHYZB_ERR_COMM, "communicator was aborted by an earlier failure");
    if (!(timeout_s > 0.0)) return fail(PHYZB_ERR_INVALID, "timeout must be > 0");
    DeviceGuard g(s->device);
    return comm_wait(c, s->stream, timeout_s);
}

int phyzb_reduce_objective(phyzb_sim* s, phyzb_comm* c, int kind, double timeout_s, double* out) {
    PZ_TRY(check_sim(s));
    if (!c || !out) return fail(PHYZB_ERR_INVALID, "communicator or output is null");
    if (c->broken) return fail(PHYZB_ERR_COMM, "communicator was aborted by an earlier failure");
    if (c->device != s->device) return fail(PHYZB_ERR_INVALID, "communicator and simulator are on different devices");
    if (!(timeout_s > 0.0)) return fail(PHYZB_ERR_INVALID, "timeout must be > 0");
    NcclApi& n = nccl();
    DeviceGuard g(s->device);
    if (!s->obj) PZ_CUDA(cudaMalloc(&s->obj, 16));
    if (!s->obj_host) PZ_CUDA(cudaHostAlloc(&s->obj_host, 16, cudaHostAllocDefault));
    if (!s->ev_obj) PZ_CUDA(cudaEventCreateWithFlags(&s->ev_obj, cudaEventDisableTiming));
    PZ_CUDA(cudaMemsetAsync(s->obj, 0, s->esz(), s->stream));
    PZ_TRY(phyzb_objective_device(s, kind, s->obj));
    const ncclResult_t r = n.AllReduce(s->obj, s->obj, 1, is_f64(s) ? ncclFloat64 : ncclFloat32, ncclSum, c->comm,
                                       s->stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        n.CommAbort(c->comm);
        c->broken = true;
        return fail(PHYZB_ERR_COMM, "ncclAllReduce: " + nccl_msg(r));
    }
    PZ_TRY(comm_settle(c, timeout_s, "objective all-reduce (enqueue)"));
    PZ_CUDA(cudaMemcpyAsync(s->obj_host, s->obj, s->esz(), cudaMemcpyDeviceToHost, s->stream));
    PZ_CUDA(cudaEventRecord(s->ev_obj, s->stream));
    // bounded wait on the collective: poll the event and NCCL's error state
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaEventQuery(s->ev_obj);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) PZ_CUDA(q);
        ncclResult_t st = ncclSuccess;
        n.CommGetAsyncError(c->comm, &st);
        if (st != ncclSuccess && st != ncclInProgress) {
            n.CommAbort(c->comm);
            c->broken = true;
            return fail(PHYZB_ERR_COMM, "objective all-reduce: " + nccl_msg(st));
        }
        if (seconds_since(t0) > timeout_s) {
            n.CommAbort(c->comm);
            c->broken = true;
            return fail(PHYZB_ERR_COMM, "objective all-reduce: timed out after " + std::to_string(timeout_s) +
                                            " s (a rank did not take part)");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    *out = is_f64(s) ? *static_cast<const double*>(s->obj_host) : (double)*static_cast<const float*>(s->obj_host);
    return PHYZB_OK;
}

}  // extern "C"
