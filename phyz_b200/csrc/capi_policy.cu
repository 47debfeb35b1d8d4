// C ABI of the on-device control loop (include/phyzb.h, "on-device control
// loop"): BatchSim's policy pass of phyz-gpu (crates/phyz-gpu/src/cuda/mod.rs
// 1081-1313, policy_pipeline.rs) over the kernels of policy.cu. The policy
// buffers belong to the simulator handle; the actions drive its PD servos.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "pz_policy.h"

using namespace pzc;


namespace pzc {

void destroy_policy(phyzb_sim* s) {
    PolicyDev* p = s->policy;
    if (!p) return;
    void* bufs[] = {p->fk,    p->d_ops,  p->d_aux, p->d_com, p->d_w,   p->d_std,  p->d_noise,
                    p->d_slots, p->d_clamp, p->d_rng, p->d_z, p->d_base, p->d_xf, p->d_obs,
                    p->d_out, p->d_rows, p->d_ret_scratch, p->d_h};
    for (void* b : bufs)
        if (b) cudaFree(b);
    delete p;
    s->policy = nullptr;
}

}  // namespace pzc

namespace {

int round_up(int x, int m) { return (x + m - 1) / m * m; }

template <class T>
pz::PolicyArgs<T> policy_args(phyzb_sim* s, int step) {
    PolicyDev* p = s->policy;
    const long long N = s->nworld;
    pz::PolicyArgs<T> a{};
    a.fk = (const pz::FkBody<T>*)p->fk;
    a.nb = s->nb;
    a.nv = s->nv;
    a.q = (const T*)s->q;
    a.v = (const T*)s->v;
    a.nworld = N;
    a.xf = p->d_xf;
    a.ops = p->d_ops;
    a.aux = p->d_aux;
    a.com = p->d_com;
    a.n_in = p->n_in;
    a.w = p->d_w;
    a.n_wf = p->n_wf;
    a.in_pad = p->in_pad;
    a.h_pad = p->h_pad;
    a.out_pad = p->out_pad;
    a.n_out = p->n_out;
    a.stdv = p->d_std;
    a.in_noise = p->d_noise;
    a.act_slots = p->d_slots;
    a.clamp = p->d_clamp;
    a.rho = p->rho;
    a.rng = p->d_rng;
    a.z = p->d_z;
    a.base = (const T*)p->d_base;
    a.targets = (T*)s->targets;
    a.npd = (int)s->cfg.pd.size();
    a.h = p->d_h;
    a.obs = p->d_obs ? p->d_obs + (size_t)step * p->n_in * N : nullptr;
    a.out = p->d_out ? p->d_out + (size_t)step * (p->n_out + 1) * N : nullptr;
    return a;
}

template <class T>
std::vector<pz::FkBody<T>> fk_table(const phyzb_model* m) {
    std::vector<pz::FkBody<T>> t(m->nbodies);
    int off = 0;
    for (int i = 0; i < m->nbodies; i++) {
        const phyzb_body& b = m->bodies[i];
        pz::FkBody<T>& f = t[i];
        f.parent = b.parent;
        f.jtype = b.joint_type;
        f.off = off;
        f.pad = 0;
        off += pz::ndof_of(b.joint_type);
        for (int k = 0; k < 3; k++) f.axis[k] = T(b.axis[k]);
        for (int k = 0; k < 9; k++) f.ptj_rot[k] = T(b.ptj_rot[k]);
        for (int k = 0; k < 3; k++) f.ptj_pos[k] = T(b.ptj_pos[k]);
    }
    return t;
}

template <class X>
int upload(X** dst, const void* src, size_t bytes) {
    if (*dst) cudaFree(*dst);
    *dst = nullptr;
    PZ_CUDA(cudaMalloc((void**)dst, bytes > 0 ? bytes : 16));
    if (bytes) PZ_CUDA(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
    return PHYZB_OK;
}

// PolicySpec::validate (policy_pipeline.rs:334-392) on the packed table.
int validate(const phyzb_sim* s, const phyzb_policy_spec* sp) {
    if (sp->n_obs < 1 || sp->n_obs > pz::POLICY_MAX_IN)
        return fail(PHYZB_ERR_INVALID, "policy input width " + std::to_string(sp->n_obs) + " not in 1..=128");
    if (sp->hidden < 1 || sp->hidden > pz::POLICY_MAX_H)
        return fail(PHYZB_ERR_INVALID, "policy hidden width " + std::to_string(sp->hidden) + " not in 1..=256");
    if (sp->hidden > 128)
        return fail(PHYZB_ERR_UNSUPPORTED, "policy hidden width " + std::to_string(sp->hidden) +
                                                " above 128: the weights do not fit the kernel's shared memory");
    if (sp->n_act < 1 || sp->n_act > pz::POLICY_MAX_OUT)
        return fail(PHYZB_ERR_INVALID, "policy output width " + std::to_string(sp->n_act) + " not in 1..=32");
    if (!sp->obs_ops || !sp->act_slots || !sp->input_noise || (sp->n_aux > 0 && !sp->obs_aux))
        return fail(PHYZB_ERR_INVALID, "policy spec has a null table");
    if (sp->history_steps < 1) return fail(PHYZB_ERR_INVALID, "policy history_steps must be at least 1");
    const int npd = (int)s->cfg.pd.size();
    for (int k = 0; k < sp->n_act; k++)
        if (sp->act_slots[k] < 0 || sp->act_slots[k] >= npd)
            return fail(PHYZB_ERR_INVALID, "action slot " + std::to_string(sp->act_slots[k]) + " exceeds the " +
                                               std::to_string(npd) + " registered PD servos");
    for (int k = 0; k < sp->n_obs; k++) {
        const float* r = sp->obs_ops + 4 * k;
        const int kind = (int)r[0], a = (int)r[1], b = (int)r[2];
        bool ok = true;
        switch (kind) {
            case PHYZB_OBS_CONST: break;
            case PHYZB_OBS_Q_MINUS:
            case PHYZB_OBS_V: ok = a >= 0 && a < s->nv; break;
            case PHYZB_OBS_BODY_PITCH:
            case PHYZB_OBS_BODY_ROLL:
            case PHYZB_OBS_BODY_YAW_ERROR:
            case PHYZB_OBS_BODY_POS_Z: ok = a >= 0 && a < s->nb; break;
            case PHYZB_OBS_BODY_POS: ok = a >= 0 && a < s->nb && b >= 0 && b < 3; break;
            case PHYZB_OBS_COM_OVER_SUPPORT: {
                const int axis = (int)r[3];
                ok = a >= 0 && b >= 0 && a + 2 + 4 * b <= sp->n_aux && axis >= 0 && axis < 3;
                if (ok) {
                    const float* x = sp->obs_aux + a;
                    if (x[0] != 0.0f) ok = (int)x[1] >= 0 && (int)x[1] < s->nb;
                    for (int i = 0; ok && i < b; i++) ok = (int)x[2 + 4 * i] >= 0 && (int)x[2 + 4 * i] < s->nb;
                }
                break;
            }
            default: ok = false;
        }
        if (!ok)
            return fail(PHYZB_ERR_INVALID, "observation op " + std::to_string(k) + " (kind " + std::to_string(kind) +
                                               ") out of range (nq " + std::to_string(s->nv) + ", nv " +
                                               std::to_string(s->nv) + ", nbodies " + std::to_string(s->nb) + ")");
    }
    return PHYZB_OK;
}

int need_policy(const phyzb_sim* s) {
    if (!s->policy) return fail(PHYZB_ERR_STATE, "policy pass not enabled — call enable_policy first");
    return PHYZB_OK;
}

template <class T>
int run_policy_t(phyzb_sim* s, int step) {
    PZ_CUDA(pz::launch_policy<T>(policy_args<T>(s, step), s->stream));
    return PHYZB_OK;
}

int run_policy(phyzb_sim* s, int step) {
    PolicyDev* p = s->policy;
    if (step < 0 || step >= p->history)
        return fail(PHYZB_ERR_INVALID, "policy step " + std::to_string(step) + " exceeds history_steps " +
                                           std::to_string(p->history));
    if (!p->has_weights) return fail(PHYZB_ERR_STATE, "policy weights not set — call set_policy_weights first");
    if (!p->has_std) return fail(PHYZB_ERR_STATE, "policy std not set — call set_policy_std first");
    return is_f64(s) ? run_policy_t<double>(s, step) : run_policy_t<float>(s, step);
}

// device SoA [width][nworld] float -> host rows [nworld][width] float
int download_float_rows(phyzb_sim* s, const float* src, int width, float* host) {
    PolicyDev* p = s->policy;
    const size_t bytes = (size_t)s->nworld * width * sizeof(float);
    if (bytes == 0) return PHYZB_OK;
    if (bytes > p->rows_bytes) {
        if (p->d_rows) cudaFree(p->d_rows);
        p->d_rows = nullptr;
        p->rows_bytes = 0;
        PZ_CUDA(cudaMalloc(&p->d_rows, bytes));
        p->rows_bytes = bytes;
    }
    const cudaError_t e = pz::launch_soa_to_aos<float, float>(src, (float*)p->d_rows, s->nworld, width, s->stream);
    PZ_CUDA(e);
    PZ_CUDA(cudaMemcpyAsync(host, p->d_rows, bytes, cudaMemcpyDeviceToHost, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    return PHYZB_OK;
}

}  // namespace

extern "C" {

int phyzb_enable_policy(phyzb_sim* s, const phyzb_policy_spec* sp) {
    PZ_TRY(check_sim(s));
    if (!sp) return fail(PHYZB_ERR_INVALID, "policy spec is null");
    if (s->cfg.pd.empty()) return fail(PHYZB_ERR_STATE, "policy pass needs PD control — call enable_pd first");
    PZ_TRY(validate(s, sp));
    DeviceGuard g(s->device);
    destroy_policy(s);
    PolicyDev* p = new PolicyDev;
    s->policy = p;
    p->n_in = sp->n_obs;
    p->n_h = sp->hidden;
    p->n_out = sp->n_act;
    p->history = sp->history_steps;
    p->in_pad = round_up(p->n_in, pz::POLICY_TILE);
    p->h_pad = round_up(p->n_h, pz::POLICY_TILE);
    p->out_pad = round_up(p->n_out, pz::POLICY_TILE);
    p->n_wf = p->in_pad * p->h_pad + p->h_pad + p->h_pad * p->h_pad + p->h_pad + p->h_pad * p->out_pad + p->out_pad;
    p->rho = (float)sp->noise_rho;
    const long long N = s->nworld;
    const int npd = (int)s->cfg.pd.size();
    const size_t esz = s->esz();
    // tables
    if (is_f64(s)) {
        auto t = fk_table<double>(&s->model);
        PZ_TRY(upload(&p->fk, t.data(), t.size() * sizeof(t[0])));
    } else {
        auto t = fk_table<float>(&s->model);
        PZ_TRY(upload(&p->fk, t.data(), t.size() * sizeof(t[0])));
    }
    PZ_TRY(upload(&p->d_ops, sp->obs_ops, (size_t)sp->n_obs * 4 * sizeof(float)));
    PZ_TRY(upload(&p->d_aux, sp->obs_aux, (size_t)std::max(sp->n_aux, 0) * sizeof(float)));
    std::vector<float> com((size_t)s->nb * 4);
    for (int i = 0; i < s->nb; i++) {  // pack_com_table (policy_pipeline.rs:258-268)
        const phyzb_body& b = s->model.bodies[i];
        com[4 * i] = (float)b.mass;
        for (int k = 0; k < 3; k++) com[4 * i + 1 + k] = (float)b.com[k];
    }
    PZ_TRY(upload(&p->d_com, com.data(), com.size() * sizeof(float)));
    std::vector<float> noise(sp->n_obs), clamp(sp->n_act);
    for (int k = 0; k < sp->n_obs; k++) noise[k] = (float)sp->input_noise[k];
    for (int k = 0; k < sp->n_act; k++)
        clamp[k] = (float)(sp->act_clamp_slots ? sp->act_clamp_slots[k] : sp->act_clamp);
    PZ_TRY(upload(&p->d_noise, noise.data(), noise.size() * sizeof(float)));
    PZ_TRY(upload(&p->d_clamp, clamp.data(), clamp.size() * sizeof(float)));
    PZ_TRY(upload(&p->d_slots, sp->act_slots, (size_t)sp->n_act * sizeof(int32_t)));
    // per-world state
    PZ_CUDA(cudaMalloc((void**)&p->d_w, (size_t)p->n_wf * sizeof(float)));
    PZ_CUDA(cudaMemsetAsync(p->d_w, 0, (size_t)p->n_wf * sizeof(float), s->stream));
    PZ_CUDA(cudaMalloc((void**)&p->d_std, (size_t)p->n_out * sizeof(float)));
    PZ_CUDA(cudaMalloc((void**)&p->d_rng, (size_t)N * sizeof(unsigned long long)));
    PZ_CUDA(cudaMalloc((void**)&p->d_z, (size_t)p->n_out * N * sizeof(float)));
    PZ_CUDA(cudaMemsetAsync(p->d_z, 0, (size_t)p->n_out * N * sizeof(float), s->stream));
    PZ_CUDA(cudaMalloc(&p->d_base, (size_t)npd * N * esz));
    PZ_CUDA(cudaMemsetAsync(p->d_base, 0, (size_t)npd * N * esz, s->stream));
    PZ_CUDA(cudaMalloc(&p->d_xf, (size_t)s->nb * pz::XF_STRIDE * N * esz));
    PZ_CUDA(cudaMalloc((void**)&p->d_h, (size_t)2 * p->h_pad * N * sizeof(float)));
    PZ_CUDA(cudaMalloc((void**)&p->d_obs, (size_t)p->history * p->n_in * N * sizeof(float)));
    PZ_CUDA(cudaMalloc((void**)&p->d_out, (size_t)p->history * (p->n_out + 1) * N * sizeof(float)));
    PZ_TRY(bounded_sync(s->stream));
    return phyzb_seed_policy(s, 0);
}

int phyzb_set_policy_weights(phyzb_sim* s, const double* w, int64_t n) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    PolicyDev* p = s->policy;
    const int64_t want = (int64_t)p->n_h * p->n_in + p->n_h + (int64_t)p->n_h * p->n_h + p->n_h +
                         (int64_t)p->n_out * p->n_h + p->n_out;
    if (!w || n != want)
        return fail(PHYZB_ERR_INVALID,
                    "policy expects " + std::to_string(want) + " weights, got " + std::to_string(n));
    // W1[h][in] -> W1^T[in_pad][h_pad] etc., zero padding (exact)
    std::vector<float> pk((size_t)p->n_wf, 0.0f);
    const double* W1 = w;
    const double* b1 = W1 + (size_t)p->n_h * p->n_in;
    const double* W2 = b1 + p->n_h;
    const double* b2 = W2 + (size_t)p->n_h * p->n_h;
    const double* W3 = b2 + p->n_h;
    const double* b3 = W3 + (size_t)p->n_out * p->n_h;
    float* o = pk.data();
    for (int j = 0; j < p->n_h; j++)
        for (int i = 0; i < p->n_in; i++) o[(size_t)i * p->h_pad + j] = (float)W1[(size_t)j * p->n_in + i];
    o += (size_t)p->in_pad * p->h_pad;
    for (int j = 0; j < p->n_h; j++) o[j] = (float)b1[j];
    o += p->h_pad;
    for (int j = 0; j < p->n_h; j++)
        for (int i = 0; i < p->n_h; i++) o[(size_t)i * p->h_pad + j] = (float)W2[(size_t)j * p->n_h + i];
    o += (size_t)p->h_pad * p->h_pad;
    for (int j = 0; j < p->n_h; j++) o[j] = (float)b2[j];
    o += p->h_pad;
    for (int k = 0; k < p->n_out; k++)
        for (int i = 0; i < p->n_h; i++) o[(size_t)i * p->out_pad + k] = (float)W3[(size_t)k * p->n_h + i];
    o += (size_t)p->h_pad * p->out_pad;
    for (int k = 0; k < p->n_out; k++) o[k] = (float)b3[k];
    DeviceGuard g(s->device);
    PZ_CUDA(cudaMemcpyAsync(p->d_w, pk.data(), pk.size() * sizeof(float), cudaMemcpyHostToDevice, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    p->has_weights = true;
    return PHYZB_OK;
}

int phyzb_set_policy_std(phyzb_sim* s, const double* sd, int32_t n) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    PolicyDev* p = s->policy;
    if (!sd || n != p->n_out)
        return fail(PHYZB_ERR_INVALID,
                    "policy has " + std::to_string(p->n_out) + " actions, got " + std::to_string(n) + " stds");
    std::vector<float> f(n);
    for (int k = 0; k < n; k++) f[k] = (float)sd[k];
    DeviceGuard g(s->device);
    PZ_CUDA(cudaMemcpyAsync(p->d_std, f.data(), f.size() * sizeof(float), cudaMemcpyHostToDevice, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    p->has_std = true;
    return PHYZB_OK;
}

int phyzb_set_policy_base_targets(phyzb_sim* s, const double* rows) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    if (!rows) return fail(PHYZB_ERR_INVALID, "rows is null");
    DeviceGuard g(s->device);
    return upload_rows(s, rows, (int)s->cfg.pd.size(), s->policy->d_base);
}

int phyzb_seed_policy(phyzb_sim* s, uint64_t seed) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    PolicyDev* p = s->policy;
    std::vector<unsigned long long> st((size_t)s->nworld);
    for (long long w = 0; w < s->nworld; w++) {
        // world_seed (policy_pipeline.rs:420-428): SplitMix64 of (seed, world)
        uint64_t z = seed + 0x9E3779B97F4A7C15ull * (uint64_t)(w + 1);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z = z ^ (z >> 31);
        st[(size_t)w] = z ? z : 1;
    }
    DeviceGuard g(s->device);
    PZ_CUDA(cudaMemcpyAsync(p->d_rng, st.data(), st.size() * sizeof(st[0]), cudaMemcpyHostToDevice, s->stream));
    PZ_CUDA(cudaMemsetAsync(p->d_z, 0, (size_t)p->n_out * s->nworld * sizeof(float), s->stream));
    PZ_TRY(bounded_sync(s->stream));
    return PHYZB_OK;
}

int phyzb_run_policy(phyzb_sim* s, int32_t step) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    DeviceGuard g(s->device);
    return run_policy(s, step);
}

int phyzb_policy_rollout(phyzb_sim* s, int32_t step0, int32_t n_control, int32_t substeps) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    if (n_control < 0 || substeps < 0) return fail(PHYZB_ERR_INVALID, "counts must be >= 0");
    if (step0 < 0 || (int64_t)step0 + n_control > s->policy->history)
        return fail(PHYZB_ERR_INVALID, "policy steps " + std::to_string(step0) + ".." +
                                           std::to_string(step0 + n_control) + " exceed history_steps " +
                                           std::to_string(s->policy->history));
    DeviceGuard g(s->device);
    for (int c = 0; c < n_control; c++) {
        PZ_TRY(run_policy(s, step0 + c));
        if (substeps > 0) PZ_TRY(launch(s, s->ctrl, 0, substeps));
    }
    return PHYZB_OK;
}

int phyzb_readback_policy_history(phyzb_sim* s, int32_t step0, int32_t n, float* obs, float* out) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    PolicyDev* p = s->policy;
    if (step0 < 0 || n < 0 || (int64_t)step0 + n > p->history)
        return fail(PHYZB_ERR_INVALID, "policy history range outside 0.." + std::to_string(p->history));
    DeviceGuard g(s->device);
    const long long N = s->nworld;
    for (int k = 0; k < n; k++) {
        const int st = step0 + k;
        if (obs)
            PZ_TRY(download_float_rows(s, p->d_obs + (size_t)st * p->n_in * N, p->n_in,
                                       obs + (size_t)k * N * p->n_in));
        if (out)
            PZ_TRY(download_float_rows(s, p->d_out + (size_t)st * (p->n_out + 1) * N, p->n_out + 1,
                                       out + (size_t)k * N * (p->n_out + 1)));
    }
    return PHYZB_OK;
}

int phyzb_readback_targets(phyzb_sim* s, double* rows) {
    PZ_TRY(check_sim(s));
    if (s->cfg.pd.empty()) return fail(PHYZB_ERR_STATE, "PD control not enabled");
    if (!rows) return fail(PHYZB_ERR_INVALID, "rows is null");
    DeviceGuard g(s->device);
    return download_rows(s, s->targets, (int)s->cfg.pd.size(), rows);
}

int phyzb_readback_kinematics(phyzb_sim* s, double* xf) {
    PZ_TRY(check_sim(s));
    PZ_TRY(need_policy(s));
    if (!xf) return fail(PHYZB_ERR_INVALID, "output is null");
    DeviceGuard g(s->device);
    PolicyDev* p = s->policy;
    cudaError_t e = is_f64(s) ? pz::launch_kinematics<double>(policy_args<double>(s, 0), s->stream)
                              : pz::launch_kinematics<float>(policy_args<float>(s, 0), s->stream);
    PZ_CUDA(e);
    const int width = s->nb * pz::XF_STRIDE;
    const size_t bytes = (size_t)s->nworld * width * sizeof(double);
    if (bytes > p->rows_bytes) {
        if (p->d_rows) cudaFree(p->d_rows);
        p->d_rows = nullptr;
        p->rows_bytes = 0;
        PZ_CUDA(cudaMalloc(&p->d_rows, bytes));
        p->rows_bytes = bytes;
    }
    e = is_f64(s) ? pz::launch_soa_to_aos<double, double>((const double*)p->d_xf, (double*)p->d_rows, s->nworld,
                                                          width, s->stream)
                  : pz::launch_soa_to_aos<float, double>((const float*)p->d_xf, (double*)p->d_rows, s->nworld,
                                                         width, s->stream);
    PZ_CUDA(e);
    PZ_CUDA(cudaMemcpyAsync(xf, p->d_rows, bytes, cudaMemcpyDeviceToHost, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    return PHYZB_OK;
}

}  // extern "C"
