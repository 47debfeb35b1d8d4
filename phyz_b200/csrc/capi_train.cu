// C ABI of the device-resident PPO update (include/phyzb.h, "PPO update"):
// phyz-gpu's TrainPipeline (crates/phyz-gpu/src/cuda/train.rs:474-810) over
// the kernels of train.cu. The update loop (epochs x minibatches, the KL
// brake read back once per minibatch) runs on the host; everything else --
// forward, surrogate and value gradients, backward, Adam with f64 master
// state -- stays on the device between updates.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "pz_policy.h"
#include "pz_train.h"

using namespace pzc;

namespace {

int pad32(int x) { return (x + 31) / 32 * 32; }

struct Net {
    pz::NetDev d{};
    std::vector<int> posf, posb;
    int* d_posf = nullptr;
    int* d_posb = nullptr;
    int mlp_params = 0;  // W1..b3
    long long t = 0;     // Adam step counter
    phyzb_adam_cfg adam{3e-4, 0.9, 0.999, 1e-8, 0.0};
};

void free_net(Net& n) {
    // (n.d.g points into the trainer's gradient block)
    void* bufs[] = {n.d.p,  n.d.m,    n.d.v,   n.d.wflat, n.d.wf,  n.d.wb,   n.d.h1,
                    n.d.h2, n.d.out,  n.d.dout, n.d.dh2,  n.d.dh1, n.d_posf, n.d_posb};
    for (void* b : bufs)
        if (b) cudaFree(b);
    n = Net{};
}

// flat index -> forward / backward pack positions (pz_train.h NetDev)
void pack_maps(Net& n) {
    const pz::NetDev& d = n.d;
    n.posf.assign(d.n_param, -1);
    n.posb.assign(d.n_param, -1);
    const int oW1f = 0, ob1f = d.in_pad * d.h_pad, oW2f = ob1f + d.h_pad, ob2f = oW2f + d.h_pad * d.h_pad,
              oW3f = ob2f + d.h_pad, ob3f = oW3f + d.h_pad * d.out_pad;
    const int oW3b = 0, oW2b = d.out_pad * d.h_pad;
    int t = 0;
    for (int j = 0; j < d.n_h; j++)
        for (int i = 0; i < d.n_in; i++) n.posf[t++] = oW1f + i * d.h_pad + j;
    for (int j = 0; j < d.n_h; j++) n.posf[t++] = ob1f + j;
    for (int j = 0; j < d.n_h; j++)
        for (int i = 0; i < d.n_h; i++) {
            n.posf[t] = oW2f + i * d.h_pad + j;
            n.posb[t] = oW2b + j * d.h_pad + i;
            t++;
        }
    for (int j = 0; j < d.n_h; j++) n.posf[t++] = ob2f + j;
    for (int k = 0; k < d.n_out; k++)
        for (int i = 0; i < d.n_h; i++) {
            n.posf[t] = oW3f + i * d.out_pad + k;
            n.posb[t] = oW3b + k * d.h_pad + i;
            t++;
        }
    for (int k = 0; k < d.n_out; k++) n.posf[t++] = ob3f + k;
}

int alloc_net(Net& n, phyzb_net_dims dims, int extra, int max_b) {
    pz::NetDev& d = n.d;
    d.n_in = dims.n_in;
    d.n_h = dims.n_h;
    d.n_out = dims.n_out;
    d.in_pad = pad32(d.n_in);
    d.h_pad = pad32(d.n_h);
    d.out_pad = pad32(d.n_out);
    n.mlp_params = d.n_h * d.n_in + d.n_h + d.n_h * d.n_h + d.n_h + d.n_out * d.n_h + d.n_out;
    d.n_param = n.mlp_params + extra;
    d.n_wf = d.in_pad * d.h_pad + d.h_pad + d.h_pad * d.h_pad + d.h_pad + d.h_pad * d.out_pad + d.out_pad;
    d.n_wb = d.out_pad * d.h_pad + d.h_pad * d.h_pad;
    d.max_b = max_b;
    const size_t P = d.n_param, L = max_b;
    PZ_CUDA(cudaMalloc((void**)&d.p, P * 8));
    PZ_CUDA(cudaMalloc((void**)&d.m, P * 8));
    PZ_CUDA(cudaMalloc((void**)&d.v, P * 8));
    PZ_CUDA(cudaMalloc((void**)&d.wflat, P * 4));
    PZ_CUDA(cudaMalloc((void**)&d.wf, (size_t)d.n_wf * 4));
    PZ_CUDA(cudaMalloc((void**)&d.wb, (size_t)d.n_wb * 4));
    PZ_CUDA(cudaMalloc((void**)&d.h1, (size_t)d.h_pad * L * 4));
    PZ_CUDA(cudaMalloc((void**)&d.h2, (size_t)d.h_pad * L * 4));
    PZ_CUDA(cudaMalloc((void**)&d.out, (size_t)d.out_pad * L * 4));
    PZ_CUDA(cudaMalloc((void**)&d.dout, (size_t)d.out_pad * L * 4));
    PZ_CUDA(cudaMalloc((void**)&d.dh2, (size_t)d.h_pad * L * 4));
    PZ_CUDA(cudaMalloc((void**)&d.dh1, (size_t)d.h_pad * L * 4));
    pack_maps(n);
    PZ_CUDA(cudaMalloc((void**)&n.d_posf, P * 4));
    PZ_CUDA(cudaMalloc((void**)&n.d_posb, P * 4));
    PZ_CUDA(cudaMemcpy(n.d_posf, n.posf.data(), P * 4, cudaMemcpyHostToDevice));
    PZ_CUDA(cudaMemcpy(n.d_posb, n.posb.data(), P * 4, cudaMemcpyHostToDevice));
    d.posf = n.d_posf;
    d.posb = n.d_posb;
    PZ_CUDA(cudaMemset(d.p, 0, P * 8));
    PZ_CUDA(cudaMemset(d.m, 0, P * 8));
    PZ_CUDA(cudaMemset(d.v, 0, P * 8));
    PZ_CUDA(cudaMemset(d.wflat, 0, P * 4));
    PZ_CUDA(cudaMemset(d.wf, 0, (size_t)d.n_wf * 4));
    PZ_CUDA(cudaMemset(d.wb, 0, (size_t)d.n_wb * 4));
    PZ_CUDA(cudaMemset(d.dout, 0, (size_t)d.out_pad * L * 4));
    return PHYZB_OK;
}

int set_net_params(Net& n, const double* flat) {
    const pz::NetDev& d = n.d;
    std::vector<float> wflat(d.n_param), wf(d.n_wf, 0.0f), wb(d.n_wb, 0.0f);
    for (int t = 0; t < d.n_param; t++) {
        const float x = (float)flat[t];
        wflat[t] = x;
        if (n.posf[t] >= 0) wf[n.posf[t]] = x;
        if (n.posb[t] >= 0) wb[n.posb[t]] = x;
    }
    PZ_CUDA(cudaMemcpy(d.p, flat, (size_t)d.n_param * 8, cudaMemcpyHostToDevice));
    PZ_CUDA(cudaMemcpy(d.wflat, wflat.data(), wflat.size() * 4, cudaMemcpyHostToDevice));
    PZ_CUDA(cudaMemcpy(d.wf, wf.data(), wf.size() * 4, cudaMemcpyHostToDevice));
    PZ_CUDA(cudaMemcpy(d.wb, wb.data(), wb.size() * 4, cudaMemcpyHostToDevice));
    return PHYZB_OK;
}

}  // namespace

struct phyzb_trainer {
    int device = 0;
    cudaStream_t stream = nullptr;
    Net actor, critic;
    long long capacity = 0, n_rows = 0;
    int max_b = 0;
    // batch columns, [F][capacity] (one block of N = n_rows rows)
    float *obs_a = nullptr, *obs_c = nullptr, *act = nullptr, *logp = nullptr, *adv = nullptr, *ret = nullptr;
    float* upload_raw = nullptr;  // row-major staging of one column
    uint32_t* order = nullptr;
    size_t order_cap = 0;
    float* dlogstd = nullptr;  // [out_pad][max_b]
    float* stats = nullptr;    // [4][max_b]
    float* reduced = nullptr;  // [4], inside gblock
    float* gblock = nullptr;   // actor g | critic g | minibatch statistics: one all-reduce
    float* reduced_host = nullptr;
    double* work = nullptr;
    float* xa = nullptr;  // a minibatch's actor / critic inputs, gathered [n_in][max_b]
    float* xc = nullptr;
    // the batch the update reads: the uploaded columns, or device arrays
    // (phyzb_trainer_set_batch_device)
    pz::BatchCol c_obs_a{}, c_obs_c{}, c_act{}, c_logp{}, c_adv{}, c_ret{};
    phyzb_comm* comm = nullptr;  // data-parallel: gradients and statistics summed over ranks
    unsigned long long* ac = nullptr;  // device order parameters
};

namespace {

void destroy_trainer(phyzb_trainer* t) {
    if (!t) return;
    DeviceGuard g(t->device);
    if (t->stream) bounded_sync(t->stream);
    free_net(t->actor);
    free_net(t->critic);
    void* bufs[] = {t->obs_a, t->obs_c,   t->act,   t->logp,    t->adv,  t->ret,  t->upload_raw,
                    t->order, t->dlogstd, t->stats, t->gblock, t->work, t->ac, t->xa, t->xc};
    for (void* b : bufs)
        if (b) cudaFree(b);
    if (t->reduced_host) cudaFreeHost(t->reduced_host);
    if (t->stream) cudaStreamDestroy(t->stream);
    delete t;
}

bool dims_ok(phyzb_net_dims d) {
    return d.n_in >= 1 && d.n_in <= pz::POLICY_MAX_IN && d.n_h >= 1 && d.n_h <= 128 && d.n_out >= 1 &&
           d.n_out <= pz::POLICY_MAX_OUT;
}

Net* net_of(phyzb_trainer* t, int which) { return which == 0 ? &t->actor : which == 1 ? &t->critic : nullptr; }

// host rows [n][F] -> device [F][n]
int upload_col(phyzb_trainer* t, const float* host, int F, long long n, float* dst) {
    PZ_CUDA(cudaMemcpyAsync(t->upload_raw, host, (size_t)n * F * 4, cudaMemcpyHostToDevice, t->stream));
    const cudaError_t e = pz::launch_aos_to_soa<float, float>(t->upload_raw, dst, n, F, 1, t->stream);
    PZ_CUDA(e);
    return PHYZB_OK;
}

// One Adam step of `n` (data-parallel: its gradient is already summed over
// the ranks; the step averages it).
int adam_step(phyzb_trainer* t, Net& n) {
    n.t += 1;
    const phyzb_adam_cfg& a = n.adam;
    const double bc1 = 1.0 - std::pow(a.beta1, (double)n.t);
    const double bc2 = 1.0 - std::pow(a.beta2, (double)n.t);
    const double gscale = 1.0 / comm_nranks(t->comm);
    PZ_CUDA(pz::train_adam(n.d, a.lr, a.beta1, a.beta2, a.eps, a.weight_decay, bc1, bc2, gscale, t->stream));
    return PHYZB_OK;
}

// The update loop of train.rs:655-795 over `t->order` (epochs x n_rows,
// already on the device).
int run_update(phyzb_trainer* t, const phyzb_ppo_cfg* cfg, phyzb_update_stats* out) {
    const long long N = t->n_rows;
    pz::PpoArgs pa{(float)cfg->clip, (float)cfg->entropy_coef, (float)cfg->vdelta, t->actor.mlp_params};
    double policy_acc = 0, value_acc = 0, brake_acc = 0, kl_acc = 0;
    long long kl_rows = 0;
    int batches = 0;
    bool stopped = false;
    cudaStream_t s = t->stream;
    const int L = t->max_b;
    const int R = comm_nranks(t->comm);
    for (int ep = 0; ep < cfg->epochs && !stopped; ep++) {
        for (long long start = 0; start < N; start += cfg->minibatch) {
            const int b = (int)std::min<long long>(cfg->minibatch, N - start);
            const uint32_t* idx = t->order + (size_t)ep * N + start;
            // the minibatch's inputs, gathered once (one copy when actor and
            // critic read the same column)
            PZ_CUDA(pz::train_gather(t->c_obs_a, idx, b, t->actor.d.n_in, t->xa, L, s));
            const bool same = t->c_obs_c.base == t->c_obs_a.base && t->c_obs_c.N == t->c_obs_a.N &&
                              t->c_obs_c.F == t->c_obs_a.F && t->critic.d.n_in == t->actor.d.n_in;
            if (!same) PZ_CUDA(pz::train_gather(t->c_obs_c, idx, b, t->critic.d.n_in, t->xc, L, s));
            const pz::BatchCol xa{t->xa, L, t->actor.d.n_in};
            const pz::BatchCol xc{same ? t->xa : t->xc, L, t->critic.d.n_in};
            // actor
            PZ_CUDA(pz::train_forward(t->actor.d, xa, nullptr, b, s));
            PZ_CUDA(pz::train_ppo_grad(t->actor.d, pa, t->c_act, t->c_logp, t->c_adv, idx, b, t->dlogstd, t->stats,
                                       s));
            PZ_CUDA(pz::train_row_sums(t->dlogstd, t->actor.d.n_out, L, b, t->actor.d.g, pa.logstd_off, t->work, s));
            PZ_CUDA(pz::train_backward(t->actor.d, xa, nullptr, b, t->work, s));
            // critic
            PZ_CUDA(pz::train_forward(t->critic.d, xc, nullptr, b, s));
            PZ_CUDA(pz::train_value_grad(t->critic.d, pa, t->c_ret, idx, b, t->stats, s));
            PZ_CUDA(pz::train_backward(t->critic.d, xc, nullptr, b, t->work, s));
            // the minibatch's statistics next to the gradients; data-parallel:
            // all of it summed over the ranks in one all-reduce
            PZ_CUDA(pz::train_stats(t->stats, L, b, t->reduced, t->work, s));
            PZ_TRY(comm_allreduce_sum(t->comm, t->gblock,
                                      (size_t)t->actor.d.n_param + t->critic.d.n_param + 4, false, s));
            // actor and critic are independent: both steps after both backward passes
            PZ_TRY(adam_step(t, t->actor));
            PZ_TRY(adam_step(t, t->critic));
            // the brake: the statistics to the host
            PZ_CUDA(cudaMemcpyAsync(t->reduced_host, t->reduced, 16, cudaMemcpyDeviceToHost, s));
            PZ_TRY(comm_wait(t->comm, s, 120.0));
            const float* r = t->reduced_host;
            const double rows = (double)b * R;
            const double ploss = r[0], kl_sum = r[1], k3_sum = r[2], vloss = r[3];
            policy_acc += ploss / rows;
            value_acc += vloss / rows;
            kl_acc += kl_sum;
            kl_rows += (long long)b * R;
            const double brake =
                (cfg->kl_mode == PHYZB_KL_CUMULATIVE ? std::fabs(kl_acc / (double)std::max<long long>(kl_rows, 1))
                                                     : k3_sum / rows) /
                cfg->kl_scale;
            brake_acc += brake;
            batches++;
            if (brake > cfg->target_kl) {
                stopped = true;
                break;
            }
        }
    }
    const double nb = std::max(batches, 1);
    *out = phyzb_update_stats{policy_acc / nb, value_acc / nb, brake_acc / nb, batches, stopped ? 1 : 0};
    return PHYZB_OK;
}

int ensure_order(phyzb_trainer* t, size_t bytes) {
    if (bytes <= t->order_cap) return PHYZB_OK;
    if (t->order) cudaFree(t->order);
    t->order = nullptr;
    t->order_cap = 0;
    PZ_CUDA(cudaMalloc((void**)&t->order, bytes));
    t->order_cap = bytes;
    return PHYZB_OK;
}

int check_update(phyzb_trainer* t, const phyzb_ppo_cfg* cfg) {
    if (cfg->minibatch < 1 || cfg->minibatch > t->max_b)
        return fail(PHYZB_ERR_INVALID, "minibatch " + std::to_string(cfg->minibatch) + " exceeds the pipeline's " +
                                           std::to_string(t->max_b));
    if (cfg->epochs < 0) return fail(PHYZB_ERR_INVALID, "epochs must be >= 0");
    return PHYZB_OK;
}

}  // namespace

extern "C" {

int phyzb_trainer_create(int32_t device, phyzb_net_dims actor, phyzb_net_dims critic, int64_t capacity,
                         int32_t max_b, phyzb_trainer** out) {
    if (!out) return fail(PHYZB_ERR_INVALID, "output is null");
    *out = nullptr;
    if (!dims_ok(actor) || !dims_ok(critic))
        return fail(PHYZB_ERR_INVALID, "network widths out of range (inputs 1..128, hidden 1..128, outputs 1..32)");
    if (critic.n_out != 1)
        return fail(PHYZB_ERR_INVALID, "critic must have one output, got " + std::to_string(critic.n_out));
    if (capacity < 1 || max_b < 1) return fail(PHYZB_ERR_INVALID, "capacity and minibatch must be >= 1");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(PHYZB_ERR_NO_DEVICE, "no CUDA device");
    }
    if (device < 0 || device >= ndev) return fail(PHYZB_ERR_INVALID, "device ordinal out of range");
    DeviceGuard g(device);
    phyzb_trainer* t = new phyzb_trainer;
    t->device = device;
    t->capacity = capacity;
    t->max_b = max_b;
    auto bail = [&](int rc) {
        destroy_trainer(t);
        return rc;
    };
    if (cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(PHYZB_ERR_CUDA, "cudaStreamCreate"));
    int rc = alloc_net(t->actor, actor, actor.n_out, max_b);
    if (rc == PHYZB_OK) rc = alloc_net(t->critic, critic, 0, max_b);
    if (rc != PHYZB_OK) return bail(rc);
    const size_t C = capacity;
    const int widest = std::max(std::max(actor.n_in, critic.n_in), actor.n_out);
    struct {
        float** p;
        size_t n;
    } cols[] = {{&t->obs_a, C * actor.n_in}, {&t->obs_c, C * critic.n_in}, {&t->act, C * actor.n_out},
                {&t->logp, C},              {&t->adv, C},                 {&t->ret, C},
                {&t->upload_raw, C * widest}, {&t->dlogstd, (size_t)pad32(actor.n_out) * max_b},
                {&t->stats, (size_t)4 * max_b},
                {&t->xa, (size_t)actor.n_in * max_b}, {&t->xc, (size_t)critic.n_in * max_b}};
    for (auto& c : cols)
        if (cudaMalloc((void**)c.p, c.n * 4) != cudaSuccess) return bail(fail(PHYZB_ERR_CUDA, "cudaMalloc batch"));
    const size_t ng = (size_t)t->actor.d.n_param + t->critic.d.n_param + 4;
    if (cudaMalloc((void**)&t->gblock, ng * 4) != cudaSuccess || cudaMemset(t->gblock, 0, ng * 4) != cudaSuccess)
        return bail(fail(PHYZB_ERR_CUDA, "cudaMalloc gradients"));
    t->actor.d.g = t->gblock;
    t->critic.d.g = t->gblock + t->actor.d.n_param;
    t->reduced = t->critic.d.g + t->critic.d.n_param;
    if (cudaHostAlloc((void**)&t->reduced_host, 16, cudaHostAllocDefault) != cudaSuccess)
        return bail(fail(PHYZB_ERR_CUDA, "cudaHostAlloc"));
    const int rows = std::max(std::max(actor.n_h, critic.n_h), actor.n_out);
    const int colsN = std::max(std::max(actor.n_in, critic.n_in), std::max(actor.n_h, critic.n_h));
    if (cudaMalloc((void**)&t->work, pz::train_work_bytes(max_b, rows, colsN)) != cudaSuccess)
        return bail(fail(PHYZB_ERR_CUDA, "cudaMalloc work"));
    *out = t;
    return PHYZB_OK;
}

int phyzb_trainer_destroy(phyzb_trainer* t) {
    destroy_trainer(t);
    return PHYZB_OK;
}

int phyzb_trainer_set_adam(phyzb_trainer* t, const phyzb_adam_cfg* a, const phyzb_adam_cfg* c) {
    if (!t || !a || !c) return fail(PHYZB_ERR_INVALID, "null argument");
    t->actor.adam = *a;
    t->critic.adam = *c;
    return PHYZB_OK;
}

int phyzb_trainer_set_params(phyzb_trainer* t, int32_t which, const double* flat, int64_t n) {
    if (!t || !flat) return fail(PHYZB_ERR_INVALID, "null argument");
    Net* net = net_of(t, which);
    if (!net) return fail(PHYZB_ERR_INVALID, "which must be 0 (actor) or 1 (critic)");
    if (n != net->d.n_param)
        return fail(PHYZB_ERR_INVALID, "parameter array is " + std::to_string(n) + " long, network wants " +
                                           std::to_string(net->d.n_param));
    DeviceGuard g(t->device);
    return set_net_params(*net, flat);
}

int phyzb_trainer_params(phyzb_trainer* t, int32_t which, double* flat, int64_t n) {
    if (!t || !flat) return fail(PHYZB_ERR_INVALID, "null argument");
    Net* net = net_of(t, which);
    if (!net) return fail(PHYZB_ERR_INVALID, "which must be 0 (actor) or 1 (critic)");
    if (n != net->d.n_param)
        return fail(PHYZB_ERR_INVALID, "parameter array is " + std::to_string(n) + " long, network has " +
                                           std::to_string(net->d.n_param));
    DeviceGuard g(t->device);
    PZ_TRY(bounded_sync(t->stream));
    PZ_CUDA(cudaMemcpy(flat, net->d.p, (size_t)n * 8, cudaMemcpyDeviceToHost));
    return PHYZB_OK;
}

int phyzb_trainer_upload_batch(phyzb_trainer* t, int64_t n, const float* obs_a, const float* obs_c, const float* act,
                               const float* logp_old, const float* adv, const float* ret) {
    if (!t) return fail(PHYZB_ERR_INVALID, "trainer is null");
    if (n < 0 || n > t->capacity)
        return fail(PHYZB_ERR_INVALID, std::to_string(n) + " samples into a pipeline built for " +
                                           std::to_string(t->capacity));
    if (n > 0 && (!obs_a || !obs_c || !act || !logp_old || !adv || !ret))
        return fail(PHYZB_ERR_INVALID, "batch column is null");
    DeviceGuard g(t->device);
    PZ_TRY(upload_col(t, obs_a, t->actor.d.n_in, n, t->obs_a));
    PZ_TRY(upload_col(t, obs_c, t->critic.d.n_in, n, t->obs_c));
    PZ_TRY(upload_col(t, act, t->actor.d.n_out, n, t->act));
    PZ_TRY(upload_col(t, logp_old, 1, n, t->logp));
    PZ_TRY(upload_col(t, adv, 1, n, t->adv));
    PZ_TRY(upload_col(t, ret, 1, n, t->ret));
    PZ_TRY(bounded_sync(t->stream));
    t->n_rows = n;
    t->c_obs_a = pz::BatchCol{t->obs_a, std::max<long long>(n, 1), t->actor.d.n_in};
    t->c_obs_c = pz::BatchCol{t->obs_c, std::max<long long>(n, 1), t->critic.d.n_in};
    t->c_act = pz::BatchCol{t->act, std::max<long long>(n, 1), t->actor.d.n_out};
    t->c_logp = pz::BatchCol{t->logp, std::max<long long>(n, 1), 1};
    t->c_adv = pz::BatchCol{t->adv, std::max<long long>(n, 1), 1};
    t->c_ret = pz::BatchCol{t->ret, std::max<long long>(n, 1), 1};
    return PHYZB_OK;
}

int phyzb_trainer_update(phyzb_trainer* t, const uint32_t* order, int32_t n_orders, const phyzb_ppo_cfg* cfg,
                         phyzb_update_stats* out) {
    if (!t || !cfg || !out) return fail(PHYZB_ERR_INVALID, "null argument");
    *out = phyzb_update_stats{0.0, 0.0, 0.0, 0, 0};
    const long long N = t->n_rows;
    if (N == 0) return PHYZB_OK;
    PZ_TRY(check_update(t, cfg));
    if (n_orders < cfg->epochs || !order)
        return fail(PHYZB_ERR_INVALID, std::to_string(n_orders) + " shuffles for " + std::to_string(cfg->epochs) +
                                           " epochs");
    for (long long k = 0; k < (long long)cfg->epochs * N; k++)
        if (order[k] >= N) return fail(PHYZB_ERR_INVALID, "shuffle index out of range");
    DeviceGuard g(t->device);
    const size_t obytes = (size_t)cfg->epochs * N * 4;
    PZ_TRY(ensure_order(t, obytes));
    PZ_CUDA(cudaMemcpyAsync(t->order, order, obytes, cudaMemcpyHostToDevice, t->stream));
    return run_update(t, cfg, out);
}

int phyzb_trainer_update_shuffled(phyzb_trainer* t, const phyzb_ppo_cfg* cfg, uint64_t seed,
                                  phyzb_update_stats* out) {
    if (!t || !cfg || !out) return fail(PHYZB_ERR_INVALID, "null argument");
    *out = phyzb_update_stats{0.0, 0.0, 0.0, 0, 0};
    const long long N = t->n_rows;
    if (N == 0) return PHYZB_OK;
    PZ_TRY(check_update(t, cfg));
    DeviceGuard g(t->device);
    // one affine permutation (a k + c) mod N per epoch, a coprime with N,
    // drawn from a SplitMix64 stream of `seed`
    std::vector<unsigned long long> ac(2 * (size_t)std::max(cfg->epochs, 1));
    uint64_t z = seed;
    auto next = [&]() {
        z += 0x9E3779B97F4A7C15ull;
        uint64_t x = z;
        x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
        x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
        return x ^ (x >> 31);
    };
    auto gcd = [](unsigned long long a, unsigned long long b) {
        while (b) {
            const unsigned long long r = a % b;
            a = b;
            b = r;
        }
        return a;
    };
    for (int e = 0; e < cfg->epochs; e++) {
        unsigned long long a = 1;
        if (N > 2)
            do a = 1 + next() % (unsigned long long)(N - 1);
            while (gcd(a, (unsigned long long)N) != 1);
        ac[2 * e] = a;
        ac[2 * e + 1] = next() % (unsigned long long)N;
    }
    if (!t->ac) PZ_CUDA(cudaMalloc((void**)&t->ac, 2 * 64 * sizeof(unsigned long long)));
    if (cfg->epochs > 64) return fail(PHYZB_ERR_INVALID, "at most 64 epochs per update");
    PZ_CUDA(cudaMemcpyAsync(t->ac, ac.data(), ac.size() * 8, cudaMemcpyHostToDevice, t->stream));
    PZ_TRY(ensure_order(t, (size_t)cfg->epochs * N * 4));
    PZ_CUDA(pz::train_orders(t->order, N, cfg->epochs, t->ac, t->stream));
    return run_update(t, cfg, out);
}

int phyzb_trainer_set_batch_device(phyzb_trainer* t, int64_t n_rows, const phyzb_batch_col* cols) {
    if (!t || !cols) return fail(PHYZB_ERR_INVALID, "null argument");
    if (n_rows < 0) return fail(PHYZB_ERR_INVALID, "n_rows must be >= 0");
    const int want[6] = {t->actor.d.n_in, t->critic.d.n_in, t->actor.d.n_out, 1, 1, 1};
    for (int k = 0; k < 6; k++) {
        if (n_rows > 0 && (!cols[k].base || cols[k].block < 1 || n_rows % cols[k].block != 0))
            return fail(PHYZB_ERR_INVALID, "batch column " + std::to_string(k) +
                                               ": null, or n_rows not a multiple of its block");
        if (cols[k].features < want[k])
            return fail(PHYZB_ERR_INVALID, "batch column " + std::to_string(k) + " has " +
                                               std::to_string(cols[k].features) + " features, needs " +
                                               std::to_string(want[k]));
    }
    if (n_rows > 0xFFFFFFFFLL) return fail(PHYZB_ERR_INVALID, "at most 2^32 - 1 rows (32-bit shuffle indices)");
    auto bc = [](const phyzb_batch_col& c) { return pz::BatchCol{c.base, c.block, c.features}; };
    t->c_obs_a = bc(cols[0]);
    t->c_obs_c = bc(cols[1]);
    t->c_act = bc(cols[2]);
    t->c_logp = bc(cols[3]);
    t->c_adv = bc(cols[4]);
    t->c_ret = bc(cols[5]);
    t->n_rows = n_rows;
    return PHYZB_OK;
}

int phyzb_trainer_evaluate(phyzb_trainer* t, int32_t which, phyzb_batch_col x, int64_t n_rows, float* out) {
    if (!t || !out) return fail(PHYZB_ERR_INVALID, "null argument");
    Net* net = net_of(t, which);
    if (!net) return fail(PHYZB_ERR_INVALID, "which must be 0 (actor) or 1 (critic)");
    if (!x.base || x.block < 1 || x.features < net->d.n_in) return fail(PHYZB_ERR_INVALID, "bad input column");
    DeviceGuard g(t->device);
    const pz::BatchCol c{x.base, x.block, x.features};
    for (long long r0 = 0; r0 < n_rows; r0 += t->max_b) {
        const int b = (int)std::min<long long>(t->max_b, n_rows - r0);
        PZ_CUDA(pz::train_forward(net->d, c, nullptr, b, t->stream, r0));
        for (int k = 0; k < net->d.n_out; k++)
            PZ_CUDA(cudaMemcpyAsync(out + (size_t)k * n_rows + r0, net->d.out + (size_t)k * t->max_b,
                                    (size_t)b * 4, cudaMemcpyDeviceToDevice, t->stream));
    }
    PZ_TRY(bounded_sync(t->stream));
    return PHYZB_OK;
}

int phyzb_trainer_set_comm(phyzb_trainer* t, phyzb_comm* comm) {
    if (!t) return fail(PHYZB_ERR_INVALID, "trainer is null");
    t->comm = comm;
    return PHYZB_OK;
}

// ── the collector side: a sim's policy history as the update's batch ────

int phyzb_policy_history_view(phyzb_sim* s, phyzb_policy_history* out) {
    PZ_TRY(check_sim(s));
    if (!out) return fail(PHYZB_ERR_INVALID, "output is null");
    if (!s->policy) return fail(PHYZB_ERR_STATE, "policy pass not enabled — call enable_policy first");
    PolicyDev* p = s->policy;
    out->obs = p->d_obs;
    out->out = p->d_out;
    out->n_obs = p->n_in;
    out->n_act = p->n_out;
    out->nworld = s->nworld;
    out->steps = p->history;
    return PHYZB_OK;
}

int phyzb_policy_advantages(phyzb_sim* s, phyzb_trainer* t, phyzb_comm* comm, const phyzb_return_cfg* cfg,
                            float* adv, float* ret, double* stats) {
    PZ_TRY(check_sim(s));
    if (!t || !cfg || !adv || !ret) return fail(PHYZB_ERR_INVALID, "null argument");
    if (!s->policy) return fail(PHYZB_ERR_STATE, "policy pass not enabled — call enable_policy first");
    PolicyDev* p = s->policy;
    const int T = cfg->steps;
    if (T < 1 || T + 1 > p->history)
        return fail(PHYZB_ERR_INVALID, "returns over " + std::to_string(T) + " steps need " + std::to_string(T + 1) +
                                           " history rows (have " + std::to_string(p->history) + ")");
    if (t->critic.d.n_in != p->n_in)
        return fail(PHYZB_ERR_INVALID, "critic input width " + std::to_string(t->critic.d.n_in) +
                                           " differs from the observation width " + std::to_string(p->n_in));
    if (!cfg->reward_coef) return fail(PHYZB_ERR_INVALID, "reward_coef is null");
    DeviceGuard g(s->device);
    const long long N = s->nworld;
    // scratch (kept on the policy state)
    const size_t need_r = (size_t)T * N * 4, need_v = (size_t)(T + 1) * N * 4,
                 need_p = (size_t)pz::gae_blocks(N) * 3 * 8 + 4 * 8;
    if (need_r + need_v + need_p + (size_t)p->n_in * 4 > p->ret_bytes) {
        if (p->d_ret_scratch) cudaFree(p->d_ret_scratch);
        p->d_ret_scratch = nullptr;
        p->ret_bytes = 0;
        const size_t bytes = need_r + need_v + need_p + (size_t)pz::POLICY_MAX_IN * 4 + 256;
        PZ_CUDA(cudaMalloc(&p->d_ret_scratch, bytes));
        p->ret_bytes = bytes;
    }
    char* base = (char*)p->d_ret_scratch;
    double* sums = (double*)base;  // 4 doubles
    double* part = sums + 4;
    float* rew = (float*)(base + need_p);
    float* val = rew + (size_t)T * N;
    float* coef = val + (size_t)(T + 1) * N;
    std::vector<float> cf(p->n_in);
    for (int j = 0; j < p->n_in; j++) cf[j] = (float)cfg->reward_coef[j];
    PZ_CUDA(cudaMemcpyAsync(coef, cf.data(), cf.size() * 4, cudaMemcpyHostToDevice, s->stream));
    PZ_CUDA(pz::rollout_rewards(p->d_obs, p->d_out, p->n_in, p->n_out, N, T, coef, (float)cfg->action_penalty, rew,
                                s->stream));
    PZ_TRY(bounded_sync(s->stream));
    // critic values of rows 0 .. T
    const phyzb_batch_col oc{p->d_obs, N, p->n_in};
    PZ_TRY(phyzb_trainer_evaluate(t, 1, oc, (int64_t)(T + 1) * N, val));
    PZ_CUDA(pz::rollout_gae(rew, val, N, T, (float)cfg->gamma, (float)cfg->lambda, adv, ret, part, sums, s->stream));
    PZ_TRY(comm_allreduce_sum(comm, sums, 3, true, s->stream));
    const double count = (double)T * N * comm_nranks(comm);
    if (cfg->normalize) PZ_CUDA(pz::normalize_advantages(adv, (long long)T * N, sums, count, s->stream));
    // bounded wait on the collective first: the read-back below then finds
    // the stream idle
    PZ_TRY(comm_wait(comm, s->stream, 120.0));
    double hs[3] = {0, 0, 0};
    PZ_CUDA(cudaMemcpyAsync(hs, sums, sizeof(hs), cudaMemcpyDeviceToHost, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    if (stats) {
        const double mean = hs[0] / count;
        stats[0] = hs[2] / ((double)N * comm_nranks(comm));  // mean return per world
        stats[1] = mean;
        stats[2] = std::sqrt(std::max(hs[1] / count - mean * mean, 0.0));
    }
    return PHYZB_OK;
}

int phyzb_policy_sync_from_trainer(phyzb_sim* s, phyzb_trainer* t) {
    PZ_TRY(check_sim(s));
    if (!t) return fail(PHYZB_ERR_INVALID, "trainer is null");
    if (!s->policy) return fail(PHYZB_ERR_STATE, "policy pass not enabled — call enable_policy first");
    PolicyDev* p = s->policy;
    const pz::NetDev& a = t->actor.d;
    if (a.n_in != p->n_in || a.n_h != p->n_h || a.n_out != p->n_out || a.n_wf != p->n_wf)
        return fail(PHYZB_ERR_INVALID, "actor shape differs from the policy's");
    DeviceGuard g(s->device);
    PZ_TRY(bounded_sync(t->stream));
    PZ_CUDA(cudaMemcpyAsync(p->d_w, a.wf, (size_t)a.n_wf * 4, cudaMemcpyDeviceToDevice, s->stream));
    std::vector<double> logstd(a.n_out);
    PZ_CUDA(cudaMemcpy(logstd.data(), a.p + t->actor.mlp_params, (size_t)a.n_out * 8, cudaMemcpyDeviceToHost));
    std::vector<float> sd(a.n_out);
    for (int k = 0; k < a.n_out; k++) sd[k] = (float)std::exp(logstd[k]);
    PZ_CUDA(cudaMemcpyAsync(p->d_std, sd.data(), sd.size() * 4, cudaMemcpyHostToDevice, s->stream));
    PZ_TRY(bounded_sync(s->stream));
    p->has_weights = p->has_std = true;
    return PHYZB_OK;
}

}  // extern "C"
