// PPO update of an actor and a critic MLP on the device (train.cu): the
// update half of phyz-gpu's training pipeline (crates/phyz-gpu/cuda/
// phyz_train.cu, src/cuda/train.rs) re-designed around per-row fused
// kernels, split-K gradient reductions and an f64-master Adam step.
// Host-side launch interface, used by capi_train.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace pz {

// A column block of per-sample data, rows r = t * N + w: feature k of row r
// lives at base[(r / N) * F * N + k * N + r % N] ("blocked SoA": the policy
// history [step][feature][world] with T = steps, and host batches uploaded
// as one block of N = n_rows).
struct BatchCol {
    const float* base;
    long long N;
    int F;
};

// One network's device state.
struct NetDev {
    int n_in, n_h, n_out;
    int in_pad, h_pad, out_pad;
    int n_param;           // flat parameters (+ the actor's log_std)
    int n_wf, n_wb;        // floats in the forward / backward packed weights
    double* p;             // f64 master parameters, flat reference order
    double* m;             // Adam moments
    double* v;
    float* g;              // gradient, flat order
    float* wflat;          // f32 mirror, flat order
    float* wf;             // forward pack: W1^T b1 W2^T b2 W3^T b3 (padded)
    float* wb;             // backward pack: W3 [out_pad][h_pad], W2 [h_pad][h_pad]
    const int* posf;       // flat index -> wf index (-1: none)
    const int* posb;       // flat index -> wb index (-1: none)
    float* h1;             // [h_pad][max_b]
    float* h2;             // [h_pad][max_b]
    float* out;            // [out_pad][max_b]
    float* dout;           // [out_pad][max_b]
    float* dh2;            // [h_pad][max_b]
    float* dh1;            // [h_pad][max_b]
    int max_b;
};

struct PpoArgs {
    float clip, entropy_coef, vdelta;
    int logstd_off;  // flat offset of the actor's log_std
};

// forward of `b` rows idx[0..b) of x (idx null: rows r0 .. r0 + b) through
// `net`, activations into its buffers
cudaError_t train_forward(const NetDev& net, BatchCol x, const uint32_t* idx, int b, cudaStream_t s,
                          long long r0 = 0);
// dst[k][r] = x(idx[r], k) for k < F, r < b (ld = row stride of dst)
cudaError_t train_gather(BatchCol x, const uint32_t* idx, int b, int F, float* dst, int ld, cudaStream_t s);
// actor: dL/dmean into net.dout, per-row dL/dlogstd, stats cols 0-2
cudaError_t train_ppo_grad(const NetDev& actor, const PpoArgs& a, BatchCol act, BatchCol logp_old, BatchCol adv,
                           const uint32_t* idx, int b, float* dlogstd, float* stats, cudaStream_t s);
// critic: dL/dvalue into net.dout, stats col 3
cudaError_t train_value_grad(const NetDev& critic, const PpoArgs& a, BatchCol ret, const uint32_t* idx, int b,
                             float* stats, cudaStream_t s);
// backprop net.dout through both hidden layers (net.dh2, net.dh1), then the
// gradient of every parameter into net.g (split-K, f64 accumulation), using
// `work` (train_work_bytes) as scratch
cudaError_t train_backward(const NetDev& net, BatchCol x, const uint32_t* idx, int b, double* work,
                           cudaStream_t s);
// sum of per-row values [rows][b] into g[off + row] (the log_std gradient)
cudaError_t train_row_sums(const float* rows, int nrows, int ld, int b, float* g, int off, double* work,
                           cudaStream_t s);
// Adam (tang's ModuleAdam, bias corrections bc1, bc2) on every parameter,
// refreshing the three f32 mirrors
cudaError_t train_adam(const NetDev& net, double lr, double beta1, double beta2, double eps, double wd,
                       double bc1, double bc2, double gscale, cudaStream_t s);
// column sums of stats [4][b] (f64 accumulation, fixed order) into out[4]
cudaError_t train_stats(const float* stats, int ld, int b, float* out, double* work, cudaStream_t s);
// scratch bytes train_backward needs for minibatches of up to max_b rows
size_t train_work_bytes(int max_b, int max_rows, int max_cols);

// epochs x n indices: order[e][k] = (a_e k + c_e) mod n, ac = [a_0, c_0, ...]
// on the device (a_e coprime with n: a permutation per epoch)
cudaError_t train_orders(uint32_t* order, long long n, int epochs, const unsigned long long* ac_dev, cudaStream_t s);
// rewards [T][N] of a policy history (obs [T+1][n_in][N], out [T][n_out+1][N]):
// r = coef . obs[t+1] - pen |act[t]|^2
cudaError_t rollout_rewards(const float* obs, const float* out, int n_in, int n_out, long long N, int T,
                            const float* coef, float pen, float* r, cudaStream_t s);
// GAE(gamma, lam) per world over values V [T+1][N]: adv, ret [T][N]; sums =
// [sum adv, sum adv^2, sum r] over the worlds (part: gae_blocks(N) x 3 scratch)
int gae_blocks(long long N);
cudaError_t rollout_gae(const float* r, const float* V, long long N, int T, float gamma, float lam, float* adv,
                        float* ret, double* part, double* sums, cudaStream_t s);
// adv <- (adv - mean) / (std + 1e-8), moments from sums over `count` rows
cudaError_t normalize_advantages(float* adv, long long n, const double* sums, double count, cudaStream_t s);

}  // namespace pz
