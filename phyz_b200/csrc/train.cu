// Kernels of the device-resident PPO update (pz_train.h).
//
// The reference walks the update as one thread per weight looping over the
// whole minibatch (phyz_train.cu:195-246); here the per-row work is fused
// (one thread per sample runs a network's forward, or its whole two-layer
// backward, out of shared memory), and every parameter gradient is one
// split-K reduction: blocks of 256 samples accumulate 32 x 32 tiles of
// sum_r dsrc[m][r] * x[r][n] (plus the bias column, x = 1) in f64 -- the
// reference's accumulator precision -- and a second pass adds the splits in a
// fixed order, so results are deterministic run to run.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "pz_mlp.cuh"
#include "pz_train.h"

namespace pz {

namespace {

constexpr int ROW_BLOCK = 128;  // samples per block of the per-row kernels
constexpr int GKC_MIN = 256;    // rows per split, at least

__device__ __forceinline__ float col(const BatchCol& c, long long r, int k) {
    return c.base[(r / c.N) * (long long)c.F * c.N + (long long)k * c.N + r % c.N];
}


__global__ void __launch_bounds__(ROW_BLOCK) fwd_kernel(const NetDev n, const BatchCol x, const uint32_t* idx,
                                                        long long r0, int b) {
    extern __shared__ __align__(16) float sm[];
    stage_weights(n.wf, n.n_wf, sm);
    const float* W1 = sm;
    const float* b1 = W1 + n.in_pad * n.h_pad;
    const float* W2 = b1 + n.h_pad;
    const float* b2 = W2 + n.h_pad * n.h_pad;
    const float* W3 = b2 + n.h_pad;
    const float* b3 = W3 + n.h_pad * n.out_pad;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= b) return;
    const long long s = idx ? (long long)idx[r] : r0 + r;
    const float* xr = x.base + (s / x.N) * (long long)x.F * x.N + s % x.N;  // feature k at xr[k * N]
    const long long L = n.max_b;
    const int n_in = n.n_in;
    float* h1 = n.h1 + r;
    float* h2 = n.h2 + r;
    float* out = n.out + r;
    dense_tiles(W1, b1, n.in_pad, n.h_pad, [&](int i) { return i < n_in ? xr[(long long)i * x.N] : 0.0f; },
                [&](int j, float a) { h1[j * L] = tanhf(a); });
    dense_tiles(W2, b2, n.h_pad, n.h_pad, [&](int i) { return h1[i * L]; },
                [&](int j, float a) { h2[j * L] = tanhf(a); });
    dense_tiles(W3, b3, n.h_pad, n.out_pad, [&](int i) { return h2[i * L]; },
                [&](int k, float a) { out[k * L] = a; });
}

// phyz_train.cu:136-186, per row; the padding rows of dout are zeroed.
__global__ void ppo_grad_kernel(const NetDev n, const PpoArgs a, const BatchCol act, const BatchCol logp_old,
                                const BatchCol adv, const uint32_t* idx, int b, float* dlogstd, float* stats) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= b) return;
    const long long L = n.max_b;
    const long long s = idx[r];
    const float LN_2PI = 1.8378770664093453f;
    const float* logstd = n.wflat + a.logstd_off;
    float logp = 0.0f;
    for (int d = 0; d < n.n_out; d++) {
        const float sd = expf(logstd[d]);
        const float z = (col(act, s, d) - n.out[d * L + r]) / sd;
        logp += -0.5f * z * z - logf(sd) - 0.5f * LN_2PI;
    }
    const float av = col(adv, s, 0);
    const float lpo = col(logp_old, s, 0);
    const float log_ratio = logp - lpo;
    const float ratio = expf(log_ratio);
    const float clipped = fminf(fmaxf(ratio, 1.0f - a.clip), 1.0f + a.clip);
    const float unclipped_obj = ratio * av;
    const float clipped_obj = clipped * av;
    stats[0 * L + r] = -(unclipped_obj < clipped_obj ? unclipped_obj : clipped_obj);
    stats[1 * L + r] = lpo - logp;
    stats[2 * L + r] = ratio - 1.0f - log_ratio;
    const bool active = unclipped_obj <= clipped_obj + 1e-12f;
    const float ent = a.entropy_coef / (float)b;
    for (int d = 0; d < n.out_pad; d++) {
        if (d >= n.n_out) {
            n.dout[d * L + r] = 0.0f;
            continue;
        }
        if (!active) {
            n.dout[d * L + r] = 0.0f;
            dlogstd[d * L + r] = -ent;
            continue;
        }
        const float coef = -av * ratio / (float)b;
        const float sd = expf(logstd[d]);
        const float z = (col(act, s, d) - n.out[d * L + r]) / sd;
        n.dout[d * L + r] = coef * (z / sd);
        dlogstd[d * L + r] = coef * (z * z - 1.0f) - ent;
    }
}

// phyz_train.cu:193-203, per row.
__global__ void value_grad_kernel(const NetDev n, const PpoArgs a, const BatchCol ret, const uint32_t* idx, int b,
                                  float* stats) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= b) return;
    const long long L = n.max_b;
    const float err = n.out[r] - col(ret, idx[r], 0);
    stats[3 * L + r] = err * err;
    const float d = fminf(fmaxf(err, -a.vdelta), a.vdelta);
    n.dout[r] = 2.0f * d / (float)b;
    for (int k = 1; k < n.out_pad; k++) n.dout[k * L + r] = 0.0f;
}

// Both hidden layers of the backward pass for one row (phyz_train.cu:213-224
// twice): dh2 = (W3^T dout) (1 - h2^2), dh1 = (W2^T dh2) (1 - h1^2).
__global__ void __launch_bounds__(ROW_BLOCK) bwd_kernel(const NetDev n, int b) {
    extern __shared__ __align__(16) float sm[];
    stage_weights(n.wb, n.n_wb, sm);
    const float* W3 = sm;                        // [out_pad][h_pad]
    const float* W2 = W3 + n.out_pad * n.h_pad;  // [h_pad][h_pad]
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= b) return;
    const long long L = n.max_b;
    const float* dout = n.dout + r;
    const float* h2 = n.h2 + r;
    const float* h1 = n.h1 + r;
    float* dh2 = n.dh2 + r;
    float* dh1 = n.dh1 + r;
    dense_tiles(W3, nullptr, n.out_pad, n.h_pad, [&](int k) { return dout[k * L]; },
                [&](int j, float a) {
                    const float h = h2[j * L];
                    dh2[j * L] = a * (1.0f - h * h);
                });
    dense_tiles(W2, nullptr, n.h_pad, n.h_pad, [&](int k) { return dh2[k * L]; },
                [&](int j, float a) {
                    const float h = h1[j * L];
                    dh1[j * L] = a * (1.0f - h * h);
                });
}

// Split-K partial sums part[split][m][n] = sum over the split's rows of
// A[m][r] * Bv(r, n) for n < N, and part[split][m][N] = sum A[m][r] (the
// bias column). A is SoA [M][lda]; Bv is SoA activations [N][ldb] or, with
// gather, batch column x at sample idx[r]. A block's output tile is TM x TN,
// shaped to the layer (64, 16 or 4 rows; 64, 32 or 4 columns), 4 x 4 per
// thread; the 256 threads that the tile leaves over split each KS-row stage
// into KG interleaved row groups, whose partials are added in group order
// before the split is written (the reduction kernel then sums the splits in
// a fixed order). Each stage
// accumulates in f32 registers and is added into f64 accumulators (the
// reference accumulates in f64); the next stage's rows are loaded into
// registers while the current one is multiplied.
template <int TM, int TN>
struct GradShape {
    static constexpr int TY = TM / 4, TX = TN / 4;
    static constexpr int KG = 256 / (TY * TX);  // row groups per stage
    // rows per stage: at least 32, two per row group, and enough that each
    // operand's stage is a whole number of elements per thread
    static constexpr int cmax(int a, int b) { return a > b ? a : b; }
    static constexpr int KS = cmax(cmax(32, 2 * KG), cmax(256 / TM, 256 / TN));
    static constexpr int PA = TM * KS / 256, PB = TN * KS / 256;  // elements each thread loads
};

template <int TM, int TN>
__global__ void __launch_bounds__(256) grad_kernel(const float* A, int lda, int M, const float* Bact, int ldb,
                                                   BatchCol x, const uint32_t* idx, int gather, int N, int b,
                                                   int kc, double* part) {
    using G = GradShape<TM, TN>;
    constexpr int KS = G::KS, KG = G::KG;
    // the stage operands, and after the last stage the row groups' partials
    constexpr int ABYTES = KS * (TM + 4) * 4, BBYTES = KS * (TN + 4) * 4, RBYTES = 256 * 20 * 8;
    constexpr int SBYTES = ABYTES + BBYTES > RBYTES ? ABYTES + BBYTES : RBYTES;
    __shared__ __align__(16) unsigned char sbuf[SBYTES];
    float(*As)[TM + 4] = reinterpret_cast<float(*)[TM + 4]>(sbuf);
    float(*Bs)[TN + 4] = reinterpret_cast<float(*)[TN + 4]>(sbuf + ABYTES);
    const int m0 = blockIdx.x * TM, n0 = blockIdx.y * TN, split = blockIdx.z;
    const int r0 = split * kc;
    const int r1 = min(b, r0 + kc);
    const int kg = threadIdx.x / (G::TY * G::TX), tt = threadIdx.x % (G::TY * G::TX);
    const int tx = tt % G::TX, ty = tt / G::TX;
    const bool bias_col = blockIdx.y == 0 && tx == 0;
    double acc[4][4], rs[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        rs[i] = 0.0;
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
    }
    float ra[G::PA], rb[G::PB];
    auto load = [&](int rst) {
#pragma unroll
        for (int u = 0; u < G::PA; u++) {
            const int e = threadIdx.x + u * 256;
            const int mm = e / KS, kk = e % KS, r = rst + kk, m = m0 + mm;
            ra[u] = (m < M && r < r1) ? A[(long long)m * lda + r] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < G::PB; u++) {
            const int e = threadIdx.x + u * 256;
            const int nn = e / KS, kk = e % KS, r = rst + kk, n = n0 + nn;
            float bv = 0.0f;
            if (r < r1 && n < N) bv = gather ? col(x, idx ? (long long)idx[r] : r, n) : Bact[(long long)n * ldb + r];
            rb[u] = bv;
        }
    };
    auto store = [&]() {
#pragma unroll
        for (int u = 0; u < G::PA; u++) {
            const int e = threadIdx.x + u * 256;
            As[e % KS][e / KS] = ra[u];
        }
#pragma unroll
        for (int u = 0; u < G::PB; u++) {
            const int e = threadIdx.x + u * 256;
            Bs[e % KS][e / KS] = rb[u];
        }
    };
    if (r0 < r1) load(r0);
    for (int rst = r0; rst < r1; rst += KS) {
        store();
        __syncthreads();
        if (rst + KS < r1) load(rst + KS);
        float fa[4][4] = {}, fr[4] = {};
#pragma unroll 4
        for (int kk = kg; kk < KS; kk += KG) {
            const float4 a4 = *reinterpret_cast<const float4*>(&As[kk][4 * ty]);
            const float4 b4 = *reinterpret_cast<const float4*>(&Bs[kk][4 * tx]);
            const float av[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
#pragma unroll
                for (int j = 0; j < 4; j++) fa[i][j] = fmaf(av[i], bv[j], fa[i][j]);
                fr[i] += av[i];
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            rs[i] += (double)fr[i];
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] += (double)fa[i][j];
        }
        __syncthreads();
    }
    if constexpr (KG > 1) {
        // the row groups' partials added in group order by group 0
        constexpr int TT = G::TY * G::TX;
        double* red = reinterpret_cast<double*>(sbuf);
        if (kg > 0) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                red[(kg * TT + tt) * 20 + 16 + i] = rs[i];
#pragma unroll
                for (int j = 0; j < 4; j++) red[(kg * TT + tt) * 20 + 4 * i + j] = acc[i][j];
            }
        }
        __syncthreads();
        if (kg > 0) return;
        for (int q = 1; q < KG; q++) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                rs[i] += red[(q * TT + tt) * 20 + 16 + i];
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] += red[(q * TT + tt) * 20 + 4 * i + j];
            }
        }
    }
    const int N1 = N + 1;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + 4 * ty + i;
        if (m >= M) continue;
        double* row = part + ((long long)split * M + m) * N1;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + 4 * tx + j;
            if (n < N) row[n] = acc[i][j];
        }
        if (bias_col) row[N] = rs[i];
    }
}

// dst[k][r] = x(idx[r], k): a minibatch's rows of a batch column made
// contiguous once (random reads), read coalesced by every later pass.
__global__ void gather_kernel(const BatchCol x, const uint32_t* idx, int b, int F, float* dst, int ld) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= b) return;
    const long long s = idx[r];
    const float* xr = x.base + (s / x.N) * (long long)x.F * x.N + s % x.N;
    for (int k = 0; k < F; k++) dst[(long long)k * ld + r] = xr[(long long)k * x.N];
}

// g[off_w + m * N + n] (n < N) and g[off_b + m] (bias) from the splits: 8
// lanes per output, each summing every 8th split, combined in a fixed
// shuffle order (deterministic).
__global__ void grad_reduce_kernel(const double* part, int nsplit, int M, int N, float* g, int off_w, int off_b) {
    const long long t = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int lane = threadIdx.x & 7;
    const int N1 = N + 1;
    const bool valid = t < (long long)M * N1;
    double s = 0.0;
    if (valid)
        for (int k = lane; k < nsplit; k += 8) s += part[(long long)k * M * N1 + t];
    for (int o = 4; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o, 8);
    if (valid && lane == 0) {
        const int m = (int)(t / N1), n = (int)(t % N1);
        if (n < N)
            g[off_w + m * N + n] = (float)s;
        else
            g[off_b + m] = (float)s;
    }
}

// tang's ModuleAdam step (phyz_train.cu:260-276) on the f64 master, then the
// f32 mirrors the forward, backward and log_std readers use.
__global__ void adam_kernel(const NetDev n, double lr, double beta1, double beta2, double eps, double wd,
                            double bc1, double bc2, double gscale) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n.n_param) return;
    double x = n.p[t];
    if (wd > 0.0) x = x * (1.0 - lr * wd);
    const double gr = gscale == 1.0 ? (double)n.g[t] : (double)n.g[t] * gscale;
    const double mt = beta1 * n.m[t] + (1.0 - beta1) * gr;
    const double vt = beta2 * n.v[t] + (1.0 - beta2) * gr * gr;
    n.m[t] = mt;
    n.v[t] = vt;
    const double m_hat = mt / bc1;
    const double v_hat = vt / bc2;
    x -= lr * m_hat / (sqrt(v_hat) + eps);
    n.p[t] = x;
    const float xf = (float)x;
    n.wflat[t] = xf;
    if (n.posf[t] >= 0) n.wf[n.posf[t]] = xf;
    if (n.posb[t] >= 0) n.wb[n.posb[t]] = xf;
}

int row_smem(int packed, int per_row, int W) { return (packed + per_row * W) * (int)sizeof(float); }

// Samples per block of a per-row kernel: the largest of 128 / 64 / 32 whose
// staged weights and per-row vectors fit the opt-in shared memory.
cudaError_t row_block(int packed, int per_row, int* W_out, int* smem_out) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
    for (int W = ROW_BLOCK; W >= 32; W /= 2)
        if (row_smem(packed, per_row, W) <= optin) {
            *W_out = W;
            *smem_out = row_smem(packed, per_row, W);
            return cudaSuccess;
        }
    return cudaErrorInvalidConfiguration;
}

// Rows per split: enough splits for about two blocks per SM over the
// output tiles, no split shorter than GKC_MIN rows, a whole number of stages.
int split_rows(int tiles, int ks, int b) {
    const int want = (2 * 148 + tiles - 1) / tiles;
    int rows = (b + want - 1) / want;
    rows = rows < GKC_MIN ? GKC_MIN : rows;
    return (rows + ks - 1) / ks * ks;
}

template <int TM, int TN>
cudaError_t grad_shaped(const float* A, int lda, int M, const float* Bact, int ldb, BatchCol x, const uint32_t* idx,
                        int gather, int N, int b, float* g, int off_w, int off_b, double* work, cudaStream_t s) {
    using G = GradShape<TM, TN>;
    const int tiles = ((M + TM - 1) / TM) * (N > 0 ? (N + TN - 1) / TN : 1);
    const int kc = split_rows(tiles, G::KS, b);
    const int nsplit = (b + kc - 1) / kc;
    dim3 grid((unsigned)((M + TM - 1) / TM), (unsigned)(N > 0 ? (N + TN - 1) / TN : 1), (unsigned)nsplit);
    grad_kernel<TM, TN><<<grid, 256, 0, s>>>(A, lda, M, Bact, ldb, x, idx, gather, N, b, kc, work);
    const long long lanes = (long long)M * (N + 1) * 8;
    grad_reduce_kernel<<<(unsigned)((lanes + 255) / 256), 256, 0, s>>>(work, nsplit, M, N, g, off_w, off_b);
    return cudaGetLastError();
}

// The tile shape of a layer: 64, 16 or 4 output rows; 64, 32 or 4 columns.
cudaError_t grad(const float* A, int lda, int M, const float* Bact, int ldb, BatchCol x, const uint32_t* idx,
                 int gather, int N, int b, float* g, int off_w, int off_b, double* work, cudaStream_t s) {
    const int rm = M > 16 ? 64 : (M > 4 ? 16 : 4), cn = N > 32 ? 64 : (N > 4 ? 32 : 4);
#define PZ_GRAD(TM_, TN_)                                                                                        \
    if (rm == TM_ && cn == TN_) return grad_shaped<TM_, TN_>(A, lda, M, Bact, ldb, x, idx, gather, N, b, g, off_w, \
                                                             off_b, work, s);
    PZ_GRAD(64, 64) PZ_GRAD(64, 32) PZ_GRAD(64, 4) PZ_GRAD(16, 64) PZ_GRAD(16, 32) PZ_GRAD(16, 4)
    PZ_GRAD(4, 64) PZ_GRAD(4, 32) PZ_GRAD(4, 4)
#undef PZ_GRAD
    return cudaErrorInvalidValue;
}

}  // namespace

size_t train_work_bytes(int max_b, int max_rows, int max_cols) {
    const size_t nsplit = (size_t)(max_b + GKC_MIN - 1) / GKC_MIN;
    return nsplit * (size_t)max_rows * (size_t)(max_cols + 1) * sizeof(double);
}

cudaError_t train_forward(const NetDev& n, BatchCol x, const uint32_t* idx, int b, cudaStream_t s, long long r0) {
    if (b <= 0) return cudaSuccess;
    int W = 0, smem = 0;
    cudaError_t e = row_block(n.n_wf, 0, &W, &smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    fwd_kernel<<<(b + W - 1) / W, W, smem, s>>>(n, x, idx, r0, b);
    return cudaGetLastError();
}

cudaError_t train_gather(BatchCol x, const uint32_t* idx, int b, int F, float* dst, int ld, cudaStream_t s) {
    if (b <= 0) return cudaSuccess;
    gather_kernel<<<(b + 255) / 256, 256, 0, s>>>(x, idx, b, F, dst, ld);
    return cudaGetLastError();
}

cudaError_t train_ppo_grad(const NetDev& actor, const PpoArgs& a, BatchCol act, BatchCol logp_old, BatchCol adv,
                           const uint32_t* idx, int b, float* dlogstd, float* stats, cudaStream_t s) {
    if (b <= 0) return cudaSuccess;
    ppo_grad_kernel<<<(b + 127) / 128, 128, 0, s>>>(actor, a, act, logp_old, adv, idx, b, dlogstd, stats);
    return cudaGetLastError();
}

cudaError_t train_value_grad(const NetDev& critic, const PpoArgs& a, BatchCol ret, const uint32_t* idx, int b,
                             float* stats, cudaStream_t s) {
    if (b <= 0) return cudaSuccess;
    value_grad_kernel<<<(b + 127) / 128, 128, 0, s>>>(critic, a, ret, idx, b, stats);
    return cudaGetLastError();
}

cudaError_t train_backward(const NetDev& n, BatchCol x, const uint32_t* idx, int b, double* work, cudaStream_t s) {
    if (b <= 0) return cudaSuccess;
    const long long L = n.max_b;
    // flat offsets (tang's Mlp::to_flat): W1 b1 W2 b2 W3 b3
    const int oW1 = 0, ob1 = n.n_h * n.n_in, oW2 = ob1 + n.n_h, ob2 = oW2 + n.n_h * n.n_h, oW3 = ob2 + n.n_h,
              ob3 = oW3 + n.n_out * n.n_h;
    // layer 3: input h2
    cudaError_t e = grad(n.dout, (int)L, n.n_out, n.h2, (int)L, x, idx, 0, n.n_h, b, n.g, oW3, ob3, work, s);
    if (e != cudaSuccess) return e;
    int W = 0, smem = 0;
    if ((e = row_block(n.n_wb, 0, &W, &smem)) != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    bwd_kernel<<<(b + W - 1) / W, W, smem, s>>>(n, b);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // layer 2: input h1; layer 1: input the batch rows
    e = grad(n.dh2, (int)L, n.n_h, n.h1, (int)L, x, idx, 0, n.n_h, b, n.g, oW2, ob2, work, s);
    if (e != cudaSuccess) return e;
    return grad(n.dh1, (int)L, n.n_h, nullptr, 0, x, idx, 1, n.n_in, b, n.g, oW1, ob1, work, s);
}

cudaError_t train_row_sums(const float* rows, int nrows, int ld, int b, float* g, int off, double* work,
                           cudaStream_t s) {
    if (b <= 0) return cudaSuccess;
    return grad(rows, ld, nrows, nullptr, 0, BatchCol{nullptr, 1, 1}, nullptr, 0, 0, b, g, 0, off, work, s);
}

cudaError_t train_adam(const NetDev& n, double lr, double beta1, double beta2, double eps, double wd, double bc1,
                       double bc2, double gscale, cudaStream_t s) {
    adam_kernel<<<(n.n_param + 255) / 256, 256, 0, s>>>(n, lr, beta1, beta2, eps, wd, bc1, bc2, gscale);
    return cudaGetLastError();
}

cudaError_t train_stats(const float* stats, int ld, int b, float* out, double* work, cudaStream_t s) {
    // four row sums: the bias column of the split-K reduction
    return grad(stats, ld, 4, nullptr, 0, BatchCol{nullptr, 1, 1}, nullptr, 0, 0, b, out, 0, 0, work, s);
}

// ── the collector side of an update: rewards, GAE, normalization ────────

namespace {

// order[e][k] = (a_e k + c_e) mod n: one affine permutation per epoch
__global__ void order_kernel(uint32_t* order, long long n, int epochs, const unsigned long long* ac) {
    const long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    for (int e = 0; e < epochs; e++) {
        const unsigned long long a = ac[2 * e], c = ac[2 * e + 1];
        // a, k < n <= 2^32: the product fits 64 bits
        order[(long long)e * n + k] = (uint32_t)((a * (unsigned long long)k % (unsigned long long)n + c) %
                                                 (unsigned long long)n);
    }
}

// r[t][w] = sum_j coef[j] obs[t+1][j][w] - pen sum_k act[t][k][w]^2
__global__ void reward_kernel(const float* obs, const float* out, int n_in, int n_out, long long N, int T,
                              const float* coef, float pen, float* r) {
    const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= N) return;
    for (int t = 0; t < T; t++) {
        const float* o = obs + (long long)(t + 1) * n_in * N + w;
        float acc = 0.0f;
        for (int j = 0; j < n_in; j++)
            if (coef[j] != 0.0f) acc += coef[j] * o[(long long)j * N];
        const float* a = out + (long long)t * (n_out + 1) * N + w;
        float e = 0.0f;
        for (int k = 0; k < n_out; k++) e += a[(long long)k * N] * a[(long long)k * N];
        r[(long long)t * N + w] = acc - pen * e;
    }
}

// GAE per world (backward over t), with per-block sums of adv, adv^2 and the
// world's return into part[block][3] (fixed tree order).
__global__ void gae_kernel(const float* r, const float* V, long long N, int T, float gamma, float lam, float* adv,
                           float* ret, double* part) {
    __shared__ double red[3][256];
    const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    double sa = 0.0, sa2 = 0.0, sr = 0.0;
    if (w < N) {
        float A = 0.0f;
        for (int t = T - 1; t >= 0; t--) {
            const float v = V[(long long)t * N + w];
            const float rt = r[(long long)t * N + w];
            const float delta = rt + gamma * V[(long long)(t + 1) * N + w] - v;
            A = delta + gamma * lam * A;
            adv[(long long)t * N + w] = A;
            ret[(long long)t * N + w] = A + v;
            sa += A;
            sa2 += (double)A * A;
            sr += rt;
        }
    }
    red[0][threadIdx.x] = sa;
    red[1][threadIdx.x] = sa2;
    red[2][threadIdx.x] = sr;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s)
            for (int c = 0; c < 3; c++) red[c][threadIdx.x] += red[c][threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0)
        for (int c = 0; c < 3; c++) part[(long long)blockIdx.x * 3 + c] = red[c][0];
}

__global__ void sum_parts_kernel(const double* part, int nblocks, double* sums) {
    const int c = threadIdx.x;
    if (c >= 3) return;
    double s = 0.0;
    for (int b = 0; b < nblocks; b++) s += part[(long long)b * 3 + c];
    sums[c] = s;
}

// adv <- (adv - mean) / (std + 1e-8) from sums = [sum adv, sum adv^2, .],
// count = rows over every rank
__global__ void normalize_kernel(float* adv, long long n, const double* sums, double count) {
    const long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n) return;
    const double mean = sums[0] / count;
    const double var = fmax(sums[1] / count - mean * mean, 0.0);
    adv[k] = (float)(((double)adv[k] - mean) / (sqrt(var) + 1e-8));
}

}  // namespace

cudaError_t train_orders(uint32_t* order, long long n, int epochs, const unsigned long long* ac_dev, cudaStream_t s) {
    order_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(order, n, epochs, ac_dev);
    return cudaGetLastError();
}

cudaError_t rollout_rewards(const float* obs, const float* out, int n_in, int n_out, long long N, int T,
                            const float* coef, float pen, float* r, cudaStream_t s) {
    reward_kernel<<<(unsigned)((N + 127) / 128), 128, 0, s>>>(obs, out, n_in, n_out, N, T, coef, pen, r);
    return cudaGetLastError();
}

int gae_blocks(long long N) { return (int)((N + 255) / 256); }

cudaError_t rollout_gae(const float* r, const float* V, long long N, int T, float gamma, float lam, float* adv,
                        float* ret, double* part, double* sums, cudaStream_t s) {
    const int nb = gae_blocks(N);
    gae_kernel<<<nb, 256, 0, s>>>(r, V, N, T, gamma, lam, adv, ret, part);
    sum_parts_kernel<<<1, 32, 0, s>>>(part, nb, sums);
    return cudaGetLastError();
}

cudaError_t normalize_advantages(float* adv, long long n, const double* sums, double count, cudaStream_t s) {
    normalize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(adv, n, sums, count);
    return cudaGetLastError();
}

}  // namespace pz
