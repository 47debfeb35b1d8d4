// Kernels of the B200 batched rigid-body stepper (sm_100a).
//
// rollout_kernel runs phyz-gpu's whole step sequence (cuda/mod.rs:879-945:
// PD -> contact -> ABA -> integrate) for `nsteps` steps in ONE launch: one
// thread per world, the model table staged once per block into shared
// memory, and each world's q, v and every per-body intermediate of the
// articulated-body algorithm held in shared memory (structure-of-arrays,
// conflict-free) for the whole rollout. Global memory sees the initial state
// read, one coalesced control row per step (prefetched a sweep ahead with
// cp.async), and the final state / accelerations / contact state written.
//
// The reference runs the same physics as 3-4 launches per step with every
// intermediate in thread-local arrays (phyz_kernels.cu:1175-1369: 255
// registers and 9.6 KB of spilled stack per thread on sm_100a).
#include <cuda_runtime.h>

#include <cstdint>
#include <cmath>
#include <cstdlib>

#include "pz_launch.h"
#include "pz_world.cuh"

namespace pz {

// Per-thread view of the shared-memory scratch: slot s of this world lives
// at base[s * W] (consecutive threads -> consecutive banks).
template <class T>
struct SmemScr {
    T* base;
    int W;
    __device__ __forceinline__ T& operator()(int s) const { return base[s * W]; }
    __device__ __forceinline__ void prefetch(int s, const T* g) const {
        const unsigned sa = (unsigned)__cvta_generic_to_shared(&base[s * W]);
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(sa), "l"(g), "n"(sizeof(T)));
    }
    __device__ __forceinline__ void commit() const { asm volatile("cp.async.commit_group;\n" ::); }
    __device__ __forceinline__ void wait() const { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
};

template <class T>
__device__ __forceinline__ ModelView<T> make_view(const RolloutArgs<T>& P, const unsigned char* blob) {
    ModelView<T> M;
    M.bt = reinterpret_cast<const BodyT<T>*>(blob);
    M.bi = reinterpret_cast<const BodyI*>(blob + P.off_bi);
    M.pd = reinterpret_cast<const PdT<T>*>(blob + P.off_pd);
    M.pd_of_dof = reinterpret_cast<const int*>(blob + P.off_pdmap);
    M.nb = P.nb;
    M.nv = P.nv;
    M.npd = P.npd;
    M.contact = P.contact;
    M.dt = T(P.dt);
    M.gx = T(P.gx);
    M.gy = T(P.gy);
    M.gz = T(P.gz);
    M.ground_h = T(P.ground_h);
    M.friction = T(P.friction);
    const double dtc = P.dt > 1e-9 ? P.dt : 1e-9;
    M.inv_dt_c = T(1.0 / dtc);
    M.kstiff_c = T(4.0 / (dtc * dtc));
    return M;
}

// Copy the model table into shared memory (16-byte chunks) and return its
// shared-memory address. All threads of the block take part.
__device__ __forceinline__ unsigned char* stage_model(const void* g, int bytes, unsigned char* smem) {
    const int4* src = reinterpret_cast<const int4*>(g);
    int4* dst = reinterpret_cast<int4*>(smem);
    for (int k = threadIdx.x; k < bytes / 16; k += blockDim.x) dst[k] = __ldg(src + k);
    __syncthreads();
    return smem;
}

template <class T, int FEAT>
__global__ void __launch_bounds__(256) rollout_kernel(const __grid_constant__ RolloutArgs<T> P) {
    extern __shared__ __align__(16) unsigned char smem[];
    const unsigned char* blob = stage_model(P.model_blob, P.model_bytes, smem);
    const ModelView<T> M = make_view<T>(P, blob);
    const int W = blockDim.x;
    const SmemScr<T> S{reinterpret_cast<T*>(smem + P.model_bytes) + threadIdx.x, W};
    const long long ntiles = (P.nworld + W - 1) / W;
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long long w = tile * W + threadIdx.x;
        if (w >= P.nworld) continue;  // no block-wide synchronisation past this point
        const long long N = P.nworld;
        for (int j = 0; j < M.nv; j++) {
            S(j) = P.q[j * N + w];
            S(M.nv + j) = P.v[j * N + w];
        }
        const WorldIO<T> io{P.ctrl, P.ctrl_stride, P.targets, N, w};
        for (int i = 0; i < M.nb; i++) prefetch_controls(M, M.bi[i], S, io, 0);
        S.commit();
        const Out<T> none{nullptr, 0};
        pass1_all<FEAT>(M, S);
        for (int s = 0; s < P.nsteps; s++) {
            S.wait();
            const bool last = s == P.nsteps - 1;
            if constexpr ((FEAT & FEAT_CONTACT) != 0) {
                // contact state of the last step, from the state it starts from
                if (last && P.contact && P.cstate)
                    contact_state_pass<FEAT>(M, S, Out<T>{P.cstate + w, N});
            }
            pass2<FEAT>(M, S);
            pass3_next<FEAT>(M, S, io, last ? -1 : s + 1, last ? Out<T>{P.qdd + w, N} : none);
            S.commit();
        }
        S.wait();
        bool finite = true;
        for (int j = 0; j < M.nv; j++) {
            const T qj = S(j), vj = S(M.nv + j);
            finite = finite && pz_finite(qj) && pz_finite(vj);
            P.q[j * N + w] = qj;
            P.v[j * N + w] = vj;
        }
        if (!finite) {
            atomicOr(P.status, 1);
            atomicMin(P.status + 1, (int)(w < 0x7fffffff ? w : 0x7fffffff));
        }
    }
}

// Kinetic energy 0.5 sum_i v_i^T I_i v_i + 0.5 sum_j armature_j qd_j^2
// (crates/phyz-rigid/src/energy.rs:8-11 with crba's armature) or sum q^2,
// reduced over the block and added into *out.
template <class T, int FEAT>
__global__ void __launch_bounds__(256) objective_kernel(const __grid_constant__ RolloutArgs<T> P, int kind,
                                                         T* out) {
    extern __shared__ __align__(16) unsigned char smem[];
    const unsigned char* blob = stage_model(P.model_blob, P.model_bytes, smem);
    ModelView<T> M = make_view<T>(P, blob);
    M.contact = 0;
    const int W = blockDim.x;
    const SmemScr<T> S{reinterpret_cast<T*>(smem + P.model_bytes) + threadIdx.x, W};
    const long long ntiles = (P.nworld + W - 1) / W;
    T acc = T(0);
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long long w = tile * W + threadIdx.x;
        if (w >= P.nworld) continue;
        const long long N = P.nworld;
        for (int j = 0; j < M.nv; j++) {
            S(j) = P.q[j * N + w];
            S(M.nv + j) = P.v[j * N + w];
        }
        if (kind == 1) {
            for (int j = 0; j < M.nv; j++) acc += S(j) * S(j);
            continue;
        }
        pass1_all<FEAT & FEAT_MULTI>(M, S);
        for (int i = 0; i < M.nb; i++) {
            const BodyI bi = M.bi[i];
            const BodyT<T>& bt = M.bt[i];
            const SV<T> v = ld_sv<T>(S, bi.s_vw);
            const V3<T> mc = ld3(bt.mcom);
            const SV<T> h = mksv<T>(symv(bt.Io, v.w) + cross(mc, v.l), v.l * bt.mass + cross(v.w, mc));
            acc += T(0.5) * dot(v, h);
            for (int k = 0; k < bi.ndof; k++) {
                const T qd = S(M.nv + bi.off + k);
                acc += T(0.5) * bt.armature * qd * qd;
            }
        }
    }
    // warp reduction, one atomic per warp (blockDim.x is a multiple of 32)
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, acc);
}

// aos [nrep][nworld][width] (Tin) -> soa [nrep][width][nworld] (Tout), 32x32 tiles.
template <class Tin, class Tout>
__global__ void aos_to_soa_kernel(const Tin* __restrict__ aos, Tout* __restrict__ soa, long long nworld,
                                  int width) {
    __shared__ Tout tile[32][33];
    const long long rep = blockIdx.z;
    const Tin* a = aos + rep * nworld * width;
    Tout* s = soa + rep * nworld * width;
    const long long w0 = (long long)blockIdx.x * 32;
    const int j0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const long long w = w0 + r;
        const int j = j0 + threadIdx.x;
        if (w < nworld && j < width) tile[r][threadIdx.x] = Tout(a[w * width + j]);
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int j = j0 + r;
        const long long w = w0 + threadIdx.x;
        if (w < nworld && j < width) s[(long long)j * nworld + w] = tile[threadIdx.x][r];
    }
}

template <class Tin, class Tout>
__global__ void soa_to_aos_kernel(const Tin* __restrict__ soa, Tout* __restrict__ aos, long long nworld,
                                  int width) {
    __shared__ Tout tile[32][33];
    const long long w0 = (long long)blockIdx.x * 32;
    const int j0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int j = j0 + r;
        const long long w = w0 + threadIdx.x;
        if (w < nworld && j < width) tile[r][threadIdx.x] = Tout(soa[(long long)j * nworld + w]);
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const long long w = w0 + r;
        const int j = j0 + threadIdx.x;
        if (w < nworld && j < width) aos[w * width + j] = tile[threadIdx.x][r];
    }
}

// ── launch helpers ───────────────────────────────────────────────────────

static int g_sm_count = -1, g_smem_optin = -1, g_device = -1;

static cudaError_t device_limits() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != g_device) {
        if ((e = cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return e;
        if ((e = cudaDeviceGetAttribute(&g_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
            cudaSuccess)
            return e;
        g_device = dev;
    }
    return cudaSuccess;
}

template <class T, int FEAT>
static cudaError_t config_variant(int scratch, int model_bytes, long long nworld, LaunchCfg* out) {
    cudaError_t e = cudaFuncSetAttribute(rollout_kernel<T, FEAT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         g_smem_optin);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(objective_kernel<T, FEAT>, cudaFuncAttributeMaxDynamicSharedMemorySize, g_smem_optin);
    if (e != cudaSuccess) return e;
    const long long per_world = (long long)scratch * (long long)sizeof(T);
    // Pick the block width (any even width up to the 256 of __launch_bounds__)
    // that keeps the most worlds resident per SM, discounted by how full the
    // last wave of tiles is. PHYZB_WORLDS_PER_BLOCK overrides it for tuning.
    int forced = 0;
    if (const char* env = getenv("PHYZB_WORLDS_PER_BLOCK")) forced = atoi(env);
    int best_w = 0, best_blocks = 0, best_smem = 0;
    double best_score = -1.0;
    for (int W = 32; W <= 256; W += 2) {
        if (forced > 0 && W != forced) continue;
        const long long smem = (long long)model_bytes + per_world * W;
        if (smem > g_smem_optin) break;
        int blocks = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, rollout_kernel<T, FEAT>, W, (size_t)smem);
        if (e != cudaSuccess) return e;
        if (blocks <= 0) continue;
        const double resident = (double)blocks * W * g_sm_count;  // worlds in flight on the GPU
        const double waves = nworld > 0 ? std::ceil((double)nworld / resident) : 1.0;
        const double used = nworld > 0 ? (double)nworld / (waves * resident) : 1.0;
        const double score = (double)blocks * W * used;
        if (score > best_score * 1.0001) {
            best_score = score;
            best_w = W;
            best_blocks = blocks;
            best_smem = (int)smem;
        }
    }
    if (best_w == 0) return cudaErrorInvalidConfiguration;
    const long long ntiles = (nworld + best_w - 1) / best_w;
    const long long cap = (long long)g_sm_count * best_blocks;
    out->W = best_w;
    out->grid = (int)(ntiles < cap ? (ntiles > 0 ? ntiles : 1) : cap);
    out->smem = best_smem;
    return cudaSuccess;
}

template <class T>
cudaError_t rollout_config(int scratch, int model_bytes, long long nworld, int feat, LaunchCfg* out) {
    cudaError_t e = device_limits();
    if (e != cudaSuccess) return e;
    switch (feat) {
        case 0: return config_variant<T, 0>(scratch, model_bytes, nworld, out);
        case FEAT_MULTI: return config_variant<T, FEAT_MULTI>(scratch, model_bytes, nworld, out);
        case FEAT_CONTACT: return config_variant<T, FEAT_CONTACT>(scratch, model_bytes, nworld, out);
        default: return config_variant<T, FEAT_MULTI | FEAT_CONTACT>(scratch, model_bytes, nworld, out);
    }
}

template <class T>
cudaError_t launch_rollout(const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s) {
    if (a.nsteps <= 0 || a.nworld <= 0) return cudaSuccess;
    switch (a.feat) {
        case 0: rollout_kernel<T, 0><<<cfg.grid, cfg.W, cfg.smem, s>>>(a); break;
        case FEAT_MULTI: rollout_kernel<T, FEAT_MULTI><<<cfg.grid, cfg.W, cfg.smem, s>>>(a); break;
        case FEAT_CONTACT: rollout_kernel<T, FEAT_CONTACT><<<cfg.grid, cfg.W, cfg.smem, s>>>(a); break;
        default: rollout_kernel<T, FEAT_MULTI | FEAT_CONTACT><<<cfg.grid, cfg.W, cfg.smem, s>>>(a); break;
    }
    return cudaGetLastError();
}

template <class T>
cudaError_t launch_objective(const RolloutArgs<T>& a, const LaunchCfg& cfg, int kind, T* out, cudaStream_t s) {
    if (a.nworld <= 0) return cudaSuccess;
    switch (a.feat) {
        case 0: objective_kernel<T, 0><<<cfg.grid, cfg.W, cfg.smem, s>>>(a, kind, out); break;
        case FEAT_MULTI: objective_kernel<T, FEAT_MULTI><<<cfg.grid, cfg.W, cfg.smem, s>>>(a, kind, out); break;
        case FEAT_CONTACT: objective_kernel<T, FEAT_CONTACT><<<cfg.grid, cfg.W, cfg.smem, s>>>(a, kind, out); break;
        default:
            objective_kernel<T, FEAT_MULTI | FEAT_CONTACT><<<cfg.grid, cfg.W, cfg.smem, s>>>(a, kind, out);
            break;
    }
    return cudaGetLastError();
}

template <class Tin, class Tout>
cudaError_t launch_aos_to_soa(const Tin* aos, Tout* soa, long long nworld, int width, int nrep, cudaStream_t s) {
    if (nworld <= 0 || width <= 0 || nrep <= 0) return cudaSuccess;
    dim3 grid((unsigned)((nworld + 31) / 32), (unsigned)((width + 31) / 32), (unsigned)nrep);
    aos_to_soa_kernel<Tin, Tout><<<grid, dim3(32, 8), 0, s>>>(aos, soa, nworld, width);
    return cudaGetLastError();
}

template <class Tin, class Tout>
cudaError_t launch_soa_to_aos(const Tin* soa, Tout* aos, long long nworld, int width, cudaStream_t s) {
    if (nworld <= 0 || width <= 0) return cudaSuccess;
    dim3 grid((unsigned)((nworld + 31) / 32), (unsigned)((width + 31) / 32), 1);
    soa_to_aos_kernel<Tin, Tout><<<grid, dim3(32, 8), 0, s>>>(soa, aos, nworld, width);
    return cudaGetLastError();
}

template cudaError_t rollout_config<float>(int, int, long long, int, LaunchCfg*);
template cudaError_t rollout_config<double>(int, int, long long, int, LaunchCfg*);
template cudaError_t launch_rollout<float>(const RolloutArgs<float>&, const LaunchCfg&, cudaStream_t);
template cudaError_t launch_rollout<double>(const RolloutArgs<double>&, const LaunchCfg&, cudaStream_t);
template cudaError_t launch_objective<float>(const RolloutArgs<float>&, const LaunchCfg&, int, float*,
                                             cudaStream_t);
template cudaError_t launch_objective<double>(const RolloutArgs<double>&, const LaunchCfg&, int, double*,
                                              cudaStream_t);
template cudaError_t launch_aos_to_soa<double, float>(const double*, float*, long long, int, int, cudaStream_t);
template cudaError_t launch_aos_to_soa<double, double>(const double*, double*, long long, int, int, cudaStream_t);
template cudaError_t launch_aos_to_soa<float, float>(const float*, float*, long long, int, int, cudaStream_t);
template cudaError_t launch_aos_to_soa<float, double>(const float*, double*, long long, int, int, cudaStream_t);
template cudaError_t launch_soa_to_aos<float, double>(const float*, double*, long long, int, cudaStream_t);
template cudaError_t launch_soa_to_aos<double, double>(const double*, double*, long long, int, cudaStream_t);

}  // namespace pz
