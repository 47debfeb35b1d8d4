// Host dispatch of the stepper's kernels and the layout-conversion kernels.
//
// The rollout and objective kernels (stepper_kernels.cuh) are compiled per
// (precision, feature set) in rollout_variants.cu; this file picks the
// variant of a model at run time and owns the device limits the launch
// configuration is sized by.
#include <cuda_runtime.h>

#include "pz_variants.h"

namespace pz {

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

static int g_device = -1;
static DeviceLimits g_limits{0, 0};

static cudaError_t device_limits() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != g_device) {
        if ((e = cudaDeviceGetAttribute(&g_limits.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return e;
        if ((e = cudaDeviceGetAttribute(&g_limits.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
            cudaSuccess)
            return e;
        g_device = dev;
    }
    return cudaSuccess;
}

// run-time feature set -> compiled variant
template <class T, bool TM, int F = 0>
static cudaError_t config_by_feat(int feat, int scratch, int model_bytes, long long nworld, int tmem_cols,
                                  LaunchCfg* out) {
    if constexpr (F < FEAT_COUNT) {
        if constexpr (feat_valid(F))
            if (feat == F) return config_variant<T, F, TM>(g_limits, scratch, model_bytes, nworld, tmem_cols, out);
        return config_by_feat<T, TM, F + 1>(feat, scratch, model_bytes, nworld, tmem_cols, out);
    } else {
        return cudaErrorInvalidValue;
    }
}
template <class T, bool TM, int F = 0>
static cudaError_t launch_by_feat(const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s) {
    if constexpr (F < FEAT_COUNT) {
        if constexpr (feat_valid(F))
            if (a.feat == F) {
                launch_variant<T, F, TM>(a, cfg, s);
                return cudaSuccess;
            }
        return launch_by_feat<T, TM, F + 1>(a, cfg, s);
    } else {
        return cudaErrorInvalidValue;
    }
}
template <class T, int F = 0>
static cudaError_t objective_by_feat(const RolloutArgs<T>& a, const LaunchCfg& cfg, int kind, T* out,
                                     cudaStream_t s) {
    if constexpr (F < FEAT_COUNT) {
        if constexpr (feat_valid(F))
            if (a.feat == F) {
                launch_objective_variant<T, F>(a, cfg, kind, out, s);
                return cudaSuccess;
            }
        return objective_by_feat<T, F + 1>(a, cfg, kind, out, s);
    } else {
        return cudaErrorInvalidValue;
    }
}

template <class T, int F = 0>
static cudaError_t lanes_config_by_feat(int feat, int lanes, int scratch, int model_bytes, long long nworld,
                                        LaunchCfg* out) {
    if constexpr (F < LANES_FEAT_COUNT) {
        if constexpr (feat_valid(F))
            if (feat == F) return config_lanes_variant<T, F>(g_limits, lanes, scratch, model_bytes, nworld, out);
        return lanes_config_by_feat<T, F + 1>(feat, lanes, scratch, model_bytes, nworld, out);
    } else {
        return cudaErrorInvalidValue;
    }
}
template <class T, int F = 0>
static cudaError_t launch_lanes_by_feat(const RolloutArgs<T>& a, const LanesArgs& la, const LaunchCfg& cfg,
                                        cudaStream_t s) {
    if constexpr (F < LANES_FEAT_COUNT) {
        if constexpr (feat_valid(F))
            if (a.feat == F) {
                launch_lanes_variant<T, F>(a, la, cfg, s);
                return cudaSuccess;
            }
        return launch_lanes_by_feat<T, F + 1>(a, la, cfg, s);
    } else {
        return cudaErrorInvalidValue;
    }
}

template <class T>
cudaError_t lanes_config(int feat, int lanes, int scratch, int model_bytes, long long nworld, LaunchCfg* out) {
    cudaError_t e = device_limits();
    if (e != cudaSuccess) return e;
    return lanes_config_by_feat<T>(feat, lanes, scratch, model_bytes, nworld, out);
}

template <class T>
cudaError_t launch_lanes(const RolloutArgs<T>& a, const LanesArgs& la, const LaunchCfg& cfg, cudaStream_t s) {
    if (a.nsteps <= 0 || a.nworld <= 0) return cudaSuccess;
    cudaError_t e = launch_lanes_by_feat<T>(a, la, cfg, s);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <class T>
cudaError_t rollout_config(int scratch, int model_bytes, long long nworld, int feat, int tmem_cols, LaunchCfg* out) {
    cudaError_t e = device_limits();
    if (e != cudaSuccess) return e;
    if (tmem_cols > 0) return config_by_feat<T, true>(feat, scratch, model_bytes, nworld, tmem_cols, out);
    return config_by_feat<T, false>(feat, scratch, model_bytes, nworld, 0, out);
}

template <class T>
cudaError_t launch_rollout(const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s) {
    if (a.nsteps <= 0 || a.nworld <= 0) return cudaSuccess;
    cudaError_t e = cfg.tm ? launch_by_feat<T, true>(a, cfg, s) : launch_by_feat<T, false>(a, cfg, s);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <class T>
cudaError_t launch_objective(const RolloutArgs<T>& a, const LaunchCfg& cfg, int kind, T* out, cudaStream_t s) {
    if (a.nworld <= 0) return cudaSuccess;
    cudaError_t e = objective_by_feat<T>(a, cfg, kind, out, s);
    if (e != cudaSuccess) return e;
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

template cudaError_t lanes_config<float>(int, int, int, int, long long, LaunchCfg*);
template cudaError_t lanes_config<double>(int, int, int, int, long long, LaunchCfg*);
template cudaError_t launch_lanes<float>(const RolloutArgs<float>&, const LanesArgs&, const LaunchCfg&, cudaStream_t);
template cudaError_t launch_lanes<double>(const RolloutArgs<double>&, const LanesArgs&, const LaunchCfg&,
                                          cudaStream_t);
template cudaError_t rollout_config<float>(int, int, long long, int, int, LaunchCfg*);
template cudaError_t rollout_config<double>(int, int, long long, int, int, LaunchCfg*);
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
template cudaError_t launch_soa_to_aos<float, float>(const float*, float*, long long, int, cudaStream_t);

}  // namespace pz
