// phyzb_gae_noalloc: generalized advantage estimation over caller-owned
// device buffers, with the reduction scratch in a fixed static device array
// instead of memory the library allocates.
//
// Who needs this: a caller whose host framework owns the whole device (a
// caching allocator that has reserved the GPU's memory, a process held to a
// fixed memory budget) or a latency-bound training loop, where a cudaMalloc
// inside the call can fail for lack of memory or stall the loop and a
// cudaFree synchronizes the device. phyzb_policy_advantages grows its scratch
// with cudaFree/cudaMalloc when a larger rollout arrives; this entry point
// takes the rewards and critic values from the caller and keeps the only
// scratch it needs -- the per-block partial sums of the GAE kernel -- in the
// array below.
//
// The array: PHYZB_GAE_NOALLOC_MAX_WORLDS worlds' worth of partial sums
// (3 doubles per 256 worlds, plus 4 doubles of totals: 1.5 MiB). Every device
// on which this library's kernels are loaded holds it until the process exits.
// All calls on one device share it: two calls whose kernels overlap on that
// device race on it, so order them (one stream, or events). Nothing in it has
// to start at zero: every word a call reads there was written earlier in the
// same call, by the GAE kernel (partials of each launched block) and then by
// the block-sum kernel (the totals).
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <string>

#include "capi_internal.h"
#include "pz_train.h"

using namespace pzc;

namespace {

constexpr long long MAX_WORLDS = PHYZB_GAE_NOALLOC_MAX_WORLDS;
constexpr int MAX_BLOCKS = (int)((MAX_WORLDS + 255) / 256);  // pz::gae_blocks(MAX_WORLDS)
constexpr int MAX_DEVICES = 64;

// [0, 4): totals (sum adv, sum adv^2, sum r, unused); [4, 4 + 3 * blocks): partials
static __device__ __align__(256) double g_gae_scratch[4 + 3 * MAX_BLOCKS];

std::mutex g_mu;
double* g_addr[MAX_DEVICES] = {};

// The device address of g_gae_scratch on `device` (current). The host-side
// name of a __device__ array is only a stand-in for it, so host code looks the
// address up once per device and hands that to the kernels. The cached
// address lives as long as the device's primary context: a cudaDeviceReset
// unloads this module's copy of the array, after which the entry point must
// not be called on that device (the header says so).
int scratch_on(int device, double** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_gae_scratch);
        if (e != cudaSuccess)
            return fail(PHYZB_ERR_CUDA, std::string("cudaGetSymbolAddress(g_gae_scratch): ") + cudaGetErrorString(e));
        g_addr[device] = (double*)p;
    }
    *out = g_addr[device];
    return PHYZB_OK;
}

}  // namespace

extern "C" {

int phyzb_gae_noalloc(const float* rewards, const float* values, int64_t nworld, int32_t steps, double gamma,
                      double lambda, int32_t normalize, int32_t device, void* stream, float* adv, float* ret,
                      double* stats) {
    // arguments first: nothing below touches the device until they pass
    if (!rewards || !values || !adv || !ret) return fail(PHYZB_ERR_INVALID, "null device buffer");
    if (nworld < 1) return fail(PHYZB_ERR_INVALID, "nworld must be >= 1");
    if (steps < 1) return fail(PHYZB_ERR_INVALID, "steps must be >= 1");
    if (nworld > MAX_WORLDS)
        return fail(PHYZB_ERR_TOO_LARGE, "nworld " + std::to_string(nworld) + " exceeds the static scratch limit of " +
                                             std::to_string(MAX_WORLDS) + " worlds per call");
    if (!std::isfinite(gamma) || !std::isfinite(lambda)) return fail(PHYZB_ERR_INVALID, "gamma/lambda not finite");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < 1) return fail(PHYZB_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev || device >= MAX_DEVICES)
        return fail(PHYZB_ERR_INVALID, "device " + std::to_string(device) + " out of range");
    DeviceGuard g(device);
    double* scr = nullptr;
    PZ_TRY(scratch_on(device, &scr));
    double* sums = scr;
    double* part = scr + 4;
    cudaStream_t s = (cudaStream_t)stream;
    PZ_CUDA(pz::rollout_gae(rewards, values, nworld, steps, (float)gamma, (float)lambda, adv, ret, part, sums, s));
    const double count = (double)steps * (double)nworld;
    if (normalize) PZ_CUDA(pz::normalize_advantages(adv, (long long)steps * nworld, sums, count, s));
    if (stats) {
        double hs[3] = {0, 0, 0};
        PZ_CUDA(cudaMemcpyAsync(hs, sums, sizeof(hs), cudaMemcpyDeviceToHost, s));
        PZ_TRY(bounded_sync(s));
        const double mean = hs[0] / count;
        stats[0] = hs[2] / (double)nworld;
        stats[1] = mean;
        stats[2] = std::sqrt(std::max(hs[1] / count - mean * mean, 0.0));
    }
    return PHYZB_OK;
}

}  // extern "C"
