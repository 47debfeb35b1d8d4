// Per-variant host entry points of the rollout kernel (stepper_kernels.cuh),
// one (precision, feature set) instantiation per translation unit
// (rollout_variants.cu), dispatched at run time by stepper.cu.
#pragma once

#include <cuda_runtime.h>

#include "pz_launch.h"

namespace pz {

// Feature bits of a kernel variant (pz_world.cuh Features): 0 .. FEAT_COUNT-1;
// the uniform-shift bit (8) only occurs with the relabel bit (4), the
// impulse (16) and heightfield (32) bits only with the contact bit (2).
constexpr int FEAT_COUNT = 64;
constexpr bool feat_valid(int f) {
    return !((f & 8) && !(f & 4)) && !((f & 16) && !(f & 2)) && !((f & 32) && !(f & 2));
}

struct DeviceLimits {
    int sm_count;
    int smem_optin;  // opt-in shared memory per block (static + dynamic)
};

template <class T, int FEAT, bool TM>
cudaError_t config_variant(const DeviceLimits& dl, int scratch, int model_bytes, long long nworld, int tmem_cols,
                           LaunchCfg* out);
template <class T, int FEAT, bool TM>
void launch_variant(const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s);
template <class T, int FEAT>
void launch_objective_variant(const RolloutArgs<T>& a, const LaunchCfg& cfg, int kind, T* out, cudaStream_t s);

}  // namespace pz
