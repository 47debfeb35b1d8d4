// One (precision, feature set) variant of the rollout and objective kernels.
// The build compiles this file once per pair, with PZ_VARIANT_T (float or
// double) and PZ_VARIANT_FEAT (0 .. FEAT_COUNT-1) defined, so the variants
// compile in parallel.
#include "stepper_kernels.cuh"

#if !defined(PZ_VARIANT_T) || !defined(PZ_VARIANT_FEAT)
#error "compile with -DPZ_VARIANT_T=float|double -DPZ_VARIANT_FEAT=<0..63>"
#endif

namespace pz {

template cudaError_t config_variant<PZ_VARIANT_T, PZ_VARIANT_FEAT, false>(const DeviceLimits&, int, int, long long, int,
                                                                          LaunchCfg*);
template cudaError_t config_variant<PZ_VARIANT_T, PZ_VARIANT_FEAT, true>(const DeviceLimits&, int, int, long long, int,
                                                                         LaunchCfg*);
template void launch_variant<PZ_VARIANT_T, PZ_VARIANT_FEAT, false>(const RolloutArgs<PZ_VARIANT_T>&, const LaunchCfg&,
                                                                   cudaStream_t);
template void launch_variant<PZ_VARIANT_T, PZ_VARIANT_FEAT, true>(const RolloutArgs<PZ_VARIANT_T>&, const LaunchCfg&,
                                                                  cudaStream_t);
template void launch_objective_variant<PZ_VARIANT_T, PZ_VARIANT_FEAT>(const RolloutArgs<PZ_VARIANT_T>&,
                                                                      const LaunchCfg&, int, PZ_VARIANT_T*,
                                                                      cudaStream_t);

}  // namespace pz
