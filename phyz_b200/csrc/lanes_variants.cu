// One (precision, feature set) variant of the lanes kernel
// (stepper_lanes.cuh). The build compiles this file once per pair, with
// PZ_VARIANT_T (float or double) and PZ_VARIANT_FEAT (a subset of the ball /
// free, contact and relabel bits: 0 .. LANES_FEAT_COUNT-1) defined.
#include "stepper_lanes.cuh"

#if !defined(PZ_VARIANT_T) || !defined(PZ_VARIANT_FEAT)
#error "compile with -DPZ_VARIANT_T=float|double -DPZ_VARIANT_FEAT=<0..15>"
#endif

namespace pz {

template cudaError_t config_lanes_variant<PZ_VARIANT_T, PZ_VARIANT_FEAT>(const DeviceLimits&, int, int, int, long long,
                                                                         LaunchCfg*);
template void launch_lanes_variant<PZ_VARIANT_T, PZ_VARIANT_FEAT>(const RolloutArgs<PZ_VARIANT_T>&, const LanesArgs&,
                                                                  const LaunchCfg&, cudaStream_t);

}  // namespace pz
