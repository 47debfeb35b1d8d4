// Per-thread dense layers for the control loop and the PPO update: one row
// (world or sample) per thread, weights staged in shared memory as
// [in_pad][out_pad] (zero-padded to POLICY_TILE multiples: exact). A row's
// vectors are read through `xin(i)` and each output goes to `epi(j, acc)`:
// callers keep them in HBM as SoA (consecutive threads, consecutive
// addresses: coalesced, mostly L1/L2 hits), so shared memory holds only the
// weights and many warps fit an SM. Each tile of 32 outputs accumulates in
// registers in the reference's order (bias, then inputs in index order),
// reading its weights as broadcast float4 loads.
#pragma once

#include "pz_policy.h"

namespace pz {

template <class Load, class Epi>
__device__ __forceinline__ void dense_tiles(const float* Wt, const float* bias, int in_pad, int out_pad, Load xin,
                                            Epi epi) {
    for (int jc = 0; jc < out_pad; jc += POLICY_TILE) {
        float acc[POLICY_TILE];
#pragma unroll
        for (int j = 0; j < POLICY_TILE; j++) acc[j] = bias ? bias[jc + j] : 0.0f;
        // (unrolled so that several inputs are loaded ahead of their FMAs)
#pragma unroll 4
        for (int i = 0; i < in_pad; i++) {
            const float xi = xin(i);
            const float4* wr = reinterpret_cast<const float4*>(Wt + i * out_pad + jc);
#pragma unroll
            for (int j4 = 0; j4 < POLICY_TILE / 4; j4++) {
                const float4 wv = wr[j4];
                acc[4 * j4 + 0] = fmaf(wv.x, xi, acc[4 * j4 + 0]);
                acc[4 * j4 + 1] = fmaf(wv.y, xi, acc[4 * j4 + 1]);
                acc[4 * j4 + 2] = fmaf(wv.z, xi, acc[4 * j4 + 2]);
                acc[4 * j4 + 3] = fmaf(wv.w, xi, acc[4 * j4 + 3]);
            }
        }
#pragma unroll
        for (int j = 0; j < POLICY_TILE; j++) epi(jc + j, acc[j]);
    }
}

// Copy `n` floats (a multiple of 4) of weights into shared memory.
__device__ __forceinline__ void stage_weights(const float* g, int n, float* sm) {
    for (int k = threadIdx.x; k < n / 4; k += blockDim.x)
        reinterpret_cast<float4*>(sm)[k] = __ldg(reinterpret_cast<const float4*>(g) + k);
    __syncthreads();
}

}  // namespace pz
