// Per-thread dense layers for the control loop and the PPO update: one row
// (world or sample) per thread, weights staged in shared memory as
// [in_pad][out_pad] (zero-padded to POLICY_TILE multiples: exact), the row's
// vectors in shared memory as SoA (slot i of this thread at x[i * W]).
// Each tile of 32 outputs accumulates in registers in the reference's order
// (bias, then inputs in index order), reading its weights as broadcast
// float4 loads.
#pragma once

#include "pz_policy.h"

namespace pz {

// y[j] = act(bias[j] + sum_i Wt[i][j] x[i]), j in [0, out_pad). bias may be
// null (zero). ACT: 0 none, 1 tanh.
template <int ACT>
__device__ __forceinline__ void dense_rows(const float* Wt, const float* bias, int in_pad, int out_pad,
                                           const float* x, float* y, int W) {
    for (int jc = 0; jc < out_pad; jc += POLICY_TILE) {
        float acc[POLICY_TILE];
#pragma unroll
        for (int j = 0; j < POLICY_TILE; j++) acc[j] = bias ? bias[jc + j] : 0.0f;
        for (int i = 0; i < in_pad; i++) {
            const float xi = x[i * W];
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
        for (int j = 0; j < POLICY_TILE; j++) y[(jc + j) * W] = ACT == 1 ? tanhf(acc[j]) : acc[j];
    }
}

}  // namespace pz
