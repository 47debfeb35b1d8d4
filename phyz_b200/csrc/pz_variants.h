// Per-variant host entry points of the rollout kernel (stepper_kernels.cuh),
// one (precision, feature set) instantiation per translation unit
// (rollout_variants.cu), dispatched at run time by stepper.cu.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>

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
    int smem_optin;         // opt-in shared memory per block (static + dynamic)
    int regs_per_sm = 65536;
    int max_threads = 1024;  // per block
};

// Pick the block width that keeps the most worlds resident per SM,
// discounted by how full the last wave of tiles is. Shared-memory layout:
// any even width up to the 256 of the kernel's launch bounds. Tensor-Memory
// layout: whole warps, one block per SM, and few enough warps per TMEM lane
// quarter that each thread's columns hold its records. `occupancy(&blocks,
// W, smem)` asks the runtime about the kernel being configured; dyn_cap is
// its dynamic shared-memory limit. `only_w` > 0 (a kernel compiled for one
// width), else PHYZB_WORLDS_PER_BLOCK for tuning, fixes the width.
// The TMEM columns each thread of a block of `warps` warps owns (warps
// w, w+4, ... share lane quarter w % 4 and split its columns, whole 8-column
// records each).
inline int tmem_cols_per_thread(int warps, int tmem_total) {
    const int per_quarter = (warps + 3) / 4;
    return (tmem_total / per_quarter) & ~7;
}

template <class Occ>
cudaError_t pick_launch(const DeviceLimits& dl, int dyn_cap, bool tm, int esz, int scratch, int model_bytes,
                        long long nworld, int tmem_cols, int tmem_total, Occ occupancy, LaunchCfg* out,
                        int only_w = 0, int max_w = 256, bool can_slice = false) {
    const long long per_world = (long long)scratch * (long long)esz;
    int forced = only_w;
    if (const char* env = getenv("PHYZB_WORLDS_PER_BLOCK"); env && forced <= 0) forced = atoi(env);
    // shared memory and resident blocks per SM of width W: 1 = fits, 0 = past
    // the layout's limits (wider blocks do not fit either), -1 = skip W,
    // -2 = the occupancy query failed (occ_err)
    cudaError_t occ_err = cudaSuccess;
    auto shape = [&](int W, long long* smem, int* blocks) -> int {
        if (tm && tmem_cols > tmem_cols_per_thread((W + 31) / 32, tmem_total)) return 0;
        *smem = (long long)model_bytes + per_world * W;
        if (*smem > dyn_cap) return 0;
        // Tensor-Memory blocks ask for more than half an SM's shared memory so
        // that no second block lands on the SM and waits on the allocation
        if (tm) *smem = std::max(*smem, (long long)(dl.smem_optin / 2 + 16) & ~15LL);
        *blocks = 0;
        occ_err = occupancy(blocks, W, (size_t)*smem);
        if (occ_err != cudaSuccess) return -2;
        if (*blocks <= 0) return -1;
        if (tm) *blocks = 1;  // each block holds the whole Tensor Memory
        return 1;
    };
    int best_w = 0, best_blocks = 0, best_smem = 0;
    double best_score = -1.0;
    const int step = tm ? 32 : 2;
    for (int W = 32; W <= max_w; W += step) {
        if (forced > 0 && W != forced) continue;
        long long smem = 0;
        int blocks = 0;
        const int r = shape(W, &smem, &blocks);
        if (r == -2) return occ_err;
        if (r == 0) break;
        if (r < 0) continue;
        const double resident = (double)blocks * W * dl.sm_count;  // worlds in flight on the GPU
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
    const long long cap = (long long)dl.sm_count * best_blocks;
    out->W = best_w;
    out->grid = (int)(ntiles < cap ? (ntiles > 0 ? ntiles : 1) : cap);
    out->smem = best_smem;
    out->tm = tm ? 1 : 0;
    out->score = best_score;
    out->blocks = best_blocks;
    // The slice-mode shape: the most resident worlds in whole-warp blocks
    // with no more warps on the busiest SM sub-partition (warps are spread
    // over the SM's four schedulers) than the tile shape has, so a step
    // takes about as long in either mode.
    out->slice_W = out->slice_grid = out->slice_smem = 0;
    if (!can_slice) return cudaSuccess;
    const int per_sub = (best_blocks * ((best_w + 31) / 32) + 3) / 4;
    long long best_res = 0;
    for (int W = 32; W <= max_w; W += 32) {
        if (only_w > 0 && W != only_w) continue;
        long long smem = 0;
        int blocks = 0;
        const int r = shape(W, &smem, &blocks);
        if (r == -2) return occ_err;
        if (r == 0) break;
        if (r < 0) continue;
        if ((blocks * (W / 32) + 3) / 4 > per_sub) continue;
        if ((long long)blocks * W > best_res) {
            best_res = (long long)blocks * W;
            out->slice_W = W;
            out->slice_grid = dl.sm_count * blocks;
            out->slice_smem = (int)smem;
        }
    }
    return cudaSuccess;
}

template <class T, int FEAT, bool TM>
cudaError_t config_variant(const DeviceLimits& dl, int scratch, int model_bytes, long long nworld, int tmem_cols,
                           LaunchCfg* out);
// lanes kernel (stepper_lanes.cuh): feature sets of the ball / free, contact
// and relabel bits only
constexpr int LANES_FEAT_COUNT = 16;
template <class T, int FEAT>
cudaError_t config_lanes_variant(const DeviceLimits& dl, int lanes, int scratch, int model_bytes, long long nworld,
                                 LaunchCfg* out);
template <class T, int FEAT>
void launch_lanes_variant(const RolloutArgs<T>& a, const LanesArgs& la, const LaunchCfg& cfg, cudaStream_t s);
template <class T, int FEAT, bool TM>
void launch_variant(const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s);
template <class T, int FEAT>
void launch_objective_variant(const RolloutArgs<T>& a, const LaunchCfg& cfg, int kind, T* out, cudaStream_t s);

}  // namespace pz
