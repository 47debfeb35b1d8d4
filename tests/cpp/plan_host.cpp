// Host harness for tests/test_slice_plan.py: the launch-shape picker
// (pz_variants.h pick_launch, with its slice-mode shape) and the per-launch
// slice planner (pz_launch.h plan_slices), driven without a GPU. The
// occupancy query is modelled on a B200 SM: 65536 registers in 256-register
// warp units, 233472 bytes of shared memory with 1 KB reserved per block,
// 2048 threads, 32 blocks.
#include <algorithm>

#include "pz_variants.h"

// out: [W, grid, blocks, slice_W, slice_grid, chunk, launch W, launch grid];
// returns the cudaError_t of pick_launch.
extern "C" int plan_host(int tm, int esz, int scratch, int model_bytes, long long nworld, int tmem_cols, int regs,
                         int can_slice, int nsteps, int force, int* out) {
    const pz::DeviceLimits dl{148, 232448};
    auto occ = [regs](int* blocks, int W, size_t smem) {
        const int warps = (W + 31) / 32;
        const int regs_warp = ((regs * 32 + 255) / 256) * 256;
        const int by_regs = 65536 / (regs_warp * warps);
        const int by_smem = (int)(233472 / (smem + 1024));
        const int by_threads = 2048 / (warps * 32);
        *blocks = std::min(std::min(by_regs, by_smem), std::min(by_threads, 32));
        return cudaSuccess;
    };
    pz::LaunchCfg c{};
    const cudaError_t e = pz::pick_launch(dl, dl.smem_optin, tm != 0, esz, scratch, model_bytes, nworld, tmem_cols,
                                          (int)pz::TMEM_COLS, occ, &c, 0, 256, can_slice != 0);
    if (e != cudaSuccess) return (int)e;
    pz::LaunchCfg run = c;
    int chunk = pz::plan_slices(c, nworld, nsteps, force, &run);
    if (chunk <= 0) {
        chunk = 0;
        run = c;
    }
    const int v[8] = {c.W, c.grid, c.blocks, c.slice_W, c.slice_grid, chunk, run.W, run.grid};
    for (int k = 0; k < 8; k++) out[k] = v[k];
    return 0;
}
