// Host-side launch interface of the stepper's kernels (stepper.cu), used by
// the C ABI (capi.cu). No kernel here has a host implementation.
#pragma once

#ifndef __CUDACC_RTC__
#include <cuda_runtime.h>

#include <string>
#include <vector>
#endif

namespace pz {

// TMEM columns allocated per block by the Tensor-Memory variant: the whole
// array (one block per SM).
constexpr unsigned TMEM_COLS = 512;

// Whether a generic rollout variant has slice mode compiled in (each mode is
// a copy of the step's code): the Tensor-Memory variants (one block per SM,
// whole warps: the layouts whose few resident worlds leave the widest
// partial waves) without impulse contact (feature bit 16) or terrain (32).
// A model-specialized kernel compiles a slice-mode twin of itself instead
// (spec_sliced), at its own whole-warp width.
template <int FEAT, bool TM>
struct SliceVariant {
    static constexpr bool value = TM && (FEAT & (16 | 32)) == 0;
};

struct LaunchCfg {
    int W;         // worlds (threads) per block
    int grid;      // blocks
    int smem;      // dynamic shared memory bytes per block
    int tm;        // 1: body records in Tensor Memory (one block per SM)
    double score;  // worlds resident per SM x fill of the last wave
    int blocks;    // blocks resident per SM at this shape
    // Slice mode (every warp takes (32 worlds, a run of steps) jobs from a
    // queue, plan_slices): the widest whole-warp block that puts no more warps
    // on an SM sub-partition than the tile shape above does; slice_W 0: none.
    int slice_W, slice_grid, slice_smem;
};

// One fused rollout launch: `nsteps` steps of every world.
template <class T>
struct RolloutArgs {
    const void* model_blob;  // BodyT[nb] | BodyI[nb] | PdT[npd] | int pd_of_dof[nv]
    int model_bytes;         // multiple of 16
    int off_bi, off_pd, off_pdmap;
    int nb, nv, npd, contact;
    int feat;              // kernel variant: Features bits (pz_world.cuh)
    double dt, gx, gy, gz, ground_h, friction;
    T* q;                  // [nv][nworld]
    T* v;                  // [nv][nworld]
    const T* ctrl;         // [nv][nworld] held, or schedule [nsteps][nv][nworld]
    long long ctrl_stride; // elements between steps of the schedule (0: held)
    const T* targets;      // [npd][nworld] or null
    T* qdd;                // [nv][nworld], last step
    T* cstate;             // [nb*8][nworld] contact state of the last step, or null
    int* status;           // [0]: bit 0 = a world went non-finite; [1]: first such world
    long long nworld;
    int nsteps;
    int scratch;           // scratch slots per world
    // impulse-mode contact (feat bit 16)
    T* imp;                // [imp_slots][nworld]: per collidable body its wrench (6) and staged
                           // impulses (3 per point), carried between steps and launches
    int imp_slots;
    int sweeps;            // [contact, backward sweep] pairs per step
    double erp, margin, restitution, rest_thr;
    double si_dmin, si_dmax, si_width, si_mid, si_power;
    // heightfield terrain (feat bit 32): f32 nodes [ny][nx] on the device
    const float* hf;
    int hf_nx, hf_ny;
    double hf_ox, hf_oy, hf_oz, hf_cell;
    // body-attached contact plane (contact variants; plane_body -1: none)
    int plane_body;
    double plane_offset, plane_max_depth, plane_half_x, plane_half_y;
    // slice mode: chunk > 0 splits every world's steps into runs of `chunk`
    // steps; a warp takes (warp tile of 32 worlds, run) jobs in run-major
    // order from the queue in `slices` ([0]: job counter, [1] unused, [2 + t]:
    // runs finished of warp tile t; zeroed before the launch) and starts a
    // run once the tile's previous one is finished (a bounded wait). 0: each
    // block takes its tiles of W worlds for all steps.
    int chunk = 0;
    int* slices = nullptr;
};

// The world split over lanes (stepper_lanes.cuh, planned by pz_lanes.h):
// the staged blob holds `lanes` sub-model tables of lane_bytes each, then
// the DOF maps.
constexpr int LANES_MAX = 8;
struct LanesArgs {
    int lanes;                  // threads per world (2, 4, 8)
    int nt;                     // trunk bodies: the first nt of every sub-model
    int trunk_nv;               // DOFs of the trunk: the first trunk_nv of every sub-model
    int lane_bytes;             // bytes of one lane's table in the staged blob
    int off_gdof;               // blob offset of the DOF maps [lanes][nv_max]
    int nv_max;
    int nb[LANES_MAX], nv[LANES_MAX];
    int off_bi[LANES_MAX], off_pd[LANES_MAX], off_pdmap[LANES_MAX];
};

#ifndef __CUDACC_RTC__
// Whether a rollout of `nsteps` steps over `nworld` worlds runs faster in
// slice mode, and with which run length. A tile launch takes ceil(tiles /
// grid) waves of the whole horizon, so a world count just past a multiple
// of the resident worlds leaves most of the GPU idle in its last wave
// (C2: 65536 worlds on 148 x 224 = 1.98 waves run as 2; at 256 worlds per
// SM, 1.73). Slices let the warps that finish early take the remaining
// worlds' runs, so the rollout takes about (warp tiles x steps) / warp
// slots step-times plus one run of tail. Each run costs about one step more
// (the state's load and store and the first step's forward sweep), counted
// here. Returns the run length (0: tile mode) and the slice launch shape in
// *out. force: -1 decide, 0 tile mode, 1 slices whenever the launch has two
// or more steps (runs of a third of them; PHYZB_SLICES=1, which the tests
// use to cover the mode at small sizes).
inline int plan_slices(const LaunchCfg& c, long long nworld, int nsteps, int force, LaunchCfg* out) {
    if (c.slice_W < 32 || c.slice_grid <= 0 || nsteps < 2 || nworld <= 0 || force == 0) return 0;
    const long long ntw = (nworld + 31) / 32;
    const int wpb = c.slice_W / 32;
    const long long need = (ntw + wpb - 1) / wpb;
    const long long grid = need < c.slice_grid ? need : c.slice_grid;
    const long long slots = grid * wpb;
    *out = c;
    out->W = c.slice_W;
    out->grid = (int)grid;
    out->smem = c.slice_smem;
    // the job counter is 32-bit: every warp's last fetch passes the job count
    auto fits = [&](long long runs) { return ntw * runs + slots < (1LL << 31); };
    if (force == 1) {
        const int chunk = nsteps >= 3 ? (nsteps / 3 < 512 ? nsteps / 3 : 512) : 1;
        return fits((nsteps + chunk - 1) / chunk) ? chunk : 0;
    }
    const long long tiles = (nworld + c.W - 1) / c.W;
    const double t_tile = (double)((tiles + c.grid - 1) / c.grid) * nsteps;
    double best = 0.97 * t_tile;
    int pick = 0;
    // every split into 2 or more runs of 8 to 512 steps: long enough that a
    // run's extra step is small, short enough that a wait for the run before
    // stays far below its bound
    for (int split = 2; split <= nsteps; split++) {
        const int chunk = (nsteps + split - 1) / split;
        if (chunk < 8) break;
        if (chunk > 512) continue;
        const long long runs = (nsteps + chunk - 1) / chunk;
        if (!fits(runs)) continue;
        const double t = (double)((ntw * runs + slots - 1) / slots) * (chunk + 1);
        if (t < best) {
            best = t;
            pick = chunk;
        }
    }
    return pick;
}

template <class T>
cudaError_t lanes_config(int feat, int lanes, int scratch, int model_bytes, long long nworld, LaunchCfg* out);
template <class T>
cudaError_t launch_lanes(const RolloutArgs<T>& a, const LanesArgs& la, const LaunchCfg& cfg, cudaStream_t s);
// tmem_cols > 0: configure the Tensor-Memory variant for a layout whose
// body records need tmem_cols columns per world.
template <class T>
cudaError_t rollout_config(int scratch, int model_bytes, long long nworld, int feat, int tmem_cols, LaunchCfg* out);
template <class T>
cudaError_t launch_rollout(const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s);

// Per-world kinetic energy (kind 0) or sum of q^2 (kind 1), summed over
// worlds into *out (accumulated; caller zeroes it).
template <class T>
cudaError_t launch_objective(const RolloutArgs<T>& a, const LaunchCfg& cfg, int kind, T* out,
                             cudaStream_t s);

// Layout conversions between host-style world-major rows and the device SoA.
// aos: [nworld][width] of Tin; soa: [width][nworld] of Tout.
template <class Tin, class Tout>
cudaError_t launch_aos_to_soa(const Tin* aos, Tout* soa, long long nworld, int width, int nrep,
                              cudaStream_t s);
template <class Tin, class Tout>
cudaError_t launch_soa_to_aos(const Tin* soa, Tout* aos, long long nworld, int width, cudaStream_t s);
// Model-specialized rollout kernels (spec.cu): the rollout kernel compiled
// at run time for one packed model, its tables literal (pz_spec.h). One
// compile per (model table, precision, feature set, layout, device) per
// process; compiled kernels are also kept on disk (PHYZB_KERNEL_CACHE,
// default $HOME/.cache/phyzb; "0" turns the disk cache off).
struct SpecKernel;
// One packed table the specialized kernel may run with.
struct SpecLayout {
    const unsigned char* blob;  // host copy of the table
    int bytes, off_bi, off_pd, off_pdmap;
    int scratch, feat, tmem_cols;
    bool tm;                    // body records in Tensor Memory
    int w0;                     // a block width the generic variant launches it with
};
// A compiled candidate: layout index, kernel, launch shape.
struct SpecChoice {
    int layout;
    const SpecKernel* k;
    LaunchCfg cfg;
};
// Compile (or fetch) the candidate kernels of each layout: at the generic
// variant's width, and at a second width -- a Tensor-Memory table as wide
// as the compiled kernel's registers and the table's on-chip memory allow
// (past the generic variants' 256 threads), a shared-memory table at whole
// warps. a supplies the model's sizes and the world count. On failure *err
// says why.
template <class T>
cudaError_t spec_candidates(const SpecLayout* lays, int nlay, const RolloutArgs<T>& a,
                            std::vector<SpecChoice>* out, std::string* err);
// The slice-mode twin of the specialized kernel of layout L at width W
// (compiled, or fetched from the caches, on a simulator's first slice-mode
// launch; its launch shape is the tile kernel's slice_W / slice_grid /
// slice_smem).
template <class T>
cudaError_t spec_sliced(const SpecLayout& L, const RolloutArgs<T>& a, int W, const SpecKernel** out,
                        std::string* err);
template <class T>
cudaError_t spec_launch(const SpecKernel* k, const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s);
// A simulator takes (retain) and gives back (release) the compiled kernel it
// runs; modules no simulator holds are unloaded, least recently used first,
// once more than kSpecModuleCap (or $PHYZB_SPEC_MODULE_CAP) are loaded (the
// on-disk cache keeps them).
constexpr int kSpecModuleCap = 32;
void spec_retain(const SpecKernel* k);
void spec_release(const SpecKernel* k);
#endif  // __CUDACC_RTC__

}  // namespace pz
