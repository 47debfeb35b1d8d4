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

struct LaunchCfg {
    int W;         // worlds (threads) per block
    int grid;      // blocks
    int smem;      // dynamic shared memory bytes per block
    int tm;        // 1: body records in Tensor Memory (one block per SM)
    double score;  // worlds resident per SM x fill of the last wave
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
