// Internals shared by the C ABI's translation units (capi.cu, capi_policy.cu):
// the simulator handle, error reporting and the host-row transfer helpers.
// Not part of the public interface (include/phyzb.h).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/phyzb.h"
#include "pz_launch.h"
#include "pz_pack.h"

namespace pzc {

// Record `msg` as the calling thread's last error and return `code`.
int fail(int code, const std::string& msg);
const char* last_error();

#define PZ_CUDA(expr)                                                                           \
    do {                                                                                        \
        cudaError_t e_ = (expr);                                                                \
        if (e_ != cudaSuccess)                                                                  \
            return fail(PHYZB_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_));    \
    } while (0)

#define PZ_TRY(expr)                \
    do {                            \
        int r_ = (expr);            \
        if (r_ != PHYZB_OK) return r_; \
    } while (0)

// Wait for everything enqueued on `stream`, at most $PHYZB_SYNC_TIMEOUT seconds
// (default 600): the kernels hold no spin, so a longer wait means a lost
// device, reported as PHYZB_ERR_CUDA instead of blocking the caller forever.
int bounded_sync(cudaStream_t stream);

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace pzc

// The on-device control loop's buffers (capi_policy.cu).
struct PolicyDev {
    // spec
    int n_in = 0, n_h = 0, n_out = 0, history = 0;
    int in_pad = 0, h_pad = 0, out_pad = 0, n_wf = 0;
    float rho = 0.0f;
    // device buffers
    void* fk = nullptr;     // FkBody<T>[nb]
    float* d_ops = nullptr;
    float* d_aux = nullptr;
    float* d_com = nullptr;  // [nb][4]
    float* d_w = nullptr;    // packed weights
    float* d_std = nullptr;
    float* d_noise = nullptr;
    int* d_slots = nullptr;
    float* d_clamp = nullptr;
    unsigned long long* d_rng = nullptr;
    float* d_z = nullptr;      // [n_out][nworld]
    void* d_base = nullptr;    // T [npd][nworld]
    void* d_xf = nullptr;      // T [nb * 18][nworld]
    float* d_h = nullptr;      // [2][h_pad][nworld] hidden-layer scratch
    float* d_obs = nullptr;    // [history][n_in][nworld]
    float* d_out = nullptr;    // [history][n_out + 1][nworld]
    void* d_rows = nullptr;    // readback transpose buffer
    size_t rows_bytes = 0;
    void* d_ret_scratch = nullptr;  // phyzb_policy_advantages: sums, rewards, values, coefficients
    size_t ret_bytes = 0;
    bool has_weights = false, has_std = false;
};

struct phyzb_comm;  // NCCL communicator (capi.cu)

struct phyzb_sim {
    int device = 0, precision = PHYZB_F64;
    long long nworld = 0;
    int nb = 0, nv = 0;
    int depth = 0;  // bodies on the model's longest root-to-leaf path
    std::vector<phyzb_body> bodies;
    phyzb_model model{};  // points into `bodies`
    pz::PackCfg cfg;
    double ground_h = 0.0, friction = 0.0;
    int collidable = 0;

    cudaStream_t own_stream = nullptr, stream = nullptr, copy_stream = nullptr;
    void *q = nullptr, *v = nullptr, *ctrl = nullptr, *qdd = nullptr;
    void *targets = nullptr, *cstate = nullptr;
    void* imp = nullptr;      // impulse mode: [imp_slots][nworld] wrenches + staged impulses
    size_t imp_bytes = 0;
    int sweeps = 16;          // impulse mode: contact sweeps per step (DEFAULT_CONTACT_SWEEPS)
    double erp = 0.0;         // impulse mode: solref error reduction at this dt
    void* hf = nullptr;       // heightfield nodes (f32), capacity hf_cap nodes
    size_t hf_cap = 0;
    int hf_nx = 0, hf_ny = 0;
    double hf_o[3] = {0, 0, 0}, hf_cell = 1.0;
    double plane[4] = {0, 0, 0, 0};  // offset, max_depth, half_x, half_y (cfg.plane_body >= 0)
    int* status = nullptr;
    // slice-mode job queue: job counter, a spare word, runs finished per warp tile
    // (pz::RolloutArgs::slices); slice_force: PHYZB_SLICES at creation
    // (-1 decide per launch, 0 never, 1 whenever a launch has two steps)
    int* slices = nullptr;
    int slice_force = -1;
    // PHYZB_SLICES_STALL=1 at creation (a test of the bounded wait): every
    // slice-mode launch starts its queue past the first run of every warp
    // tile, so each later run's wait runs out and the status reports it
    bool slice_stall = false;
    unsigned slice_stall_start = 0;
    size_t slices_bytes() const { return 8 + 4 * (size_t)((nworld + 31) / 32); }
    // lay[0]: every record in shared memory (the objective kernel's layout
    // and the fallback); lay[1]: hinge records in Tensor Memory. `use` is the
    // layout the rollout kernel runs with.
    struct Layout {
        pz::PackInfo info;
        void* blob = nullptr;
        size_t cap = 0;
        pz::LaunchCfg launch{};
        std::vector<unsigned char> host;  // the table as uploaded
    } lay[2];
    int use = 0;
    // the model-specialized kernel (null: not compiled since the last repack),
    // its table layout and launch
    const pz::SpecKernel* spec = nullptr;
    const pz::SpecKernel* spec_sliced = nullptr;  // its slice-mode twin (compiled on first use)
    Layout spec_lay;
    // PHYZB_SPECIALIZE_*: whether rollouts run the model-specialized kernel
    // (compiled at the first launch after each repack) or the generic variants
    int specialize = 0;
    // one world over several threads (pz_lanes.h): requested lanes (0: off),
    // and the packed sub-model tables (rebuilt at the first launch after a
    // repack); lanes_ok false with lanes_why when the model or its settings
    // keep one thread per world
    int lanes = 0;
    bool lanes_built = false, lanes_ok = false;
    std::string lanes_why;
    void* lanes_blob = nullptr;
    size_t lanes_cap = 0;
    int lanes_bytes = 0, lanes_scratch = 0, lanes_feat = 0;
    pz::LanesArgs la{};
    pz::LaunchCfg lanes_launch{};
    void* staging = nullptr;  // device, AoS f64 rows for host copies
    void* hist_q = nullptr;   // state history [slot][nv][nworld] (enable_state_history)
    void* hist_v = nullptr;
    int hist_slots = 0;
    size_t staging_bytes = 0;
    // bulk per-step control pipeline (phyzb_step_with_controls)
    void* pipe_raw[2] = {nullptr, nullptr};
    void* pipe_soa[2] = {nullptr, nullptr};
    size_t pipe_raw_bytes = 0, pipe_soa_bytes = 0;
    cudaEvent_t ev_copied[2] = {nullptr, nullptr}, ev_converted[2] = {nullptr, nullptr};
    PolicyDev* policy = nullptr;  // phyzb_enable_policy
    void* obj = nullptr;       // device scalar of phyzb_reduce_objective
    void* obj_host = nullptr;  // pinned: the read-back never blocks the host
    cudaEvent_t ev_obj = nullptr;

    size_t esz() const { return precision == PHYZB_F64 ? 8 : 4; }
    size_t state_bytes() const { return (size_t)nworld * nv * esz(); }
};

namespace pzc {

bool is_f64(const phyzb_sim* s);
bool specialized(const phyzb_sim* s);  // the next rollout launch runs the specialized kernel
int check_sim(const phyzb_sim* s);
void free_ptr(void*& p);
// one fused rollout launch of nsteps under `ctrl` (schedule stride or 0)
int launch(phyzb_sim* s, const void* ctrl, long long stride, int nsteps);
// host rows [nworld][width] f64 <-> device SoA [width][nworld] (sim precision)
int upload_rows(phyzb_sim* s, const double* host, int width, void* dst);
int download_rows(phyzb_sim* s, const void* src, int width, double* host);
void destroy_policy(phyzb_sim* s);  // capi_policy.cu
// NCCL (capi.cu): sum all-reduce of `count` f32 / f64 values in place, enqueued
// on `stream`; and a bounded wait for everything enqueued on `stream` so far
// (the communicator is aborted on failure or timeout).
int comm_allreduce_sum(phyzb_comm* c, void* buf, size_t count, bool f64, cudaStream_t stream);
int comm_wait(phyzb_comm* c, cudaStream_t stream, double timeout_s);
int comm_nranks(const phyzb_comm* c);

}  // namespace pzc
