// On-device control loop of the batched stepper: the kinematics readout,
// the observation row, a two-hidden-layer tanh MLP and a diagonal-Gaussian
// action written into the PD targets -- phyz-gpu's phyz_fk / phyz_obs /
// phyz_policy passes (crates/phyz-gpu/cuda/phyz_kernels.cu:1436-1715,
// crates/phyz-gpu/src/policy_pipeline.rs) as one launch per control step.
// Host-side launch interface (policy.cu).
#pragma once

#include <cuda_runtime.h>

namespace pz {

// Kinematics table of one body, in the model's own (not relabelled) frames:
// the joint transform and the parent->joint transform of phyz's Joint.
template <class T>
struct alignas(16) FkBody {
    int parent, jtype, off, pad;
    T axis[3];
    T ptj_rot[9];  // row-major, parent -> joint frame
    T ptj_pos[3];  // joint origin in the parent frame
};

// Floats per body in the kinematics readout (policy_pipeline.rs XF_STRIDE):
// world->body rotation (9, row-major), body origin in world (3), angular and
// linear velocity in the body frame (3 + 3).
constexpr int XF_STRIDE = 18;
constexpr int OBS_OP_STRIDE = 4;
constexpr int POLICY_MAX_IN = 128;
constexpr int POLICY_MAX_H = 256;
constexpr int POLICY_MAX_OUT = 32;
// MLP tiles: widths are padded to multiples of this (zero weights: exact).
constexpr int POLICY_TILE = 32;

template <class T>
struct PolicyArgs {
    const FkBody<T>* fk;  // [nb]
    int nb, nv;
    const T* q;  // state, SoA [nv][nworld]
    const T* v;
    long long nworld;
    void* xf;          // kinematics readout (T), SoA [(body * XF_STRIDE + k)][nworld]
    // observation
    const float* ops;  // [n_in][OBS_OP_STRIDE]: kind, a, b, c
    const float* aux;  // ComOverSupport payloads
    const float* com;  // [nb][4]: mass, com (body frame)
    int n_in;
    // MLP, packed for the kernel (policy.cu pack_weights): W1^T [in_pad][h_pad],
    // b1 [h_pad], W2^T [h_pad][h_pad], b2 [h_pad], W3^T [h_pad][out_pad], b3 [out_pad]
    const float* w;
    int n_wf;  // floats in w
    int in_pad, h_pad, out_pad, n_out;
    const float* stdv;      // [n_out]
    const float* in_noise;  // [n_in]
    const int* act_slots;   // [n_out] PD servo slot of each action
    const float* clamp;     // [n_out] applied-action clamp
    float rho;
    unsigned long long* rng;  // [nworld] xorshift64 state
    float* z;                 // [n_out][nworld] AR(1) noise state
    const T* base;            // [npd][nworld] base PD targets
    T* targets;               // [npd][nworld] PD targets (written)
    int npd;
    float* h;    // hidden-layer scratch, SoA [2][h_pad][nworld]
    float* obs;  // this step's observation rows, SoA [n_in][nworld]
    float* out;  // this step's actions + log-prob, SoA [n_out + 1][nworld]
};

// Kinematics readout only (phyz_fk): fills args.xf from q, v.
template <class T>
cudaError_t launch_kinematics(const PolicyArgs<T>& a, cudaStream_t s);
// One control step: kinematics, observation, MLP, sample, PD targets.
template <class T>
cudaError_t launch_policy(const PolicyArgs<T>& a, cudaStream_t s);


}  // namespace pz
