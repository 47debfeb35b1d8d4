// TEST INFRASTRUCTURE ONLY -- the reference's own CUDA kernels on this GPU.
//
// oracle/Makefile compiles crates/phyz-gpu/cuda/phyz_kernels.cu from the
// reference tree with nvcc for sm_100a (IEEE division and square root, no
// fast math: the reference's NVRTC options, cuda/nvrtc.rs:83-90) and links
// it with this driver into oracle/_ref/libphyz_ref_cuda.so. The driver
// replays the reference's step sequence (cuda/mod.rs:879-945: penalty
// contact -> aba -> integrate, or impulse mode's aba, sweeps x [contact ->
// aba], integrate; 64-thread blocks, nvrtc.rs:120-126) as one
// captured CUDA graph per rollout, the way BatchSim::step_many replays its
// graph cache (mod.rs:843-875). Used by the GPU tests for parity of the B200
// stepper with the reference's GPU path and for its throughput on the same
// GPU.
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

typedef unsigned int u32;

extern "C" __global__ void phyz_contact(const float* cparams, const float* bodies, const float* geometry,
                                        const float* q, const float* v, float* ext_forces, float* contact_state,
                                        const float* hf_heights, const float* qdd);
extern "C" __global__ void phyz_aba(u32 nworld, u32 nv, float dt, u32 nbodies, float gx, float gy, float gz,
                                    const float* bodies, const float* q, const float* v, const float* ctrl,
                                    float* qdd, const float* ext_forces);
extern "C" __global__ void phyz_integrate(u32 nworld, u32 nv, float dt, u32 nbodies, float* q, float* v,
                                          const float* qdd, const float* bodies);

namespace {

const int BODY_STRIDE = 36, GEOM_STRIDE = 24, CP_STRIDE = 32, CS_STRIDE = 56, BLOCK = 64;

#define RC(x)                                   \
    do {                                        \
        if ((x) != cudaSuccess) return -(int)(x); \
    } while (0)

struct Bufs {
    float *bodies = nullptr, *geom = nullptr, *cp = nullptr, *q = nullptr, *v = nullptr, *ctrl = nullptr,
          *qdd = nullptr, *ext = nullptr, *cs = nullptr, *hf = nullptr;
    ~Bufs() {
        for (float* p : {bodies, geom, cp, q, v, ctrl, qdd, ext, cs, hf})
            if (p) cudaFree(p);
    }
};

// sweeps == 0: the penalty sequence contact -> aba -> integrate; sweeps > 0
// (impulse mode, cparams solve_mode 1): aba, sweeps x [contact -> aba],
// integrate (cuda/mod.rs:916-927).
int enqueue(cudaStream_t s, const Bufs& b, u32 n, u32 nv, u32 nb, float dt, float gx, float gy, float gz,
            int64_t stride, int nsteps, int sweeps) {
    const unsigned gw = (n + BLOCK - 1) / BLOCK, gi = (n * nb + BLOCK - 1) / BLOCK;
    for (int k = 0; k < nsteps; k++) {
        const float* c = b.ctrl + (size_t)k * stride;
        if (sweeps > 0) {
            phyz_aba<<<gw, BLOCK, 0, s>>>(n, nv, dt, nb, gx, gy, gz, b.bodies, b.q, b.v, c, b.qdd, b.ext);
            for (int w = 0; w < sweeps; w++) {
                phyz_contact<<<gw, BLOCK, 0, s>>>(b.cp, b.bodies, b.geom, b.q, b.v, b.ext, b.cs, b.hf, b.qdd);
                phyz_aba<<<gw, BLOCK, 0, s>>>(n, nv, dt, nb, gx, gy, gz, b.bodies, b.q, b.v, c, b.qdd, b.ext);
            }
        } else {
            if (b.geom)
                phyz_contact<<<gw, BLOCK, 0, s>>>(b.cp, b.bodies, b.geom, b.q, b.v, b.ext, b.cs, b.hf, b.qdd);
            phyz_aba<<<gw, BLOCK, 0, s>>>(n, nv, dt, nb, gx, gy, gz, b.bodies, b.q, b.v, c, b.qdd, b.ext);
        }
        phyz_integrate<<<gi, BLOCK, 0, s>>>(n, nv, dt, nb, b.q, b.v, b.qdd, b.bodies);
    }
    return (int)cudaGetLastError();
}

}  // namespace

extern "C" {

// nsteps of the reference's GPU step on nworld worlds (AoS f32 rows, as its
// buffers hold them): q, v updated in place, qdd and the contact state of
// the last step returned. ctrl: [nsteps][nworld][nv] when ctrl_step_stride
// = nworld * nv, or one held row set when 0. With reps > 0 the same rollout
// is then replayed reps times from the same initial state and *ms_min gets
// the fastest replay (CUDA events around one graph launch).
// `sweeps` > 0 runs the impulse-mode sequence (cparams must say solve_mode
// 1); the wrench and impulse buffers start from zero on every call.
int phyzref_cuda_rollout_sweeps(u32 nworld, u32 nv, u32 nb, float dt, float gx, float gy, float gz,
                                const float* bodies, const float* geometry, const float* cparams, float* q, float* v,
                                const float* ctrl, int64_t ctrl_step_stride, int32_t nsteps, int32_t sweeps,
                                int32_t reps, float* qdd_out, float* cs_out, float* ms_min) {
    if (sweeps > 0 && !geometry) return -1;
    Bufs b;
    const size_t n = nworld, S = (size_t)n * nv * 4;
    const size_t ctrl_bytes = ctrl_step_stride ? (size_t)nsteps * ctrl_step_stride * 4 : S;
    RC(cudaMalloc(&b.bodies, (size_t)nb * BODY_STRIDE * 4));
    RC(cudaMemcpy(b.bodies, bodies, (size_t)nb * BODY_STRIDE * 4, cudaMemcpyHostToDevice));
    if (geometry) {
        RC(cudaMalloc(&b.geom, (size_t)nb * GEOM_STRIDE * 4));
        RC(cudaMemcpy(b.geom, geometry, (size_t)nb * GEOM_STRIDE * 4, cudaMemcpyHostToDevice));
        RC(cudaMalloc(&b.cp, CP_STRIDE * 4));
        RC(cudaMemcpy(b.cp, cparams, CP_STRIDE * 4, cudaMemcpyHostToDevice));
    }
    RC(cudaMalloc(&b.q, S));
    RC(cudaMalloc(&b.v, S));
    RC(cudaMalloc(&b.ctrl, ctrl_bytes));
    RC(cudaMalloc(&b.qdd, S));
    RC(cudaMalloc(&b.ext, n * nb * 6 * 4));
    RC(cudaMalloc(&b.cs, n * nb * CS_STRIDE * 4));
    RC(cudaMalloc(&b.hf, 16));
    RC(cudaMemset(b.ext, 0, n * nb * 6 * 4));
    RC(cudaMemset(b.cs, 0, n * nb * CS_STRIDE * 4));
    RC(cudaMemset(b.hf, 0, 16));
    RC(cudaMemset(b.qdd, 0, S));
    RC(cudaMemcpy(b.ctrl, ctrl, ctrl_bytes, cudaMemcpyHostToDevice));
    cudaStream_t s;
    RC(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int rc = 0;
    auto load = [&]() -> int {
        RC(cudaMemcpyAsync(b.q, q, S, cudaMemcpyHostToDevice, s));
        RC(cudaMemcpyAsync(b.v, v, S, cudaMemcpyHostToDevice, s));
        return 0;
    };
    do {
        if ((rc = load())) break;
        if ((rc = -(int)cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal))) break;
        const int er = enqueue(s, b, nworld, nv, nb, dt, gx, gy, gz, ctrl_step_stride, nsteps, sweeps);
        const cudaError_t ec = cudaStreamEndCapture(s, &graph);
        if (er || ec != cudaSuccess) {
            rc = er ? -er : -(int)ec;
            break;
        }
        if ((rc = -(int)cudaGraphInstantiate(&exec, graph, 0))) break;
        if ((rc = -(int)cudaGraphLaunch(exec, s))) break;
        if ((rc = -(int)cudaStreamSynchronize(s))) break;
        // the parity result
        std::vector<float> hq(n * nv), hv(n * nv);
        if ((rc = -(int)cudaMemcpy(hq.data(), b.q, S, cudaMemcpyDeviceToHost))) break;
        if ((rc = -(int)cudaMemcpy(hv.data(), b.v, S, cudaMemcpyDeviceToHost))) break;
        if (qdd_out && (rc = -(int)cudaMemcpy(qdd_out, b.qdd, S, cudaMemcpyDeviceToHost))) break;
        if (cs_out && (rc = -(int)cudaMemcpy(cs_out, b.cs, n * nb * CS_STRIDE * 4, cudaMemcpyDeviceToHost))) break;
        if (reps > 0 && ms_min) {
            cudaEvent_t e0, e1;
            cudaEventCreate(&e0);
            cudaEventCreate(&e1);
            float best = 1e30f;
            for (int r = 0; r < reps && !rc; r++) {
                if ((rc = load())) break;
                cudaEventRecord(e0, s);
                cudaGraphLaunch(exec, s);
                cudaEventRecord(e1, s);
                if ((rc = -(int)cudaEventSynchronize(e1))) break;
                float ms = 0.0f;
                cudaEventElapsedTime(&ms, e0, e1);
                if (ms < best) best = ms;
            }
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
            *ms_min = best;
        }
        std::copy(hq.begin(), hq.end(), q);
        std::copy(hv.begin(), hv.end(), v);
    } while (0);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
    return rc;
}

int phyzref_cuda_rollout(u32 nworld, u32 nv, u32 nb, float dt, float gx, float gy, float gz, const float* bodies,
                         const float* geometry, const float* cparams, float* q, float* v, const float* ctrl,
                         int64_t ctrl_step_stride, int32_t nsteps, int32_t reps, float* qdd_out, float* cs_out,
                         float* ms_min) {
    return phyzref_cuda_rollout_sweeps(nworld, nv, nb, dt, gx, gy, gz, bodies, geometry, cparams, q, v, ctrl,
                                       ctrl_step_stride, nsteps, 0, reps, qdd_out, cs_out, ms_min);
}

}  // extern "C"
