// The rollout kernel with one world split over L threads (2, 4 or 8 lanes of
// a warp): pz_lanes.h plans the split, each lane steps its own sub-model
// (the trunk, then its limbs) with the same sweep code as rollout_kernel,
// and the backward sweep sums the limbs' articulated inertias and bias
// forces over the lanes before the trunk is swept. For a branching tree the
// limbs then run in parallel: a world step takes the trunk's time plus the
// longest lane's limbs instead of every body in turn, the point when worlds
// are too few to fill the GPU with one thread each.
//
// Shared-memory record layout only; no PD servos, impulse contact,
// heightfield or plane (the host keeps those on one thread per world). The
// kernel leaves the final step of a launch to the one-thread kernel, which
// writes the accelerations and contact state of that step.
#pragma once

#include "pz_lanes_sweep.cuh"
#include "stepper_kernels.cuh"

namespace pz {

// x summed over the L lanes of this thread's world; every lane gets the same
// bits (each pairwise sum is a + b on one lane and b + a on the other).
template <class T>
__device__ __forceinline__ T lane_sum(T x, int L) {
    for (int o = 1; o < L; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// The backward sweep of a lane: its limbs, then the sum over lanes of what
// the limbs pass to trunk bodies (the carry into the last trunk body and the
// trunk bodies' branch accumulators), then the trunk.
template <int FEAT, class T, class Scr>
__device__ __forceinline__ void pass2_lanes(const ModelView<T>& M, const Scr& S, int nt, int L) {
    AI<T> I;
    SV<T> pA;
    pass2_limbs<FEAT>(M, S, nt, I, pA);
#pragma unroll
    for (int k = 0; k < 6; k++) I.a[k] = lane_sum(I.a[k], L);
#pragma unroll
    for (int k = 0; k < 9; k++) I.h[k] = lane_sum(I.h[k], L);
#pragma unroll
    for (int k = 0; k < 6; k++) I.m[k] = lane_sum(I.m[k], L);
    pA = mksv<T>(mk3<T>(lane_sum(pA.w.x, L), lane_sum(pA.w.y, L), lane_sum(pA.w.z, L)),
                 mk3<T>(lane_sum(pA.l.x, L), lane_sum(pA.l.y, L), lane_sum(pA.l.z, L)));
    for (int t = 0; t < nt; t++) {
        const BodyI bi = M.bi[t];
        if (bi.flags & F_BRANCH)
            for (int k = 0; k < 27; k++) S(bi.s_acc + k) = lane_sum(S(bi.s_acc + k), L);
    }
    pass2_trunk<FEAT>(M, S, nt, I, pA);
}

template <class T, int FEAT>
__global__ void __launch_bounds__(256, 1) lanes_kernel(const __grid_constant__ RolloutArgs<T> P,
                                                       const __grid_constant__ LanesArgs La) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int F = FEAT | FEAT_LANES;
    const unsigned char* blob = stage_model(P.model_blob, P.model_bytes, smem);
    const int L = La.lanes;
    const int lane = threadIdx.x % L;
    // this lane's sub-model table
    const unsigned char* tab = blob + lane * La.lane_bytes;
    ModelView<T> M = make_view<T>(P, tab);
    M.bi = reinterpret_cast<const BodyI*>(tab + La.off_bi[lane]);
    M.pd = reinterpret_cast<const PdT<T>*>(tab + La.off_pd[lane]);
    M.pd_of_dof = reinterpret_cast<const int*>(tab + La.off_pdmap[lane]);
    M.nb = La.nb[lane];
    M.nv = La.nv[lane];
    const int* gdof = reinterpret_cast<const int*>(blob + La.off_gdof) + lane * La.nv_max;
    const int W = blockDim.x;
    SmemScr<T> S;
    S.base = reinterpret_cast<T*>(smem + P.model_bytes) + threadIdx.x;
    S.W = W;
    const int per_block = W / L;  // worlds per block (W is a multiple of 32, L divides 32)
    const long long N = P.nworld;
    const long long ntiles = (N + per_block - 1) / per_block;
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long long wt = tile * per_block + threadIdx.x / L;
        // lanes past the last world run world N-1 again and write nothing, so
        // every group of lanes takes part in the shuffles
        const bool active = wt < N;
        const long long w = active ? wt : N - 1;
        for (int j = 0; j < M.nv; j++) {
            S(j) = P.q[(long long)gdof[j] * N + w];
            S(M.nv + j) = P.v[(long long)gdof[j] * N + w];
        }
        WorldIO<T> io{P.ctrl, P.ctrl_stride, P.targets, N, w};
        io.gdof = gdof;
        for (int i = 0; i < M.nb; i++) prefetch_controls<false, T, SmemScr<T>, true>(M, M.bi[i], S, io, 0);
        S.commit();
        const Out<T> none{nullptr, 0};
        pass1_all<F>(M, S);
        for (int s = 0; s < P.nsteps; s++) {
            S.wait();
            pass2_lanes<F>(M, S, La.nt, L);
            pass3_next<F, false>(M, S, io, s + 1, none);
            S.commit();
        }
        S.wait();
        if (active) {
            bool finite = true;
            // the trunk's DOFs are the same on every lane: lane 0 writes them
            for (int j = lane == 0 ? 0 : La.trunk_nv; j < M.nv; j++) {
                const T qj = S(j), vj = S(M.nv + j);
                finite = finite && pz_finite(qj) && pz_finite(vj);
                P.q[(long long)gdof[j] * N + w] = qj;
                P.v[(long long)gdof[j] * N + w] = vj;
            }
            if (!finite) {
                atomicOr(P.status, 1);
                atomicMin(P.status + 1, (int)(w < 0x7fffffff ? w : 0x7fffffff));
            }
        }
    }
}

#ifndef __CUDACC_RTC__
// Block width (a multiple of 32 threads, at most 256) with the most worlds
// resident per SM, discounted by the fill of the last wave.
template <class T, int FEAT>
cudaError_t config_lanes_variant(const DeviceLimits& dl, int lanes, int scratch, int model_bytes, long long nworld,
                                 LaunchCfg* out) {
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, lanes_kernel<T, FEAT>);
    if (e != cudaSuccess) return e;
    const int dyn_cap = dl.smem_optin - (int)fa.sharedSizeBytes;
    e = cudaFuncSetAttribute(lanes_kernel<T, FEAT>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_cap);
    if (e != cudaSuccess) return e;
    double best = -1.0;
    for (int W = 32; W <= 256; W += 32) {
        const long long smem = (long long)model_bytes + (long long)scratch * (long long)sizeof(T) * W;
        if (smem > dyn_cap) break;
        int blocks = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, lanes_kernel<T, FEAT>, W, (size_t)smem);
        if (e != cudaSuccess) return e;
        if (blocks <= 0) continue;
        const double resident = (double)blocks * (W / lanes) * dl.sm_count;
        const double waves = std::ceil((double)nworld / resident);
        const double score = (double)blocks * (W / lanes) * ((double)nworld / (waves * resident));
        if (score > best * 1.0001) {
            best = score;
            const long long ntiles = (nworld + W / lanes - 1) / (W / lanes);
            const long long cap = (long long)dl.sm_count * blocks;
            out->W = W;
            out->grid = (int)(ntiles < cap ? (ntiles > 0 ? ntiles : 1) : cap);
            out->smem = (int)smem;
            out->tm = 0;
            out->score = score;
        }
    }
    return best < 0 ? cudaErrorInvalidConfiguration : cudaSuccess;
}

template <class T, int FEAT>
void launch_lanes_variant(const RolloutArgs<T>& a, const LanesArgs& la, const LaunchCfg& cfg, cudaStream_t s) {
    lanes_kernel<T, FEAT><<<cfg.grid, cfg.W, cfg.smem, s>>>(a, la);
}
#endif  // __CUDACC_RTC__

}  // namespace pz
