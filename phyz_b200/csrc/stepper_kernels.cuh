// Kernels of the B200 batched rigid-body stepper (sm_100a).
//
// rollout_kernel runs phyz-gpu's whole step sequence (cuda/mod.rs:879-945:
// PD -> contact -> ABA -> integrate) for `nsteps` steps in ONE launch: one
// thread per world, the model table staged once per block into shared
// memory, and each world's q, v and every per-body intermediate of the
// articulated-body algorithm held on chip (shared memory, structure-of-arrays
// and conflict-free, plus Tensor Memory for hinge records) for the whole
// rollout. Global memory sees the initial state read, one coalesced control
// row per step (prefetched a sweep ahead with cp.async), and the final state
// / accelerations / contact state written.
//
// The reference runs the same physics as 3-4 launches per step with every
// intermediate in thread-local arrays (phyz_kernels.cu:1175-1369: 255
// registers and 9.6 KB of spilled stack per thread on sm_100a).
//
// This header holds the kernel templates and their per-variant host
// wrappers (pz_variants.h); rollout_variants.cu instantiates one
// (precision, feature set) pair per translation unit.
#pragma once

#ifndef __CUDACC_RTC__
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>

#include "pz_variants.h"
#endif
#include "pz_launch.h"
#include "pz_world.cuh"

namespace pz {


// Per-thread view of the shared-memory scratch: slot s of this world lives
// at base[s * W] (consecutive threads -> consecutive banks). A specialized
// build fixes W (the block width) at compile time, so every slot access is
// one load or store at an immediate offset from `base`.
template <class T>
struct SmemScr {
    T* base;
#ifdef PZ_SPEC
    static constexpr int W = PZ_SPEC_W;
#else
    int W;
#endif
    __device__ __forceinline__ T& operator()(int s) const { return base[s * W]; }
    // Queue an asynchronous copy of *g into slot s. The "memory" clobber keeps
    // the compiler from moving a read of the slot's previous contents (the
    // sweep's D^-1 u, read just before the next control is queued into the
    // same slot) past the copy's issue, where the copy could land first.
    __device__ __forceinline__ void prefetch(int s, const T* g) const {
        const unsigned sa = (unsigned)__cvta_generic_to_shared(&base[s * W]);
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(sa), "l"(g), "n"(sizeof(T)) : "memory");
    }
    __device__ __forceinline__ void commit() const { asm volatile("cp.async.commit_group;\n" ::); }
    __device__ __forceinline__ void wait() const { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
    __device__ __forceinline__ void fence_st() const {}
    __device__ __forceinline__ Rec<T> rec_get(const BodyI& bi) const {
        Rec<T> r;
        r.c = (*this)(bi.s_xj);
        r.s = (*this)(bi.s_xj + 1);
        r.v = ld_sv<T>(*this, bi.s_vw);
        return r;
    }
    __device__ __forceinline__ void rec_put(const BodyI& bi, const Rec<T>& r) const {
        (*this)(bi.s_xj) = r.c;
        (*this)(bi.s_xj + 1) = r.s;
        st_sv(*this, bi.s_vw, r.v);
    }
    __device__ __forceinline__ void rec_put_vw(const BodyI& bi, const SV<T>& v) const { st_sv(*this, bi.s_vw, v); }
    // the external (contact) wrench of an F_EXTF body
    __device__ __forceinline__ SV<T> ext_get(const BodyI& bi) const { return ld_sv<T>(*this, bi.s_f); }
    __device__ __forceinline__ void ext_put(const BodyI& bi, const SV<T>& f) const { st_sv(*this, bi.s_f, f); }
};

// Tensor Memory scratch for body records: each thread owns the TMEM lane of
// its position in its warp (the warp's lane quarter is warp % 4) and a range
// of columns; a record [c, s, v0..v5] is 8 consecutive 32-bit columns (16 in
// f64) moved with one tcgen05.ld / tcgen05.st of shape 32x32b. In a
// Tensor-Memory layout every relabelled hinge (the only bodies whose
// records go through this interface) has its record here (t_rec >= 0). All
// record accesses are warp-uniform (every thread of a warp processes the
// same body).
template <class T>
struct TmemScr : SmemScr<T> {
    unsigned tbase;  // (lane quarter << 16) | this warp's first column
    __device__ __forceinline__ Rec<T> rec_get(const BodyI& bi) const {
        const unsigned a = tbase + (unsigned)bi.t_rec;
        Rec<T> r;
        if constexpr (sizeof(T) == 4) {
            unsigned x0, x1, x2, x3, x4, x5, x6, x7;
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                         : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3), "=r"(x4), "=r"(x5), "=r"(x6), "=r"(x7)
                         : "r"(a));
            asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                         : "+r"(x0), "+r"(x1), "+r"(x2), "+r"(x3), "+r"(x4), "+r"(x5), "+r"(x6), "+r"(x7)::"memory");
            r.c = __uint_as_float(x0);
            r.s = __uint_as_float(x1);
            r.v = mksv<T>(mk3<T>(__uint_as_float(x2), __uint_as_float(x3), __uint_as_float(x4)),
                          mk3<T>(__uint_as_float(x5), __uint_as_float(x6), __uint_as_float(x7)));
        } else {
            unsigned x[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                "%14, %15}, [%16];\n"
                : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]),
                  "=r"(x[8]), "=r"(x[9]), "=r"(x[10]), "=r"(x[11]), "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15])
                : "r"(a));
            asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                         : "+r"(x[0]), "+r"(x[1]), "+r"(x[2]), "+r"(x[3]), "+r"(x[4]), "+r"(x[5]), "+r"(x[6]),
                           "+r"(x[7]), "+r"(x[8]), "+r"(x[9]), "+r"(x[10]), "+r"(x[11]), "+r"(x[12]), "+r"(x[13]),
                           "+r"(x[14]), "+r"(x[15])::"memory");
            T d[8];
#pragma unroll
            for (int k = 0; k < 8; k++) d[k] = T(__hiloint2double((int)x[2 * k + 1], (int)x[2 * k]));
            r.c = d[0];
            r.s = d[1];
            r.v = mksv<T>(mk3<T>(d[2], d[3], d[4]), mk3<T>(d[5], d[6], d[7]));
        }
        return r;
    }
    __device__ __forceinline__ void put_words(unsigned a, const T* d, int n) const {
        // n = 8 (whole record) or 6 (columns 2..7: v / W only)
        if constexpr (sizeof(T) == 4) {
            unsigned x[8];
#pragma unroll
            for (int k = 0; k < 8; k++) x[k] = __float_as_uint(d[k]);
            if (n == 8)
                asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"r"(a),
                             "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(x[4]), "r"(x[5]), "r"(x[6]), "r"(x[7])
                             : "memory");
            else {
                asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};\n" ::"r"(a + 2u), "r"(x[2]),
                             "r"(x[3])
                             : "memory");
                asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(a + 4u),
                             "r"(x[4]), "r"(x[5]), "r"(x[6]), "r"(x[7])
                             : "memory");
            }
        } else {
            unsigned x[16];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                x[2 * k] = (unsigned)__double2loint((double)d[k]);
                x[2 * k + 1] = (unsigned)__double2hiint((double)d[k]);
            }
            if (n == 8)
                asm volatile(
                    "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15, %16};\n" ::"r"(a),
                    "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(x[4]), "r"(x[5]), "r"(x[6]), "r"(x[7]), "r"(x[8]),
                    "r"(x[9]), "r"(x[10]), "r"(x[11]), "r"(x[12]), "r"(x[13]), "r"(x[14]), "r"(x[15])
                    : "memory");
            else {
                asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(a + 4u),
                             "r"(x[4]), "r"(x[5]), "r"(x[6]), "r"(x[7])
                             : "memory");
                asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"r"(
                                 a + 8u),
                             "r"(x[8]), "r"(x[9]), "r"(x[10]), "r"(x[11]), "r"(x[12]), "r"(x[13]), "r"(x[14]),
                             "r"(x[15])
                             : "memory");
            }
        }
    }
    __device__ __forceinline__ void rec_put(const BodyI& bi, const Rec<T>& r) const {
        const T d[8] = {r.c, r.s, r.v.w.x, r.v.w.y, r.v.w.z, r.v.l.x, r.v.l.y, r.v.l.z};
        put_words(tbase + (unsigned)bi.t_rec, d, 8);
    }
    __device__ __forceinline__ void rec_put_vw(const BodyI& bi, const SV<T>& v) const {
        const T d[8] = {T(0), T(0), v.w.x, v.w.y, v.w.z, v.l.x, v.l.y, v.l.z};
        put_words(tbase + (unsigned)bi.t_rec, d, 6);
    }
    // the external (contact) wrench of an F_EXTF body: a record [f, 0, 0] at
    // column t_f, or its shared-memory slots when the layout keeps it there
    __device__ __forceinline__ SV<T> ext_get(const BodyI& bi) const {
        if (bi.t_f < 0) return ld_sv<T>(*this, bi.s_f);
        const unsigned a = tbase + (unsigned)bi.t_f;
        T d[6];
        if constexpr (sizeof(T) == 4) {
            unsigned x0, x1, x2, x3, x4, x5, x6, x7;
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                         : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3), "=r"(x4), "=r"(x5), "=r"(x6), "=r"(x7)
                         : "r"(a));
            asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                         : "+r"(x0), "+r"(x1), "+r"(x2), "+r"(x3), "+r"(x4), "+r"(x5), "+r"(x6), "+r"(x7)::"memory");
            d[0] = __uint_as_float(x0);
            d[1] = __uint_as_float(x1);
            d[2] = __uint_as_float(x2);
            d[3] = __uint_as_float(x3);
            d[4] = __uint_as_float(x4);
            d[5] = __uint_as_float(x5);
        } else {
            unsigned x[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                "%14, %15}, [%16];\n"
                : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]),
                  "=r"(x[8]), "=r"(x[9]), "=r"(x[10]), "=r"(x[11]), "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15])
                : "r"(a));
            asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                         : "+r"(x[0]), "+r"(x[1]), "+r"(x[2]), "+r"(x[3]), "+r"(x[4]), "+r"(x[5]), "+r"(x[6]),
                           "+r"(x[7]), "+r"(x[8]), "+r"(x[9]), "+r"(x[10]), "+r"(x[11]), "+r"(x[12]), "+r"(x[13]),
                           "+r"(x[14]), "+r"(x[15])::"memory");
#pragma unroll
            for (int k = 0; k < 6; k++) d[k] = T(__hiloint2double((int)x[2 * k + 1], (int)x[2 * k]));
        }
        return mksv<T>(mk3<T>(d[0], d[1], d[2]), mk3<T>(d[3], d[4], d[5]));
    }
    __device__ __forceinline__ void ext_put(const BodyI& bi, const SV<T>& f) const {
        if (bi.t_f < 0) {
            st_sv(*this, bi.s_f, f);
            return;
        }
        const T d[8] = {f.w.x, f.w.y, f.w.z, f.l.x, f.l.y, f.l.z, T(0), T(0)};
        put_words(tbase + (unsigned)bi.t_f, d, 8);
    }
    // stores complete before later loads of the same columns
    __device__ __forceinline__ void fence_st() const { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
};

template <class T>
__device__ __forceinline__ ModelView<T> make_view(const RolloutArgs<T>& P, const unsigned char* blob) {
    ModelView<T> M;
    M.btp = reinterpret_cast<const BodyT<T>*>(blob);
#ifndef PZ_SPEC
    M.bt = M.btp;
    M.bi = reinterpret_cast<const BodyI*>(blob + P.off_bi);
    M.pd = reinterpret_cast<const PdT<T>*>(blob + P.off_pd);
    M.pd_of_dof = reinterpret_cast<const int*>(blob + P.off_pdmap);
    M.nb = P.nb;
    M.nv = P.nv;
#endif
    M.npd = P.npd;
    M.contact = P.contact;
    M.dt = T(P.dt);
    M.gx = T(P.gx);
    M.gy = T(P.gy);
    M.gz = T(P.gz);
    M.ground_h = T(P.ground_h);
    M.friction = T(P.friction);
    const double dtc = P.dt > 1e-9 ? P.dt : 1e-9;
    M.inv_dt_c = T(1.0 / dtc);
    M.kstiff_c = T(4.0 / (dtc * dtc));
    M.im.ground_h = T(P.ground_h);
    M.im.friction = T(P.friction);
    M.im.dt = T(P.dt);
    M.im.erp = T(P.erp);
    M.im.margin = T(P.margin);
    M.im.restitution = T(P.restitution);
    M.im.rest_thr = T(P.rest_thr);
    M.im.dmin = T(P.si_dmin);
    M.im.dmax = T(P.si_dmax);
    M.im.width = T(P.si_width);
    M.im.mid = T(P.si_mid);
    M.im.power = T(P.si_power);
    impmat_finish(M.im);
    M.ter.h = P.hf;
    M.ter.nx = P.hf_nx;
    M.ter.ny = P.hf_ny;
    M.ter.ox = T(P.hf_ox);
    M.ter.oy = T(P.hf_oy);
    M.ter.oz = T(P.hf_oz);
    M.ter.cell = T(P.hf_cell);
    M.plane.body = P.plane_body;
    M.plane.offset = T(P.plane_offset);
    M.plane.max_depth = T(P.plane_max_depth);
    M.plane.half_x = T(P.plane_half_x);
    M.plane.half_y = T(P.plane_half_y);
    return M;
}

// Copy the model table into shared memory (16-byte chunks) and return its
// shared-memory address. All threads of the block take part.
__device__ __forceinline__ unsigned char* stage_model(const void* g, int bytes, unsigned char* smem) {
    const int4* src = reinterpret_cast<const int4*>(g);
    int4* dst = reinterpret_cast<int4*>(smem);
    for (int k = threadIdx.x; k < bytes / 16; k += blockDim.x) dst[k] = __ldg(src + k);
    __syncthreads();
    return smem;
}


#ifndef PZ_STEP_SYNC
#define PZ_STEP_SYNC 0
#endif

// Slice mode (RolloutArgs::chunk > 0). The warp's next job from the queue:
// lane 0 takes it and a warp reduction (its result is the same on every
// lane by construction) hands it to every lane.
__device__ __forceinline__ int slice_next(int* slices) {
    unsigned j = 0;
    if ((threadIdx.x & 31) == 0) j = atomicAdd(reinterpret_cast<unsigned*>(slices), 1u);
    return (int)__reduce_max_sync(0xffffffffu, j);
}

// Wait until a warp tile has finished `want` runs (*flag, published by
// slice_done). Every lane reads the flag with acquire semantics, so the
// state stores of the run before are visible to every lane's loads after.
// The job order makes the wait short (the run before was taken a whole
// round of jobs earlier) and a run is only ever held by a running warp, so
// it ends; it is still bounded: after 4 s of device time the status word's
// bit 1 is set and the run goes on.
__device__ __forceinline__ void slice_wait(const int* flag, int want, int* status) {
    int got;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];\n" : "=r"(got) : "l"(flag) : "memory");
    if (got < want) {
        unsigned long long t0, t;
        asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t0));
        for (;;) {
            __nanosleep(256);
            asm volatile("ld.acquire.gpu.global.s32 %0, [%1];\n" : "=r"(got) : "l"(flag) : "memory");
            if (got >= want) break;
            asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
            if (t - t0 > 4000000000ull) {
                atomicOr(status, 2);
                break;
            }
        }
    }
    __syncwarp();
}

// Publish that a warp tile has finished `done` runs, after every lane's
// state stores.
__device__ __forceinline__ void slice_done(int* flag, int done) {
    __threadfence();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) asm volatile("st.release.gpu.global.s32 [%0], %1;\n" ::"l"(flag), "r"(done) : "memory");
}

template <bool TM, class T>
struct PickScr {
    using type = SmemScr<T>;
};
template <class T>
struct PickScr<true, T> {
    using type = TmemScr<T>;
};

// Threads per block the kernel is compiled for: any width up to 256 in the
// generic variants (up to 255 registers a thread); a specialized build is
// compiled for its one width, which may go past 256 when its registers,
// shared memory and Tensor Memory per world allow.
#ifdef PZ_SPEC
#define PZ_MAX_THREADS PZ_SPEC_W
#else
#define PZ_MAX_THREADS 256
#endif

// One job of the rollout kernel: this thread's world wt from step s0 to
// step s1 of the launch (state in from q, v and the impulse buffer, out to
// them; accelerations and contact state when s1 is the launch's last step).
template <class T, int FEAT, class Scr>
__device__ __forceinline__ void run_job(const RolloutArgs<T>& P, const ModelView<T>& M, const Scr& S,
                                        const long long wt, const int s0, const int s1) {
    const long long N = P.nworld;
    // lanes past the last world run world N-1 again and write nothing, so
    // every warp stays converged for the warp-wide tcgen05 operations
    const bool active = wt < N;
    const long long w = active ? wt : N - 1;
    PZ_UNROLL_BODIES
    for (int j = 0; j < M.nv; j++) {
        S(j) = P.q[j * N + w];
        S(M.nv + j) = P.v[j * N + w];
    }
    const WorldIO<T> io{P.ctrl, P.ctrl_stride, P.targets, N, w};
    PZ_UNROLL_BODIES
    for (int i = 0; i < M.nb; i++) prefetch_controls<(FEAT & FEAT_IMPULSE) != 0>(M, M.bi[i], S, io, s0);
    S.commit();
    if constexpr ((FEAT & FEAT_IMPULSE) != 0) {
        // the wrenches of the previous step's last sweep and the staged
        // impulses that warm-start this one
        PZ_UNROLL_BODIES
        for (int i = 0; i < M.nb; i++) {
            const BodyI bi = M.bi[i];
            if (bi.c_imp < 0) continue;
            // rows: wrench (6), ground impulses, plane impulses (3 per point each)
            const int np3 = 3 * (bi.gtype == 2 ? 8 : 1);
            int r = bi.c_imp;
            for (int k = 0; k < 6; k++) S(bi.s_f + k) = P.imp[(long long)(r++) * N + w];
            if (bi.s_imp >= 0)
                for (int k = 0; k < np3; k++) S(bi.s_imp + k) = P.imp[(long long)(r++) * N + w];
            if (bi.s_pimp >= 0)
                for (int k = 0; k < np3; k++) S(bi.s_pimp + k) = P.imp[(long long)(r++) * N + w];
        }
    }
    const Out<T> none{nullptr, 0};
    pass1_all<FEAT>(M, S);
    for (int s = s0; s < s1; s++) {
        S.wait();
#if PZ_STEP_SYNC
        // keep the block's warps on the same stretch of code (they share
        // its instruction fetches); every thread runs every step
        __syncthreads();
#endif
        const bool last = s == P.nsteps - 1;
        if constexpr ((FEAT & FEAT_CONTACT) != 0 && (FEAT & FEAT_IMPULSE) == 0) {
            // contact state of the last step, from the state it starts from
            // (every lane runs it, warp-wide record loads; only active lanes write)
            if (last && P.contact && P.cstate)
                contact_state_pass<FEAT>(M, S, active ? Out<T>{P.cstate + w, N} : none);
        }
        if constexpr ((FEAT & FEAT_TERRAIN) != 0 && (FEAT & FEAT_IMPULSE) == 0) {
            // the plane contacts of this step's state join the ground wrenches of pass 1
            if (M.plane.body >= 0) plane_pass<false, FEAT>(M, S);
        }
        pass2<FEAT>(M, S);
        if constexpr ((FEAT & FEAT_IMPULSE) != 0) {
            // sweeps x [contact at the free velocity -> the response to
            // the wrench change], from the step's backward sweep
            keep_backward_state(M, S);
            for (int k = 0; k < P.sweeps; k++) {
                sweep_forward<FEAT>(M, S);
                if constexpr ((FEAT & FEAT_TERRAIN) != 0)
                    if (M.plane.body >= 0) plane_pass<true, FEAT>(M, S);
                wrench_response<FEAT>(M, S);
            }
            if (last && P.cstate) contact_state_impulse_pass<FEAT>(M, S, active ? Out<T>{P.cstate + w, N} : none);
        }
        if (last)
            pass3_next<FEAT, true>(M, S, io, -1, active ? Out<T>{P.qdd + w, N} : none);
        else
            pass3_next<FEAT, false>(M, S, io, s + 1, none);
        S.commit();
    }
    S.wait();
    if constexpr ((FEAT & FEAT_IMPULSE) != 0) {
        if (active)
            PZ_UNROLL_BODIES
            for (int i = 0; i < M.nb; i++) {
                const BodyI bi = M.bi[i];
                if (bi.c_imp < 0) continue;
                const int np3 = 3 * (bi.gtype == 2 ? 8 : 1);
                int r = bi.c_imp;
                for (int k = 0; k < 6; k++) P.imp[(long long)(r++) * N + w] = S(bi.s_f + k);
                if (bi.s_imp >= 0)
                    for (int k = 0; k < np3; k++) P.imp[(long long)(r++) * N + w] = S(bi.s_imp + k);
                if (bi.s_pimp >= 0)
                    for (int k = 0; k < np3; k++) P.imp[(long long)(r++) * N + w] = S(bi.s_pimp + k);
            }
    }
    if (active) {
        bool finite = true;
        PZ_UNROLL_BODIES
        for (int j = 0; j < M.nv; j++) {
            const T qj = S(j), vj = S(M.nv + j);
            finite = finite && pz_finite(qj) && pz_finite(vj);
            P.q[j * N + w] = qj;
            P.v[j * N + w] = vj;
        }
        if (!finite) {
            atomicOr(P.status, 1);
            atomicMin(P.status + 1, (int)(w < 0x7fffffff ? w : 0x7fffffff));
        }
    }
}

template <class T, int FEAT, bool TM>
__global__ void __launch_bounds__(PZ_MAX_THREADS, 1) rollout_kernel(const __grid_constant__ RolloutArgs<T> P) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ unsigned tmem_slot;
    const unsigned char* blob = stage_model(P.model_blob, P.model_bytes, smem);
    const ModelView<T> M = make_view<T>(P, blob);
#ifdef PZ_SPEC
    constexpr int W = PZ_SPEC_W;  // the launch's block width
#else
    const int W = blockDim.x;
#endif
    using Scr = typename PickScr<TM, T>::type;
    Scr S;
    S.base = reinterpret_cast<T*>(smem + P.model_bytes) + threadIdx.x;
#ifndef PZ_SPEC
    S.W = W;
#endif
    const int warp = threadIdx.x >> 5;
    if constexpr (TM) {
        if (warp == 0) {
            const unsigned dst = (unsigned)__cvta_generic_to_shared(&tmem_slot);
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst),
                         "r"(TMEM_COLS));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
        }
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        // warps w, w+4, w+8, ... share lane quarter w % 4 and split its columns
        const int nwarps = (W + 31) >> 5;
        const unsigned per_quarter = (unsigned)((nwarps + 3) >> 2);
        const unsigned cols = (TMEM_COLS / per_quarter) & ~7u;  // whole 8-column records
        S.tbase = tmem_slot + ((unsigned)(32 * (warp & 3)) << 16) + (unsigned)(warp >> 2) * cols;
    }
    const long long N = P.nworld;
#if PZ_STEP_SYNC
    constexpr bool sliced = false;
#elif defined(PZ_SPEC)
    // a model-specialized build holds one of the two loops (a second copy of
    // its unrolled step would double the compile): the tile kernel and its
    // slice-mode twin are compiled apart
    constexpr bool sliced = PZ_SPEC_SLICED != 0;
#else
    constexpr bool can_slice = SliceVariant<FEAT, TM>::value;
    const bool sliced = can_slice && P.chunk > 0;
#endif
    // Tile mode: the blocks stride over tiles of W worlds, each for every
    // step. Slice mode: every warp takes jobs (a tile of 32 worlds, one run
    // of P.chunk steps) from the queue in run-major order, the state going
    // through q and v between runs. The two loops are written out apart so
    // that tile mode's step range stays the kernel parameters (measured:
    // one loop over either kind of job ran C2's tile launches 2 % slower).
    if (!sliced) {
        const long long ntiles = (N + W - 1) / W;
        for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x)
            run_job<T, FEAT>(P, M, S, tile * W + threadIdx.x, 0, P.nsteps);
    } else {
        const long long ntiles = (N + 31) / 32;
        const long long njobs = ntiles * ((P.nsteps + P.chunk - 1) / P.chunk);
        for (long long job = slice_next(P.slices); job < njobs; job = slice_next(P.slices)) {
            const long long tile = job % ntiles;
            const int run = (int)(job / ntiles);
            const int s0 = run * P.chunk;
            if (run > 0) slice_wait(P.slices + 2 + tile, run, P.status);
            run_job<T, FEAT>(P, M, S, tile * 32 + (threadIdx.x & 31), s0,
                             s0 + P.chunk < P.nsteps ? s0 + P.chunk : P.nsteps);
            slice_done(P.slices + 2 + tile, run + 1);
        }
    }
    if constexpr (TM) {
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        if (warp == 0)
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_slot), "r"(TMEM_COLS));
    }
}

// Kinetic energy 0.5 sum_i v_i^T I_i v_i + 0.5 sum_j armature_j qd_j^2
// (crates/phyz-rigid/src/energy.rs:8-11 with crba's armature) or sum q^2,
// reduced over the block and added into *out.
template <class T, int FEAT>
__global__ void __launch_bounds__(256) objective_kernel(const __grid_constant__ RolloutArgs<T> P, int kind,
                                                         T* out) {
    extern __shared__ __align__(16) unsigned char smem[];
    const unsigned char* blob = stage_model(P.model_blob, P.model_bytes, smem);
    ModelView<T> M = make_view<T>(P, blob);
    M.contact = 0;
    const int W = blockDim.x;
    const SmemScr<T> S{reinterpret_cast<T*>(smem + P.model_bytes) + threadIdx.x, W};
    const long long ntiles = (P.nworld + W - 1) / W;
    T acc = T(0);
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long long w = tile * W + threadIdx.x;
        if (w >= P.nworld) continue;
        const long long N = P.nworld;
        PZ_UNROLL_BODIES
        for (int j = 0; j < M.nv; j++) {
            S(j) = P.q[j * N + w];
            S(M.nv + j) = P.v[j * N + w];
        }
        if (kind == 1) {
            PZ_UNROLL_BODIES
            for (int j = 0; j < M.nv; j++) acc += S(j) * S(j);
            continue;
        }
        pass1_all<FEAT & (FEAT_MULTI | FEAT_PERM | FEAT_PERM1)>(M, S);
        PZ_UNROLL_BODIES
        for (int i = 0; i < M.nb; i++) {
            const BodyI bi = M.bi[i];
            const BodyT<T>& bt = M.bt[i];
            const SV<T> v = ld_sv<T>(S, bi.s_vw);
            const V3<T> mc = ld3(bt.mcom);
            const SV<T> h = mksv<T>(symv(bt.Io, v.w) + cross(mc, v.l), v.l * bt.mass + cross(v.w, mc));
            acc += T(0.5) * dot(v, h);
            for (int k = 0; k < bi.ndof; k++) {
                const T qd = S(M.nv + bi.off + k);
                acc += T(0.5) * bt.armature * qd * qd;
            }
        }
    }
    // warp reduction, one atomic per warp (blockDim.x is a multiple of 32)
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, acc);
}

#ifndef __CUDACC_RTC__
template <class T, int FEAT, bool TM>
cudaError_t config_variant(const DeviceLimits& dl, int scratch, int model_bytes, long long nworld, int tmem_cols,
                           LaunchCfg* out) {
    // the opt-in limit covers static and dynamic shared memory together
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, rollout_kernel<T, FEAT, TM>);
    if (e != cudaSuccess) return e;
    const int dyn_cap = dl.smem_optin - (int)fa.sharedSizeBytes;
    e = cudaFuncSetAttribute(rollout_kernel<T, FEAT, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_cap);
    if (e != cudaSuccess) return e;
    if (!TM) {
        e = cudaFuncSetAttribute(objective_kernel<T, FEAT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 dl.smem_optin);
        if (e != cudaSuccess) return e;
    }
    auto occupancy = [](int* blocks, int W, size_t smem) {
        return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, rollout_kernel<T, FEAT, TM>, W, smem);
    };
    return pick_launch(dl, dyn_cap, TM, (int)sizeof(T), scratch, model_bytes, nworld, tmem_cols, (int)TMEM_COLS,
                       occupancy, out, 0, 256, SliceVariant<FEAT, TM>::value);
}

template <class T, int FEAT, bool TM>
void launch_variant(const RolloutArgs<T>& a, const LaunchCfg& cfg, cudaStream_t s) {
    rollout_kernel<T, FEAT, TM><<<cfg.grid, cfg.W, cfg.smem, s>>>(a);
}

template <class T, int FEAT>
void launch_objective_variant(const RolloutArgs<T>& a, const LaunchCfg& cfg, int kind, T* out, cudaStream_t s) {
    objective_kernel<T, FEAT><<<cfg.grid, cfg.W, cfg.smem, s>>>(a, kind, out);
}
#endif  // __CUDACC_RTC__

}  // namespace pz
