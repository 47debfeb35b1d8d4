// Kernels of the on-device control loop (pz_policy.h): kinematics readout,
// observation, tanh MLP, Gaussian action -> PD targets.
//
// One thread per world. The kinematics of every body go to a readout buffer
// in HBM (SoA, the reference's XF_STRIDE record); the observation ops read
// it back (the same thread wrote it). The MLP runs out of shared memory: the
// block stages the packed weights once (transposed, padded to 32-wide tiles
// with zeros, so a tile of outputs reads its weights as broadcast float4
// loads), every world keeps its input and hidden rows in shared memory
// (SoA, conflict-free), and each output tile accumulates in 32 registers in
// the reference's summation order (bias first, then inputs in index order).
// Random draws follow phyz's per-world xorshift64 + Box-Muller stream
// (phyz_kernels.cu:1600-1640) bit for bit.
#include <cuda_runtime.h>

#include <cstdint>

#include "pz_mlp.cuh"
#include "pz_policy.h"
#include "pz_world.cuh"

namespace pz {

namespace {

constexpr int POLICY_BLOCK = 128;

template <class T>
struct Xf {
    R3<T> E;  // world -> body
    V3<T> p;  // body origin, world
    V3<T> w, l;  // body velocity, body frame
};

template <class T>
__device__ __forceinline__ V3<T> rmul_t(const R3<T>& E, const V3<T>& x) {  // E^T x
    return mk3<T>(E.m[0] * x.x + E.m[3] * x.y + E.m[6] * x.z, E.m[1] * x.x + E.m[4] * x.y + E.m[7] * x.z,
                  E.m[2] * x.x + E.m[5] * x.y + E.m[8] * x.z);
}
template <class T>
__device__ __forceinline__ V3<T> rmul_(const R3<T>& E, const V3<T>& x) {  // E x
    return mk3<T>(E.m[0] * x.x + E.m[1] * x.y + E.m[2] * x.z, E.m[3] * x.x + E.m[4] * x.y + E.m[5] * x.z,
                  E.m[6] * x.x + E.m[7] * x.y + E.m[8] * x.z);
}
template <class T>
__device__ __forceinline__ R3<T> rmat(const R3<T>& A, const R3<T>& B) {  // A B
    R3<T> C;
#pragma unroll
    for (int r = 0; r < 3; r++)
#pragma unroll
        for (int c = 0; c < 3; c++)
            C.m[r * 3 + c] = A.m[r * 3 + 0] * B.m[0 * 3 + c] + A.m[r * 3 + 1] * B.m[1 * 3 + c] +
                             A.m[r * 3 + 2] * B.m[2 * 3 + c];
    return C;
}

// World transforms and velocities of every body (phyz-rigid forward
// kinematics with tang's compose: rot = A B, pos = B.pos + B.rot^T A.pos;
// apply_motion = [R w; R (v - p x w)]), written to the readout.
template <class T>
__device__ void kinematics_world(const PolicyArgs<T>& P, long long w) {
    const long long N = P.nworld;
    Xf<T> prev;
    for (int i = 0; i < P.nb; i++) {
        const FkBody<T>& b = P.fk[i];
        const V3<T> ax = mk3<T>(b.axis[0], b.axis[1], b.axis[2]);
        R3<T> EJ;
        EJ.m[0] = EJ.m[4] = EJ.m[8] = T(1);
        EJ.m[1] = EJ.m[2] = EJ.m[3] = EJ.m[5] = EJ.m[6] = EJ.m[7] = T(0);
        V3<T> rJ = zero3<T>(), vw = zero3<T>(), vl = zero3<T>();
        const T* q = P.q + (long long)b.off * N + w;
        const T* v = P.v + (long long)b.off * N + w;
        switch (b.jtype) {
            case J_REVOLUTE: {
                T s, c;
                pz_sincos(-q[0], &s, &c);
                EJ = hinge_matrix(ax, c, s);
                vw = ax * v[0];
                break;
            }
            case J_PRISMATIC:
                rJ = ax * q[0];
                vl = ax * v[0];
                break;
            case J_BALL:
            case J_FREE: {
                EJ = qjoint_rot(qexp(mk3<T>(q[0], q[N], q[2 * N])));
                vw = mk3<T>(v[0], v[N], v[2 * N]);
                if (b.jtype == J_FREE) {
                    rJ = mk3<T>(q[3 * N], q[4 * N], q[5 * N]);
                    vl = mk3<T>(v[3 * N], v[4 * N], v[5 * N]);
                }
                break;
            }
            default: break;
        }
        R3<T> Rp;
#pragma unroll
        for (int k = 0; k < 9; k++) Rp.m[k] = b.ptj_rot[k];
        const V3<T> pp = mk3<T>(b.ptj_pos[0], b.ptj_pos[1], b.ptj_pos[2]);
        // X_tree = X_J o X_ptj
        const R3<T> Et = rmat(EJ, Rp);
        const V3<T> pt = pp + rmul_t(Rp, rJ);
        Xf<T> cur;
        if (b.parent < 0) {
            cur.E = Et;
            cur.p = pt;
            cur.w = vw;
            cur.l = vl;
        } else {
            Xf<T> par;
            if (b.parent == i - 1) {
                par = prev;
            } else {
                const T* base = reinterpret_cast<const T*>(P.xf) + (long long)b.parent * XF_STRIDE * N + w;
#pragma unroll
                for (int k = 0; k < 9; k++) par.E.m[k] = base[k * N];
                par.p = mk3<T>(base[9 * N], base[10 * N], base[11 * N]);
                par.w = mk3<T>(base[12 * N], base[13 * N], base[14 * N]);
                par.l = mk3<T>(base[15 * N], base[16 * N], base[17 * N]);
            }
            cur.E = rmat(Et, par.E);
            cur.p = par.p + rmul_t(par.E, pt);
            // X_tree applied to the parent's velocity, plus the joint's
            cur.w = rmul_(Et, par.w) + vw;
            cur.l = rmul_(Et, par.l - cross(pt, par.w)) + vl;
        }
        T* o = reinterpret_cast<T*>(P.xf) + (long long)i * XF_STRIDE * N + w;
#pragma unroll
        for (int k = 0; k < 9; k++) o[k * N] = cur.E.m[k];
        o[9 * N] = cur.p.x;
        o[10 * N] = cur.p.y;
        o[11 * N] = cur.p.z;
        o[12 * N] = cur.w.x;
        o[13 * N] = cur.w.y;
        o[14 * N] = cur.w.z;
        o[15 * N] = cur.l.x;
        o[16 * N] = cur.l.y;
        o[17 * N] = cur.l.z;
        prev = cur;
    }
}

template <class T>
__global__ void __launch_bounds__(POLICY_BLOCK) kinematics_kernel(const __grid_constant__ PolicyArgs<T> P) {
    const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (w < P.nworld) kinematics_world(P, w);
}

__device__ __forceinline__ float wrap_pi(float a) {
    const float PI_F = 3.14159265358979323846f;
    while (a > PI_F) a -= 2.0f * PI_F;
    while (a < -PI_F) a += 2.0f * PI_F;
    return a;
}

// Readout element k of body b as float (the reference's readout is f32).
template <class T>
__device__ __forceinline__ float xfv(const PolicyArgs<T>& P, long long w, int b, int k) {
    return (float)reinterpret_cast<const T*>(P.xf)[((long long)b * XF_STRIDE + k) * P.nworld + w];
}
// A body-frame point in world coordinates (double, as phyz_kernels.cu:1506-1511).
template <class T>
__device__ __forceinline__ void point_world(const PolicyArgs<T>& P, long long w, int b, float ox, float oy, float oz,
                                            double* px, double* py, double* pz) {
    float r[12];
#pragma unroll
    for (int k = 0; k < 12; k++) r[k] = xfv(P, w, b, k);
    *px = (double)r[9] + (double)(r[0] * ox + r[3] * oy + r[6] * oz);
    *py = (double)r[10] + (double)(r[1] * ox + r[4] * oy + r[7] * oz);
    *pz = (double)r[11] + (double)(r[2] * ox + r[5] * oy + r[8] * oz);
}

// Observation feature k (phyz_kernels.cu:1477-1576, policy_pipeline.rs ObsOp).
template <class T>
__device__ float obs_feature(const PolicyArgs<T>& P, long long w, int k) {
    const long long N = P.nworld;
    const float* op = P.ops + k * OBS_OP_STRIDE;
    const int kind = (int)op[0];
    const int a = (int)op[1];
    const int b = (int)op[2];
    const float c = op[3];
    switch (kind) {
        case 0: return c;
        case 1: return (float)P.q[(long long)a * N + w] - c;
        case 2: return (float)P.v[(long long)a * N + w];
        case 3: return atan2f(-xfv(P, w, a, 2), xfv(P, w, a, 8));
        case 4: return atan2f(xfv(P, w, a, 5), xfv(P, w, a, 8));
        case 5: return wrap_pi(c - atan2f(xfv(P, w, a, 1), xfv(P, w, a, 0)));
        case 6: return xfv(P, w, a, 11);
        case 7: return xfv(P, w, a, 9 + (b > 2 ? 2 : b));
        case 8: {
            const int n_sup = b;
            if (n_sup <= 0) return 0.0f;
            double cx = 0.0, cy = 0.0, cz = 0.0, mtot = 0.0;
            for (int i = 0; i < P.nb; i++) {
                const float m = P.com[i * 4];
                if (m <= 0.0f) continue;
                double px, py, pz;
                point_world(P, w, i, P.com[i * 4 + 1], P.com[i * 4 + 2], P.com[i * 4 + 3], &px, &py, &pz);
                cx += (double)m * px;
                cy += (double)m * py;
                cz += (double)m * pz;
                mtot += (double)m;
            }
            if (mtot > 0.0) {
                cx /= mtot;
                cy /= mtot;
                cz /= mtot;
            } else {
                cx = cy = cz = 0.0;
            }
            double tx = 0.0, ty = 0.0, tz = 0.0;
            for (int i = 0; i < n_sup; i++) {
                const float* sp = P.aux + a + 2 + i * 4;
                double px, py, pz;
                point_world(P, w, (int)sp[0], sp[1], sp[2], sp[3], &px, &py, &pz);
                tx += px;
                ty += py;
                tz += pz;
            }
            const double inv = 1.0 / (double)n_sup;
            const double ex = cx - tx * inv, ey = cy - ty * inv, ez = cz - tz * inv;
            const int axis = (int)c;
            if (P.aux[a] != 0.0f) {
                const int hb = (int)P.aux[a + 1];
                const double yaw = atan2((double)xfv(P, w, hb, 1), (double)xfv(P, w, hb, 0));
                const double sy = sin(yaw), cyw = cos(yaw);
                if (axis == 0) return (float)(cyw * ex + sy * ey);
                if (axis == 1) return (float)(-sy * ex + cyw * ey);
                return (float)ez;
            }
            return (float)(axis == 0 ? ex : (axis == 1 ? ey : ez));
        }
        default: return 0.0f;
    }
}

// phyz's per-world stream: xorshift64, uniform = (x >> 11) / 2^53, normal by
// Box-Muller in double (phyz_kernels.cu:1612-1640).
__device__ __forceinline__ double rng_uniform(unsigned long long& x) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return (double)(x >> 11) / 9007199254740992.0;
}
__device__ __forceinline__ double rng_normal(unsigned long long& x) {
    double u1 = rng_uniform(x);
    const double u2 = rng_uniform(x);
    if (u1 < 1e-300) u1 = 1e-300;
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586476925286766559 * u2);
}

template <class T>
__global__ void __launch_bounds__(POLICY_BLOCK) policy_kernel(const __grid_constant__ PolicyArgs<T> P) {
    extern __shared__ __align__(16) float sm[];
    stage_weights(P.w, P.n_wf, sm);
    const float* W1 = sm;
    const float* b1 = W1 + P.in_pad * P.h_pad;
    const float* W2 = b1 + P.h_pad;
    const float* b2 = W2 + P.h_pad * P.h_pad;
    const float* W3 = b2 + P.h_pad;
    const float* b3 = W3 + P.h_pad * P.out_pad;

    const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= P.nworld) return;
    const long long N = P.nworld;

    kinematics_world(P, w);
    unsigned long long r = P.rng[w];
    float* xo = P.obs + w;  // the observation row, as recorded (noise included)
    for (int k = 0; k < P.n_in; k++) {
        float xk = obs_feature(P, w, k);
        const float sc = P.in_noise[k];
        if (sc != 0.0f) xk += sc * (float)rng_normal(r);
        xo[(long long)k * N] = xk;
    }
    const int n_in = P.n_in;
    float* h1 = P.h + w;
    float* h2 = P.h + (long long)P.h_pad * N + w;
    dense_tiles(W1, b1, P.in_pad, P.h_pad, [&](int i) { return i < n_in ? xo[(long long)i * N] : 0.0f; },
                [&](int j, float a) { h1[(long long)j * N] = tanhf(a); });
    dense_tiles(W2, b2, P.h_pad, P.h_pad, [&](int i) { return h1[(long long)i * N]; },
                [&](int j, float a) { h2[(long long)j * N] = tanhf(a); });
    // the action means stay in registers (out_pad is one tile)
    float mean[POLICY_TILE];
#pragma unroll
    for (int k = 0; k < POLICY_TILE; k++) mean[k] = b3[k];
    for (int i = 0; i < P.h_pad; i++) {
        const float xi = h2[(long long)i * N];
        const float4* wr = reinterpret_cast<const float4*>(W3 + i * P.out_pad);
#pragma unroll
        for (int k4 = 0; k4 < POLICY_TILE / 4; k4++) {
            const float4 wv = wr[k4];
            mean[4 * k4 + 0] = fmaf(wv.x, xi, mean[4 * k4 + 0]);
            mean[4 * k4 + 1] = fmaf(wv.y, xi, mean[4 * k4 + 1]);
            mean[4 * k4 + 2] = fmaf(wv.z, xi, mean[4 * k4 + 2]);
            mean[4 * k4 + 3] = fmaf(wv.w, xi, mean[4 * k4 + 3]);
        }
    }

    // every servo tracks its base target; actions add onto their slots
    for (int j = 0; j < P.npd; j++) P.targets[(long long)j * N + w] = P.base[(long long)j * N + w];
    const float keep = sqrtf(fmaxf(0.0f, 1.0f - P.rho * P.rho));
    const float LN_2PI = 1.8378770664093453f;
    float logp = 0.0f;
#pragma unroll
    for (int k = 0; k < POLICY_TILE; k++) {
        if (k >= P.n_out) break;
        const float m = mean[k];
        const float zk = P.rho * P.z[(long long)k * N + w] + keep * (float)rng_normal(r);
        P.z[(long long)k * N + w] = zk;
        const float sd = P.stdv[k];
        const float act = m + sd * zk;
        const float zi = (act - m) / sd;
        logp += -0.5f * zi * zi - logf(sd) - 0.5f * LN_2PI;
        P.out[(long long)k * N + w] = act;
        const int slot = P.act_slots[k];
        const float lim = P.clamp[k];
        const float applied = fminf(fmaxf(act, -lim), lim);
        P.targets[(long long)slot * N + w] = P.base[(long long)slot * N + w] + (T)applied;
    }
    P.out[(long long)P.n_out * N + w] = logp;
    P.rng[w] = r;
}

}  // namespace

template <class T>
cudaError_t launch_kinematics(const PolicyArgs<T>& a, cudaStream_t s) {
    if (a.nworld <= 0) return cudaSuccess;
    const unsigned grid = (unsigned)((a.nworld + POLICY_BLOCK - 1) / POLICY_BLOCK);
    kinematics_kernel<T><<<grid, POLICY_BLOCK, 0, s>>>(a);
    return cudaGetLastError();
}

template <class T>
cudaError_t launch_policy(const PolicyArgs<T>& a, cudaStream_t s) {
    if (a.nworld <= 0) return cudaSuccess;
    const int smem = a.n_wf * (int)sizeof(float);  // the weights; a world's rows live in HBM
    cudaError_t e = cudaFuncSetAttribute(policy_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)((a.nworld + POLICY_BLOCK - 1) / POLICY_BLOCK);
    policy_kernel<T><<<grid, POLICY_BLOCK, smem, s>>>(a);
    return cudaGetLastError();
}

template cudaError_t launch_kinematics<float>(const PolicyArgs<float>&, cudaStream_t);
template cudaError_t launch_kinematics<double>(const PolicyArgs<double>&, cudaStream_t);
template cudaError_t launch_policy<float>(const PolicyArgs<float>&, cudaStream_t);
template cudaError_t launch_policy<double>(const PolicyArgs<double>&, cudaStream_t);

}  // namespace pz
