// Spatial-algebra value types of the B200 stepper, in the reduced form the
// kernel computes in:
//
//   * spatial vectors are [angular; linear] (Featherstone order, as phyz's
//     tang::SpatialVec, crates/phyz-math/src/spatial.rs:3-12);
//   * an articulated inertia is kept as its three distinct 3x3 blocks
//     |Ia  H|        Ia, M symmetric (6 entries each), H full (9):
//     |H^T M|        21 numbers instead of phyz's dense 36;
//   * Plücker transforms (tang::SpatialTransform, spatial.rs:24-35) are
//     applied as a rotation E followed by a translation r, never as 6x6
//     matrices: X = [E 0; -E r^x E] (phyz_kernels.cu:180-200 builds the
//     same matrix densely).
//
// Everything is templated on the scalar T: float and double on the device,
// and a counting scalar on the host, which is how the algorithmic flop
// count of a world-step is taken from this exact code.
#pragma once

#if defined(__CUDACC__)
#define PZ_HD __host__ __device__ __forceinline__
#define PZ_OUTLINE __host__ __device__ __noinline__
#else
#define PZ_HD inline
#define PZ_OUTLINE inline
#endif

#if defined(__CUDA_ARCH__) && !defined(__CUDACC_RTC__)
#include <cuda_runtime.h>
#endif

namespace pz {

// ── scalar shims (device versions; the host counting scalar overloads these) ──
#if defined(__CUDA_ARCH__)
__device__ __forceinline__ void pz_sincos(float x, float* s, float* c) { sincosf(x, s, c); }
__device__ __forceinline__ void pz_sincos(double x, double* s, double* c) { sincos(x, s, c); }
__device__ __forceinline__ float pz_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double pz_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float pz_atan2(float y, float x) { return atan2f(y, x); }
__device__ __forceinline__ double pz_atan2(double y, double x) { return atan2(y, x); }
__device__ __forceinline__ float pz_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double pz_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float pz_pow(float x, float y) { return powf(x, y); }
__device__ __forceinline__ double pz_pow(double x, double y) { return pow(x, y); }
__device__ __forceinline__ float pz_abs(float x) { return fabsf(x); }
__device__ __forceinline__ double pz_abs(double x) { return fabs(x); }
__device__ __forceinline__ float pz_min(float a, float b) { return fminf(a, b); }
__device__ __forceinline__ double pz_min(double a, double b) { return fmin(a, b); }
__device__ __forceinline__ float pz_max(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double pz_max(double a, double b) { return fmax(a, b); }
__device__ __forceinline__ bool pz_finite(float x) { return isfinite(x); }
__device__ __forceinline__ bool pz_finite(double x) { return isfinite(x); }
__device__ __forceinline__ int pz_trunc_int(float x) { return (int)x; }
__device__ __forceinline__ int pz_trunc_int(double x) { return (int)x; }
#endif

// Small-angle threshold of the exp/log maps: f64 uses f64::EPSILON like
// crates/phyz-math/src/lib.rs:48,67; f32 uses the 1e-6 of the reference's
// f32 kernels (phyz_kernels.cu:262,292).
// Counting(T): T is the host op-counting scalar (flops.cpp), which tallies
// only algorithmic work. The kernel does some structurally zero work
// unconditionally (a zero offset, a zero spring) because it is cheaper than
// a branch; under counting those terms are skipped.
template <class T> struct Counting { static constexpr bool value = false; };

template <class T> struct Eps;
template <> struct Eps<float> { static constexpr double quat = 1e-6; };
template <> struct Eps<double> { static constexpr double quat = 2.220446049250313e-16; };

// ── 3-vectors ──────────────────────────────────────────────────────────────
template <class T>
struct V3 {
    T x, y, z;
};
template <class T>
PZ_HD V3<T> mk3(T x, T y, T z) {
    V3<T> r;
    r.x = x;
    r.y = y;
    r.z = z;
    return r;
}
template <class T>
PZ_HD V3<T> zero3() {
    return mk3<T>(T(0), T(0), T(0));
}
template <class T>
PZ_HD V3<T> operator+(const V3<T>& a, const V3<T>& b) {
    return mk3<T>(a.x + b.x, a.y + b.y, a.z + b.z);
}
template <class T>
PZ_HD V3<T> operator-(const V3<T>& a, const V3<T>& b) {
    return mk3<T>(a.x - b.x, a.y - b.y, a.z - b.z);
}
template <class T>
PZ_HD V3<T> operator-(const V3<T>& a) {
    return mk3<T>(-a.x, -a.y, -a.z);
}
template <class T>
PZ_HD V3<T> operator*(const V3<T>& a, const T& s) {
    return mk3<T>(a.x * s, a.y * s, a.z * s);
}
template <class T>
PZ_HD T dot(const V3<T>& a, const V3<T>& b) {
    return a.x * b.x + a.y * b.y + a.z * b.z;
}
template <class T>
PZ_HD V3<T> cross(const V3<T>& a, const V3<T>& b) {
    return mk3<T>(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}

// ── products with model-table constants ────────────────────────────────────
// A model table is full of exact zeros (off-diagonal inertias, offsets and
// centres of mass along one axis). In a specialized build the table is
// literal, and a term whose table factor is zero is left out of its sum:
// kzero() is then a compile-time constant per term. The compiler cannot drop
// such a term itself (0 x is not 0 for infinite or NaN x, and x + 0 is not x
// for x = -0), so the sums below start from -0 (-0 + t = t for every t) and
// add their terms conditionally; in the generic build every term is added.
// Leaving a term out changes a result only in the sign of a zero or in NaN
// propagation. PZ_KSKIP makes a host build take the same decisions at run
// time (for checking them against the oracle). The host flop counter's
// scalar (Counting<T>) takes them at run time when its kskip_on() says so,
// to count what a specialized kernel executes.
#if defined(PZ_SPEC) || defined(PZ_KSKIP)
#define PZ_KSKIP_ON 1
#else
#define PZ_KSKIP_ON 0
#endif
template <class T>
PZ_HD bool kzero(const T& k) {
    if constexpr (Counting<T>::value) {
        return Counting<T>::kskip_on() && !(k > T(0) || k < T(0));
    } else {
        if constexpr (PZ_KSKIP_ON != 0) return !(k > T(0) || k < T(0));
        return false;
    }
}
// k x, or -0 when k is a zero table constant (a sum's first term)
template <class T>
PZ_HD T kmul(const T& k, const T& x) {
    return kzero(k) ? T(-0.0) : k * x;
}
template <class T>
PZ_HD T kmadd(const T& acc, const T& k, const T& x) {
    return kzero(k) ? acc : acc + k * x;
}
template <class T>
PZ_HD T kmsub(const T& acc, const T& k, const T& x) {
    return kzero(k) ? acc : acc - k * x;
}
// x + k, x - k for a table constant k
template <class T>
PZ_HD T kadd(const T& x, const T& k) {
    return kzero(k) ? x : x + k;
}
template <class T>
PZ_HD T ksub(const T& x, const T& k) {
    return kzero(k) ? x : x - k;
}
// k x b and a x k with k a table constant
template <class T>
PZ_HD V3<T> kcross(const V3<T>& k, const V3<T>& b) {
    return mk3<T>(kmsub(kmul(k.y, b.z), k.z, b.y), kmsub(kmul(k.z, b.x), k.x, b.z),
                  kmsub(kmul(k.x, b.y), k.y, b.x));
}
template <class T>
PZ_HD V3<T> crossk(const V3<T>& a, const V3<T>& k) {
    return mk3<T>(kmsub(kmul(k.z, a.y), k.y, a.z), kmsub(kmul(k.x, a.z), k.z, a.x),
                  kmsub(kmul(k.y, a.x), k.x, a.y));
}
// H x and H^T x for a row-major 3x3 table matrix H
template <class T>
PZ_HD V3<T> km3v(const T* H, const V3<T>& x) {
    return mk3<T>(kmadd(kmadd(kmul(H[0], x.x), H[1], x.y), H[2], x.z),
                  kmadd(kmadd(kmul(H[3], x.x), H[4], x.y), H[5], x.z),
                  kmadd(kmadd(kmul(H[6], x.x), H[7], x.y), H[8], x.z));
}
template <class T>
PZ_HD V3<T> km3tv(const T* H, const V3<T>& x) {
    return mk3<T>(kmadd(kmadd(kmul(H[0], x.x), H[3], x.y), H[6], x.z),
                  kmadd(kmadd(kmul(H[1], x.x), H[4], x.y), H[7], x.z),
                  kmadd(kmadd(kmul(H[2], x.x), H[5], x.y), H[8], x.z));
}
// A x for a symmetric table matrix A (xx, yy, zz, xy, xz, yz)
template <class T>
PZ_HD V3<T> ksymv(const T* A, const V3<T>& x) {
    return mk3<T>(kmadd(kmadd(kmul(A[0], x.x), A[3], x.y), A[4], x.z),
                  kmadd(kmadd(kmul(A[3], x.x), A[1], x.y), A[5], x.z),
                  kmadd(kmadd(kmul(A[4], x.x), A[5], x.y), A[2], x.z));
}
template <class T>
PZ_HD T get(const V3<T>& a, int i) {
    return i == 0 ? a.x : (i == 1 ? a.y : a.z);
}
template <int I, class T>
PZ_HD T& at(V3<T>& a) {
    return I == 0 ? a.x : (I == 1 ? a.y : a.z);
}
template <int I, class T>
PZ_HD const T& at(const V3<T>& a) {
    return I == 0 ? a.x : (I == 1 ? a.y : a.z);
}

// ── spatial vectors [angular; linear] ─────────────────────────────────────
template <class T>
struct SV {
    V3<T> w, l;
};
template <class T>
PZ_HD SV<T> mksv(const V3<T>& w, const V3<T>& l) {
    SV<T> r;
    r.w = w;
    r.l = l;
    return r;
}
template <class T>
PZ_HD SV<T> zerosv() {
    return mksv<T>(zero3<T>(), zero3<T>());
}
template <class T>
PZ_HD SV<T> operator+(const SV<T>& a, const SV<T>& b) {
    return mksv<T>(a.w + b.w, a.l + b.l);
}
template <class T>
PZ_HD SV<T> operator-(const SV<T>& a, const SV<T>& b) {
    return mksv<T>(a.w - b.w, a.l - b.l);
}
template <class T>
PZ_HD T dot(const SV<T>& a, const SV<T>& b) {
    return dot(a.w, b.w) + dot(a.l, b.l);
}
// motion cross v x m (phyz_kernels.cu:110-116)
template <class T>
PZ_HD SV<T> crm(const SV<T>& v, const SV<T>& m) {
    return mksv<T>(cross(v.w, m.w), cross(v.w, m.l) + cross(v.l, m.w));
}
// force cross v x* f (phyz_kernels.cu:118-124)
template <class T>
PZ_HD SV<T> crf(const SV<T>& v, const SV<T>& f) {
    return mksv<T>(cross(v.w, f.w) + cross(v.l, f.l), cross(v.w, f.l));
}
template <class T>
PZ_HD T svget(const SV<T>& a, int i) {
    return i < 3 ? get(a.w, i) : get(a.l, i - 3);
}

// symmetric 3x3 packed as xx, yy, zz, xy, xz, yz
PZ_HD constexpr int sidx(int i, int j) {
    return i == j ? i : (i + j == 1 ? 3 : (i + j == 2 ? 4 : 5));
}

// ── articulated inertia in three blocks ────────────────────────────────────
template <class T>
struct AI {
    T a[6];  // angular-angular (symmetric)
    T h[9];  // angular-linear, row-major
    T m[6];  // linear-linear (symmetric)
};

template <class T>
PZ_HD void ai_zero(AI<T>& I) {
#pragma unroll
    for (int k = 0; k < 6; k++) I.a[k] = T(0), I.m[k] = T(0);
#pragma unroll
    for (int k = 0; k < 9; k++) I.h[k] = T(0);
}
template <class T>
PZ_HD void ai_add(AI<T>& I, const AI<T>& B) {
#pragma unroll
    for (int k = 0; k < 6; k++) I.a[k] = I.a[k] + B.a[k], I.m[k] = I.m[k] + B.m[k];
#pragma unroll
    for (int k = 0; k < 9; k++) I.h[k] = I.h[k] + B.h[k];
}
template <class T>
PZ_HD V3<T> symv(const T* A, const V3<T>& x) {
    return mk3<T>(A[0] * x.x + A[3] * x.y + A[4] * x.z, A[3] * x.x + A[1] * x.y + A[5] * x.z,
                  A[4] * x.x + A[5] * x.y + A[2] * x.z);
}
template <class T>
PZ_HD V3<T> m3v(const T* H, const V3<T>& x) {
    return mk3<T>(H[0] * x.x + H[1] * x.y + H[2] * x.z, H[3] * x.x + H[4] * x.y + H[5] * x.z,
                  H[6] * x.x + H[7] * x.y + H[8] * x.z);
}
template <class T>
PZ_HD V3<T> m3tv(const T* H, const V3<T>& x) {
    return mk3<T>(H[0] * x.x + H[3] * x.y + H[6] * x.z, H[1] * x.x + H[4] * x.y + H[7] * x.z,
                  H[2] * x.x + H[5] * x.y + H[8] * x.z);
}
// I v = [Ia w + H l; H^T w + M l]
template <class T>
PZ_HD SV<T> ai_mul(const AI<T>& I, const SV<T>& v) {
    return mksv<T>(symv(I.a, v.w) + m3v(I.h, v.l), m3tv(I.h, v.w) + symv(I.m, v.l));
}

// ── transforms ─────────────────────────────────────────────────────────────
// A rotation E as a row-major 3x3.
template <class T>
struct R3 {
    T m[9];
};
template <class T>
PZ_HD V3<T> rmul(const R3<T>& E, const V3<T>& x) {
    return m3v(E.m, x);
}
template <class T>
PZ_HD V3<T> rtmul(const R3<T>& E, const V3<T>& x) {
    return m3tv(E.m, x);
}

// apply_motion with E, r: [E w; E (l - r x w)] (phyz_kernels.cu:314-320)
template <class T>
PZ_HD SV<T> xm_apply(const R3<T>& E, const V3<T>& r, const SV<T>& m) {
    return mksv<T>(rmul(E, m.w), rmul(E, m.l - cross(r, m.w)));
}
template <class T>
PZ_HD SV<T> xm_apply_rot(const R3<T>& E, const SV<T>& m) {
    return mksv<T>(rmul(E, m.w), rmul(E, m.l));
}
template <class T>
PZ_HD SV<T> xm_apply_trans(const V3<T>& r, const SV<T>& m) {
    return mksv<T>(m.w, m.l - cross(r, m.w));
}
// inv_apply_force: X^T f = [E^T t + r x E^T f; E^T f] (phyz_kernels.cu:322-329)
template <class T>
PZ_HD SV<T> xf_tapply_rot(const R3<T>& E, const SV<T>& f) {
    return mksv<T>(rtmul(E, f.w), rtmul(E, f.l));
}
template <class T>
PZ_HD SV<T> xf_tapply_trans(const V3<T>& r, const SV<T>& f) {
    return mksv<T>(f.w + cross(r, f.l), f.l);
}
// The same two translations by a table constant r (a specialized build
// forms l - r x w as l + w x r, so that left-out terms are -0 added; the
// generic build keeps the original expression)
template <class T>
PZ_HD SV<T> kxm_apply_trans(const V3<T>& r, const SV<T>& m) {
#if PZ_KSKIP_ON
    return mksv<T>(m.w, m.l + crossk(m.w, r));
#else
    if constexpr (Counting<T>::value)
        if (Counting<T>::kskip_on()) return mksv<T>(m.w, m.l + crossk(m.w, r));
    return xm_apply_trans(r, m);
#endif
}
template <class T>
PZ_HD SV<T> kxf_tapply_trans(const V3<T>& r, const SV<T>& f) {
    return mksv<T>(f.w + kcross(r, f.l), f.l);
}

// Planar rotation about the coordinate axis K by the angle whose cosine
// and sine are (c, s): E e_i = c e_i + s e_j, E e_j = -s e_i + c e_j with
// (i, j, K) cyclic. This is revolute_rot of a unit coordinate axis
// (phyz_kernels.cu:245-256 / joint.rs:259-266).
template <int K, class T>
PZ_HD V3<T> prot(const T& c, const T& s, const V3<T>& x) {
    constexpr int I = (K + 1) % 3, J = (K + 2) % 3;
    V3<T> r = x;
    at<I>(r) = c * at<I>(x) - s * at<J>(x);
    at<J>(r) = s * at<I>(x) + c * at<J>(x);
    return r;
}
template <int K, class T>
PZ_HD V3<T> prot_t(const T& c, const T& s, const V3<T>& x) {
    constexpr int I = (K + 1) % 3, J = (K + 2) % 3;
    V3<T> r = x;
    at<I>(r) = c * at<I>(x) + s * at<J>(x);
    at<J>(r) = -s * at<I>(x) + c * at<J>(x);
    return r;
}

// Inertia congruence by a rotation: I <- X^T I X for X = [E 0; 0 E]:
// Ia <- E^T Ia E, H <- E^T H E, M <- E^T M E.
template <class T>
PZ_HD void sym_rot(const R3<T>& E, T* A) {
    // B = A E (full), A' = E^T B (symmetric part)
    T B[9];
#pragma unroll
    for (int i = 0; i < 3; i++)
#pragma unroll
        for (int j = 0; j < 3; j++)
            B[i * 3 + j] = A[sidx(i, 0)] * E.m[0 * 3 + j] + A[sidx(i, 1)] * E.m[1 * 3 + j] +
                           A[sidx(i, 2)] * E.m[2 * 3 + j];
#pragma unroll
    for (int i = 0; i < 3; i++)
#pragma unroll
        for (int j = i; j < 3; j++)
            A[sidx(i, j)] = E.m[0 * 3 + i] * B[0 * 3 + j] + E.m[1 * 3 + i] * B[1 * 3 + j] +
                            E.m[2 * 3 + i] * B[2 * 3 + j];
}
template <class T>
PZ_HD void full_rot(const R3<T>& E, T* H) {
    T B[9];
#pragma unroll
    for (int i = 0; i < 3; i++)
#pragma unroll
        for (int j = 0; j < 3; j++)
            B[i * 3 + j] =
                H[i * 3 + 0] * E.m[0 * 3 + j] + H[i * 3 + 1] * E.m[1 * 3 + j] + H[i * 3 + 2] * E.m[2 * 3 + j];
#pragma unroll
    for (int i = 0; i < 3; i++)
#pragma unroll
        for (int j = 0; j < 3; j++)
            H[i * 3 + j] =
                E.m[0 * 3 + i] * B[0 * 3 + j] + E.m[1 * 3 + i] * B[1 * 3 + j] + E.m[2 * 3 + i] * B[2 * 3 + j];
}
template <class T>
PZ_HD void ai_rot(const R3<T>& E, AI<T>& I) {
    sym_rot(E, I.a);
    full_rot(E, I.h);
    sym_rot(E, I.m);
}

// Planar versions of the same congruence (rotation about axis K).
template <int K, class T>
PZ_HD void sym_prot(const T& c, const T& s, const T& cc, const T& ss, const T& cs, T* A) {
    constexpr int I = (K + 1) % 3, J = (K + 2) % 3;
    const T aii = A[sidx(I, I)], ajj = A[sidx(J, J)], aij = A[sidx(I, J)];
    const T aik = A[sidx(I, K)], ajk = A[sidx(J, K)];
    const T two_cs_aij = (cs + cs) * aij;
    A[sidx(I, I)] = cc * aii + two_cs_aij + ss * ajj;
    A[sidx(J, J)] = ss * aii - two_cs_aij + cc * ajj;
    A[sidx(I, J)] = cs * (ajj - aii) + (cc - ss) * aij;
    A[sidx(I, K)] = c * aik + s * ajk;
    A[sidx(J, K)] = c * ajk - s * aik;
}
template <int K, class T>
PZ_HD void full_prot(const T& c, const T& s, T* H) {
    constexpr int I = (K + 1) % 3, J = (K + 2) % 3;
    // columns: B = H E
#pragma unroll
    for (int r = 0; r < 3; r++) {
        const T hi = H[r * 3 + I], hj = H[r * 3 + J];
        H[r * 3 + I] = c * hi + s * hj;
        H[r * 3 + J] = c * hj - s * hi;
    }
    // rows: H' = E^T B
#pragma unroll
    for (int q = 0; q < 3; q++) {
        const T hi = H[I * 3 + q], hj = H[J * 3 + q];
        H[I * 3 + q] = c * hi + s * hj;
        H[J * 3 + q] = c * hj - s * hi;
    }
}
template <int K, class T>
PZ_HD void ai_prot(const T& c, const T& s, AI<T>& I) {
    const T cc = c * c, ss = s * s, cs = c * s;
    sym_prot<K>(c, s, cc, ss, cs, I.a);
    full_prot<K>(c, s, I.h);
    sym_prot<K>(c, s, cc, ss, cs, I.m);
}

// Inertia congruence by a translation r (X = [1 0; -r^x 1]):
//   M' = M, H' = H + r^x M, Ia' = Ia - Z - Z^T - (r^x M) r^x with Z = H r^x.
// Row i of (A r^x) is (row i of A) x r; column j of (r^x M) is r x M e_j.
template <class T>
PZ_HD void ai_trans(const V3<T>& r, AI<T>& I) {
    // T1 = r^x M (full), columns r x M_col
    T t1[9];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        V3<T> col = mk3<T>(I.m[sidx(0, j)], I.m[sidx(1, j)], I.m[sidx(2, j)]);
        V3<T> rc = cross(r, col);
        t1[0 * 3 + j] = rc.x;
        t1[1 * 3 + j] = rc.y;
        t1[2 * 3 + j] = rc.z;
    }
    // Z = H r^x (rows of H crossed with r)
    T z[9];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        V3<T> row = mk3<T>(I.h[i * 3 + 0], I.h[i * 3 + 1], I.h[i * 3 + 2]);
        V3<T> rr = cross(row, r);
        z[i * 3 + 0] = rr.x;
        z[i * 3 + 1] = rr.y;
        z[i * 3 + 2] = rr.z;
    }
    // W = T1 r^x (symmetric): rows of T1 crossed with r
#pragma unroll
    for (int i = 0; i < 3; i++) {
        V3<T> row = mk3<T>(t1[i * 3 + 0], t1[i * 3 + 1], t1[i * 3 + 2]);
        V3<T> w = cross(row, r);
#pragma unroll
        for (int j = i; j < 3; j++) {
            const T wij = get(w, j);
            I.a[sidx(i, j)] = I.a[sidx(i, j)] - z[i * 3 + j] - z[j * 3 + i] - wij;
        }
    }
#pragma unroll
    for (int k = 0; k < 9; k++) I.h[k] = I.h[k] + t1[k];
}
// ai_trans by a table constant r, every product with r through the k
// helpers: Ia' = Ia + Y + Y^T + V with Y = -(H r^x) (rows r x H_row) and
// V = -(T1 r^x) (rows r x T1_row), so that a left-out term is a -0 added.
template <class T>
PZ_HD void kai_trans_skip(const V3<T>& r, AI<T>& I) {
    T t1[9];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const V3<T> rc = kcross(r, mk3<T>(I.m[sidx(0, j)], I.m[sidx(1, j)], I.m[sidx(2, j)]));
        t1[0 * 3 + j] = rc.x;
        t1[1 * 3 + j] = rc.y;
        t1[2 * 3 + j] = rc.z;
    }
    T y[9];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const V3<T> rr = kcross(r, mk3<T>(I.h[i * 3 + 0], I.h[i * 3 + 1], I.h[i * 3 + 2]));
        y[i * 3 + 0] = rr.x;
        y[i * 3 + 1] = rr.y;
        y[i * 3 + 2] = rr.z;
    }
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const V3<T> w = kcross(r, mk3<T>(t1[i * 3 + 0], t1[i * 3 + 1], t1[i * 3 + 2]));
#pragma unroll
        for (int j = i; j < 3; j++) I.a[sidx(i, j)] = I.a[sidx(i, j)] + y[i * 3 + j] + y[j * 3 + i] + get(w, j);
    }
#pragma unroll
    for (int k = 0; k < 9; k++) I.h[k] = I.h[k] + t1[k];
}
template <class T>
PZ_HD void kai_trans(const V3<T>& r, AI<T>& I) {
#if PZ_KSKIP_ON
    kai_trans_skip(r, I);
#else
    if constexpr (Counting<T>::value) {
        if (Counting<T>::kskip_on()) {
            kai_trans_skip(r, I);
            return;
        }
    }
    ai_trans(r, I);  // the generic build: the original expression order
#endif
}

}  // namespace pz
