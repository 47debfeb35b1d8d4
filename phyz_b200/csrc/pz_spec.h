// Source text of a model-specialized rollout kernel.
//
// The generic rollout kernel (stepper_kernels.cuh) reads the packed body
// table from shared memory and loops over bodies whose count, kinds and
// scratch slots it learns at run time. For one packed model this header
// writes a translation unit that defines the same tables as literal
// constants (namespace pz::spec, declared in pz_model.cuh) and includes the
// unchanged kernel source with PZ_SPEC set: every body loop then unrolls,
// the per-body kind dispatch and flag tests fold away, table entries become
// immediates of the instructions that use them, and with the block width
// fixed every scratch slot is an immediate shared-memory offset. The source
// and its operations are the generic kernel's (the compiler may fuse a
// different product of a sum into an FMA once constants fold, so results
// agree to rounding); the runtime compiler (spec.cu) turns the text into a
// kernel for the device in use.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "pz_model.cuh"

namespace pz {

// Exact literal of a table scalar: hexadecimal for finite values, the bit
// pattern for infinities and NaNs.
inline void spec_lit(std::string& o, float x) {
    char b[64];
    if (std::isfinite(x)) {
        std::snprintf(b, sizeof b, "%af", (double)x);
    } else {
        uint32_t u;
        std::memcpy(&u, &x, 4);
        std::snprintf(b, sizeof b, "__int_as_float(0x%08x)", u);
    }
    o += b;
}
inline void spec_lit(std::string& o, double x) {
    char b[64];
    if (std::isfinite(x)) {
        std::snprintf(b, sizeof b, "%a", x);
    } else {
        uint64_t u;
        std::memcpy(&u, &x, 8);
        std::snprintf(b, sizeof b, "__longlong_as_double(0x%016llxll)", (unsigned long long)u);
    }
    o += b;
}

template <class T>
constexpr const char* spec_type_name() {
    return sizeof(T) == 8 ? "double" : "float";
}

// The kernel's name expression, as the runtime compiler resolves it.
template <class T>
std::string spec_kernel_name(int feat, bool tm) {
    return std::string("pz::rollout_kernel<") + spec_type_name<T>() + ", " + std::to_string(feat) + ", " +
           (tm ? "true" : "false") + ">";
}

// The translation unit for the model packed in `blob` (BodyT[nb] at 0,
// BodyI[nb] at off_bi, PdT[npd] at off_pd, int[nv] at off_pdmap), launched
// with blocks of W threads (W worlds per block). `sliced`: the kernel's
// slice-mode loop instead of its tile loop (each build holds one of them).
template <class T>
std::string spec_source(const unsigned char* blob, int off_bi, int off_pd, int off_pdmap, int nb, int nv, int npd,
                        int W, bool sliced = false) {
    const char* tn = spec_type_name<T>();
    std::string o;
    o.reserve(4096 + (size_t)nb * 1536);
    o += "// model-specialized rollout kernel: " + std::to_string(nb) + " bodies, " + std::to_string(nv) +
         " DOFs, " + tn + ", " + std::to_string(W) + " worlds per block\n";
    o += "#define PZ_SPEC 1\n#define PZ_SPEC_NB " + std::to_string(nb) + "\n#define PZ_SPEC_NV " +
         std::to_string(nv) + "\n#define PZ_SPEC_W " + std::to_string(W) + "\n#define PZ_SPEC_SLICED " +
         (sliced ? "1" : "0") + "\n#include \"pz_model.cuh\"\n\nnamespace pz {\nnamespace spec {\n\n";
    // body integer table
    o += "__device__ __forceinline__ BodyI body(int i) {\n    switch (i) {\n";
    for (int i = 0; i < nb; i++) {
        int w[BODYI_WORDS];
        std::memcpy(w, blob + off_bi + (size_t)i * sizeof(BodyI), sizeof w);
        o += "    case " + std::to_string(i) + ": return BodyI{";
        for (int k = 0; k < BODYI_WORDS; k++) o += (k ? ", " : "") + std::to_string(w[k]);
        o += "};\n";
    }
    o += "    default: return BodyI{};\n    }\n}\n\n";
    // body scalar table
    o += std::string("template <>\n__device__ __forceinline__ BodyT<") + tn + "> bodyt<" + tn +
         ">(int i) {\n    switch (i) {\n";
    for (int i = 0; i < nb; i++) {
        T x[BODYT_WORDS];
        std::memcpy(x, blob + (size_t)i * sizeof(BodyT<T>), sizeof x);
        o += "    case " + std::to_string(i) + std::string(": return BodyT<") + tn + ">{";
        for (int k = 0; k < BODYT_WORDS; k++) {
            if (k) o += ", ";
            spec_lit(o, x[k]);
        }
        o += "};\n";
    }
    o += std::string("    default: return BodyT<") + tn + ">{};\n    }\n}\n\n";
    // PD servo tables
    o += "__device__ __forceinline__ int pd_of(int d) {\n    switch (d) {\n";
    for (int d = 0; d < nv; d++) {
        int e;
        std::memcpy(&e, blob + off_pdmap + (size_t)d * sizeof(int), sizeof e);
        if (e >= 0) o += "    case " + std::to_string(d) + ": return " + std::to_string(e) + ";\n";
    }
    o += "    default: return -1;\n    }\n}\n\n";
    o += std::string("template <>\n__device__ __forceinline__ PdT<") + tn + "> pdt<" + tn +
         ">(int k) {\n    switch (k) {\n";
    for (int k = 0; k < npd; k++) {
        PdT<T> e;
        std::memcpy(&e, blob + off_pd + (size_t)k * sizeof(PdT<T>), sizeof e);
        o += "    case " + std::to_string(k) + std::string(": return PdT<") + tn + ">{";
        spec_lit(o, e.kp);
        o += ", ";
        spec_lit(o, e.kd);
        o += ", ";
        spec_lit(o, e.maxf);
        o += ", " + std::to_string(e.qi) + ", " + std::to_string(e.vi) + "};\n";
    }
    o += std::string("    default: return PdT<") + tn + ">{};\n    }\n}\n\n";
    o += "}  // namespace spec\n}  // namespace pz\n\n#include \"stepper_kernels.cuh\"\n";
    return o;
}

}  // namespace pz
