// The two halves of a lane's backward sweep (stepper_lanes.cuh): first its
// limbs, then -- once the limbs' contributions to trunk bodies have been
// summed over the lanes -- the trunk. Host-compilable, so the host test of
// the split (tests/cpp/lanes_host.cpp) runs the same sweep code.
#pragma once

#include "pz_world.cuh"

namespace pz {

// Zero the branch accumulators and sweep the limbs (bodies nt .. nb-1). On
// return the carry (I, pA) holds what the lane's first limb body passes to
// the last trunk body, or zero when that body is not its parent.
template <int FEAT, class T, class Scr>
PZ_HD void pass2_limbs(const ModelView<T>& M, const Scr& S, int nt, AI<T>& I, SV<T>& pA) {
    for (int i = 0; i < M.nb; i++) {
        const BodyI bi = M.bi[i];
        if (bi.flags & F_BRANCH)
            for (int k = 0; k < 27; k++) S(bi.s_acc + k) = T(0);
    }
    pA = zerosv<T>();
    ai_zero(I);
    for (int i = M.nb - 1; i >= nt; i--) {
        const BodyI bi = M.bi[i];
#define PZ_P2(AX) pass2_body<AX, FEAT>(M, S, i, bi, I, pA)
        PZ_BY_KIND(body_kind(bi), PZ_P2)
#undef PZ_P2
    }
    if (!(M.nb > nt && M.bi[nt].parent == nt - 1)) {
        ai_zero(I);
        pA = zerosv<T>();
    }
}

// Sweep the trunk (bodies nt-1 .. 0) from the summed carry and accumulators.
template <int FEAT, class T, class Scr>
PZ_HD void pass2_trunk(const ModelView<T>& M, const Scr& S, int nt, AI<T>& I, SV<T>& pA) {
    for (int i = nt - 1; i >= 0; i--) {
        const BodyI bi = M.bi[i];
#define PZ_P2(AX) pass2_body<AX, FEAT>(M, S, i, bi, I, pA)
        PZ_BY_KIND(body_kind(bi), PZ_P2)
#undef PZ_P2
    }
}

}  // namespace pz
