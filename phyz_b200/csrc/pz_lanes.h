// Splitting one world over several threads ("lanes") for branching trees.
//
// The trunk is every body whose subtree holds two or more leaves; a limb is
// a chain hanging off the trunk (or off the world). Lane l steps its own
// sub-model: the whole trunk, in the model's order, then the limbs it is
// given. Every lane runs the trunk (the same values on every lane); the
// limbs run in parallel. The only exchange is in the backward sweep: once
// every lane has swept its limbs, the articulated inertias and bias forces
// its limbs passed to trunk bodies are summed over the lanes (warp shuffles)
// and every lane finishes the trunk with the sums. Forward sweeps need
// nothing: each lane holds the trunk's state.
//
// The planner below builds the sub-models; pack_model packs each of them
// with the trunk bodies' flags made the same on every lane (branch slots for
// every trunk body any lane's limb hangs off; the chain flag on the last
// trunk body if any lane's first limb continues it), so the lanes run the
// trunk through identical code.
#pragma once

#include <algorithm>
#include <string>
#include <vector>

#include "pz_pack.h"

namespace pz {

struct LanePlan {
    int lanes = 0;
    int nt = 0;                                  // trunk bodies (first nt of every sub-model)
    std::vector<std::vector<int>> bodies;        // per lane: model body index of each sub-model body
    std::vector<std::vector<phyzb_body>> sub;    // per lane: the sub-model's bodies (parents renumbered)
    std::vector<std::vector<int>> dof;           // per lane: model DOF of each sub-model DOF
    std::vector<int> force_branch;               // sub-model indices (trunk), the same on every lane
    int force_chain = -1;
};

// Split `m` over `lanes` threads. Returns "" or why the model does not split
// (no branching: a chain is one limb).
inline std::string plan_lanes(const phyzb_model* m, int lanes, LanePlan* out) {
    const int nb = m->nbodies;
    if (lanes < 2) return "fewer than two lanes";
    std::vector<std::vector<int>> kids(nb);
    for (int i = 0; i < nb; i++)
        if (m->bodies[i].parent >= 0) kids[m->bodies[i].parent].push_back(i);
    std::vector<int> leaves(nb, 0);
    for (int i = nb - 1; i >= 0; i--) {
        if (kids[i].empty()) leaves[i] = 1;
        for (int c : kids[i]) leaves[i] += leaves[c];
    }
    std::vector<char> trunk(nb, 0);
    int nt = 0;
    for (int i = 0; i < nb; i++)
        if (leaves[i] >= 2) {
            trunk[i] = 1;
            nt++;
        }
    if (nt == 0) return "the model does not branch (a chain has one limb)";
    // limbs: chains whose first body hangs off the trunk or the world
    std::vector<std::vector<int>> limbs;
    for (int i = 0; i < nb; i++) {
        const int p = m->bodies[i].parent;
        if (trunk[i] || (p >= 0 && !trunk[p])) continue;
        std::vector<int> chain{i};
        while (!kids[chain.back()].empty()) chain.push_back(kids[chain.back()][0]);
        limbs.push_back(chain);
    }
    // the largest limbs first, each to the lane with the fewest DOFs so far
    auto dofs = [&](const std::vector<int>& c) {
        int n = 0;
        for (int b : c) n += ndof_of(m->bodies[b].joint_type);
        return n;
    };
    std::stable_sort(limbs.begin(), limbs.end(),
                     [&](const std::vector<int>& a, const std::vector<int>& b) { return dofs(a) > dofs(b); });
    std::vector<std::vector<int>> own(lanes);
    std::vector<int> load(lanes, 0);
    for (const auto& c : limbs) {
        const int l = (int)(std::min_element(load.begin(), load.end()) - load.begin());
        for (int b : c) own[l].push_back(b);
        load[l] += dofs(c);
    }
    std::vector<int> gdof(nb + 1, 0);
    for (int i = 0; i < nb; i++) gdof[i + 1] = gdof[i] + ndof_of(m->bodies[i].joint_type);

    LanePlan P;
    P.lanes = lanes;
    P.nt = nt;
    P.bodies.resize(lanes);
    P.sub.resize(lanes);
    P.dof.resize(lanes);
    std::vector<char> branch(nt, 0);
    bool chain = false;
    for (int l = 0; l < lanes; l++) {
        std::vector<int>& order = P.bodies[l];
        for (int i = 0; i < nb; i++)
            if (trunk[i]) order.push_back(i);
        std::sort(own[l].begin(), own[l].end());  // model order keeps parents first within a lane
        order.insert(order.end(), own[l].begin(), own[l].end());
        std::vector<int> at(nb, -1);
        for (int k = 0; k < (int)order.size(); k++) at[order[k]] = k;
        for (int k = 0; k < (int)order.size(); k++) {
            phyzb_body b = m->bodies[order[k]];
            b.parent = b.parent >= 0 ? at[b.parent] : -1;
            P.sub[l].push_back(b);
            for (int d = gdof[order[k]]; d < gdof[order[k] + 1]; d++) P.dof[l].push_back(d);
        }
        // the trunk's flags as this lane's sub-model would set them
        const int n = (int)order.size();
        for (int t = 0; t < nt; t++)
            for (int j = t + 2; j < n; j++)
                if (P.sub[l][j].parent == t) branch[t] = 1;
        if (n > nt && P.sub[l][nt].parent == nt - 1) chain = true;
    }
    for (int t = 0; t < nt; t++)
        if (branch[t]) P.force_branch.push_back(t);
    P.force_chain = chain ? nt - 1 : -1;
    *out = std::move(P);
    return "";
}

}  // namespace pz
