// Host helper for tests/test_spec_compile.py: the model-specialized rollout
// kernel's source for a packed model (pz_spec.h), without a GPU.
#include <cstring>
#include <string>
#include <vector>

#include "pz_pack.h"
#include "pz_spec.h"

// contact: 0 none, 1 penalty, 2 impulse; sliced: the slice-mode twin. Writes
// the source (NUL-terminated) and the kernel's name expression; returns the
// source length, or -needed when a buffer is too small.
extern "C" int spec_source_for(const phyzb_model* m, int nv, int contact, int f64, int W, int sliced, char* src,
                               int src_cap, char* name, int name_cap) {
    pz::PackCfg cfg;
    cfg.contact = contact != 0;
    cfg.impulse = contact == 2;
    cfg.gk.assign(m->nbodies, 1e4);
    cfg.gd.assign(m->nbodies, 100.0);
    std::vector<unsigned char> blob;
    const pz::PackInfo info =
        f64 ? pz::pack_model<double>(m, nv, cfg, blob, 0) : pz::pack_model<float>(m, nv, cfg, blob, 0);
    const std::string s = f64 ? pz::spec_source<double>(blob.data(), info.off_bi, info.off_pd, info.off_pdmap,
                                                        m->nbodies, nv, 0, W, sliced != 0)
                              : pz::spec_source<float>(blob.data(), info.off_bi, info.off_pd, info.off_pdmap,
                                                       m->nbodies, nv, 0, W, sliced != 0);
    const std::string k = f64 ? pz::spec_kernel_name<double>(info.feat, false)
                              : pz::spec_kernel_name<float>(info.feat, false);
    if ((int)s.size() + 1 > src_cap || (int)k.size() + 1 > name_cap) return -(int)(s.size() + k.size() + 2);
    std::memcpy(src, s.c_str(), s.size() + 1);
    std::memcpy(name, k.c_str(), k.size() + 1);
    return (int)s.size();
}
