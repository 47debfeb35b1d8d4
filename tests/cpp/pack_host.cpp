// Host harness for tests/test_pack_tmem.py: the scratch layout pz_pack.h
// gives a model, with and without a Tensor-Memory budget.
#include <vector>

#include "pz_pack.h"

// contact: 0 none, 1 penalty, 2 impulse. out: [scratch words per world,
// Tensor-Memory columns, bodies whose wrench is a Tensor-Memory record,
// bodies whose wrench has shared-memory slots, hinge records in Tensor
// Memory, the largest column any record reaches].
extern "C" void pack_host(const phyzb_model* m, int nv, int contact, int plane_body, int f64, int budget, int* out) {
    pz::PackCfg cfg;
    cfg.contact = contact != 0;
    cfg.impulse = contact == 2;
    cfg.plane_body = plane_body;
    cfg.terrain = plane_body >= 0;
    cfg.gk.assign(m->nbodies, 1e4);
    cfg.gd.assign(m->nbodies, 100.0);
    std::vector<unsigned char> blob;
    const pz::PackInfo info =
        f64 ? pz::pack_model<double>(m, nv, cfg, blob, budget) : pz::pack_model<float>(m, nv, cfg, blob, budget);
    const pz::BodyI* bi = reinterpret_cast<const pz::BodyI*>(blob.data() + info.off_bi);
    const int rec = f64 ? 16 : 8;
    int tf = 0, sf = 0, trec = 0, top = 0;
    for (int i = 0; i < m->nbodies; i++) {
        if (bi[i].t_f >= 0) {
            tf++;
            top = bi[i].t_f + rec > top ? bi[i].t_f + rec : top;
        }
        if (bi[i].s_f >= 0) sf++;
        if (bi[i].t_rec >= 0) {
            trec++;
            top = bi[i].t_rec + rec > top ? bi[i].t_rec + rec : top;
        }
    }
    const int v[6] = {info.scratch, info.tmem_cols, tf, sf, trec, top};
    for (int k = 0; k < 6; k++) out[k] = v[k];
}
