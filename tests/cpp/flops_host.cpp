// The flop counter of the library (phyz_b200/csrc/flops.cpp) built for the
// host with a C shim, so tests/test_flops.py can check its counts without a
// GPU: the generic and the executed (specialized) counts, with the contact
// force law where bodies touch the ground.
#include "../../phyz_b200/csrc/flops.cpp"

extern "C" {

// contact: 0 none, 1 penalty (gains k, d on every body), 2 impulse
int host_flops(const phyzb_model* m, int contact, double k, double d, double ground, double mu, int sweeps,
               const double* q, const double* v, const double* ctrl, long long nworld, int nsteps, int specialized,
               double* out) {
    pz::PackCfg cfg;
    cfg.contact = contact != 0;
    cfg.impulse = contact == 2;
    cfg.gk.assign(m->nbodies, k);
    cfg.gd.assign(m->nbodies, d);
    int nv = 0;
    for (int i = 0; i < m->nbodies; i++) nv += pz::ndof_of(m->bodies[i].joint_type);
    const double erp = 0.2;
    pz::FlopCount fc;
    if (nsteps <= 0)
        fc = pz::count_world_step(m, nv, cfg, sweeps);
    else
        fc = pz::count_rollout(m, nv, cfg, sweeps, ground, mu, erp, q, v, ctrl, nworld, nsteps, specialized != 0);
    out[0] = fc.flops;
    out[1] = fc.transcendentals;
    return 0;
}
}
