// C++ host driving libphyzb200 through include/phyzb.hpp the way phyz's
// examples/gpu_batch.rs drives BatchSim: the C1 double pendulum over N
// worlds with fanned-out initial angles, stepped, read back. Prints one
// JSON object: either {"error": code, ...} (BatchSim::new returned Err) or
// the final q rows.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "phyzb.hpp"

static phyzb_body rod(int parent, double m, double h) {
    phyzb_body b{};
    b.parent = parent;
    b.joint_type = PHYZB_JOINT_REVOLUTE;
    b.mass = m;
    b.com[1] = -h;
    const double L = 2.0 * h, i = m * L * L / 12.0;
    b.inertia[0] = i;
    b.inertia[2] = i;
    b.ptj_rot[0] = b.ptj_rot[4] = b.ptj_rot[8] = 1.0;
    b.axis[2] = 1.0;
    b.geom_origin_rot[0] = b.geom_origin_rot[4] = b.geom_origin_rot[8] = 1.0;
    return b;
}

int main(int argc, char** argv) {
    const int nworld = argc > 1 ? std::atoi(argv[1]) : 8;
    const int steps = argc > 2 ? std::atoi(argv[2]) : 100;
    std::vector<phyzb_body> bodies = {rod(-1, 1.0, 0.5), rod(0, 0.8, 0.4)};
    phyzb_model m{};
    m.nbodies = 2;
    m.gravity[1] = -9.81;
    m.dt = 0.002;
    m.bodies = bodies.data();
    auto made = phyzb::BatchSim::create(m, nworld, PHYZB_F64);
    if (!made.ok()) {
        std::printf("{\"error\": %d, \"message\": \"%s\"}\n", made.code, made.error.c_str());
        return 0;
    }
    phyzb::BatchSim sim = std::move(made.value);
    std::vector<std::vector<double>> q(nworld, std::vector<double>(2)), v(nworld, std::vector<double>(2, 0.0));
    for (int i = 0; i < nworld; i++) {
        const double t = (double)i / nworld;
        q[i] = {0.2 + 1.2 * t, -0.4 + 0.8 * t};
    }
    sim.load_states(q, v);
    if (!sim.step_many(steps).ok()) return 2;
    auto out = sim.readback_states();
    auto contact = sim.readback_contacts();  // contact never enabled: Err, like the reference
    std::printf("{\"contacts_err\": %d, \"q\": [", contact.ok() ? 0 : contact.code);
    for (int i = 0; i < nworld; i++)
        std::printf("%s[%.17g, %.17g]", i ? ", " : "", out.first[i][0], out.first[i][1]);
    std::printf("]}\n");
    return 0;
}
