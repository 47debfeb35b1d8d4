"""Model-specialized rollout kernels (phyzb_set_kernel_specialization): the
kernel compiled at run time for one packed model runs the generic kernel's
source with the tables literal, so its states, accelerations and contact
records match the generic variant's to rounding -- the compiler may fuse a
different product of a sum into an FMA once constants are folded, so f32
agrees to ~1e-6 relative per step and the tolerance below covers 60-120
steps -- for every feature set: articulated chains, ball and free joints with
penalty contact, PD servos, impulse contact, heightfield terrain, and the
Tensor-Memory record layout."""
import numpy as np
import pytest

from phyz_b200 import BatchSim, BodyContactGains, Heightfield, PdDof, configs

pytestmark = pytest.mark.gpu

N = 96  # worlds: a ragged last block at every block width


def bumpy(seed=5, n=9):
    rng = np.random.default_rng(seed)
    hf = Heightfield.new((-1.0, -1.0, -0.05), 0.25, n, n)
    hf.heights[:] = (0.05 * rng.standard_normal(n * n)).astype(np.float32)
    return hf


def setup(sim, m, mode):
    if mode == "penalty":
        sim.enable_ground_contact(0.0, 1e4, 100.0, 1.0)
    elif mode == "impulse":
        sim.enable_contact_impulse(0.0, 1.0)
    elif mode == "terrain":
        sim.enable_contact_terrain(0.0, 1.0, [BodyContactGains(1e4, 100.0)] * m.nbodies, heightfield=bumpy())
    elif mode == "pd":
        dofs = [PdDof(j, j, 50.0, 2.0, 20.0) for j in range(m.nv)]
        sim.enable_pd_control(dofs)
        sim.set_position_targets(np.full((sim.nworld, len(dofs)), 0.1))


TOL = {"f32": 2e-4, "f64": 1e-10}


def close(a, b, precision, frac=1.0):
    """b within tolerance of a; with frac < 1, for at least that fraction of
    worlds (rows): the staged impulse law is discontinuous (the friction-disc
    clamp, a contact point entering or leaving the margin), so a rounding
    difference can send one world down another branch, as in the impulse
    parity tests."""
    assert np.all(np.isfinite(a)) and np.all(np.isfinite(b))
    tol = TOL[precision]
    atol = tol * max(1.0, float(np.abs(a).max()))
    if frac >= 1.0:
        np.testing.assert_allclose(b, a, rtol=tol, atol=atol)
        return
    ok = np.all(np.abs(b - a) <= atol + tol * np.abs(a), axis=tuple(range(1, a.ndim)))
    assert ok.mean() >= frac, f"{ok.mean():.3f} of worlds within tolerance"


def run(name, precision, mode, specialize, chunks=3, per=20):
    m = configs.CONFIGS[name].builder()
    q0, v0 = configs.initial_state(name, m, range(N))
    rng = np.random.default_rng(11)
    c = 0.5 * rng.standard_normal((N, m.nv)) * configs.actuated(m)
    sim = BatchSim(m, N, precision=precision)
    sim.specialize = specialize
    setup(sim, m, mode)
    sim.load_states(q0, v0, c)
    out = []
    for _ in range(chunks):
        sim.step_many(per)
        q, v = sim.readback_states()
        out += [q, v, sim.readback_qdd()]
    if mode in ("penalty", "impulse", "terrain"):
        out.append(sim.readback_contacts())
    info = sim.launch_info()
    assert sim.specialize == specialize
    sim.close()
    return out, info


CASES = [
    ("c2_chain32", "f32", None),
    ("c2_chain32", "f64", None),
    ("c1_double_pendulum", "f64", "pd"),
    ("c3_quadruped", "f32", "penalty"),
    ("c3_quadruped", "f64", "penalty"),
    ("c4_humanoid", "f32", "penalty"),
    ("c3_quadruped", "f32", "impulse"),
    ("c3_quadruped", "f32", "terrain"),
]


@pytest.mark.parametrize("name,precision,mode", CASES)
def test_specialized_matches_generic(name, precision, mode):
    gen, _ = run(name, precision, mode, False)
    spec, info = run(name, precision, mode, True)
    assert info["worlds_per_block"] > 0 and info["blocks"] > 0
    for a, b in zip(gen, spec):
        close(a, b, precision, frac=0.95 if mode == "impulse" else 1.0)


@pytest.mark.parametrize("name", ["c2_chain32", "c3_quadruped"])
def test_specialized_tensor_memory_layout(monkeypatch, name):
    monkeypatch.setenv("PHYZB_TMEM", "1")
    mode = "penalty" if name == "c3_quadruped" else None
    gen, ginfo = run(name, "f32", mode, False, chunks=2)
    spec, sinfo = run(name, "f32", mode, True, chunks=2)
    assert ginfo["tmem_cols"] > 0 and sinfo["tmem_cols"] == ginfo["tmem_cols"]
    for a, b in zip(gen, spec):
        close(a, b, "f32")


def test_table_change_recompiles():
    """A contact change repacks the table; the next launch specializes again
    and matches a fresh generic simulator with the same settings."""
    name = "c3_quadruped"
    m = configs.CONFIGS[name].builder()
    q0, v0 = configs.initial_state(name, m, range(N))
    sims = [BatchSim(m, N, precision="f32") for _ in range(2)]
    sims[1].specialize = True
    for s in sims:
        s.load_states(q0, v0)
        s.step_many(5)  # no contact
        s.enable_ground_contact(0.0, 1e4, 100.0, 1.0)
        s.step_many(30)
    a, b = (s.readback_states() for s in sims)
    for x, y in zip(a, b):
        close(x, y, "f32")
    for s in sims:
        s.close()


def test_auto_mode_and_invalid_mode():
    """"auto" specializes trees whose longest chain has at most 16 bodies (the
    quadruped, the 22-body humanoid), not the 32-body chain; a mode outside
    {0, 1, 2} is refused."""
    from phyz_b200 import PhyzbError, _lib

    for name, expect in (("c3_quadruped", True), ("c4_humanoid", True), ("c2_chain32", False)):
        m = configs.CONFIGS[name].builder()
        sim = BatchSim(m, 64, precision="f32")
        sim.specialize = False
        assert sim.specialize is False and not sim.specialized
        sim.specialize = "auto"
        assert sim.specialize == "auto" and sim.specialized == expect
        with pytest.raises(PhyzbError):
            _lib.check(sim._lib.phyzb_set_kernel_specialization(sim._h, 7))
        sim.close()


MODULE_CAP_SCRIPT = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from phyz_b200 import BatchSim, configs
name = "c3_quadruped"
m = configs.CONFIGS[name].builder()
n = 96
q0, v0 = configs.initial_state(name, m, range(n))
gen = BatchSim(m, n, precision="f32")
sims = [BatchSim(m, n, precision="f32") for _ in range(2)]
for s in sims:
    s.specialize = True
for s in [gen] + sims:
    s.load_states(q0, v0)
    s.step_many(5)  # no contact: one module each table
    s.enable_ground_contact(0.0, 1e4, 100.0, 1.0)  # a table change: compile again, release the old module
    s.step_many(30)
sims[0].close()  # its module is now unused and may be unloaded
for s in [gen, sims[1]]:
    s.step_many(10)
a, b = gen.readback_states(), sims[1].readback_states()
for x, y in zip(a, b):
    np.testing.assert_allclose(y, x, rtol=2e-4, atol=2e-4 * max(1.0, float(np.abs(x).max())))
print("ok")
"""


def test_module_cache_unloads_unused_modules():
    """With the cache capped at one loaded module, table changes and a closed
    simulator unload the modules no simulator holds, and the simulator still
    running its specialized kernel keeps stepping it correctly."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = str(Path(__file__).resolve().parents[1])
    r = subprocess.run([sys.executable, "-c", MODULE_CAP_SCRIPT, root], capture_output=True, text=True, timeout=900,
                       env=dict(os.environ, PHYZB_SPEC_MODULE_CAP="1"))
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]
