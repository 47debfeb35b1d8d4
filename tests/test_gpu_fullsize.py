"""Parity at the benchmarked sizes: every config at its own world count and
horizon, with the launch shape the bench runs (grid-stride tiles, several
waves, a Tensor-Memory block reused for its next tile, the model-specialized
kernel where `auto` picks it), compared on a sample of worlds chosen to land
in different blocks, tiles and waves.

The controls are the bench's own: a device schedule `[step][nv][nworld]`
drawn with torch.randn from the bench seed; the sampled worlds' columns are
gathered back for the checkers.

* One step, f64: max normwise relative error <= 1e-5 on q, v, qdd (the north
  star's bound), also asserted <= 1e-9 (the formulations agree to rounding);
  f32: <= 1e-3.
* Full horizon, f64: for every sampled world, |device - oracle| <= 100 x the
  oracle's own divergence under a 1-ulp perturbation of q0 (+1e-12), the
  drift bound of test_double_pendulum_500_step_drift and the reference's
  determinism method (crates/phyz/src/determinism.rs:180,333).
* Full horizon, f32: the device's divergence from the f64 oracle is no worse
  than that of the reference's own f32 kernels (crates/phyz-gpu/cuda/
  phyz_kernels.cu compiled as host C++) on the same worlds and controls: its
  median and 90th percentile over the sampled worlds are within 4x the
  reference's. Every world of the launch is finite.
* Every world of the launch is checked for finiteness and the sampled worlds
  for cross-world independence (crates/phyz-gpu/tests/cuda_vs_cpu.rs:246-270
  at full scale: each matches its own oracle trajectory).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err
from phyz_b200 import BatchSim, configs

pytestmark = pytest.mark.gpu

SAMPLE = 256

# (config, precision, kernel): kernel "auto" = what bench.py runs by default;
# "tmem" / "smem" = the generic variant with that record layout forced
CASES = [
    ("c1_double_pendulum", "f64", "auto"),
    ("c1_double_pendulum", "f64", "tmem"),
    ("c1_double_pendulum", "f64", "smem"),
    ("c2_chain32", "f32", "auto"),
    ("c2_chain32", "f32", "smem"),
    ("c2_chain32", "f64", "tmem"),
    ("c2_chain32", "f64", "smem"),
    ("c3_quadruped", "f32", "auto"),
    ("c3_quadruped", "f32", "tmem"),
    ("c3_quadruped", "f32", "smem"),
    ("c3_quadruped", "f64", "auto"),
    ("c4_humanoid", "f32", "auto"),
    ("c4_humanoid", "f32", "tmem"),
    ("c4_humanoid", "f64", "auto"),
    ("c4_humanoid", "f64", "smem"),
]


def sample_worlds(nworld: int, W: int, grid: int, seed: int = 0) -> np.ndarray:
    """Worlds at the edges of tiles of the first, middle and last blocks,
    in their first three tiles (a block walks tiles b, b + grid, ...), the
    last worlds of the launch, and a uniform fill up to SAMPLE."""
    ntiles = -(-nworld // W)
    picks = set()
    for b in sorted({0, 1, grid // 2, grid - 1}):
        for k in range(3):
            t = b + k * grid
            if t >= ntiles:
                break
            for off in (0, 1, 31, 32, W - 1):
                w = t * W + off
                if 0 <= off < W and w < nworld:
                    picks.add(w)
    picks.update({nworld - 1, nworld - 2, nworld // 2})
    rng = np.random.default_rng(seed)
    while len(picks) < SAMPLE:
        picks.add(int(rng.integers(0, nworld)))
    return np.array(sorted(picks))[:SAMPLE] if len(picks) > SAMPLE else np.array(sorted(picks))


def device_run(name, precision, kernel, steps, monkeypatch):
    """Run the config at full size; returns (sim info, sampled worlds, their
    q0/v0, their control schedule [steps][n][nv] as applied, device q, v,
    qdd of those worlds, all-finite flag)."""
    import torch

    cfg = configs.CONFIGS[name]
    model = cfg.builder()
    nworld, nv = cfg.nworld, model.nv
    if kernel in ("tmem", "smem"):
        monkeypatch.setenv("PHYZB_TMEM", "1" if kernel == "tmem" else "0")
    sim = BatchSim(model, nworld, precision=precision)
    sim.specialize = "auto" if kernel == "auto" else False
    if cfg.contact is not None:
        sim.enable_ground_contact(*cfg.contact)
    tdt = torch.float32 if precision == "f32" else torch.float64
    q0, v0 = configs.initial_state(name, model, np.arange(nworld))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(configs.CTRL_SEED)
    mask = torch.tensor(configs.actuated(model), dtype=tdt, device="cuda").view(1, nv, 1)
    sched = torch.randn(steps, nv, nworld, generator=gen, dtype=tdt, device="cuda") * (cfg.ctrl_sigma * mask)
    # the schedule is written on torch's stream and read on the simulator's
    # own (non-blocking) stream: finish it first
    torch.cuda.synchronize()
    sim.load_states(q0, v0)
    sim.step_device_controls(sched.data_ptr(), nv * nworld, steps)
    sim.sync()
    info = dict(sim.launch_info(), specialized=sim.specialized)
    q, v = sim.readback_states()
    qdd = sim.readback_qdd()
    sim.close()
    finite = bool(np.isfinite(q).all() and np.isfinite(v).all())
    ws = sample_worlds(nworld, info["worlds_per_block"], info["blocks"])
    ctrl = sched[:, :, torch.as_tensor(ws, device="cuda")].permute(0, 2, 1).double().cpu().numpy()
    del sched
    torch.cuda.empty_cache()
    return info, ws, q0[ws], v0[ws], ctrl, q[ws], v[ws], qdd[ws], finite


def oracle_contact(cfg, model):
    if cfg.contact is None:
        return None
    g, k, d, mu = cfg.contact
    return g, mu, [k] * model.nbodies, [d] * model.nbodies


@pytest.mark.parametrize("name,precision,kernel", CASES)
def test_one_step_full_size(oracle, monkeypatch, name, precision, kernel):
    cfg = configs.CONFIGS[name]
    model = cfg.builder()
    info, ws, q0, v0, ctrl, q, v, qdd, finite = device_run(name, precision, kernel, 1, monkeypatch)
    assert finite
    if name != "c1_double_pendulum":  # C1's 4096 worlds fit one wave
        tiles = -(-cfg.nworld // info["worlds_per_block"])
        assert tiles > info["blocks"], f"every block runs a single tile: {info}"
    if kernel == "auto" and name != "c2_chain32":
        assert info["specialized"], info
    qo, vo, qddo, _ = oracle.rollout(model, q0, v0, ctrl, 1, schedule=True, contact=oracle_contact(cfg, model),
                                     nthreads=8)
    tol = 1e-5 if precision == "f64" else 1e-3
    for nm, a, b in (("q", q, qo), ("v", v, vo), ("qdd", qdd, qddo)):
        e = rel_err(a, b)
        assert e <= tol, f"{name} {precision} {kernel} {nm}: {e:.3e} ({info})"
        if precision == "f64":
            assert e <= 1e-9, f"{name} f64 {kernel} {nm}: {e:.3e} (formulations should agree to rounding)"


@pytest.mark.parametrize("name,precision,kernel", CASES)
def test_full_horizon_full_size(oracle, refhost, monkeypatch, name, precision, kernel):
    cfg = configs.CONFIGS[name]
    model = cfg.builder()
    steps = cfg.steps
    info, ws, q0, v0, ctrl, q, v, _, finite = device_run(name, precision, kernel, steps, monkeypatch)
    assert finite, f"non-finite worlds after {steps} steps ({info})"
    oc = oracle_contact(cfg, model)
    qo, vo, _, _ = oracle.rollout(model, q0, v0, ctrl, steps, schedule=True, contact=oc, nthreads=8)
    dev = np.abs(q - qo).max(axis=1)
    # worlds stay apart: the sample's trajectories are not copies of each other
    assert len({tuple(np.round(r, 9)) for r in q}) == len(ws)
    if precision == "f64":
        qp, _, _, _ = oracle.rollout(model, np.nextafter(q0, np.inf), v0, ctrl, steps, schedule=True, contact=oc,
                                     nthreads=8)
        env = np.maximum(np.abs(qp - qo).max(axis=1), 1e-15)
        ratio = dev / (100 * env + 1e-12)
        assert np.all(ratio <= 1.0), (f"{name} f64 {kernel}: world {ws[np.argmax(ratio)]} drifts "
                                      f"{float(ratio.max()):.2f}x past 100x the 1-ulp envelope ({info})")
    else:
        rc = None if cfg.contact is None else cfg.contact
        if rc is not None:
            g, k, d, mu = rc
            rc = (g, mu, k, d)
        qr, _, _, _ = refhost.rollout(model, q0, v0, ctrl.astype(np.float32), steps, schedule=True, contact=rc,
                                      nthreads=8)
        ref = np.abs(qr - qo).max(axis=1)
        for p in (0.5, 0.9):
            a, b = float(np.quantile(dev, p)), float(np.quantile(ref, p))
            assert a <= 4 * b + 1e-7, (f"{name} f32 {kernel}: divergence quantile {p} {a:.3e} vs the "
                                       f"reference's f32 kernels {b:.3e} ({info})")


@pytest.mark.parametrize("name", ["c2_chain32", "c3_quadruped"])
@pytest.mark.parametrize("layout", ["0", "1"])
def test_second_tiles_narrow_blocks(oracle, monkeypatch, name, layout):
    """32-world blocks over 40000 worlds: more tiles than the grid's blocks
    (one Tensor-Memory block or a few shared-memory blocks per SM), so blocks
    walk to second and later tiles (and a Tensor-Memory block reuses its
    columns for them). Worlds of first and later tiles match the oracle over
    a 10-step schedule."""
    monkeypatch.setenv("PHYZB_WORLDS_PER_BLOCK", "32")
    monkeypatch.setenv("PHYZB_TMEM", layout)
    cfg = configs.CONFIGS[name]
    model = cfg.builder()
    n, steps = 40000, 10
    q0, v0 = configs.initial_state(name, model, range(n))
    sched = configs.control_schedule(name, model, range(n), steps)
    sim = BatchSim(model, n, precision="f64")
    if cfg.contact is not None:
        sim.enable_ground_contact(*cfg.contact)
    info = sim.launch_info()
    assert info["worlds_per_block"] == 32 and -(-n // 32) > info["blocks"], info
    assert (info["tmem_cols"] > 0) == (layout == "1"), info
    sim.load_states(q0, v0)
    sim.step_with_controls(np.ascontiguousarray(sched))
    sim.sync()
    q, v = sim.readback_states()
    sim.close()
    G = info["blocks"]
    ws = np.unique(np.concatenate([np.arange(0, 64), np.arange(G * 32, G * 32 + 64), np.arange(n - 64, n),
                                   np.random.default_rng(2).integers(64, n - 64, 64)]))
    qo, vo, _, _ = oracle.rollout(model, q0[ws], v0[ws], sched[:, ws], steps, schedule=True,
                                  contact=oracle_contact(cfg, model), nthreads=8)
    assert rel_err(q[ws], qo) <= 1e-9 and rel_err(v[ws], vo) <= 1e-9, (rel_err(q[ws], qo), rel_err(v[ws], vo))
