"""The B200 stepper against the reference's own CUDA kernels running on the
same GPU (crates/phyz-gpu/cuda/phyz_kernels.cu compiled for sm_100a, driven
in the reference's step sequence as one CUDA graph: oracle/ref_cuda_driver.cu):
the same f32 results within f32 rounding on C1-C4, and the fused kernel
faster on every config. The measured throughputs are printed (pytest -s)."""
import time

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle.oracle import RefCuda
from phyz_b200 import BatchSim, configs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def refcuda(refhost):
    return RefCuda(refhost)


def inputs(name, n, steps):
    cfg = configs.CONFIGS[name]
    m = cfg.builder()
    q0, v0 = configs.initial_state(name, m, range(n))
    sched = configs.control_schedule(name, m, range(n), steps)
    return cfg, m, q0, v0, sched


@pytest.mark.parametrize("name", list(configs.CONFIGS))
def test_matches_the_reference_gpu_kernels(refhost, refcuda, name):
    n, steps = 256, 10
    cfg, m, q0, v0, sched = inputs(name, n, steps)
    contact = None if cfg.contact is None else (cfg.contact[0], cfg.contact[3], cfg.contact[1], cfg.contact[2])
    qr, vr, qddr, csr, _ = refcuda.rollout(m, q0, v0, sched, steps, schedule=True, contact=contact)
    # the reference's GPU kernels equal its host-compiled kernels up to f32 rounding
    qh, vh, _, _ = refhost.rollout(m, q0, v0, sched, steps, schedule=True, contact=contact)
    assert rel_err(qr, qh) < 1e-4 and rel_err(vr, vh) < 1e-3
    sim = BatchSim(m, n, precision="f32")
    if cfg.contact:
        sim.enable_ground_contact(*cfg.contact)
    sim.load_states(q0, v0)
    sim.step_with_controls(np.ascontiguousarray(sched))
    qd, vd = sim.readback_states()
    assert rel_err(qd, qr) < 2e-3, rel_err(qd, qr)
    assert rel_err(vd, vr) < 2e-2, rel_err(vd, vr)
    sim.close()


@pytest.mark.parametrize("name,nworld,steps", [("c1_double_pendulum", 4096, 500), ("c2_chain32", 65536, 100),
                                              ("c3_quadruped", 262144, 100), ("c4_humanoid", 131072, 100)])
def test_faster_than_the_reference_gpu_kernels(refcuda, name, nworld, steps):
    cfg, m, q0, v0, _ = inputs(name, nworld, 1)
    contact = None if cfg.contact is None else (cfg.contact[0], cfg.contact[3], cfg.contact[1], cfg.contact[2])
    ctrl = np.zeros((nworld, m.nv), np.float32)
    _, _, _, _, ms_ref = refcuda.rollout(m, q0, v0, ctrl, steps, contact=contact, reps=3)
    sim = BatchSim(m, nworld, precision="f32")
    if cfg.contact:
        sim.enable_ground_contact(*cfg.contact)
    st = torch.cuda.Stream()
    sim.set_stream(st.cuda_stream)
    best = 1e30
    for _ in range(4):
        sim.load_states(q0, v0, ctrl)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        sim.step_many(steps)
        e1.record(st)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    sim.close()
    ours, ref = nworld * steps / best * 1e3, nworld * steps / ms_ref * 1e3
    print(f"\n{name}: B200 stepper {ours:.3e} world-steps/s, reference CUDA kernels {ref:.3e} "
          f"world-steps/s on the same GPU: {ours / ref:.1f}x")
    assert ours > 2 * ref


def impulse_inputs(n):
    m = configs.quadruped()
    q0, v0 = configs.initial_state("c3_quadruped", m, range(n))
    q0[:, 5] = np.linspace(0.55, 0.62, n)  # feet on or just above the ground
    return m, q0, v0, np.zeros((n, m.nv), np.float32)


def test_impulse_mode_matches_the_reference_gpu_kernels(refhost, refcuda):
    """Impulse-mode contact (16 sweeps) on the quadruped: the reference's GPU
    sequence (35 launches per step) against the fused kernel, f32, from a
    fresh warm start."""
    n, steps = 256, 40
    m, q0, v0, ctrl = impulse_inputs(n)
    qr, vr, _, csr, _ = refcuda.rollout(m, q0, v0, ctrl, steps, contact=(0.0, 1.0), sweeps=16)
    qh, vh, _, _, _ = refhost.rollout_impulse(m, q0, v0, ctrl, nsteps=steps, contact=(0.0, 1.0))
    assert rel_err(qr, qh) < 1e-4
    sim = BatchSim(m, n, precision="f32")
    sim.enable_contact_impulse(0.0, 1.0)
    sim.load_states(q0, v0, ctrl)
    sim.step_many(steps)
    qd, vd = sim.readback_states()
    cs = sim.readback_contacts()
    sim.close()
    assert cs[:, :, 0].sum() > 0
    assert rel_err(qd, qr) < 2e-3, rel_err(qd, qr)
    assert np.array_equal(cs[:, :, 0], csr[:, :, 0])


def test_impulse_mode_faster_than_the_reference_gpu_kernels(refcuda):
    n, steps = 65536, 20
    m, q0, v0, ctrl = impulse_inputs(n)
    _, _, _, _, ms_ref = refcuda.rollout(m, q0, v0, ctrl, steps, contact=(0.0, 1.0), sweeps=16, reps=3)
    sim = BatchSim(m, n, precision="f32")
    sim.enable_contact_impulse(0.0, 1.0)
    st = torch.cuda.Stream()
    sim.set_stream(st.cuda_stream)
    best = 1e30
    for _ in range(4):
        sim.load_states(q0, v0, ctrl)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        sim.step_many(steps)
        e1.record(st)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    sim.close()
    ours, ref = n * steps / best * 1e3, n * steps / ms_ref * 1e3
    print(f"\nimpulse C3: B200 stepper {ours:.3e} world-steps/s, reference CUDA kernels {ref:.3e} "
          f"world-steps/s on the same GPU: {ours / ref:.1f}x")
    assert ours > 2 * ref
