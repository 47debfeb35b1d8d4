"""The multi-GPU collective of the C ABI on the device: the NCCL
all-reduce of the per-world objective (phyzb_reduce_objective), with one
rank on one GPU, two ranks on two GPUs where the box has them, and the
bounded wait when a rank never joins (a host-side failure: no kernel of
the missing rank exists, nothing on the GPU faults or hangs)."""
import json
import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

from phyz_b200 import BatchSim, PhyzbError, configs
from phyz_b200 import _lib
from phyz_b200.parallel import Comm, new_unique_id, shard_bounds

pytestmark = pytest.mark.gpu

# no NVLink multicast objects in tests that may lose a rank
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")


def _sim(name, lo, hi, precision="f64"):
    m = configs.CONFIGS[name].builder()
    sim = BatchSim(m, hi - lo, precision=precision)
    q, v = configs.initial_state(name, m, range(lo, hi))
    sim.load_states(q, v + 0.25)
    return m, q, v + 0.25, sim


def test_reduce_objective_single_rank(oracle):
    import torch

    name = "c4_humanoid"
    m, q, v, sim = _sim(name, 0, 300)
    with Comm(0, 1, 0, timeout=30.0, id_channel=lambda p, r: p) as comm:
        total = comm.reduce_objective(sim, 0)
        total_again = comm.reduce_objective(sim, 0)
        sq = comm.reduce_objective(sim, 1)
        # enqueued without waiting, read after one bounded wait
        dev = torch.full((2,), -1.0, dtype=torch.float64, device="cuda")
        torch.cuda.synchronize()
        comm.reduce_objective_device(sim, dev[0].data_ptr(), 0)
        comm.reduce_objective_device(sim, dev[1].data_ptr(), 1)
        comm.sync(sim)
        total_dev, sq_dev = (float(x) for x in dev.cpu())
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    sim.objective_device(0, out.data_ptr())
    torch.cuda.synchronize()
    ke, _ = oracle.energy(m, q, v)
    assert abs(total - ke.sum()) <= 1e-10 * ke.sum()
    # the per-warp partial sums are added atomically (order varies by run)
    assert abs(total - total_again) <= 1e-12 * total and abs(total - out.item()) <= 1e-12 * total
    assert abs(sq - np.sum(q * q)) <= 1e-10 * np.sum(q * q)
    assert abs(total_dev - total) <= 1e-12 * total and abs(sq_dev - sq) <= 1e-12 * sq
    sim.close()


def test_comm_init_times_out_when_a_rank_never_joins():
    """World of 2, only rank 0 present: init returns ERR_COMM after the
    timeout instead of blocking (the communicator is aborted)."""
    uid = new_unique_id()
    import time

    t0 = time.time()
    with pytest.raises(PhyzbError) as ex:
        Comm(0, 2, 0, timeout=3.0, id_channel=lambda p, r: uid)
    assert ex.value.code == _lib.ERR_COMM
    assert time.time() - t0 < 60


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, name, total, out_dir):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)  # id exchange only
    try:
        lo, hi = shard_bounds(total, rank, world)
        m = configs.CONFIGS[name].builder()
        sim = BatchSim(m, hi - lo, device=rank, precision="f64")
        q, v = configs.initial_state(name, m, range(lo, hi))
        sim.load_states(q, v + 0.25)
        with Comm(rank, world, rank, timeout=60.0) as comm:
            val = comm.reduce_objective(sim, 0)
        sim.close()
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps({"total": val}))
    finally:
        dist.destroy_process_group()


def test_reduce_objective_two_gpus(oracle, tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    name, total, world = "c3_quadruped", 1000, 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, name, total, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    m = configs.CONFIGS[name].builder()
    q, v = configs.initial_state(name, m, range(total))
    ke, _ = oracle.energy(m, q, v + 0.25)
    for r in range(world):
        got = json.loads(Path(tmp_path, f"rank{r}.json").read_text())["total"]
        assert abs(got - ke.sum()) <= 1e-10 * ke.sum()


def _dp_rank(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phyz_b200.train import NetDims, PpoCfg, Trainer

        pa, pc, batches, orders = _dp_problem()
        t = Trainer(NetDims(8, 32, 3), NetDims(8, 32, 1), 256, 64, device=rank)
        t.set_params(0, pa)
        t.set_params(1, pc)
        with Comm(rank, world, rank, timeout=60.0) as comm:
            t.set_comm(comm)
            t.upload_batch(*batches[rank])
            st = t.update(orders[rank], PpoCfg(minibatch=64, epochs=2, entropy_coef=0.01))
            a, c = t.params(0), t.params(1)
            t.set_comm(None)
        t.close()
        np.savez(Path(out_dir, f"dp{rank}.npz"), a=a, c=c, pl=st["policy_loss"], vl=st["value_loss"])
    finally:
        dist.destroy_process_group()


def _dp_problem():
    rng = np.random.default_rng(5)
    from phyz_b200.train import NetDims

    A, Cn = NetDims(8, 32, 3), NetDims(8, 32, 1)
    pa = np.concatenate([rng.normal(0, 0.3, A.param_count()), np.full(3, -0.6)])
    pc = rng.normal(0, 0.3, Cn.param_count())
    batches = [[rng.normal(0, 1, (256, 8)), rng.normal(0, 1, (256, 8)), rng.normal(0, 0.5, (256, 3)),
                rng.normal(-2.5, 0.3, 256), rng.normal(0, 1, 256), rng.normal(0, 1, 256)] for _ in range(2)]
    orders = [np.stack([rng.permutation(256) for _ in range(2)]).astype(np.uint32) for _ in range(2)]
    return pa, pc, batches, orders


def test_data_parallel_update_two_gpus(tmp_path):
    """Two ranks, each with its own batch, gradients all-reduced: both end
    with the same networks, equal to one trainer stepping on the union of
    the ranks' minibatches."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from phyz_b200.train import NetDims, PpoCfg, Trainer

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dp_rank, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    r0, r1 = (np.load(Path(tmp_path, f"dp{r}.npz")) for r in range(2))
    assert np.array_equal(r0["a"], r1["a"]) and np.array_equal(r0["c"], r1["c"])
    # one trainer on both batches: minibatch k = rank 0's chunk k + rank 1's
    pa, pc, batches, orders = _dp_problem()
    union = [np.concatenate([batches[0][i], batches[1][i]]) for i in range(6)]
    order = np.stack([np.concatenate([np.concatenate([orders[0][e][k:k + 64], 256 + orders[1][e][k:k + 64]])
                                      for k in range(0, 256, 64)]) for e in range(2)]).astype(np.uint32)
    t = Trainer(NetDims(8, 32, 3), NetDims(8, 32, 1), 512, 128)
    t.set_params(0, pa)
    t.set_params(1, pc)
    t.upload_batch(*union)
    st = t.update(order, PpoCfg(minibatch=128, epochs=2, entropy_coef=0.01))
    for got, want, before in ((r0["a"], t.params(0), pa), (r0["c"], t.params(1), pc)):
        assert np.linalg.norm((got - before) - (want - before)) <= 1e-5 * np.linalg.norm(want - before)
    assert abs(float(r0["pl"]) - st["policy_loss"]) <= 1e-4 * max(abs(st["policy_loss"]), 1e-9)
    assert abs(float(r0["vl"]) - st["value_loss"]) <= 1e-4 * abs(st["value_loss"])
    t.close()
