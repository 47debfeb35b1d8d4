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
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    sim.objective_device(0, out.data_ptr())
    torch.cuda.synchronize()
    ke, _ = oracle.energy(m, q, v)
    assert abs(total - ke.sum()) <= 1e-10 * ke.sum()
    # the per-warp partial sums are added atomically (order varies by run)
    assert abs(total - total_again) <= 1e-12 * total and abs(total - out.item()) <= 1e-12 * total
    assert abs(sq - np.sum(q * q)) <= 1e-10 * np.sum(q * q)
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
