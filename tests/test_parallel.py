"""Host side of the multi-GPU path on CPU: contiguous world shards, the
communicator id handed from rank 0 to the others, and the end-of-rollout
sum of a per-world objective over shards -- run as two gloo ranks. The
per-world objective here is the oracle's kinetic energy (the quantity
phyzb_reduce_objective sums on device)."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

from phyz_b200 import configs
from phyz_b200.parallel import shard_bounds, weak_block

ROOT = Path(__file__).resolve().parents[1]


def test_shard_bounds_partition_contiguously():
    for total in (0, 1, 7, 4096, 65537):
        for world in (1, 2, 3, 8):
            got = [shard_bounds(total, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [hi - lo for lo, hi in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_weak_blocks_draw_the_global_worlds():
    """A rank's seeded initial state is the slice of the whole batch's: the
    per-world seeds depend on the global world index only."""
    name = "c3_quadruped"
    m = configs.CONFIGS[name].builder()
    q, v = configs.initial_state(name, m, range(0, 64))
    for rank in range(4):
        lo, hi = weak_block(16, rank)
        qr, vr = configs.initial_state(name, m, range(lo, hi))
        assert np.array_equal(qr, q[lo:hi]) and np.array_equal(vr, v[lo:hi])
    sched = configs.control_schedule(name, m, range(0, 64), 3)
    assert np.array_equal(configs.control_schedule(name, m, range(32, 48), 3), sched[:, 32:48])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, name, total, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch

        from oracle.oracle import Oracle
        from phyz_b200.parallel import share_bytes

        uid = share_bytes(bytes(range(128)) if rank == 0 else None, rank)
        m = configs.CONFIGS[name].builder()
        lo, hi = shard_bounds(total, rank, world)
        q, v = configs.initial_state(name, m, range(lo, hi))
        ke, _ = Oracle().energy(m, q, v)
        part = torch.tensor([ke.sum()], dtype=torch.float64)
        dist.all_reduce(part)
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps(
            {"uid_ok": uid == bytes(range(128)), "lo": lo, "hi": hi, "total_ke": float(part.item())}))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_the_sharded_objective(oracle, tmp_path):
    name, total, world = "c4_humanoid", 50, 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, name, total, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, p.exitcode
    res = [json.loads(Path(tmp_path, f"rank{r}.json").read_text()) for r in range(world)]
    assert all(r["uid_ok"] for r in res)
    assert res[0]["hi"] == res[1]["lo"] and res[0]["lo"] == 0 and res[1]["hi"] == total
    m = configs.CONFIGS[name].builder()
    q, v = configs.initial_state(name, m, range(total))
    ke, _ = oracle.energy(m, q, v)
    for r in res:
        assert abs(r["total_ke"] - ke.sum()) <= 1e-12 * abs(ke.sum())


def test_reference_arm_under_two_ranks(tmp_path):
    """`bench.py --impl reference` under a 2-rank launch: rank 0 times the
    reference's CPU path and prints one line; rank 1 exits 0 silently."""
    base = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1",
            "--warmup", "0", "--nworld", "64", "--horizon", "8"]
    env = dict(os.environ, WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    r1 = subprocess.run(base, env=dict(env, RANK="1", LOCAL_RANK="1"), capture_output=True, text=True, timeout=300)
    assert r1.returncode == 0, r1.stderr
    assert r1.stdout.strip() == ""
    r0 = subprocess.run(base, env=dict(env, RANK="0", LOCAL_RANK="0"), capture_output=True, text=True, timeout=300)
    assert r0.returncode == 0, r0.stderr
    line = json.loads(r0.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference" and line["e2e"]["h2d_bytes_per_step"] == 0
