"""bench.py's config block and L2 rule (no GPU): both arms print the same
`config` for the same arguments, zero-control configs step under held
controls and flush L2, and streamed schedules larger than L2 do not."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from phyz_b200 import configs  # noqa: E402


def test_config_block_is_the_same_for_both_arms():
    m = configs.chain()
    a = bench.bench_config("c2_chain32", m, 65536, 1000, "f32", 1)
    b = bench.bench_config("c2_chain32", m, 65536, 1000, "f32", 1)
    assert a == b and a["nworld_per_gpu"] == 65536 and a["horizon"] == 1000
    s = bench.bench_config("c1_double_pendulum", configs.double_pendulum(), 4096, 500, "f64", 8, strong=True)
    assert s["nworld_total"] == 4096 and "strong" in s["parallelism"]


def test_l2_rule():
    flush, note = bench.l2_rule("c1_double_pendulum", configs.double_pendulum(), 4096, 500, "f64")
    assert flush and "held" in note and bench.held_controls("c1_double_pendulum")
    flush, note = bench.l2_rule("c2_chain32", configs.chain(), 65536, 1000, "f32")
    assert not flush and "larger than L2" in note
    flush, _ = bench.l2_rule("c2_chain32", configs.chain(), 64, 8, "f32")
    assert flush  # a small schedule fits L2: flushed between rollouts
