"""The byte and FLOP accounting bench.py reports against (no GPU): the
algorithmic bytes of a decode step and the traffic figure read back from the
committed ncu summaries."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
import moe_configs as C  # noqa: E402


def test_decode_step_bytes_bf16_batch1():
    # per layer: 6 experts x 12,582,912 + shared 25,165,824 + router 524,288 = 101,187,584
    total, gate_up = bench.decode_bytes(C.CONFIGS[1], [6] * 24, fmt_int8=False)
    assert total == 101_187_584 * 24
    assert gate_up == [6 * 2 * 1024 * 2048 * 2 + 2 * 2048 * 2048 * 2] * 24


def test_decode_step_bytes_int8_batch1():
    # per layer: 6 x 6,307,840 (int8 rows + fp32 row scales) + shared 12,607,488 + router 524,288
    total, _ = bench.decode_bytes(C.CONFIGS[2], [6] * 24, fmt_int8=True)
    assert total == 50_978_816 * 24


def test_decode_bytes_follow_the_distinct_experts():
    a, _ = bench.decode_bytes(C.CONFIGS[1], [35], fmt_int8=False)
    b, _ = bench.decode_bytes(C.CONFIGS[1], [6], fmt_int8=False)
    assert a - b == 29 * 12_582_912


def test_traffic_figures_are_read_from_the_profiles():
    t1 = bench.traffic_from_profile("decode_gate_up_bf16_t1.txt")
    assert t1 is not None and abs(t1 - 67_108_864) / 67_108_864 < 0.05  # DRAM bytes ~ algorithmic bytes
    assert bench.traffic_from_profile("no_such_profile.txt") is None
