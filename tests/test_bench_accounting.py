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


def test_route_check_counts_exempt_and_bad_rows():
    """The bench's ids check against the oracle: the oracle's own ids pass,
    a swapped pair in a row with a wide margin counts as a mismatch outside
    the exemption (a mistake planted on the CPU)."""
    import dataclasses

    import numpy as np
    import oracle as O
    cfg = dataclasses.replace(C.CONFIGS[1], hidden=64, experts=8, top_k=2, layers=2)
    rng = np.random.default_rng(5)
    inputs, ids = [], []
    for layer in range(cfg.layers):
        h = rng.standard_normal((6, cfg.hidden)).astype(np.float32)
        r = O.round_bf16(O.synth(cfg.seed, layer, O.KIND_ROUTER, 0, cfg.experts * cfg.hidden, 0.02))
        z = np.zeros
        w = O.MoeWeights(r.reshape(cfg.experts, cfg.hidden), z((cfg.experts, cfg.hidden), np.float32),
                         z((cfg.experts, cfg.hidden), np.float32), z((cfg.experts * cfg.hidden, 1), np.float32),
                         z((0, cfg.hidden), np.float32), z((0, cfg.hidden), np.float32), z((cfg.hidden, 0), np.float32))
        want = O.moe_forward(w, O.rms_norm(h, None, 1e-6), cfg.top_k, True)
        inputs.append(h)
        ids.append(want.ids.copy())
    ok = bench.route_check(cfg, inputs, ids)
    assert ok["rows_checked"] == 12 and ok["margin_exempt_rows"] == 0 and ok["mismatched_rows_outside_margin"] == 0
    ids[1][3] = ids[1][3][::-1].copy()  # order swapped: wrong unless the two logits are within 1e-3
    bad = bench.route_check(cfg, inputs, ids)
    assert bad["margin_exempt_rows"] + bad["mismatched_rows_outside_margin"] == 1
