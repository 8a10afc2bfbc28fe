"""The CPU oracle, pinned before anything is checked against it.

1. Golden vectors produced by the reference's own MixtureOfExperts::forward
   (tests/golden/make_golden.py): the oracle reproduces them bit for bit, and
   the input digests pin the synthetic generator.
2. When oracle/_ref is built (reference sources present), a live comparison
   against the reference on fresh shapes, edge cases included.
3. Known answers of the reference ops (tests/ops_test.cpp:17-57 of the
   reference) and its thread-count independence (:108-120).
4. The int8 quantiser bound (tests/cuda_ops_test.cpp:187-200) per output channel.
"""
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
import sys  # noqa: E402
sys.path.insert(0, GOLDEN)
import make_golden as MG  # noqa: E402


def _load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.mark.parametrize("name", ["c0", "c1_layer0_t8"])
def test_golden_generated_inputs(name):
    g = _load(name)
    w, x = MG.make_inputs(int(g["seed"]), int(g["tokens"]), int(g["hidden"]), int(g["experts"]), int(g["ffn"]),
                          int(g["shared_ffn"]), bool(g["bf16"]))
    assert MG.digest(x) == str(g["x_sha"]), "generator drifted (x)"
    assert MG.digest(w.router) == str(g["router_sha"])
    assert MG.digest(w.gate) == str(g["gate_sha"])
    assert MG.digest(w.down) == str(g["down_sha"])
    r = O.moe_forward(w, x, int(g["top_k"]), renormalize=False)
    assert np.array_equal(r.y.view(np.uint32), g["y"].view(np.uint32)), "oracle != reference golden"
    assert np.array_equal(r.ids, g["ids"])


def test_golden_tiny_stored_inputs():
    g = _load("tiny")
    w = O.MoeWeights(g["router"], g["gate"], g["up"], g["down"], g["shared_gate"], g["shared_up"], g["shared_down"])
    r = O.moe_forward(w, g["x"], int(g["top_k"]), renormalize=False)
    assert np.array_equal(r.y.view(np.uint32), g["y"].view(np.uint32))


def _random_layer(rng, H, E, F, S):
    f = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float32)  # noqa: E731
    return O.MoeWeights(f(E, H), f(E * F, H), f(E * F, H), f(E * H, F), f(S, H), f(S, H), f(H, S))


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (reference sources absent)")


@needs_ref
@pytest.mark.parametrize("T,H,E,K,F,S", [(1, 64, 8, 3, 32, 32), (0, 32, 4, 1, 16, 16), (13, 40, 5, 5, 24, 8),
                                         (37, 96, 16, 2, 48, 64), (5, 16, 128, 8, 16, 16)])
def test_oracle_matches_reference_live(T, H, E, K, F, S):
    rng = np.random.default_rng(T * 1000 + E)
    w = _random_layer(rng, H, E, F, S)
    x = rng.standard_normal((T, H)).astype(np.float32)
    ref = O.RefMoe(w, K)
    want = ref(x)
    got = O.moe_forward(w, x, K, renormalize=False).y
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_ref
def test_oracle_matches_reference_on_ties():
    """Identical router rows give tied scores: the lower expert id wins (feed_forward.cpp:47)."""
    rng = np.random.default_rng(11)
    w = _random_layer(rng, 32, 6, 16, 16)
    w.router[3] = w.router[1]
    w.router[5] = w.router[1]
    x = rng.standard_normal((9, 32)).astype(np.float32)
    r = O.moe_forward(w, x, 3, renormalize=False)
    ref = O.RefMoe(w, 3)
    assert np.array_equal(r.y.view(np.uint32), ref(x).view(np.uint32))
    for row in r.ids:
        picked = [e for e in row if e in (1, 3, 5)]
        assert picked == sorted(picked)


def test_renormalisation_semantics():
    rng = np.random.default_rng(3)
    w = _random_layer(rng, 48, 8, 16, 0)
    x = rng.standard_normal((6, 48)).astype(np.float32)
    a = O.moe_forward(w, x, 3, renormalize=False)
    b = O.moe_forward(w, x, 3, renormalize=True)
    assert np.array_equal(a.ids, b.ids)
    s = a.weights.sum(axis=1, dtype=np.float32)
    np.testing.assert_allclose(b.weights, a.weights / s[:, None], rtol=1e-6)
    np.testing.assert_allclose(b.weights.sum(axis=1), 1.0, rtol=1e-6)


def test_router_bias_enters_logits():
    rng = np.random.default_rng(4)
    w = _random_layer(rng, 32, 8, 16, 16)
    x = rng.standard_normal((4, 32)).astype(np.float32)
    plain = O.moe_forward(w, x, 2, renormalize=True)
    w.router_bias = np.linspace(-1, 1, 8).astype(np.float32)
    biased = O.moe_forward(w, x, 2, renormalize=True)
    np.testing.assert_array_equal(biased.logits, (plain.logits + w.router_bias).astype(np.float32))


def test_reference_op_known_answers():
    """ops_test.cpp:18-24 (linear) and :48-56 (silu, softmax) of the reference."""
    x = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    wt = np.array([[1, 0, -1], [0.5, 0.5, 0.5]], np.float32)
    b = np.array([10, 20], np.float32)
    y = np.empty((2, 2), np.float32)
    O.lib().oracle_linear(O._p(x), 2, 3, O._p(wt), 2, O._p(b), O._p(y), 1)
    np.testing.assert_allclose(y, [[8, 23], [8, 27.5]], rtol=1e-5)
    # A one-expert, one-token MoE exposes silu: gate = 2, up = 1, down = 1 -> silu(2).
    w1 = O.MoeWeights(np.ones((1, 1), np.float32), np.full((1, 1), 2.0, np.float32), np.ones((1, 1), np.float32),
                      np.ones((1, 1), np.float32), np.zeros((0, 1), np.float32), np.zeros((0, 1), np.float32),
                      np.zeros((1, 0), np.float32))
    r = O.moe_forward(w1, np.ones((1, 1), np.float32), 1, renormalize=False)
    assert abs(r.y[0, 0] - 2 / (1 + np.exp(-2.0))) < 1e-6
    assert r.weights[0, 0] == 1.0  # softmax over one expert


def test_softmax_values_through_router():
    """ops_test.cpp:52-55: softmax([0, 0, log 2]) = [.25, .25, .5]; top-1 picks the 0.5."""
    H = 1
    router = np.array([[0.0], [0.0], [np.log(2.0)]], np.float32)
    z = np.zeros((3, H), np.float32)
    w = O.MoeWeights(router, np.zeros((3, H), np.float32), z.copy(), z.copy(), np.zeros((0, H), np.float32),
                     np.zeros((0, H), np.float32), np.zeros((H, 0), np.float32))
    r = O.moe_forward(w, np.ones((1, H), np.float32), 2, renormalize=False)
    assert r.ids.tolist() == [[2, 0]]  # tie between 0 and 1 -> lower id
    np.testing.assert_allclose(r.weights, [[0.5, 0.25]], rtol=1e-6)


def test_thread_count_independence():
    rng = np.random.default_rng(5)
    w = _random_layer(rng, 72, 12, 24, 40)
    x = rng.standard_normal((33, 72)).astype(np.float32)
    base = O.moe_forward(w, x, 4, renormalize=True, threads=1).y
    for th in (2, 7):
        assert np.array_equal(base, O.moe_forward(w, x, 4, renormalize=True, threads=th).y)


def test_quantiser_half_step_bound_per_channel():
    rng = np.random.default_rng(6)
    w = (rng.standard_normal((40, 96)) * 0.1).astype(np.float32)
    w[3] = 0.0  # an all-zero row takes scale 1 (device_weight.cpp:19)
    q, s = O.quantize_q8(w)
    assert s.shape == (40, 1) and s[3, 0] == 1.0 and not q[3].any()
    deq = O.dequantize_q8(q, s)
    peak = np.abs(w).max(axis=1, keepdims=True)
    assert np.all(np.abs(deq - w) <= peak / 254.0 + 1e-7)
    assert np.abs(q).max() <= 127
    q32, s32 = O.quantize_q8(w, group=32)  # the reference's own per-32 format
    assert s32.shape == (40, 3)


def test_synth_statistics_and_determinism():
    a = O.synth(9, 2, O.KIND_GATE, 5, 200000, 0.02)
    b = O.synth(9, 2, O.KIND_GATE, 5, 200000, 0.02)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 0.02 * 0.01 and abs(a.std() / 0.02 - 1) < 0.01
    tail = O.synth(9, 2, O.KIND_GATE, 5, 1000, 0.02, offset=199000)
    assert np.array_equal(tail, a[199000:])
    other = O.synth(9, 2, O.KIND_GATE, 6, 1000, 0.02)
    assert not np.array_equal(other, a[:1000])


def test_rms_norm_known_answer():
    # one row [3, 4]: ss = 25, mean 12.5, inv = 1/sqrt(12.5) in float
    x = np.array([[3.0, 4.0]], np.float32)
    inv = np.float32(1.0 / np.sqrt(12.5))
    got = O.rms_norm(x, np.array([1.0, 2.0], np.float32), 0.0)
    assert np.array_equal(got, np.array([[np.float32(3.0) * inv, np.float32(2.0) * (np.float32(4.0) * inv)]],
                                        np.float32))


@pytest.mark.skipif(not O.ref_available(), reason="reference sources not present (oracle/_ref not built)")
@pytest.mark.parametrize("H", [64, 1280, 2048])
def test_rms_norm_matches_reference(H):
    """The restatement of ref::rms_norm (ops.cpp:129-141) against the reference's own, bit for bit."""
    rng = np.random.default_rng(H)
    x = (rng.standard_normal((40, H)) * rng.choice([1e-3, 1.0, 50.0], (40, 1))).astype(np.float32)
    x[0] = 0.0  # an all-zero row: inv = 1 / sqrt(eps)
    g = rng.standard_normal(H).astype(np.float32)
    for gain in (None, g):
        for eps in (1e-6, 1e-5):
            a = O.rms_norm(x, gain, eps)
            b = O.ref_rms_norm(x, gain, eps)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))

