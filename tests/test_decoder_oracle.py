"""The page-decoder oracle on the CPU: its attention and rotation against the
reference's own attention_head and PageRope (oracle/_ref), and the
decode-equals-prefill property the reference's decoder test holds
(tests/decoder_test.cpp:92-97): a prefill of n rows followed by one decode
step gives the same last-row logits as a prefill of the n + 1 rows."""
import numpy as np
import pytest

import decoder_oracle as D
import oracle as O

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref (the reference's own build) not present")


@needs_ref
@pytest.mark.parametrize("lq,lk,d", [(1, 1, 128), (5, 17, 128), (32, 64, 64)])
def test_attention_head_matches_the_reference(lq, lk, d):
    rng = np.random.default_rng(lq * 31 + lk)
    q = rng.standard_normal((lq, d)).astype(np.float32)
    k = rng.standard_normal((lk, d)).astype(np.float32)
    v = rng.standard_normal((lk, d)).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    want = O.ref_attention_head(q, k, v, scale)
    got = D.attention_head(q, k, v, scale, np.full(lq, lk - 1))  # every key visible
    assert np.abs(got - want).max() <= 2e-6 * max(1.0, np.abs(want).max())


@needs_ref
def test_rotation_matches_page_rope():
    """The rotate-half arithmetic and fp32 angles of PageRope::apply: with the
    page coordinate 0 its page pair turns by angle 0, so the reference's
    table (63 token pairs, then the page pair) drives the oracle's rope."""
    rng = np.random.default_rng(3)
    rows, heads, dim = 9, 3, 128
    x = rng.standard_normal((rows, heads * dim)).astype(np.float32)
    tok = np.array([0, 1, 2, 7, 100, 1000, 4095, 5119, 40000])
    want, inv = O.ref_page_rope(x, dim, 1e4, 256.0, 1, 2, tok, np.zeros(rows, np.int64))
    inv = inv.copy()
    inv[-1] = 0.0  # the page pair: page coordinate 0, so angle 0 whatever the token
    got = D.rope(x, tok, dim, inv)
    assert np.abs(got - want).max() <= 1e-6 * max(1.0, np.abs(want).max())


def test_rope_table_is_plain_rope():
    inv = D.rope_inv_freq(128, 1e4)
    assert inv[0] == 1.0 and inv.shape == (64,)
    assert np.allclose(inv, 1e4 ** (-np.arange(64) / 64), rtol=1e-6)


def _tiny(int8=False):
    d = D.DecoderDims(hidden=256, layers=2, heads=2, kv_heads=1, head_dim=128, vocab=96, experts=4, top_k=2, ffn=32,
                      shared_ffn=64)
    return d, D.synth_weights(d, seed=7, int8=int8, norm_sigma=0.1)


@pytest.mark.parametrize("int8", [False, True])
def test_decode_step_equals_prefill_of_one_more_row(int8):
    d, w = _tiny(int8)
    rows = D.synth_prompt(d, 7, 6)
    a = D.DecoderOracle(d, w)
    a.prefill(rows[:5])
    tok = 17
    step = a.step(tok)
    b = D.DecoderOracle(d, w)
    full = np.concatenate([rows[:5], w.embed[tok][None, :]])
    last = b.prefill(full)
    np.testing.assert_allclose(step, last, rtol=0, atol=1e-5 * np.abs(last).max())
    assert a.length == 6 and b.length == 6


def test_gqa_head_sharing_and_causality():
    """A query head reads its group's key/value head, and a row never sees
    later rows: changing the last row leaves earlier rows' outputs alone."""
    rng = np.random.default_rng(11)
    q = rng.standard_normal((4, 128)).astype(np.float32)
    k = rng.standard_normal((4, 128)).astype(np.float32)
    v = rng.standard_normal((4, 128)).astype(np.float32)
    pos = np.arange(4)
    base = D.attention_head(q, k, v, 0.1, pos)
    k2, v2 = k.copy(), v.copy()
    k2[3] += 5.0
    v2[3] -= 3.0
    moved = D.attention_head(q, k2, v2, 0.1, pos)
    np.testing.assert_array_equal(base[:3], moved[:3])
    assert not np.array_equal(base[3], moved[3])
    np.testing.assert_allclose(base[0], v[0], rtol=1e-6)  # the first row sees only itself


def test_greedy_takes_the_lowest_id_on_a_tie():
    assert D.greedy(np.array([0.5, 2.0, 2.0, -1.0], np.float32)) == 1
