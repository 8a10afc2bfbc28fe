"""The arithmetic claim behind the decode softmax's warp-tree total.

The reference sums a row's softmax numerators in double in index order
(src/backend/reference/ops.cpp:179-183). The device sums them as a warp tree
(four strided elements per lane, then a butterfly) when every numerator is 0
or at least 2^-22, because then every partial sum is exact and the order of
the adds cannot matter; otherwise it sums sequentially. These tests check that
claim on adversarial rows, and that below the floor the order does matter (so
the fallback is needed).
"""
import numpy as np
import pytest

FLOOR = np.float32(2.0 ** -22)


def sequential(v):
    t = 0.0
    for a in v.astype(np.float64):
        t += a
    return t


def warp_tree(v):
    """Lane l holds elements l, l+32, l+64, l+96; then a shfl_xor butterfly."""
    E = v.shape[0]
    part = np.zeros(32)
    for lane in range(32):
        p = 0.0
        for i in range(4):
            e = lane + 32 * i
            if e < E:
                p += float(v[e])
        part[lane] = p
    off = 16
    while off:
        part = np.array([part[lane] + part[lane ^ off] for lane in range(32)])
        off //= 2
    assert np.all(part == part[0])
    return part[0]


def adversarial_rows(rng, E, n):
    rows = []
    for _ in range(n):
        kind = rng.integers(0, 4)
        if kind == 0:  # values just above the floor with one at 1.0
            v = (FLOOR * (1 + rng.random(E) * 3)).astype(np.float32)
        elif kind == 1:  # spread over the whole admissible range
            v = np.exp2(-rng.random(E) * 22).astype(np.float32)
        elif kind == 2:  # mantissas full of bits, near 1 and near the floor
            v = np.where(rng.random(E) < 0.5, 1 - rng.random(E) * 1e-3, FLOOR * (1 + rng.random(E))).astype(np.float32)
        else:  # exp() of standard-normal logits, with zeros mixed in
            v = np.exp(rng.standard_normal(E).astype(np.float32) * 4).astype(np.float32)
            v = np.where(v >= FLOOR, v, 0).astype(np.float32)
        v[rng.integers(0, E)] = 1.0
        v = np.minimum(v, np.float32(1.9999999))
        rows.append(v)
    return rows


@pytest.mark.parametrize("E", [8, 37, 64, 100, 128])
def test_tree_total_equals_sequential_above_floor(E):
    rng = np.random.default_rng(E)
    for v in adversarial_rows(rng, E, 300):
        assert np.all((v == 0) | (v >= FLOOR))
        assert warp_tree(v) == sequential(v)


def test_order_matters_below_floor():
    # 1 followed by 63 numerators of 2^-53: each sequential add rounds back to
    # 1, while the tree first adds the small ones to each other.
    w = np.array([1.0] + [2.0 ** -53] * 63, np.float32)
    assert sequential(w) == 1.0
    assert warp_tree(w) != sequential(w)
