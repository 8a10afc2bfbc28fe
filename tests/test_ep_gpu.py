"""Expert parallelism on one GPU: a local group of virtual ranks (plans on the
same device, phases run rank after rank on one stream) against a single
plan over the same rows. Every output row must be bitwise the single plan's:
the exchange moves rows, it does not re-associate any sum.
"""
import numpy as np
import pytest

import oracle as O
import uocr_moe as M
from conftest import max_rel
from test_decode_gpu import BF16_TOL, _tiny_layer, _upload, to_np

pytestmark = pytest.mark.gpu


def _group(n, dims, max_rows, w, torch, cuda, strided=False, owner=None):
    flags = M.PLAN_EP_STRIDED if strided else 0
    plans = [M.Plan(dims, max_rows=max_rows, router_bias=w.router_bias is not None, flags=flags, ep_world=n,
                    ep_rank=r, ep_owner=owner) for r in range(n)]
    keep = [_upload(p, w, torch, cuda) for p in plans]
    M.ep_connect_local(plans)
    return plans, keep


def _skewed(rng, H, E, F, S):
    w = _tiny_layer(rng, H, E, F, S)
    # Zipf-like popularity: a few hot experts, a cold tail.
    w.router_bias = (1.2 * np.log(1.0 / np.arange(1, E + 1))).astype(np.float32)
    return w


@pytest.mark.parametrize("n,strided,rows", [
    (2, False, [40, 300]), (4, True, [0, 17, 129, 64]), (4, False, [100, 100, 100, 100]), (8, False, [33] * 8),
    (8, True, [1, 0, 5, 200, 16, 0, 77, 3])])
def test_local_group_equals_single_plan(cuda, n, strided, rows):
    import torch
    rng = np.random.default_rng(sum(rows) + n)
    H, E, K, F, S = 256, 32, 4, 128, 128
    w = _skewed(rng, H, E, F, S)
    dims = M.Dims(H, E, K, F, S)
    plans, keep = _group(n, dims, max(max(rows), 1), w, torch, cuda, strided)
    x = torch.from_numpy(rng.standard_normal((sum(rows), H)).astype(np.float32)).to(cuda)
    xs = list(torch.split(x, rows))
    xs = [t.contiguous() for t in xs]
    ys = [torch.full_like(t, float("nan")) for t in xs]
    M.ep_forward_local(plans, 0, xs, ys)
    for p in plans:
        p.check()
    single = M.Plan(dims, max_rows=sum(rows), router_bias=True)
    _upload(single, w, torch, cuda)
    y = torch.empty_like(x)
    single.forward(0, x, y)
    single.check()
    assert torch.equal(torch.cat(ys), y)
    want = O.moe_forward(w, to_np(x), K, renormalize=True)
    assert max_rel(to_np(torch.cat(ys)), want.y) <= BF16_TOL
    del keep


def test_local_group_pre_norm_equals_single_plan(cuda):
    """PLAN_PRE_NORM under expert parallelism: each rank normalises its own rows
    (the same summation order as a single plan), so the group's output is
    still bitwise the single plan's."""
    import torch
    rng = np.random.default_rng(21)
    H, E, K, F, S, n = 256, 16, 4, 128, 128, 2
    w = _skewed(rng, H, E, F, S)
    dims = M.Dims(H, E, K, F, S)
    g = torch.from_numpy((1.0 + 0.3 * rng.standard_normal(H)).astype(np.float32)).to(cuda)
    plans = [M.Plan(dims, max_rows=64, router_bias=True, flags=M.PLAN_PRE_NORM, rms_norm_eps=1e-5, ep_world=n,
                    ep_rank=r) for r in range(n)]
    single = M.Plan(dims, max_rows=128, router_bias=True, flags=M.PLAN_PRE_NORM, rms_norm_eps=1e-5)
    keep = []
    for p in plans + [single]:
        k = _upload(p, w, torch, cuda)
        p.set_layer(0, k["router"], k["gate"], k["up"], k["down"], k["shared_gate"], k["shared_up"],
                    k["shared_down"], router_bias=k["router_bias"], norm=g)
        keep.append(k)
    M.ep_connect_local(plans)
    x = torch.from_numpy((rng.standard_normal((90, H)) * 4.0).astype(np.float32)).to(cuda)
    rows = [64, 26]
    xs = [t.contiguous() for t in torch.split(x, rows)]
    ys = [torch.empty_like(t) for t in xs]
    M.ep_forward_local(plans, 0, xs, ys)
    y = torch.empty_like(x)
    single.forward(0, x, y)
    for p in plans + [single]:
        p.check()
    assert torch.equal(torch.cat(ys), y)
    want = O.moe_forward(w, O.rms_norm(to_np(x), to_np(g), 1e-5), K, renormalize=True)
    assert max_rel(to_np(y), want.y) <= BF16_TOL
    del keep


def test_local_group_repeats_and_stacks(cuda):
    """Several layers and repeated calls reuse the exchange buffers safely."""
    import torch
    rng = np.random.default_rng(3)
    H, E, K, F, S, n = 256, 16, 2, 128, 0, 2
    layers = [_skewed(rng, H, E, F, S) for _ in range(3)]
    dims = M.Dims(H, E, K, F, S, layers=3)
    plans = [M.Plan(dims, max_rows=64, router_bias=True, ep_world=n, ep_rank=r) for r in range(n)]
    keep = [[_upload(p, wl, torch, cuda, layer=i) for i, wl in enumerate(layers)] for p in plans]
    M.ep_connect_local(plans)
    single = M.Plan(dims, max_rows=128, router_bias=True)
    keep.append([_upload(single, wl, torch, cuda, layer=i) for i, wl in enumerate(layers)])
    x = torch.from_numpy(rng.standard_normal((100, H)).astype(np.float32)).to(cuda)
    rows = [64, 36]
    for layer in (0, 1, 2, 1):
        xs = [t.contiguous() for t in torch.split(x, rows)]
        ys = [torch.empty_like(t) for t in xs]
        M.ep_forward_local(plans, layer, xs, ys)
        y = torch.empty_like(x)
        single.forward(layer, x, y)
        for p in plans + [single]:
            p.check()
        assert torch.equal(torch.cat(ys), y)
        x = y


def test_ep_plan_misuse_is_reported(cuda):
    import torch
    rng = np.random.default_rng(4)
    H, E, K, F, S = 256, 16, 2, 128, 128
    w = _tiny_layer(rng, H, E, F, S)
    lone = M.Plan(M.Dims(H, E, K, F, S), max_rows=32, ep_world=2, ep_rank=0)
    _upload(lone, w, torch, cuda)
    x = torch.zeros(20, H, device=cuda)
    y = torch.zeros(20, H, device=cuda)
    with pytest.raises(M.UocrError) as e:
        lone.forward(0, x, y)  # not connected
    assert e.value.code == 1
    plans, keep = _group(2, M.Dims(H, E, K, F, S), 32, w, torch, cuda)
    with pytest.raises(M.UocrError) as e:
        plans[0].forward(0, x, y)  # local-group ranks only run through ep_forward_local
    assert e.value.code == 1
    with pytest.raises(M.UocrError) as e:
        M.ep_forward_local(plans[::-1], 0, [x, x], [y, y])  # not in rank order
    assert e.value.code == 1
    # Two ranks on one GPU may not connect through IPC handles.
    a = M.Plan(M.Dims(H, E, K, F, S), max_rows=32, ep_world=2, ep_rank=0)
    b = M.Plan(M.Dims(H, E, K, F, S), max_rows=32, ep_world=2, ep_rank=1)
    with pytest.raises(M.UocrError) as e:
        a.ep_connect([a.ep_handle(), b.ep_handle()])
    assert e.value.code == 2
    # A handle of a differently shaped plan is refused.
    c = M.Plan(M.Dims(H, E, K, F, S), max_rows=64, ep_world=2, ep_rank=1)
    with pytest.raises(M.UocrError) as e:
        a.ep_connect([a.ep_handle(), c.ep_handle()])
    assert e.value.code == 1
    del keep


@pytest.mark.parametrize("n,rows", [(2, [300, 257]), (4, [0, 129, 500, 64]), (8, [100] * 8)])
def test_balanced_placement_equals_single_plan(cuda, n, rows):
    """A load-balanced owner table (hot experts replicated, their rows split
    by source rank; ranks holding different numbers of experts) moves rows
    differently but must still give the single plan's output bit for bit."""
    import torch

    import ep
    rng = np.random.default_rng(7 * n + sum(rows))
    H, E, K, F, S = 256, 32, 4, 128, 128
    w = _skewed(rng, H, E, F, S)
    dims = M.Dims(H, E, K, F, S)
    x = torch.from_numpy(rng.standard_normal((sum(rows), H)).astype(np.float32)).to(cuda)
    single = M.Plan(dims, max_rows=sum(rows), router_bias=True)
    _upload(single, w, torch, cuda)
    y = torch.empty_like(x)
    ids = torch.empty(sum(rows), K, dtype=torch.int32, device=cuda)
    single.forward(0, x, y, ids)
    single.check()
    # the calibration histogram: rows each source rank routes to each expert
    flat = ids.cpu().numpy()
    starts = np.concatenate([[0], np.cumsum(rows)])
    cbs = [np.bincount(flat[starts[r]:starts[r + 1]].ravel(), minlength=E) for r in range(n)]
    owner = ep.balanced_owner_table(cbs, n, share=0.1)  # a small share: the hot experts are replicated
    assert len({owner[e * n + s] for e in range(E) for s in range(n)}) == n
    assert any(len({owner[e * n + s] for s in range(n)}) > 1 for e in range(E))  # some expert is replicated
    plans, keep = _group(n, dims, max(max(rows), 1), w, torch, cuda, owner=owner)
    xs = [t.contiguous() for t in torch.split(x, rows)]
    ys = [torch.full_like(t, float("nan")) for t in xs]
    M.ep_forward_local(plans, 0, xs, ys)
    for p in plans:
        p.check()
    assert torch.equal(torch.cat(ys), y)
    del keep
