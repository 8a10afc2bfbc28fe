"""uocr_expert_ffn_one_noalloc, the entry point for callers that cannot
allocate device memory (a pool reserved up front by another allocator, a
decode step that must not synchronise on cudaMalloc, a runtime that forbids
allocations after start-up). It launches the same kernels as
uocr_expert_ffn_one, whose scratch comes from cudaMallocAsync, so on two calls
in a row — the second reusing the static scratch the first one left behind —
its outputs must equal that entry point's bit for bit, and match a float64
restatement of the expert sum within the decode tests' bf16 tolerance. The
device's free memory must not move across those calls. This file is collected
last on purpose; it needs nothing from the other test files, so it also runs
alone in a fresh process.
"""
import numpy as np
import pytest

import oracle as O
import uocr_moe as M
from conftest import max_rel

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2  # the decode tests' bf16 tolerance


def _stack(torch, cuda, rows, cols, seed, kind, experts):
    t = torch.empty(experts * rows, cols, dtype=torch.bfloat16, device=cuda)
    for e in range(experts):
        M.synth_fill(t[e * rows:(e + 1) * rows], seed, 0, kind, e, 0.02)
    return t


def _fp64_expert_sum(x, gate, up, down, ids, wts, H, F):
    """out = sum_j w_j down_j(bf16(silu(gate_j x) up_j x)), x rounded to bf16,
    every product and sum in float64 (the op's definition, not its order)."""
    xh = O.round_bf16(x).astype(np.float64)
    out = np.zeros(H)
    for e, w in zip(ids, wts):
        g = gate[e * F:(e + 1) * F].astype(np.float64) @ xh
        u = up[e * F:(e + 1) * F].astype(np.float64) @ xh
        a = O.round_bf16((g / (1 + np.exp(-g)) * u).astype(np.float32)).astype(np.float64)
        out += float(np.float32(w)) * (down[e * H:(e + 1) * H].astype(np.float64) @ a)
    return out


def test_noalloc_matches_allocating_entry_point_twice(cuda):
    import torch
    H, F, E, K = 2048, 1024, 16, 6
    gate = _stack(torch, cuda, F, H, 21, M.KIND_GATE, E)
    up = _stack(torch, cuda, F, H, 21, M.KIND_UP, E)
    down = _stack(torch, cuda, H, F, 21, M.KIND_DOWN, E)
    calls = [([3, 0, 15, 7, 9, 1], [0.3, 0.2, 0.15, 0.15, 0.1, 0.1], 1),
             ([12, 4, 5, 2, 8, 14], [0.25, 0.25, 0.2, 0.1, 0.1, 0.1], 2)]
    inputs, wants = [], []
    for chosen, wts, xseed in calls:
        x = torch.empty(1, H, dtype=torch.float32, device=cuda)
        M.synth_fill(x, xseed, 0, M.KIND_X, 0, 1.0)
        ids = torch.tensor([chosen], dtype=torch.int64, device=cuda)
        w = torch.tensor([wts], dtype=torch.float32, device=cuda)
        want = torch.empty(H, dtype=torch.float32, device=cuda)
        M.expert_ffn_one(x, H, F, gate, up, down, ids, w, K, want)
        inputs.append((x, ids, w))
        wants.append(want)
    outs = [torch.full((H,), float("nan"), dtype=torch.float32, device=cuda) for _ in calls]
    # A first call on this device looks the static array's address up; it
    # runs before the free-memory reading so that only the calls under test
    # are inside it.
    warm = torch.empty(H, dtype=torch.float32, device=cuda)
    x0, ids0, w0 = inputs[0]
    M.expert_ffn_one_noalloc(x0, H, F, gate, up, down, ids0, w0, K, warm)
    torch.cuda.synchronize()
    # Nothing may be allocated across the two calls: the device's free bytes
    # and torch's allocated bytes must not grow (a collection of other
    # tests' garbage may shrink the latter meanwhile).
    import gc
    gc.collect()
    free_before = torch.cuda.mem_get_info()[0]
    torch_before = torch.cuda.memory_allocated()
    for (x, ids, w), got in zip(inputs, outs):
        M.expert_ffn_one_noalloc(x, H, F, gate, up, down, ids, w, K, got)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free_before
    assert torch.cuda.memory_allocated() <= torch_before
    M.ops_check()
    for got, want in zip(outs, wants):
        assert torch.equal(got, want)
    hg, hu, hd = (t.float().cpu().numpy() for t in (gate, up, down))
    for (x, ids, w), got, (chosen, wts, _) in zip(inputs, outs, calls):
        ref = _fp64_expert_sum(x.cpu().numpy()[0], hg, hu, hd, chosen, wts, H, F)
        g = got.cpu().numpy()
        assert np.isfinite(g).all()
        assert max_rel(g, ref) <= BF16_TOL


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    import torch
    x = torch.zeros(1, 64, device=cuda)
    out = torch.zeros(64, device=cuda)
    ids = torch.zeros(1, 8, dtype=torch.int64, device=cuda)
    w = torch.zeros(1, 8, device=cuda)
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(M.UocrError) as e:
        M.expert_ffn_one_noalloc(x, 64, 8192 + 16, dummy, dummy, dummy, ids, w, 8, out)
    assert e.value.code == 1 and "8192" in str(e.value)
    with pytest.raises(M.UocrError) as e:
        M.expert_ffn_one_noalloc(x, 64, 32, dummy, dummy, dummy, ids, w, 9, out)
    assert e.value.code == 1
