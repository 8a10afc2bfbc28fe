"""uocr_expert_ffn_one_noalloc, the entry point for callers that cannot
allocate device memory (a pool reserved up front by another allocator, a
decode step that must not synchronise on cudaMalloc, a runtime that forbids
allocations after start-up). It must give the results of
uocr_expert_ffn_one, whose scratch comes from cudaMallocAsync, on two calls
in a row — the second call reuses the static scratch the first one left
behind. This file is collected last on purpose; it needs nothing from the
other test files, so it also runs alone in a fresh process.
"""
import numpy as np
import pytest

import uocr_moe as M
from conftest import max_rel

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2  # the decode tests' bf16 tolerance


def _stack(torch, cuda, rows, cols, seed, kind, experts):
    t = torch.empty(experts * rows, cols, dtype=torch.bfloat16, device=cuda)
    for e in range(experts):
        M.synth_fill(t[e * rows:(e + 1) * rows], seed, 0, kind, e, 0.02)
    return t


def test_noalloc_matches_allocating_entry_point_twice(cuda):
    import torch
    H, F, E, K = 2048, 1024, 16, 6
    gate = _stack(torch, cuda, F, H, 21, M.KIND_GATE, E)
    up = _stack(torch, cuda, F, H, 21, M.KIND_UP, E)
    down = _stack(torch, cuda, H, F, 21, M.KIND_DOWN, E)
    calls = [([3, 0, 15, 7, 9, 1], [0.3, 0.2, 0.15, 0.15, 0.1, 0.1], 1),
             ([12, 4, 5, 2, 8, 14], [0.25, 0.25, 0.2, 0.1, 0.1, 0.1], 2)]
    for chosen, wts, xseed in calls:
        x = torch.empty(1, H, dtype=torch.float32, device=cuda)
        M.synth_fill(x, xseed, 0, M.KIND_X, 0, 1.0)
        ids = torch.tensor([chosen], dtype=torch.int64, device=cuda)
        w = torch.tensor([wts], dtype=torch.float32, device=cuda)
        want = torch.empty(H, dtype=torch.float32, device=cuda)
        got = torch.full((H,), float("nan"), dtype=torch.float32, device=cuda)
        M.expert_ffn_one(x, H, F, gate, up, down, ids, w, K, want)
        M.expert_ffn_one_noalloc(x, H, F, gate, up, down, ids, w, K, got)
        torch.cuda.synchronize()
        g, r = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        assert max_rel(g, r) <= BF16_TOL


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
