"""Decode path (rows <= 16) on the GPU, through the C ABI, against the oracle.

Bars: expert ids and their order bit-exact except rows
whose k-th vs (k+1)-th router-logit margin is below 1e-3 (counted); layer
output max_rel (max|got-want| / max|want|) <= 2e-2 for bf16, <= 5e-2 for int8.
"""
import numpy as np
import pytest

import moe_configs as C
import oracle as O
import uocr_moe as M
from conftest import max_rel

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
INT8_TOL = 5e-2
MARGIN = 1e-3


def to_np(t):
    return t.detach().float().cpu().numpy()


def host_weights(t: dict) -> O.MoeWeights:
    H = t["router"].shape[1]
    z = lambda *s: np.zeros(s, np.float32)  # noqa: E731
    return O.MoeWeights(
        router=to_np(t["router"]), gate=to_np(t["gate"]), up=to_np(t["up"]), down=to_np(t["down"]),
        shared_gate=to_np(t["shared_gate"]) if "shared_gate" in t else z(0, H),
        shared_up=to_np(t["shared_up"]) if "shared_up" in t else z(0, H),
        shared_down=to_np(t["shared_down"]) if "shared_down" in t else z(H, 0),
        router_bias=to_np(t["router_bias"]) if "router_bias" in t else None)


def check_ids(got_ids, want: O.MoeResult):
    """ids and order exact except near-tie rows; returns the number of exempt rows."""
    exempt = 0
    for t in range(got_ids.shape[0]):
        if np.array_equal(got_ids[t], want.ids[t]):
            continue
        assert want.margin[t] < MARGIN or want.order_margin[t] < MARGIN, (
            f"row {t}: ids {got_ids[t]} != {want.ids[t]} with margin {want.margin[t]}")
        exempt += 1
    return exempt


def run_plan(plan, layer, x, k, torch):
    T = x.shape[0]
    y = torch.empty_like(x)
    ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, k, dtype=torch.float32, device=x.device)
    plan.forward(layer, x, y, ids, w)
    plan.check()
    return to_np(y), ids.cpu().numpy(), w.cpu().numpy()


def test_device_generator_matches_host(cuda):
    import torch
    for dt, sigma in ((torch.float32, 0.02), (torch.bfloat16, 1.0)):
        t = torch.empty(300001, dtype=dt, device=cuda)
        M.synth_fill(t, 5, 3, M.KIND_UP, 9, sigma, offset=77)
        want = O.synth(5, 3, M.KIND_UP, 9, 300001, sigma, offset=77)
        if dt == torch.bfloat16:
            want = O.round_bf16(want)
        assert np.array_equal(to_np(t).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("group", [None, 32])
def test_device_quantiser_matches_oracle(cuda, group):
    import torch
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((67, 256)) * 0.05).astype(np.float32)
    w[5] = 0
    q = torch.empty(67, 256, dtype=torch.int8, device=cuda)
    s = torch.empty(67, 256 // (group or 256), dtype=torch.float32, device=cuda)
    M.quantize_q8(torch.from_numpy(w).to(cuda), q, s, group=group)
    torch.cuda.synchronize()
    wq, ws = O.quantize_q8(w, group=group)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ws.view(np.uint32))


def _tiny_layer(rng, H, E, F, S, bf16=True):
    f = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float32)  # noqa: E731
    w = O.MoeWeights(f(E, H), f(E * F, H), f(E * F, H), f(E * H, F), f(S, H), f(S, H), f(H, S))
    if bf16:
        for name in ("router", "gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
            setattr(w, name, O.round_bf16(getattr(w, name)).reshape(getattr(w, name).shape))
    return w


def _upload(plan, w: O.MoeWeights, torch, cuda, layer=0):
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    keep = {k: d(getattr(w, k)) for k in ("router", "gate", "up", "down", "shared_gate", "shared_up", "shared_down")}
    if w.router_bias is not None:
        keep["router_bias"] = d(w.router_bias)
    plan.set_layer(layer, keep["router"], keep["gate"], keep["up"], keep["down"], keep["shared_gate"],
                   keep["shared_up"], keep["shared_down"], router_bias=keep.get("router_bias"))
    return keep


# (16, 2048, 128, ...): the router rows and x rows exceed the cluster router's
# shared memory, so the block-per-expert router with its last-block table build runs.
SMALL_SHAPES = [
    (16, 2048, 128, 8, 128, 128, True, 0),
    (1, 64, 8, 3, 32, 32, True, 0), (5, 128, 16, 1, 48, 0, True, 0), (16, 256, 128, 8, 64, 64, True, 0),
    (3, 96, 12, 4, 32, 48, False, 0), (16, 64, 2, 2, 16, 16, True, 0), (7, 128, 32, 6, 64, 128, True, 1),
    (16, 512, 64, 6, 256, 512, True, 1), (2, 1024, 16, 2, 1536, 2560, True, 0), (9, 2048, 16, 4, 2560, 128, True, 1)]
# hidden, ffn and shared widths that are all multiples of 128
TC_SHAPES = [(1, 256, 8, 3, 128, 128, True, 0), (5, 128, 128, 8, 128, 0, True, 0),
             (16, 512, 64, 6, 256, 256, False, 0), (11, 384, 24, 5, 384, 128, True, 0)]


@pytest.mark.parametrize("T,H,E,K,F,S,renorm,fmt,flags",
                         [s + (0,) for s in SMALL_SHAPES + TC_SHAPES])
def test_small_shapes_against_oracle(cuda, T, H, E, K, F, S, renorm, fmt, flags):
    import torch
    rng = np.random.default_rng(T * 7919 + E)
    w = _tiny_layer(rng, H, E, F, S)
    x = rng.standard_normal((T, H)).astype(np.float32)
    plan = M.Plan(M.Dims(H, E, K, F, S), max_rows=16, weight_format=fmt, renormalize=renorm, flags=flags)
    _upload(plan, w, torch, cuda)
    y, ids, wts = run_plan(plan, 0, torch.from_numpy(x).to(cuda), K, torch)
    ww = w
    if fmt == M.WEIGHT_INT8:
        ww = O.MoeWeights(w.router, *[O.dequantize_q8(*O.quantize_q8(getattr(w, n))) for n in
                                      ("gate", "up", "down", "shared_gate", "shared_up")],
                          O.dequantize_q8(*O.quantize_q8(w.shared_down)) if S else w.shared_down)
    want = O.moe_forward(ww, x, K, renormalize=renorm)
    check_ids(ids, want)
    assert max_rel(y, want.y) <= (INT8_TOL if fmt else BF16_TOL)
    np.testing.assert_allclose(wts, want.weights, rtol=1e-5, atol=1e-7)


def test_tied_router_rows_pick_lower_id(cuda):
    import torch
    rng = np.random.default_rng(2)
    w = _tiny_layer(rng, 64, 8, 32, 32)
    w.router[6] = w.router[2]
    w.router[4] = w.router[2]
    x = rng.standard_normal((9, 64)).astype(np.float32)
    plan = M.Plan(M.Dims(64, 8, 3, 32, 32), max_rows=16)
    _upload(plan, w, torch, cuda)
    _, ids, _ = run_plan(plan, 0, torch.from_numpy(x).to(cuda), 3, torch)
    want = O.moe_forward(w, x, 3, renormalize=True)
    assert np.array_equal(ids, want.ids)  # exact ties are not near-ties: no exemption


def _topk_want(logits, K):
    """float64 softmax of each row and its order: higher first, lower id on a tie."""
    l64 = logits.astype(np.float64)
    p = np.exp(l64 - l64.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    order = np.stack([np.lexsort((np.arange(row.size), -row)) for row in p])
    return p, order


@pytest.mark.parametrize("E,K", [(8, 3), (37, 6), (64, 6), (64, 8), (100, 1), (128, 8)])
@pytest.mark.parametrize("renorm", [False, True])
def test_expert_topk_edge_rows(cuda, E, K, renorm):
    """uocr_expert_topk on rows that take both totals of the softmax (numerators
    all >= 2^-22, or some smaller: logits scaled by 40), rows with exact ties,
    and a fully masked row (softmax of zeros, ops.cpp:175-177)."""
    import torch
    rng = np.random.default_rng(E * 31 + K)
    rows = 64
    logits = rng.standard_normal((rows, E)).astype(np.float32)
    logits[rows // 2:] *= 40
    for r in range(0, rows, 5):  # exact ties, one of them at the top
        a, b = rng.choice(E, 2, replace=False)
        logits[r, b] = logits[r, a]
        if r % 10 == 0:
            logits[r, a] = logits[r, b] = logits[r].max()
    logits[3] = -np.inf
    dl = torch.from_numpy(logits).to(cuda)
    ids = torch.empty(rows, K, dtype=torch.int64, device=cuda)
    wts = torch.empty(rows, K, dtype=torch.float32, device=cuda)
    M.expert_topk(dl, K, renorm, ids, wts)
    got_ids, got_w = ids.cpu().numpy(), wts.cpu().numpy()
    p, order = _topk_want(np.where(np.isinf(logits), 0, logits), K)
    assert np.array_equal(got_ids[3], np.arange(K))
    if not renorm:
        assert np.all(got_w[3] == 0)
    for r in range(rows):
        if r == 3:
            continue
        want = order[r, :K]
        if not np.array_equal(got_ids[r], want):
            srt = p[r, order[r, :K + 1]]
            gaps = np.abs(np.diff(srt)) / np.maximum(srt[:-1], 1e-300)
            assert gaps.min() < 1e-5, f"row {r}: {got_ids[r]} != {want}"
            continue
        w = p[r, want]
        if renorm:
            w = w / w.sum()
        np.testing.assert_allclose(got_w[r], w, rtol=2e-6, atol=1e-30)


# (16, 2048, 128, ...) does not fit the 8-CTA cluster router's shared memory:
# it runs the 128-block router (its last block builds the table), which then
# normalises the rows it stages too.
@pytest.mark.parametrize("T,H,E,K,F,S,fmt", [(1, 64, 8, 3, 32, 32, 0), (5, 128, 16, 4, 48, 0, 1),
                                              (16, 256, 64, 6, 64, 64, 0), (9, 2048, 16, 4, 256, 128, 1),
                                              (16, 2048, 128, 8, 128, 128, 0)])
def test_pre_norm_against_oracle(cuda, T, H, E, K, F, S, fmt):
    """PLAN_PRE_NORM: y = MoE(RMSNorm(x)) with a per-layer gain, the decoder's
    feed-forward block (decoder.cpp:180-181) without its residual."""
    import torch
    rng = np.random.default_rng(T * 131 + H)
    w = _tiny_layer(rng, H, E, F, S)
    g = (1.0 + 0.3 * rng.standard_normal(H)).astype(np.float32)
    x = (rng.standard_normal((T, H)) * 7.0).astype(np.float32)  # not unit scale: the norm matters
    eps = 1e-5
    plan = M.Plan(M.Dims(H, E, K, F, S), max_rows=16, weight_format=fmt, flags=M.PLAN_PRE_NORM, rms_norm_eps=eps)
    keep = _upload(plan, w, torch, cuda)
    gd = torch.from_numpy(g).to(cuda)
    plan.set_layer(0, keep["router"], keep["gate"], keep["up"], keep["down"], keep["shared_gate"], keep["shared_up"],
                   keep["shared_down"], norm=gd)
    y, ids, _ = run_plan(plan, 0, torch.from_numpy(x).to(cuda), K, torch)
    ww = w
    if fmt == M.WEIGHT_INT8:
        ww = O.MoeWeights(w.router, *[O.dequantize_q8(*O.quantize_q8(getattr(w, n))) for n in
                                      ("gate", "up", "down", "shared_gate", "shared_up")],
                          O.dequantize_q8(*O.quantize_q8(w.shared_down)) if S else w.shared_down)
    want = O.moe_forward(ww, O.rms_norm(x, g, eps), K, renormalize=True)
    check_ids(ids, want)
    assert max_rel(y, want.y) <= (INT8_TOL if fmt else BF16_TOL)


@pytest.mark.parametrize("T,fmt,flags", [(1, 0, M.PLAN_PRE_NORM), (8, 0, M.PLAN_PRE_NORM), (1, 1, M.PLAN_PRE_NORM),
                                         (8, 0, 0), (300, 0, M.PLAN_PRE_NORM),
                                         (300, 1, M.PLAN_PRE_NORM)])
def test_checkpoint_dims(cuda, T, fmt, flags):
    """The checkpoint's own MoE shapes (src/weights/architecture.h:21-30:
    hidden 1280, 64 experts, top-6, expert ffn 896, 2 shared experts = 1792)
    with its own semantics (raw softmax weights, feed_forward.cpp:40), decode
    and prefill row counts, bf16 and int8, behind the pre-feed-forward norm."""
    import torch
    H, E, K, F, S = 1280, 64, 6, 896, 1792
    rng = np.random.default_rng(T + 7 * fmt + flags)
    w = _tiny_layer(rng, H, E, F, S)
    g = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    x = (rng.standard_normal((T, H)) * 2.0).astype(np.float32)
    plan = M.Plan(M.Dims(H, E, K, F, S), max_rows=max(T, 16), weight_format=fmt, renormalize=False, flags=flags)
    keep = _upload(plan, w, torch, cuda)
    pre = (flags & M.PLAN_PRE_NORM) != 0
    if pre:
        gd = torch.from_numpy(g).to(cuda)
        plan.set_layer(0, keep["router"], keep["gate"], keep["up"], keep["down"], keep["shared_gate"],
                       keep["shared_up"], keep["shared_down"], norm=gd)
    y, ids, _ = run_plan(plan, 0, torch.from_numpy(x).to(cuda), K, torch)
    ww = w
    if fmt == M.WEIGHT_INT8:
        ww = O.MoeWeights(w.router, *[O.dequantize_q8(*O.quantize_q8(getattr(w, n))) for n in
                                      ("gate", "up", "down", "shared_gate", "shared_up", "shared_down")])
    want = O.moe_forward(ww, O.rms_norm(x, g, 1e-6) if pre else x, K, renormalize=False)
    check_ids(ids, want)
    assert max_rel(y, want.y) <= (INT8_TOL if fmt else BF16_TOL)


def test_router_bias(cuda):
    import torch
    rng = np.random.default_rng(3)
    w = _tiny_layer(rng, 128, 16, 32, 32)
    w.router_bias = np.array(C.zipf_bias(16, 1.2), np.float32)
    x = rng.standard_normal((12, 128)).astype(np.float32)
    plan = M.Plan(M.Dims(128, 16, 4, 32, 32), max_rows=16, router_bias=True)
    _upload(plan, w, torch, cuda)
    y, ids, _ = run_plan(plan, 0, torch.from_numpy(x).to(cuda), 4, torch)
    want = O.moe_forward(w, x, 4, renormalize=True)
    check_ids(ids, want)
    assert max_rel(y, want.y) <= BF16_TOL


@pytest.fixture(scope="module")
def c1_layer(cuda):
    cfg = C.CONFIGS[1]
    t = C.device_layer(cfg, 0)
    return cfg, t, host_weights(t)


# The decode kernel set: CUDA-core weight streaming, one PDL-chained launch
# per phase.
DECODE_PATHS = {"layered": 0}


# 14 and 16 rows: the down kernel's activations no longer all fit in shared
# memory, so it stages the routed slots alone.
@pytest.mark.parametrize("path", list(DECODE_PATHS))
@pytest.mark.parametrize("T", [1, 4, 8, 14, 16])
def test_config1_layer_bf16(cuda, c1_layer, T, path):
    import torch
    cfg, t, hw = c1_layer
    plan = M.Plan(cfg.dims(layers=1), max_rows=16, renormalize=True, flags=DECODE_PATHS[path])
    C.load_layer(plan, cfg, 0, t)
    x = C.device_input(cfg, T)
    y, ids, _ = run_plan(plan, 0, x, cfg.top_k, torch)
    want = O.moe_forward(hw, to_np(x), cfg.top_k, renormalize=True)
    exempt = check_ids(ids, want)
    err = max_rel(y, want.y)
    print(f"config1 T={T}: max_rel {err:.2e}, exempt rows {exempt}")
    assert err <= BF16_TOL


@pytest.mark.parametrize("path", list(DECODE_PATHS))
@pytest.mark.parametrize("T", [1, 8, 16])
def test_config2_layer_int8(cuda, c1_layer, T, path):
    import torch
    cfg = C.CONFIGS[2]
    t = C.device_layer(cfg, 0)
    hw = host_weights(t)
    plan = M.Plan(cfg.dims(layers=1), max_rows=16, weight_format=M.WEIGHT_INT8, renormalize=True,
                  flags=DECODE_PATHS[path])
    C.load_layer(plan, cfg, 0, t)
    x = C.device_input(cfg, T)
    y, ids, _ = run_plan(plan, 0, x, cfg.top_k, torch)
    deq = lambda a: O.dequantize_q8(*O.quantize_q8(a))  # noqa: E731
    hq = O.MoeWeights(hw.router, deq(hw.gate), deq(hw.up), deq(hw.down), deq(hw.shared_gate), deq(hw.shared_up),
                      deq(hw.shared_down))
    want = O.moe_forward(hq, to_np(x), cfg.top_k, renormalize=True)
    exempt = check_ids(ids, want)
    err = max_rel(y, want.y)
    print(f"config2 T={T}: max_rel {err:.2e}, exempt rows {exempt}")
    assert err <= INT8_TOL


@pytest.mark.parametrize("path", list(DECODE_PATHS))
def test_stack_residual_two_layers(cuda, path):
    import torch
    cfg = C.CONFIGS[1]
    layers = [C.device_layer(cfg, l) for l in range(2)]
    plan = M.Plan(cfg.dims(layers=2), max_rows=8, flags=DECODE_PATHS[path])
    for l, t in enumerate(layers):
        C.load_layer(plan, cfg, l, t)
    x = C.device_input(cfg, 4)
    h = x.clone()
    plan.forward_stack(h)
    plan.check()
    want = to_np(x)
    for t in layers:
        want = want + O.moe_forward(host_weights(t), want, cfg.top_k, renormalize=True).y
    assert max_rel(to_np(h), want) <= BF16_TOL


def test_pre_norm_stack_two_layers_and_24_stay_finite(cuda):
    """forward_stack with PLAN_PRE_NORM: h <- h + MoE(RMSNorm(h)) per layer
    (unit gains). Two layers against the oracle; the full 24-layer config-1
    stack keeps finite values and varied routing (the plain residual stack
    of N(0, 0.02) SwiGLU layers grows quadratically and overflows)."""
    import torch
    cfg = C.CONFIGS[1]
    layers = [C.device_layer(cfg, l) for l in range(2)]
    plan = M.Plan(cfg.dims(layers=2), max_rows=8, flags=M.PLAN_PRE_NORM)
    for l, t in enumerate(layers):
        C.load_layer(plan, cfg, l, t)
    x = C.device_input(cfg, 4)
    h = x.clone()
    plan.forward_stack(h)
    plan.check()
    want = to_np(x)
    for t in layers:
        want = want + O.moe_forward(host_weights(t), O.rms_norm(want, None, 1e-6), cfg.top_k, renormalize=True).y
    assert max_rel(to_np(h), want) <= BF16_TOL
    del plan, layers
    plan = M.Plan(cfg.dims(), max_rows=8, flags=M.PLAN_PRE_NORM)
    for l in range(cfg.layers):
        C.load_layer(plan, cfg, l, C.device_layer(cfg, l))
    h = C.device_input(cfg, 8)
    y = torch.empty_like(h)
    ids = torch.empty(8, cfg.top_k, dtype=torch.int32, device=cuda)
    distinct = []
    for l in range(cfg.layers):
        plan.forward(l, h, y, ids)
        h = h + y
        distinct.append(len(set(ids.cpu().numpy().ravel().tolist())))
    plan.check()
    assert torch.isfinite(h).all()
    assert min(distinct) >= 20  # eight rows with independent routing touch ~35 of 64 experts


@pytest.mark.parametrize("path", list(DECODE_PATHS))
def test_stack_graph_replay_matches_plain_launches(cuda, path):
    """forward_stack on a capturable stream is captured once (with programmatic
    dependent launches between the kernels) and replayed; the replays give the
    bits of plain stream-ordered launches."""
    import torch
    cfg = C.CONFIGS[1]
    layers = [C.device_layer(cfg, l) for l in range(3)]
    extra = DECODE_PATHS[path]
    graphed = M.Plan(cfg.dims(layers=3), max_rows=8, flags=extra)
    plain = M.Plan(cfg.dims(layers=3), max_rows=8, flags=extra | M.PLAN_NO_GRAPHS)
    for l, t in enumerate(layers):
        C.load_layer(graphed, cfg, l, t)
        C.load_layer(plain, cfg, l, t)
    x = C.device_input(cfg, 8)
    s = torch.cuda.Stream()
    h1 = x.clone()
    h2 = x.clone()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for h in (h1, h2):
            for _ in range(3):  # capture, then two replays on the same buffer
                h.copy_(x)
                graphed.forward_stack(h, stream=s) if h is h1 else plain.forward_stack(h, stream=s)
    torch.cuda.synchronize()
    graphed.check()
    plain.check()
    assert torch.equal(h1, h2)


def test_forward_is_deterministic(cuda, c1_layer):
    import torch
    cfg, t, _ = c1_layer
    plan = M.Plan(cfg.dims(layers=1), max_rows=8)
    C.load_layer(plan, cfg, 0, t)
    x = C.device_input(cfg, 8)
    a, _, _ = run_plan(plan, 0, x, cfg.top_k, torch)
    b, _, _ = run_plan(plan, 0, x, cfg.top_k, torch)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_op_mirrors(cuda, c1_layer):
    """uocr_expert_topk / uocr_expert_ffn_one(_q8), the reference's op shapes."""
    import torch
    cfg, t, hw = c1_layer
    H, F, K = cfg.hidden, cfg.ffn, cfg.top_k
    x = C.device_input(cfg, 1)
    logits = (x @ t["router"].T).contiguous()
    ids = torch.empty(1, K, dtype=torch.int64, device=cuda)
    wts = torch.empty(1, K, dtype=torch.float32, device=cuda)
    M.expert_topk(logits, K, False, ids, wts)
    out = torch.empty(H, dtype=torch.float32, device=cuda)
    M.expert_ffn_one(x, H, F, t["gate"], t["up"], t["down"], ids, wts, K, out)
    torch.cuda.synchronize()
    xh = O.round_bf16(to_np(x)[0]).astype(np.float64)
    want = np.zeros(H)
    for j, e in enumerate(ids.cpu().numpy()[0]):
        g = hw.gate[e * F:(e + 1) * F].astype(np.float64) @ xh
        u = hw.up[e * F:(e + 1) * F].astype(np.float64) @ xh
        a = O.round_bf16((g / (1 + np.exp(-g)) * u).astype(np.float32)).astype(np.float64)
        want += wts.cpu().numpy()[0, j] * (hw.down[e * H:(e + 1) * H].astype(np.float64) @ a)
    assert max_rel(to_np(out), want) <= BF16_TOL
    sc = torch.softmax(logits.double(), dim=1)
    top = torch.topk(sc, K, dim=1)
    assert torch.equal(top.indices, ids)
    # int8 stacks, per output channel
    q = {n: torch.empty_like(t[n], dtype=torch.int8) for n in ("gate", "up", "down")}
    s = {n: torch.empty(t[n].shape[0], 1, dtype=torch.float32, device=cuda) for n in q}
    for n in q:
        M.quantize_q8(t[n], q[n], s[n])
    out8 = torch.empty(H, dtype=torch.float32, device=cuda)
    M.expert_ffn_one_q8(x, H, F, q["gate"], s["gate"], q["up"], s["up"], q["down"], s["down"], ids, wts, K, out8)
    torch.cuda.synchronize()
    assert max_rel(to_np(out8), want) <= INT8_TOL


def test_op_mirrors_report_bad_expert_ids(cuda):
    """An expert id outside [0, 128) given to the expert_ffn_one mirrors is
    reported by uocr_ops_check as UOCR_ERR_DEVICE (a host-visible status, the
    word is cleared by the check); the slot adds nothing to the output."""
    import torch
    H, F, E, K = 256, 128, 8, 4
    gate = torch.empty(E * F, H, dtype=torch.bfloat16, device=cuda)
    up = torch.empty_like(gate)
    down = torch.empty(E * H, F, dtype=torch.bfloat16, device=cuda)
    for i, t in enumerate((gate, up, down)):
        M.synth_fill(t, 31, 0, M.KIND_GATE + i, 0, 0.02)
    x = torch.empty(1, H, device=cuda)
    M.synth_fill(x, 31, 0, M.KIND_X, 0, 1.0)
    w = torch.tensor([[0.4, 0.3, 0.2, 0.1]], device=cuda)
    M.ops_check()  # clean before the test
    fns = {"bf16": lambda ids, ww, out: M.expert_ffn_one(x, H, F, gate, up, down, ids, ww, K, out),
           "noalloc": lambda ids, ww, out: M.expert_ffn_one_noalloc(x, H, F, gate, up, down, ids, ww, K, out)}
    for name, fn in fns.items():
        for bad in (200, -1):
            ids = torch.tensor([[3, bad, 1, 6]], dtype=torch.int64, device=cuda)
            got = torch.empty(H, device=cuda)
            fn(ids, w, got)
            with pytest.raises(M.UocrError) as e:
                M.ops_check()
            assert e.value.code == 5, name
            assert f"expert id {bad} at position 1" in str(e.value), name
            M.ops_check()  # the check cleared the word
            ids0 = torch.tensor([[3, 0, 1, 6]], dtype=torch.int64, device=cuda)
            w0 = w.clone()
            w0[0, 1] = 0.0
            want = torch.empty(H, device=cuda)
            fn(ids0, w0, want)
            M.ops_check()
            assert torch.equal(got, want), name


def test_forward_errors(cuda):
    import torch
    plan = M.Plan(M.Dims(64, 8, 2, 32, 32), max_rows=32)
    x = torch.zeros(4, 64, device=cuda)
    y = torch.zeros(4, 64, device=cuda)
    with pytest.raises(M.UocrError) as e:
        plan.forward(0, x, y)  # weights never set
    assert e.value.code == 1
    with pytest.raises(M.UocrError) as e:
        plan.forward(0, x, x)
    assert e.value.code == 1
    xm = torch.zeros(4 * 64 + 1, device=cuda)[1:].view(4, 64)  # 4 bytes past a 16-byte boundary
    with pytest.raises(M.UocrError, match="aligned") as e:
        plan.forward(0, xm, y)
    assert e.value.code == 1
    with pytest.raises(M.UocrError, match="aligned"):
        plan.forward_stack(xm)
