"""Loading MoE layers from a checkpoint (uocr_moe_set_layer_parts) on the GPU.

A synthetic checkpoint under the published tensor names, spread over two
shards, is loaded one tensor per expert straight from the mapped files; the
plan must compute exactly what a plan loaded from the host-stacked matrices
computes (uocr_moe_set_layer): bitwise equal outputs, ids and weights, on the
decode path (rows <= 16) and the prefill path, bf16 and int8, with the
checkpoint's pre-norm gain.
"""
import numpy as np
import pytest

import safetensors_py as C
import uocr_moe as M
from test_checkpoint import write_moe_checkpoint
from test_decode_gpu import run_plan

pytestmark = pytest.mark.gpu

H, E, K, F, S = 256, 8, 2, 128, 256
LAYERS = [1, 2]  # checkpoint layers -> plan layers 0, 1


def _widen(a):
    return (a.astype(np.uint32) << 16).view(np.float32) if a.dtype == np.uint16 else a


def _load_stacked(plan, arrays, layer, plan_layer, dtype, torch, cuda):
    """The same layer through uocr_moe_set_layer: experts stacked on the host."""
    p = f"model.layers.{layer}."

    def dev(a):
        a = np.ascontiguousarray(a)
        return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).to(cuda)

    stack = lambda proj: dev(np.concatenate([arrays[f"{p}mlp.experts.{e}.{proj}.weight"] for e in range(E)]))  # noqa: E731
    keep = [dev(_widen(arrays[p + "mlp.gate.weight"])), stack("gate_proj"), stack("up_proj"), stack("down_proj"),
            dev(arrays[p + "mlp.shared_experts.gate_proj.weight"]), dev(arrays[p + "mlp.shared_experts.up_proj.weight"]),
            dev(arrays[p + "mlp.shared_experts.down_proj.weight"]), dev(_widen(arrays[p + "post_attention_layernorm.weight"]))]
    plan.set_layer(plan_layer, *keep[:7], dtype=dtype, norm=keep[7])
    torch.cuda.synchronize()
    return keep


@pytest.mark.parametrize("fmt", [M.WEIGHT_BF16, M.WEIGHT_INT8])
@pytest.mark.parametrize("ckpt_dtype", ["BF16", "F32"])
def test_checkpoint_load_matches_stacked_upload(cuda, tmp_path, fmt, ckpt_dtype):
    import torch
    idx, arrays = write_moe_checkpoint(tmp_path, LAYERS, H, E, F, S, seed=7, dtype=ckpt_dtype)
    w = C.ShardedWeights.open(idx)
    dims = M.Dims(H, E, K, F, S, layers=len(LAYERS))
    a = M.Plan(dims, max_rows=64, weight_format=fmt, flags=M.PLAN_PRE_NORM)
    b = M.Plan(dims, max_rows=64, weight_format=fmt, flags=M.PLAN_PRE_NORM)
    dtype = M.DTYPE_BF16 if ckpt_dtype == "BF16" else M.DTYPE_F32
    for i, l in enumerate(LAYERS):
        C.load_moe_layer(a, w, l, plan_layer=i)
        _keep = _load_stacked(b, arrays, l, i, dtype, torch, cuda)
    rng = np.random.default_rng(3)
    for T in (1, 5, 16, 40):
        x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(cuda)
        for i in range(len(LAYERS)):
            ya, ia, wa = run_plan(a, i, x, K, torch)
            yb, ib, wb = run_plan(b, i, x, K, torch)
            assert np.isfinite(ya).all()
            np.testing.assert_array_equal(ia, ib)
            assert np.array_equal(wa.view(np.int32), wb.view(np.int32))
            assert np.array_equal(ya.view(np.int32), yb.view(np.int32)), (T, i)
        ha, hb = x.clone(), x.clone()
        a.forward_stack(ha)
        b.forward_stack(hb)
        torch.cuda.synchronize()
        assert torch.equal(ha.view(torch.int32), hb.view(torch.int32)), T
    a.close()
    b.close()


def test_checkpoint_parts_from_device_memory(cuda, tmp_path):
    """The same entry point with every part already on the device (a loader
    that uploads tensors one by one)."""
    import torch
    idx, arrays = write_moe_checkpoint(tmp_path, [1], H, E, F, S, seed=9)
    w = C.ShardedWeights.open(idx)
    dims = M.Dims(H, E, K, F, S)
    a = M.Plan(dims, max_rows=16, flags=M.PLAN_PRE_NORM)
    b = M.Plan(dims, max_rows=16, flags=M.PLAN_PRE_NORM)
    C.load_moe_layer(a, w, 1, plan_layer=0)
    p = "model.layers.1."
    dev = lambda n: torch.from_numpy(np.ascontiguousarray(arrays[p + n]).view(np.int16)).to(cuda)  # noqa: E731
    parts = {proj: [dev(f"mlp.experts.{e}.{proj}.weight") for e in range(E)] for proj in C.PROJS}
    shared = [dev(f"mlp.shared_experts.{proj}.weight") for proj in C.PROJS]
    b.set_layer_parts(0, dev("mlp.gate.weight"), parts["gate_proj"], parts["up_proj"], parts["down_proj"], *shared,
                      memory=M.MEMORY_DEVICE, dtype=M.DTYPE_BF16, norm=dev("post_attention_layernorm.weight"))
    x = torch.from_numpy(np.random.default_rng(4).standard_normal((3, H)).astype(np.float32)).to(cuda)
    ya, ia, _ = run_plan(a, 0, x, K, torch)
    yb, ib, _ = run_plan(b, 0, x, K, torch)
    np.testing.assert_array_equal(ia, ib)
    assert np.array_equal(ya.view(np.int32), yb.view(np.int32))
    a.close()
    b.close()


def test_checkpoint_load_rejects_a_bad_layer(cuda, tmp_path):
    gone = "model.layers.1.mlp.experts.5.down_proj.weight"
    idx, _ = write_moe_checkpoint(tmp_path, [1], H, E, F, S, drop=gone)
    plan = M.Plan(M.Dims(H, E, K, F, S), max_rows=16)
    with pytest.raises(C.CheckpointError, match=f"missing {gone}"):
        C.load_moe_layer(plan, C.ShardedWeights.open(idx), 1, plan_layer=0)
    with pytest.raises(M.UocrError, match="set_layer_parts: gate, up and down"):
        plan.set_layer_parts(0, 0, None, None, None)
    plan.close()


@pytest.mark.parametrize("strided", [False, True])
def test_checkpoint_load_into_expert_parallel_ranks(cuda, tmp_path, strided):
    """Each virtual rank of a local expert-parallel group reads only its own
    experts from the checkpoint; the group computes what one plan does."""
    import torch
    idx, _ = write_moe_checkpoint(tmp_path, [1], H, E, F, S, seed=11)
    w = C.ShardedWeights.open(idx)
    dims = M.Dims(H, E, K, F, S)
    flags = M.PLAN_PRE_NORM | (M.PLAN_EP_STRIDED if strided else 0)
    plans = [M.Plan(dims, max_rows=64, flags=flags, ep_world=2, ep_rank=r) for r in range(2)]
    for p in plans:
        C.load_moe_layer(p, w, 1, plan_layer=0)
    M.ep_connect_local(plans)
    single = M.Plan(dims, max_rows=128, flags=M.PLAN_PRE_NORM)
    C.load_moe_layer(single, w, 1, plan_layer=0)
    rows = [40, 24]
    x = torch.from_numpy(np.random.default_rng(5).standard_normal((sum(rows), H)).astype(np.float32)).to(cuda)
    xs = [t.contiguous() for t in torch.split(x, rows)]
    ys = [torch.full_like(t, float("nan")) for t in xs]
    M.ep_forward_local(plans, 0, xs, ys)
    for p in plans:
        p.check()
    y = torch.empty_like(x)
    single.forward(0, x, y)
    single.check()
    assert torch.equal(torch.cat(ys), y)


@pytest.mark.parametrize("fmt,ckpt_dtype", [(M.WEIGHT_BF16, "BF16"), (M.WEIGHT_INT8, "BF16"), (M.WEIGHT_BF16, "F32")])
def test_native_loader_matches_python_loader(cuda, tmp_path, fmt, ckpt_dtype):
    """uocr_moe_load_layer (the library's own reader and packing) loads what
    safetensors_py.load_moe_layer loads, bit for bit."""
    import torch
    idx, _ = write_moe_checkpoint(tmp_path, LAYERS, H, E, F, S, seed=13, dtype=ckpt_dtype, shards=3)
    dims = M.Dims(H, E, K, F, S, layers=len(LAYERS))
    a = M.Plan(dims, max_rows=64, weight_format=fmt, flags=M.PLAN_PRE_NORM)
    b = M.Plan(dims, max_rows=64, weight_format=fmt, flags=M.PLAN_PRE_NORM)
    ck = M.Checkpoint(idx)
    w = C.ShardedWeights.open(idx)
    for i, l in enumerate(LAYERS):
        ck.load_layer(a, l, i)
        C.load_moe_layer(b, w, l, plan_layer=i)
    rng = np.random.default_rng(6)
    for T in (1, 8, 33):
        x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(cuda)
        ha, hb = x.clone(), x.clone()
        a.forward_stack(ha)
        b.forward_stack(hb)
        a.check()
        b.check()
        assert torch.equal(ha.view(torch.int32), hb.view(torch.int32)), T
    ck.close()
    a.close()
    b.close()


def test_native_loader_rejects_a_bad_layer(cuda, tmp_path):
    gone = "model.layers.1.mlp.experts.2.gate_proj.weight"
    flat = "model.layers.1.mlp.shared_experts.up_proj.weight"
    idx, _ = write_moe_checkpoint(tmp_path, [1], H, E, F, S, drop=gone)
    plan = M.Plan(M.Dims(H, E, K, F, S), max_rows=16)
    ck = M.Checkpoint(idx)
    with pytest.raises(M.UocrError, match=f"load_layer: missing {gone}"):
        ck.load_layer(plan, 1, 0)
    with pytest.raises(M.UocrError, match="load_layer: missing model.layers.4.mlp.gate.weight"):
        ck.load_layer(plan, 4, 0)
    d2 = tmp_path / "flat"
    d2.mkdir()
    idx2, _ = write_moe_checkpoint(d2, [1], H, E, F, S, reshape=flat)
    with pytest.raises(M.UocrError, match=f"{flat}: shape \\[65536\\], expected \\[256, 256\\]"):
        M.Checkpoint(idx2).load_layer(plan, 1, 0)
    biased = M.Plan(M.Dims(H, E, K, F, S), max_rows=16, router_bias=True)
    with pytest.raises(M.UocrError, match="router bias"):
        M.Checkpoint(idx2).load_layer(biased, 1, 0)
    ck.close()
    plan.close()
    biased.close()
