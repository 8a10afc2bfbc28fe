"""The page decoder on the GPU (uocr_decoder through the C ABI) against the CPU
restatement (oracle/decoder_oracle.py): prefill logits, then each greedy decode
step's logits with the device's own tokens fed back to the oracle (teacher
forcing). Bars: max_rel (max|got-want| / max|want|) <= 2e-2 for bf16 and
<= 5e-2 for int8 weights, the north star's layer tolerances."""
import numpy as np
import pytest

import decoder_oracle as D
import uocr_moe as M
from conftest import max_rel

pytestmark = pytest.mark.gpu

TOL = {M.WEIGHT_BF16: 2e-2, M.WEIGHT_INT8: 5e-2}

# (hidden, layers, heads, kv_heads, vocab, experts, top_k, ffn, shared, prefill rows, decode steps)
SHAPES = [
    (512, 2, 4, 1, 1024, 8, 2, 128, 256, 70, 6),    # 4 query heads per kv head, two prefill tiles
    (1024, 2, 8, 4, 768, 16, 4, 128, 128, 17, 5),  # 2 per kv head, the MoE prefill path at 17 rows
    (512, 1, 4, 2, 512, 8, 2, 128, 256, 9, 4),     # a prefill short enough for the MoE decode kernels
]


def _device_layer(torch, cuda, L: D.DecoderLayer):
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda)  # noqa: E731
    return {"input_norm": f(L.input_norm), "wq": f(L.wq), "wk": f(L.wk), "wv": f(L.wv), "wo": f(L.wo),
            "post_norm": f(L.post_norm), "router": f(L.moe.router), "gate": f(L.moe.gate), "up": f(L.moe.up),
            "down": f(L.moe.down), "shared_gate": f(L.moe.shared_gate), "shared_up": f(L.moe.shared_up),
            "shared_down": f(L.moe.shared_down)}


def _build(torch, cuda, shape, fmt, seed=5, flags=0):
    H, layers, heads, kv, vocab, E, K, F, S, n, steps = shape
    dims = D.DecoderDims(H, layers, heads, kv, 128, vocab, E, K, F, S)
    w_dev = D.synth_weights(dims, seed, int8=False, norm_sigma=0.1)  # the device quantises these itself
    w_ora = D.synth_weights(dims, seed, int8=fmt == M.WEIGHT_INT8, norm_sigma=0.1)
    dec = M.Decoder(H, layers, heads, kv, vocab, max_positions=n + steps + 3, max_prefill=n, experts=E, top_k=K,
                    ffn=F, shared_ffn=S, weight_format=fmt, flags=flags)
    keep = []
    for li, L in enumerate(w_dev.layers):
        t = _device_layer(torch, cuda, L)
        dec.set_layer(li, t, dtype=M.DTYPE_F32)
        keep.append(t)
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda)  # noqa: E731
    head = (f(w_dev.embed), f(w_dev.final_norm), f(w_dev.lm_head))
    dec.set_head(*head, dtype=M.DTYPE_F32)
    torch.cuda.synchronize()
    return dims, dec, w_ora


def _run(torch, cuda, dec, prompt, vocab, steps, stream):
    logits0 = torch.empty(vocab, device=cuda)
    tok0 = torch.empty(1, dtype=torch.int32, device=cuda)
    toks = torch.empty(steps, dtype=torch.int32, device=cuda)
    lg = torch.empty(steps, vocab, device=cuda)
    x = torch.from_numpy(prompt).to(cuda)
    torch.cuda.synchronize()  # x comes from the default stream; `stream` does not wait for it
    with torch.cuda.stream(stream):
        dec.prefill(x, logits0, tok0, stream=stream)
        dec.decode(steps, toks, lg, stream=stream)
        dec.check(stream=stream)
    torch.cuda.synchronize()
    return logits0.cpu().numpy(), int(tok0.item()), toks.cpu().numpy(), lg.cpu().numpy()


# The decode attention on the tensor cores (the default) and on the CUDA cores.
ATTENTION = {"tensor_cores": 0, "cuda_cores": M.DECODER_CUDA_CORE_ATTENTION}


@pytest.mark.parametrize("attention", list(ATTENTION))
@pytest.mark.parametrize("fmt", [M.WEIGHT_BF16, M.WEIGHT_INT8])
@pytest.mark.parametrize("shape", SHAPES)
def test_decoder_against_oracle(cuda, shape, fmt, attention):
    import torch
    dims, dec, w_ora = _build(torch, cuda, shape, fmt, flags=ATTENTION[attention])
    n, steps = shape[-2], shape[-1]
    prompt = D.synth_prompt(dims, 5, n)
    side = torch.cuda.Stream()
    l0, t0, toks, lg = _run(torch, cuda, dec, prompt, dims.vocab, steps, side)  # replays the captured step
    ora = D.DecoderOracle(dims, w_ora)
    want0 = ora.prefill(prompt)
    tol = TOL[fmt]
    errs = [max_rel(l0, want0)]
    assert t0 == int(np.argmax(l0))
    fed = [t0] + toks.tolist()
    for s in range(steps):
        want = ora.step(fed[s])
        errs.append(max_rel(lg[s], want))
        assert toks[s] == int(np.argmax(lg[s])), f"step {s}: the token is not its own logits' argmax"
    print(f"decoder {shape} fmt {fmt}: max_rel per step {[f'{e:.1e}' for e in errs]}")
    assert max(errs) <= tol, errs
    # The same sequence again on the legacy stream (plain launches, no graph)
    # and again on the side stream: bitwise the same.
    l0b, t0b, toksb, lgb = _run(torch, cuda, dec, prompt, dims.vocab, steps, torch.cuda.default_stream())
    assert np.array_equal(l0, l0b) and t0 == t0b and np.array_equal(toks, toksb) and np.array_equal(lg, lgb)
    l0c, _, toksc, lgc = _run(torch, cuda, dec, prompt, dims.vocab, steps, side)
    assert np.array_equal(lg, lgc) and np.array_equal(toks, toksc)
    dec.close()


def test_decoder_sequence_limits(cuda):
    import torch
    shape = (512, 1, 4, 1, 256, 8, 2, 128, 256, 20, 2)
    dims, dec, _ = _build(torch, cuda, shape, M.WEIGHT_BF16)
    toks = torch.empty(8, dtype=torch.int32, device=cuda)
    with pytest.raises(M.UocrError) as e:
        dec.decode(1, toks)  # nothing prefilled yet
    assert e.value.code == 1
    x = torch.from_numpy(D.synth_prompt(dims, 5, 20)).to(cuda)
    dec.prefill(x)
    dec.decode(5, toks)  # 20 + 5 == max_positions
    with pytest.raises(M.UocrError) as e:
        dec.decode(1, toks)
    assert e.value.code == 1 and "max_positions" in str(e.value)
    with pytest.raises(M.UocrError):
        dec.prefill(torch.zeros(21, 512, device=cuda))  # above max_prefill
    dec.check()
    dec.close()
