"""The drop-in inside the reference's own decoder: the reference's CUDA
decoder test (tests/cuda_decoder_test.cpp — CudaDecoder against the reference
decoder on a tiny random model, bf16 and int8 weights, the logits after the
prompt and after 44 decode steps within 2e-2) built from its sources by
oracle/Makefile, with the decode path of CudaDecoder::moe
(src/model/cuda/cuda_decoder.cpp:137-192) calling this library: expert_topk
and expert_ffn_one are bound to uocr_expert_topk / uocr_expert_ffn_one
(oracle/ref_cuda_bind.cpp). The int8 decoder keeps the reference's own
expert_ffn_one_q8 (one scale per 32 inputs, against one per row here)."""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

EXE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "cuda_decoder_test")


def test_reference_cuda_decoder_with_the_library_ops():
    if not os.path.exists(EXE):
        pytest.skip("oracle/_ref/cuda_decoder_test was not built (the reference sources were absent at build time)")
    r = subprocess.run([EXE], capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0, (r.stdout + r.stderr)[-2000:]
    assert "ok" in r.stdout.split()
    m = re.search(r"uocr binding: expert_topk (\d+), expert_ffn_one (\d+)", r.stdout)
    assert m is not None
    assert int(m.group(1)) > 0 and int(m.group(2)) > 0  # the library's kernels ran inside the reference decoder
