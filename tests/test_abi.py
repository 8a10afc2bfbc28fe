"""The C ABI without a GPU: the library loads, exports every entry point the
header declares, and rejects bad arguments with the documented status codes
before touching a device."""
import ctypes
import os
import re

import pytest

import uocr_moe as M

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
HEADER = os.path.join(INCLUDE, "uocr_moe.h")
DECODER_HEADER = os.path.join(INCLUDE, "uocr_decoder.h")


def declared_symbols(header=None):
    names = set()
    for h in ([header] if header else [HEADER, DECODER_HEADER]):
        text = open(h).read()
        names |= set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\**\s+\**(uocr_[a-z_0-9]+)\s*\(", text, re.M))
    return sorted(names)


def test_header_and_binding_agree():
    assert declared_symbols(HEADER) == sorted(M.EXPORTS)
    assert declared_symbols(DECODER_HEADER) == sorted(M.DECODER_EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = M.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.uocr_abi_version() == 5


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors have the C layouts of the header's structs: a small C
    program compiled against include/uocr_moe.h prints sizeof and offsetof."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"uocr_moe_desc": M.MoeDesc, "uocr_moe_layer_src": M.LayerSrc, "uocr_moe_layer_parts": M.LayerParts,
               "uocr_tensor_view": M.TensorView, "uocr_decoder_desc": M.DecoderDesc,
               "uocr_decoder_layer_src": M.DecoderLayerSrc}
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "uocr_decoder.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for ln in out:
        parts = ln.split()
        if len(parts) == 3:
            got[(parts[0], parts[1])] = int(parts[2])
    for cname, cls in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(cls), cname
        for field, _ in cls._fields_:
            assert got[(cname, field)] == getattr(cls, field).offset, (cname, field)
    assert ctypes.sizeof(M.EpHandle) == 256


def _desc(**kw):
    d = dict(hidden=64, routed_experts=8, experts_per_token=2, expert_ffn=32, shared_ffn=32, layers=1, max_rows=4,
             weight_format=0, renormalize=1, router_bias=0, device=0, flags=0)
    d.update(kw)
    return M.MoeDesc(**d)


@pytest.mark.parametrize("bad", [dict(hidden=0), dict(hidden=40), dict(routed_experts=129), dict(routed_experts=0),
                                 dict(experts_per_token=9), dict(experts_per_token=9, routed_experts=8),
                                 dict(expert_ffn=24), dict(shared_ffn=-16), dict(layers=0), dict(max_rows=0),
                                 dict(weight_format=2)])
def test_plan_create_rejects_bad_shapes(bad):
    h = ctypes.c_void_p()
    rc = M.lib().uocr_moe_plan_create(ctypes.byref(_desc(**bad)), ctypes.byref(h))
    assert rc == 1 and not h.value
    assert M.lib().uocr_last_error().decode().startswith("plan_create")


@pytest.mark.parametrize("bad,code", [
    (dict(ep_world=9, ep_rank=0), 1), (dict(ep_world=-1), 1), (dict(ep_world=2, ep_rank=2), 1),
    (dict(ep_world=3, ep_rank=0, hidden=256, expert_ffn=128, shared_ffn=128), 1),  # 8 experts over 3 ranks, no table
    (dict(ep_world=2, ep_rank=0), 2),  # hidden 64: not a prefill shape
    (dict(ep_world=2, ep_rank=1, hidden=256, expert_ffn=128, shared_ffn=128, weight_format=1), 2)])
def test_plan_create_rejects_bad_expert_parallel_setups(bad, code):
    h = ctypes.c_void_p()
    rc = M.lib().uocr_moe_plan_create(ctypes.byref(_desc(**bad)), ctypes.byref(h))
    assert rc == code and not h.value


@pytest.mark.parametrize("table,why", [
    ([0, 1] * 7 + [0, 2], "is not a rank"),       # expert 7's rows from rank 1 to rank 2 of 2
    ([0, 0] * 8, "holds no expert"),              # rank 1 would hold nothing
])
def test_plan_create_rejects_bad_owner_tables(table, why):
    owner = (ctypes.c_int32 * len(table))(*table)
    d = _desc(ep_world=2, ep_rank=0, hidden=256, expert_ffn=128, shared_ffn=128)
    d.ep_owner = ctypes.cast(owner, ctypes.c_void_p).value
    h = ctypes.c_void_p()
    assert M.lib().uocr_moe_plan_create(ctypes.byref(d), ctypes.byref(h)) == 1 and not h.value
    assert why in M.lib().uocr_last_error().decode()


def test_ep_entry_points_reject_bad_arguments():
    lib = M.lib()
    assert lib.uocr_moe_ep_handle(None, None) == 1
    assert lib.uocr_moe_ep_connect(None, None) == 1
    assert lib.uocr_moe_ep_connect_local(None, 2) == 1
    assert lib.uocr_moe_ep_forward_local(None, 2, 0, None, None, None, None) == 1
    assert ctypes.sizeof(M.EpHandle) == 256


def test_null_arguments_are_rejected():
    lib = M.lib()
    assert lib.uocr_moe_plan_create(None, None) == 1
    assert lib.uocr_moe_forward(None, 0, None, 1, None, None, None, None) == 1
    assert lib.uocr_moe_set_layer(None, 0, None, None) == 1
    assert lib.uocr_moe_set_layer_parts(None, 0, None, None) == 1
    assert lib.uocr_moe_load_layer(None, None, 0, 0, None) == 1
    assert lib.uocr_moe_plan_destroy(None) == 0
    assert lib.uocr_checkpoint_open(None, None) == 1
    assert lib.uocr_checkpoint_count(None, None) == 1
    assert lib.uocr_checkpoint_tensor(None, b"x", None) == 1
    assert lib.uocr_checkpoint_close(None) == 0


def test_op_mirror_argument_checks():
    lib = M.lib()
    # the reference throws invalid_argument above 128 experts (ops.cu:653)
    assert lib.uocr_expert_topk(None, 1, 129, 2, 1, None, None, None) == 1
    assert "128" in lib.uocr_last_error().decode()
    assert lib.uocr_expert_topk(None, 1, 8, 9, 1, None, None, None) == 1
    assert lib.uocr_quantize_q8(None, 0, 4, 96, 40, None, None, None) == 1
    assert lib.uocr_expert_ffn_one(None, 40, 32, None, None, None, None, None, 2, None, None) == 1
    assert lib.uocr_synth_fill(1, 2, 1.0, 0, -1, 0, None, None) == 1


def test_synth_stream_layout():
    assert M.synth_stream(3, M.KIND_DOWN, 17) == (3 << 40) | (M.KIND_DOWN << 32) | 17


def _ddesc(**kw):
    d = dict(hidden=512, layers=1, heads=4, kv_heads=1, head_dim=128, vocab=1024, max_positions=64, max_prefill=32,
             routed_experts=8, experts_per_token=2, expert_ffn=128, shared_ffn=256, rope_theta=1e4,
             rms_norm_eps=1e-6, weight_format=0, renormalize=1, device=0, flags=0)
    d.update(kw)
    return M.DecoderDesc(**d)


@pytest.mark.parametrize("bad,code", [(dict(head_dim=64), 2), (dict(heads=3), 1), (dict(kv_heads=3), 1),
                                      (dict(heads=16, kv_heads=1, hidden=2048), 1), (dict(hidden=384, heads=3), 1),
                                      (dict(max_positions=32), 1), (dict(vocab=1), 1), (dict(weight_format=2), 1),
                                      (dict(layers=0), 1), (dict(rope_theta=0.0), 1)])
def test_decoder_create_rejects_bad_shapes(bad, code):
    h = ctypes.c_void_p()
    rc = M.lib().uocr_decoder_create(ctypes.byref(_ddesc(**bad)), ctypes.byref(h))
    assert rc == code and not h.value
    assert M.lib().uocr_last_error().decode().startswith("decoder_create")


def test_decoder_calls_reject_null_handles():
    lib = M.lib()
    assert lib.uocr_decoder_prefill(None, None, 1, None, None, None) == 1
    assert lib.uocr_decoder_decode(None, 1, None, None, None) == 1
    assert lib.uocr_decoder_set_layer(None, 0, None, None) == 1
    assert lib.uocr_decoder_destroy(None) == 0
