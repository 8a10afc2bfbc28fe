"""Checkpoint readers on the CPU: one safetensors shard, the shard index, and
the MoE tensor table of a layer. The failure cases are the reference's
(tests/safetensors_test.cpp): each malformed header, file and index is
rejected with the tensor or file named."""
import json
import struct

import numpy as np
import pytest

import safetensors_py as C


def _raw_shard(path, header: dict | str, data: bytes, hlen: int | None = None):
    h = header if isinstance(header, str) else json.dumps(header)
    hb = h.encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb) if hlen is None else hlen))
        f.write(hb)
        f.write(data)


def test_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    b = rng.integers(0, 1 << 16, size=(4, 2), dtype=np.uint16)
    c = np.arange(7, dtype=np.uint8)
    p = tmp_path / "one.safetensors"
    C.write_safetensors(p, {"a": ("F32", a), "b": ("BF16", b), "c": ("U8", c)}, metadata={"format": "pt"})
    f = C.SafetensorsFile(p)
    assert sorted(f.tensors) == ["a", "b", "c"]
    assert f.find("a").dtype == "F32" and f.find("a").shape == (3, 5)
    np.testing.assert_array_equal(f.array("a"), a)
    np.testing.assert_array_equal(f.array("b"), b)
    np.testing.assert_array_equal(f.array("c"), c)
    assert f.find("absent") is None
    assert not f.array("a").flags.writeable  # a view into the read-only map


def test_zero_sized_tensor(tmp_path):
    p = tmp_path / "z.safetensors"
    C.write_safetensors(p, {"e": ("F32", np.zeros((0, 4), np.float32)), "x": ("I32", np.arange(3, dtype=np.int32))})
    f = C.SafetensorsFile(p)
    assert f.array("e").shape == (0, 4)
    np.testing.assert_array_equal(f.array("x"), [0, 1, 2])


HEADER_CASES = [
    ("[]", 0, "not a JSON object"),
    ("{not json", 0, "not a JSON object"),
    ('{"a":{"dtype":"F64","shape":[1],"data_offsets":[0,8]}}', 8, "unsupported dtype"),
    ('{"a":{"dtype":"F32","shape":[-1],"data_offsets":[0,4]}}', 4, "negative dim"),
    ('{"a":{"dtype":"F32","shape":[1.5],"data_offsets":[0,4]}}', 4, "non-integer"),
    ('{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', 4, "bytes stored"),
    ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', 8, "data section is 8 bytes"),
    ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[4,8]}}', 8, "previous tensor ends at 0"),
    ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', 2, "outside a 2-byte"),
    ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},"b":{"dtype":"F32","shape":[1],"data_offsets":[2,6]}}',
     6, "previous tensor ends at 4"),
    ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[8,4]}}', 8, "outside"),
    ('{"a":{"dtype":"F32","shape":[1]}}', 4, "lacks dtype, shape or data_offsets"),
    ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0]}}', 4, "two unsigned integers"),
    ('{"a":{"dtype":"U8","shape":[4294967296,4294967296,16],"data_offsets":[0,0]}}', 0, "overflows"),
    ('{"a":{"dtype":"F32","shape":3,"data_offsets":[0,4]}}', 4, "not an array"),
    ('{"a":{"dtype":"F32","shape":[9223372036854775808],"data_offsets":[0,4]}}', 4, "non-integer or negative dim"),
    ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,18446744073709551616]}}', 4, "two unsigned integers"),
    ('{"b":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},"a":{"dtype":"F64","shape":[1],"data_offsets":[4,12]}}',
     12, "tensor a: unsupported"),  # entries are checked in name order
]


@pytest.mark.parametrize("header,size,why", HEADER_CASES)
def test_header_rejections(header, size, why):
    with pytest.raises(C.CheckpointError, match=why):
        C.parse_header(header, size)


def test_metadata_is_skipped():
    t = C.parse_header('{"__metadata__":{"k":"v"},"a":{"dtype":"I64","shape":[2],"data_offsets":[0,16]}}', 16)
    assert list(t) == ["a"] and t["a"].element_count() == 2


def test_file_rejections(tmp_path):
    short = tmp_path / "short.safetensors"
    short.write_bytes(b"\x01\x02\x03")
    with pytest.raises(C.CheckpointError, match="too short"):
        C.SafetensorsFile(short)
    huge = tmp_path / "huge.safetensors"
    _raw_shard(huge, "{}", b"", hlen=1 << 40)
    with pytest.raises(C.CheckpointError, match="does not fit the file"):
        C.SafetensorsFile(huge)
    with pytest.raises(C.CheckpointError, match="cannot open"):
        C.SafetensorsFile(tmp_path / "absent.safetensors")
    bad = tmp_path / "bad.safetensors"
    _raw_shard(bad, '{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', b"\0" * 4)
    with pytest.raises(C.CheckpointError, match="bad.safetensors: tensor a"):
        C.SafetensorsFile(bad)


def _two_shards(d):
    C.write_safetensors(d / "s1.safetensors", {"x": ("F32", np.ones(2, np.float32)), "y": ("U8", np.arange(3, dtype=np.uint8))})
    C.write_safetensors(d / "s2.safetensors", {"z": ("I32", np.arange(4, dtype=np.int32))})


def test_sharded_weights(tmp_path):
    _two_shards(tmp_path)
    C.write_index(tmp_path / "good.json", {"x": "s1.safetensors", "y": "s1.safetensors", "z": "s2.safetensors"})
    w = C.ShardedWeights.open(tmp_path / "good.json")
    assert w.tensor_count() == 3 and w.names() == ["x", "y", "z"]
    np.testing.assert_array_equal(w.array("z"), [0, 1, 2, 3])
    assert w.find("q") is None
    with pytest.raises(KeyError, match="no tensor named q"):
        w.at("q")


INDEX_CASES = [
    ({"x": "s2.safetensors", "y": "s1.safetensors", "z": "s2.safetensors"}, "holds x, which the index places in s2"),
    ({"y": "s1.safetensors", "z": "s2.safetensors"}, "holds x, which the index does not list"),
    ({"x": "s1.safetensors", "y": "s1.safetensors", "z": "s2.safetensors", "w": "s2.safetensors"},
     "places w here but the shard lacks it"),
    ({"x": "../s1.safetensors", "y": "s1.safetensors", "z": "s2.safetensors"}, "not a plain file name"),
    ({"x": "..", "y": "s1.safetensors", "z": "s2.safetensors"}, "not a plain file name"),
    ({"x": 3, "y": "s1.safetensors", "z": "s2.safetensors"}, "is not a file name"),
    ({"x": "s1.safetensors", "y": "s1.safetensors", "z": "absent.safetensors"}, "cannot open"),
]


@pytest.mark.parametrize("wmap,why", INDEX_CASES)
def test_index_rejections(tmp_path, wmap, why):
    _two_shards(tmp_path)
    C.write_index(tmp_path / "idx.json", wmap)
    with pytest.raises(C.CheckpointError, match=why):
        C.ShardedWeights.open(tmp_path / "idx.json")


def test_index_file_rejections(tmp_path):
    with pytest.raises(C.CheckpointError, match="cannot open the shard index"):
        C.ShardedWeights.open(tmp_path / "absent.json")
    (tmp_path / "bad.json").write_text('{"metadata": {}}')
    with pytest.raises(C.CheckpointError, match="no weight_map object"):
        C.ShardedWeights.open(tmp_path / "bad.json")


def write_moe_checkpoint(d, layers, H, E, F, S, seed=0, shards=2, dtype="BF16", drop=None, reshape=None):
    """A synthetic checkpoint of `layers` MoE layers under the published
    names, spread over `shards` shards; returns (index path, name -> array)."""
    rng = np.random.default_rng(seed)
    arrays = {}
    for l in layers:
        for name, shape in C.moe_layer_tensors(l, H, E, F, S).items():
            sigma = 1.0 if name.endswith("layernorm.weight") else 0.05
            v = (rng.standard_normal(shape) * sigma + (1.0 if name.endswith("layernorm.weight") else 0.0))
            v = v.astype(np.float32)
            if dtype == "BF16":
                u = v.view(np.uint32)
                v = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
            arrays[name] = v
    if drop is not None:
        arrays.pop(drop)
    if reshape is not None:
        arrays[reshape] = arrays[reshape].reshape(-1)
    names = sorted(arrays)
    wmap = {}
    for s in range(shards):
        part = {n: (dtype, arrays[n]) for i, n in enumerate(names) if i % shards == s}
        fn = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        C.write_safetensors(d / fn, part)
        wmap.update({n: fn for n in part})
    C.write_index(d / "model.safetensors.index.json", wmap)
    return d / "model.safetensors.index.json", arrays


def test_moe_layer_table(tmp_path):
    idx, arrays = write_moe_checkpoint(tmp_path, [1, 2], H=64, E=4, F=32, S=64)
    w = C.ShardedWeights.open(idx)
    assert C.check_moe_layer(w, 1, 64, 4, 32, 64) == []
    assert C.check_moe_layer(w, 2, 64, 4, 32, 64) == []
    probs = C.check_moe_layer(w, 0, 64, 4, 32, 64)
    assert len(probs) == 3 + 4 * 3 + 2 and all(p.startswith("missing model.layers.0.") for p in probs)
    assert C.check_moe_layer(w, 1, 64, 4, 16, 64) != []  # wrong ffn width
    name = "model.layers.1.mlp.experts.3.down_proj.weight"
    np.testing.assert_array_equal(w.array(name), arrays[name])
    assert w.at(name).shape == (64, 32)


def test_moe_layer_table_names_each_problem(tmp_path):
    gone = "model.layers.1.mlp.experts.2.up_proj.weight"
    flat = "model.layers.1.mlp.shared_experts.down_proj.weight"
    idx, _ = write_moe_checkpoint(tmp_path, [1], H=64, E=4, F=32, S=64, drop=gone, reshape=flat)
    probs = C.check_moe_layer(C.ShardedWeights.open(idx), 1, 64, 4, 32, 64)
    assert probs == [f"missing {gone}", f"{flat}: shape [4096], expected [64, 64]"]


# ---- the library's own reader (uocr_checkpoint_*, host only) --------------

def _native(path):
    import uocr_moe as M
    return M.Checkpoint(path)


def test_native_reader_matches(tmp_path):
    import ctypes
    idx, arrays = write_moe_checkpoint(tmp_path, [1, 3], H=64, E=4, F=32, S=64, shards=3)
    ck = _native(idx)
    py = C.ShardedWeights.open(idx)
    assert len(ck) == py.tensor_count() == len(arrays)
    for name, arr in arrays.items():
        dtype, shape, addr, nbytes = ck.tensor(name)
        assert (dtype, shape) == ("BF16", arr.shape)
        assert nbytes == arr.nbytes and ctypes.string_at(addr, nbytes) == arr.tobytes()
    one = tmp_path / "one.safetensors"
    C.write_safetensors(one, {"a": ("F32", np.arange(6, dtype=np.float32).reshape(2, 3)), "b": ("I64", np.arange(2))})
    ck1 = _native(one)
    assert len(ck1) == 2
    dtype, shape, addr, nbytes = ck1.tensor("a")
    assert (dtype, shape, nbytes) == ("F32", (2, 3), 24)
    assert np.frombuffer(ctypes.string_at(addr, nbytes), np.float32).tolist() == [0, 1, 2, 3, 4, 5]
    import uocr_moe as M
    with pytest.raises(M.UocrError, match="no tensor named q"):
        ck1.tensor("q")
    ck.close()
    ck1.close()


@pytest.mark.parametrize("header,size,why", HEADER_CASES)
def test_native_header_rejections(tmp_path, header, size, why):
    import uocr_moe as M
    p = tmp_path / "h.safetensors"
    _raw_shard(p, header, b"\0" * size)
    with pytest.raises(M.UocrError, match=why) as e:
        _native(p)
    assert e.value.code == 1 and "h.safetensors: " in str(e.value)


def test_native_file_rejections(tmp_path):
    import uocr_moe as M
    short = tmp_path / "short.safetensors"
    short.write_bytes(b"\x01\x02\x03")
    huge = tmp_path / "huge.safetensors"
    _raw_shard(huge, "{}", b"", hlen=1 << 40)
    for path, why in ((short, "too short"), (huge, "does not fit the file"),
                      (tmp_path / "absent.safetensors", "cannot open")):
        with pytest.raises(M.UocrError, match=why):
            _native(path)
    with pytest.raises(M.UocrError, match="cannot open the shard index"):
        _native(tmp_path / "absent.json")
    (tmp_path / "bad.json").write_text('{"metadata": {}}')
    with pytest.raises(M.UocrError, match="no weight_map object"):
        _native(tmp_path / "bad.json")


@pytest.mark.parametrize("wmap,why", INDEX_CASES)
def test_native_index_rejections(tmp_path, wmap, why):
    import uocr_moe as M
    _two_shards(tmp_path)
    C.write_index(tmp_path / "idx.json", wmap)
    with pytest.raises(M.UocrError, match=why):
        _native(tmp_path / "idx.json")


def test_native_json_strictness(tmp_path):
    """What a strict JSON reader must refuse (trailing commas, bare words,
    unterminated strings, bad escapes, content after the value) and accept
    (escapes, surrogate pairs, nesting in the metadata)."""
    import uocr_moe as M
    for bad in ('{"a":1,}', "{a:1}", '{"a":"x}', '{"a":"\\q"}', '{} {}', '{"a":[1,2]', '{"a":01}',
                '{"a":"\\ud800"}', '{"a":tru}'):
        with pytest.raises(M.UocrError, match="header is not a JSON object"):
            _native_header(tmp_path, bad, 0)
    ok = ('{"__metadata__":{"k":["v",{"n":null,"t":true,"f":-1.5e3}]},'
          '"\\u00e9\\ud83d\\ude00\\n":{"dtype":"U8","shape":[2],"data_offsets":[0,2]}}')
    ck = _native_header(tmp_path, ok, 2)
    assert ck.tensor("\u00e9\U0001F600\n")[1] == (2,)
    py = C.parse_header(ok, 2)
    assert list(py) == ["\u00e9\U0001F600\n"]


def _native_header(tmp_path, header, size):
    p = tmp_path / "j.safetensors"
    _raw_shard(p, header, b"\0" * size)
    return _native(p)


def test_native_and_python_readers_agree_on_mutated_headers(tmp_path):
    """Random single-byte mutations of a valid shard: the library's reader and
    the Python reader accept exactly the same files, and name the same first
    problem when both reject (both restate the reference's checks and order)."""
    import uocr_moe as M
    good = tmp_path / "g.safetensors"
    C.write_safetensors(good, {"b.w": ("BF16", np.arange(6, dtype=np.uint16).reshape(2, 3)),
                               "a.w": ("F32", np.ones((2, 2), np.float32)), "c": ("U8", np.arange(5, dtype=np.uint8))},
                        metadata={"format": "pt"})
    raw = bytearray(good.read_bytes())
    hlen = int.from_bytes(raw[:8], "little")
    rng = np.random.default_rng(1)
    alphabet = b'0123456789[]{},:"-.eE ABFIU'
    agree = accepted = 0
    for trial in range(400):
        b = bytearray(raw)
        pos = 8 + int(rng.integers(0, hlen))
        b[pos] = alphabet[int(rng.integers(0, len(alphabet)))]
        p = tmp_path / f"m{trial % 4}.safetensors"
        p.write_bytes(bytes(b))
        try:
            C.SafetensorsFile(p)
            py = None
        except C.CheckpointError as e:
            py = str(e)
        try:
            M.Checkpoint(p).close()
            nat = None
        except M.UocrError as e:
            nat = str(e).split(": ", 1)[1]  # drop the status name
        if py is None or nat is None:
            assert py is None and nat is None, (bytes(b[8:8 + hlen]), py, nat)
            accepted += py is None
        else:
            # Python's json module accepts a few texts a strict reader refuses
            # (NaN, lone surrogates); everything else names the same problem.
            if "header is not a JSON object" in nat and "header is not a JSON object" not in py:
                continue
            assert py == nat, (bytes(b[8:8 + hlen]), py, nat)
        agree += 1
    assert agree > 350 and accepted > 0


def test_moe_layer_table_dtype_problems(tmp_path):
    """A layer must be all BF16 or all F32: another dtype, or a mix, is named."""
    H, E, F, S = 64, 2, 32, 64
    tensors = {}
    for name, shape in C.moe_layer_tensors(1, H, E, F, S).items():
        tensors[name] = ("BF16", np.zeros(shape, np.uint16))
    f16 = "model.layers.1.mlp.experts.1.up_proj.weight"
    f32 = "model.layers.1.mlp.gate.weight"
    tensors[f16] = ("F16", np.zeros((F, H), np.float16))
    tensors[f32] = ("F32", np.zeros((E, H), np.float32))
    C.write_safetensors(tmp_path / "one.safetensors", tensors)
    C.write_index(tmp_path / "idx.json", {n: "one.safetensors" for n in tensors})
    probs = C.check_moe_layer(C.ShardedWeights.open(tmp_path / "idx.json"), 1, H, E, F, S)
    assert f"{f16}: dtype F16, expected BF16 or F32" in probs
    assert probs[-1] == "layer 1: mixed dtypes ['BF16', 'F16', 'F32']"


def test_readers_close(tmp_path):
    _two_shards(tmp_path)
    C.write_index(tmp_path / "good.json", {"x": "s1.safetensors", "y": "s1.safetensors", "z": "s2.safetensors"})
    with C.ShardedWeights.open(tmp_path / "good.json") as w:
        assert w.array("z").sum() == 6  # the view is gone before the close
    assert all(s._map.closed for s in w.shards)
    f = C.SafetensorsFile(tmp_path / "s1.safetensors")
    view = f.array("x")
    with pytest.raises(BufferError):
        f.close()  # a live view keeps the map open
    del view
    f.close()
