"""TEST INFRASTRUCTURE: a second, independent reader of the checkpoint
format in Python — safetensors shards, the shard index, and a layer's MoE
weights loaded into a plan straight from the mapped files through
uocr_moe_set_layer_parts — against which the library's own reader
(uocr_checkpoint_open / uocr_checkpoint_tensor / uocr_moe_load_layer) is
checked; it also writes the fixture shards the tests use. The product loads
checkpoints through the library alone.

The readers keep the reference's checks and failure cases:
  * one shard — parse_safetensors_header and SafetensorsFile
    (src/weights/safetensors.cpp:69-124, 126-163): an 8-byte little-endian
    header length of at most 100 MiB that fits the file, a JSON object header
    (``__metadata__`` skipped), a known dtype, non-negative integer dims, two
    unsigned data offsets inside the data section, a byte count equal to
    shape x dtype size, and data extents that tile the data section exactly;
  * the index — ShardedWeights::open (src/weights/sharded_weights.cpp:12-61):
    a ``weight_map`` object of plain file names, every indexed tensor in the
    shard the index names and no shard holding a tensor the index does not
    list.
Tensors are numpy views into a read-only memory map; bf16 tensors are their
uint16 bit patterns.

The MoE tensor names and shapes are the published checkpoint's
(src/weights/architecture.cpp:108-117), read the way CudaDecoder reads them
(src/model/cuda/cuda_decoder.cpp:44-84): ``model.layers.{l}.mlp.gate.weight``
[E, H], ``mlp.experts.{e}.{gate,up}_proj.weight`` [F, H],
``mlp.experts.{e}.down_proj.weight`` [H, F], ``mlp.shared_experts.*`` with
width S, and ``post_attention_layernorm.weight`` [H], the gain of the RMSNorm
in front of the feed-forward block (src/model/decoder.cpp:180, 200).
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from dataclasses import dataclass

import numpy as np

# dtype name -> (numpy view type, bytes per element); the reference's table
# (src/tensor/dtype.cpp:15-22).
DTYPES = {
    "BF16": (np.uint16, 2),
    "F16": (np.float16, 2),
    "F32": (np.float32, 4),
    "I64": (np.int64, 8),
    "I32": (np.int32, 4),
    "U8": (np.uint8, 1),
}
MAX_HEADER_BYTES = 100 * 1024 * 1024


class CheckpointError(RuntimeError):
    """A malformed shard, index or tensor table (the reference's runtime_error)."""


@dataclass(frozen=True)
class TensorInfo:
    dtype: str
    shape: tuple
    begin: int  # byte offsets inside the data section
    end: int

    def element_count(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


def _is_uint(v, bits: int = 64) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and 0 <= v < (1 << bits)


def parse_header(header_json, data_size: int) -> dict:
    """name -> TensorInfo for a header against a data section of data_size
    bytes; raises CheckpointError naming the first problem."""
    try:
        header = json.loads(header_json)
    except (ValueError, UnicodeDecodeError):
        raise CheckpointError("header is not a JSON object") from None
    if not isinstance(header, dict):
        raise CheckpointError("header is not a JSON object")
    tensors = {}
    for name, entry in sorted(header.items()):  # key order, as the reference's JSON object iterates
        if name == "__metadata__":
            continue
        if not isinstance(entry, dict) or not all(k in entry for k in ("dtype", "shape", "data_offsets")):
            raise CheckpointError(f"tensor {name}: entry lacks dtype, shape or data_offsets")
        dtype = entry["dtype"]
        if not isinstance(dtype, str) or dtype not in DTYPES:
            raise CheckpointError(f"tensor {name}: unsupported dtype {json.dumps(dtype)}")
        shape = entry["shape"]
        if not isinstance(shape, list):
            raise CheckpointError(f"tensor {name}: shape is not an array")
        if not all(_is_uint(d, 63) for d in shape):
            raise CheckpointError(f"tensor {name}: shape holds a non-integer or negative dim")
        offsets = entry["data_offsets"]
        if not isinstance(offsets, list) or len(offsets) != 2 or not all(_is_uint(v) for v in offsets):
            raise CheckpointError(f"tensor {name}: data_offsets is not two unsigned integers")
        begin, end = offsets
        if begin > end or end > data_size:
            raise CheckpointError(f"tensor {name}: data_offsets [{begin}, {end}) outside a {data_size}-byte "
                                  "data section")
        need = DTYPES[dtype][1]
        for d in shape:
            need *= d
        if need >= 1 << 64:
            raise CheckpointError(f"tensor {name}: shape overflows")
        if end - begin != need:
            raise CheckpointError(f"tensor {name}: {end - begin} bytes stored, shape and dtype need {need}")
        tensors[name] = TensorInfo(dtype, tuple(shape), begin, end)
    cursor = 0
    for name, info in sorted(tensors.items(), key=lambda kv: kv[1].begin):
        if info.begin != cursor:
            raise CheckpointError(f"tensor {name}: starts at {info.begin} but the previous tensor ends at {cursor}")
        cursor = info.end
    if cursor != data_size:
        raise CheckpointError(f"tensors end at {cursor} but the data section is {data_size} bytes")
    return tensors


class SafetensorsFile:
    """One shard, memory-mapped read-only; tensors are views into the map."""

    def __init__(self, path):
        self.path = os.fspath(path)
        try:
            fd = os.open(self.path, os.O_RDONLY | getattr(os, "O_CLOEXEC", 0))
        except OSError as e:
            raise CheckpointError(f"{self.path}: cannot open: {e.strerror}") from None
        try:
            size = os.fstat(fd).st_size
            if size < 8:
                raise CheckpointError(f"{self.path}: {size} bytes is too short for a safetensors file")
            self._map = mmap.mmap(fd, size, access=mmap.ACCESS_READ)
        finally:
            os.close(fd)
        try:
            (hlen,) = struct.unpack_from("<Q", self._map, 0)
            if hlen > MAX_HEADER_BYTES or hlen > size - 8:
                raise CheckpointError(f"header length {hlen} does not fit the file")
            self._data = 8 + hlen
            self.tensors = parse_header(bytes(self._map[8:8 + hlen]), size - 8 - hlen)
        except CheckpointError as e:
            self._map.close()
            raise CheckpointError(f"{self.path}: {e}") from None

    def find(self, name: str):
        return self.tensors.get(name)

    def close(self) -> None:
        """Unmaps the file. Arrays from array() must be gone first (the map
        refuses to close under live views: BufferError)."""
        self._map.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def array(self, name: str) -> np.ndarray:
        info = self.tensors[name]
        typ, _ = DTYPES[info.dtype]
        return np.frombuffer(self._map, dtype=typ, count=info.element_count(),
                             offset=self._data + info.begin).reshape(info.shape)


class ShardedWeights:
    """A checkpoint split across shards, addressed by tensor name through the
    shard index (model.safetensors.index.json)."""

    def __init__(self):
        self.shards = []
        self._where = {}  # name -> shard

    @classmethod
    def open(cls, index_path) -> "ShardedWeights":
        index_path = os.fspath(index_path)
        try:
            with open(index_path, "rb") as f:
                text = f.read()
        except OSError:
            raise CheckpointError(f"{index_path}: cannot open the shard index") from None
        try:
            index = json.loads(text)
        except (ValueError, UnicodeDecodeError):
            index = None
        if not isinstance(index, dict) or not isinstance(index.get("weight_map"), dict):
            raise CheckpointError(f"{index_path}: not a shard index (no weight_map object)")
        w = cls()
        expected, by_file = {}, {}
        base = os.path.dirname(index_path)
        for name, file in sorted(index["weight_map"].items()):
            if not isinstance(file, str):
                raise CheckpointError(f"{index_path}: weight_map[{name}] is not a file name")
            if "/" in file or file == ".." or not file:
                raise CheckpointError(f"{index_path}: shard name {file} is not a plain file name")
            expected[name] = file
            if file not in by_file:
                by_file[file] = SafetensorsFile(os.path.join(base, file))
                w.shards.append(by_file[file])
        for file in sorted(by_file):
            shard = by_file[file]
            for name in sorted(shard.tensors):
                if name not in expected:
                    raise CheckpointError(f"{file}: holds {name}, which the index does not list")
                if expected[name] != file:
                    raise CheckpointError(f"{file}: holds {name}, which the index places in {expected[name]}")
                w._where[name] = shard
        for name, file in sorted(expected.items()):
            if name not in w._where:
                raise CheckpointError(f"{file}: the index places {name} here but the shard lacks it")
        return w

    def find(self, name: str):
        s = self._where.get(name)
        return None if s is None else s.tensors[name]

    def at(self, name: str) -> TensorInfo:
        info = self.find(name)
        if info is None:
            raise KeyError(f"no tensor named {name}")
        return info

    def array(self, name: str) -> np.ndarray:
        self.at(name)
        return self._where[name].array(name)

    def names(self) -> list:
        return sorted(self._where)

    def tensor_count(self) -> int:
        return len(self._where)

    def close(self) -> None:
        for shard in self.shards:
            shard.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """Writes name -> (dtype name, array) as one shard, data in name order and
    the header padded with spaces to 8 bytes. bf16 arrays are uint16 bits."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name in sorted(tensors):
        dtype, arr = tensors[name]
        typ, _ = DTYPES[dtype]
        b = np.ascontiguousarray(arr, dtype=typ).tobytes()
        header[name] = {"dtype": dtype, "shape": list(np.shape(arr)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_index(path, weight_map: dict) -> None:
    with open(path, "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)


# ---- the MoE tensors of one decoder layer ----------------------------------

PROJS = ("gate_proj", "up_proj", "down_proj")


def moe_layer_tensors(layer: int, hidden: int, experts: int, ffn: int, shared_ffn: int) -> dict:
    """name -> shape of every tensor a plan layer reads from the checkpoint."""
    p = f"model.layers.{layer}."
    out = {p + "post_attention_layernorm.weight": (hidden,), p + "mlp.gate.weight": (experts, hidden)}
    for e in range(experts):
        q = f"{p}mlp.experts.{e}."
        out[q + "gate_proj.weight"] = (ffn, hidden)
        out[q + "up_proj.weight"] = (ffn, hidden)
        out[q + "down_proj.weight"] = (hidden, ffn)
    if shared_ffn > 0:
        q = p + "mlp.shared_experts."
        out[q + "gate_proj.weight"] = (shared_ffn, hidden)
        out[q + "up_proj.weight"] = (shared_ffn, hidden)
        out[q + "down_proj.weight"] = (hidden, shared_ffn)
    return out


def check_moe_layer(weights: ShardedWeights, layer: int, hidden: int, experts: int, ffn: int,
                    shared_ffn: int) -> list:
    """Problems with one layer's MoE tensors (each missing tensor, each shape
    or dtype other than the plan needs), in the manner of
    check_architecture (src/weights/architecture.h:75-78). Empty means the
    layer loads."""
    problems, dtypes = [], set()
    for name, shape in moe_layer_tensors(layer, hidden, experts, ffn, shared_ffn).items():
        info = weights.find(name)
        if info is None:
            problems.append(f"missing {name}")
            continue
        if info.dtype not in ("BF16", "F32"):
            problems.append(f"{name}: dtype {info.dtype}, expected BF16 or F32")
        dtypes.add(info.dtype)
        if info.shape != tuple(shape):
            problems.append(f"{name}: shape {list(info.shape)}, expected {list(shape)}")
    if len(dtypes) > 1:
        problems.append(f"layer {layer}: mixed dtypes {sorted(dtypes)}")
    return problems


def load_moe_layer(plan, weights: ShardedWeights, layer: int, plan_layer: int | None = None, stream=None) -> None:
    """Loads checkpoint layer `layer` into plan layer `plan_layer` (default the
    same index) through uocr_moe_set_layer_parts, each expert's tensors passed
    as pointers into the mapped shards (host memory)."""
    import uocr_moe as M

    d = plan.desc
    H, E, F, S = d.hidden, d.routed_experts, d.expert_ffn, d.shared_ffn
    if d.router_bias:
        raise CheckpointError("the plan expects a router bias, which the checkpoint does not hold")
    problems = check_moe_layer(weights, layer, H, E, F, S)
    if problems:
        raise CheckpointError(f"layer {layer}: " + "; ".join(problems))
    p = f"model.layers.{layer}."
    router = weights.array(p + "mlp.gate.weight")
    dtype = M.DTYPE_BF16 if weights.at(p + "mlp.gate.weight").dtype == "BF16" else M.DTYPE_F32
    experts = [[weights.array(f"{p}mlp.experts.{e}.{proj}.weight") for e in range(E)] for proj in PROJS]
    shared = [weights.array(f"{p}mlp.shared_experts.{proj}.weight") if S > 0 else None for proj in PROJS]
    norm = weights.array(p + "post_attention_layernorm.weight")

    def addr(a):
        return None if a is None else a.ctypes.data

    plan.set_layer_parts(layer if plan_layer is None else plan_layer, addr(router),
                         [addr(a) for a in experts[0]], [addr(a) for a in experts[1]], [addr(a) for a in experts[2]],
                         addr(shared[0]), addr(shared[1]), addr(shared[2]), memory=M.MEMORY_HOST, dtype=dtype,
                         stream=stream, norm=addr(norm))
