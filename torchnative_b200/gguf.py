"""GGUF checkpoints straight to the device, keeping the file's own blocks.

The container half reads a GGUF file as the format specification
(llama.cpp's docs/gguf.md) defines it, from a read-only memory map:

    magic "GGUF" | u32 version (2, 3) | u64 tensor count | u64 metadata count
    metadata:  { string key | u32 value type | value } *
    tensors:   { string name | u32 rank | u64 extent * rank (fastest first)
                 | u32 GGML type | u64 offset into the data section } *
    padding to `general.alignment` (32 unless the metadata says otherwise)
    data section

Strings are a u64 byte length and UTF-8 bytes; all integers little-endian.
The device half (`load_tensor`, `quantized_linear`) moves one tensor's bytes
through a pinned staging buffer to HBM: the block formats with B200 kernels
(Q4_0, Q8_0, Q4_K) become a QTensor holding the file's blocks unchanged; dense
F32 / F16 / BF16 arrive bit for bit. The loader contract it serves is the
reference's torchnative.gguf (torchnative/python/torchnative/gguf/).
"""

from __future__ import annotations

import mmap
import os
from collections import namedtuple

import numpy as np

__all__ = ["GGML_TYPE_TABLE", "GGUFContainer", "GGUFMalformed", "GGUFUnsupported", "TensorSlot", "ggml_type_name",
           "load_tensor", "quantized_linear", "why_refused"]


class GGUFMalformed(ValueError):
    """The bytes do not form a GGUF file (wrong magic, short, inconsistent)."""


class GGUFUnsupported(NotImplementedError):
    """A valid GGUF construct that this loader declines, with the reason."""


# Why a GGML type is not turned into a tensor here.
_ONLY_ACTIVATIONS = "exists only as llama.cpp's activation-side operand, never as a stored weight"
_NO_B200_KERNEL = ("has no B200 kernel in this backend (the block formats with one are Q4_0, Q8_0 and Q4_K); "
                   "GGUFContainer.bytes_of still returns its stored bytes")
_NOT_IN_CANDLE = "is not a candle GgmlDType in the reference, so no path on either side stores or computes it"
_INTEGER_OR_F64 = "is a plain integer / float64 type that no checkpoint stores weights in; declined"
_REMOVED_REPACK = "is one of the repacked layouts llama.cpp dropped from the file format"

GGMLType = namedtuple("GGMLType", "name block_elems block_bytes handling target")
# The GGML type ids with their block geometry (ggml's type traits, checked
# against gguf-py's GGML_QUANT_SIZES by the tests) and this loader's handling:
# "dense" (read as the torch dtype `target`), "block" (a device QTensor of
# format `target`), "bytes" (readable bytes, no kernel) or "declined".
GGML_TYPE_TABLE = {
    0: GGMLType("F32", 1, 4, "dense", "float32"),
    1: GGMLType("F16", 1, 2, "dense", "float16"),
    2: GGMLType("Q4_0", 32, 18, "block", "q4_0"),
    3: GGMLType("Q4_1", 32, 20, "bytes", _NO_B200_KERNEL),
    6: GGMLType("Q5_0", 32, 22, "bytes", _NO_B200_KERNEL),
    7: GGMLType("Q5_1", 32, 24, "bytes", _NO_B200_KERNEL),
    8: GGMLType("Q8_0", 32, 34, "block", "q8_0"),
    9: GGMLType("Q8_1", 32, 36, "declined", _ONLY_ACTIVATIONS),
    10: GGMLType("Q2_K", 256, 84, "bytes", _NO_B200_KERNEL),
    11: GGMLType("Q3_K", 256, 110, "bytes", _NO_B200_KERNEL),
    12: GGMLType("Q4_K", 256, 144, "block", "q4_k"),
    13: GGMLType("Q5_K", 256, 176, "bytes", _NO_B200_KERNEL),
    14: GGMLType("Q6_K", 256, 210, "bytes", _NO_B200_KERNEL),
    15: GGMLType("Q8_K", 256, 292, "declined", _ONLY_ACTIVATIONS),
    16: GGMLType("IQ2_XXS", 256, 66, "declined", _NOT_IN_CANDLE),
    17: GGMLType("IQ2_XS", 256, 74, "declined", _NOT_IN_CANDLE),
    18: GGMLType("IQ3_XXS", 256, 98, "declined", _NOT_IN_CANDLE),
    19: GGMLType("IQ1_S", 256, 50, "declined", _NOT_IN_CANDLE),
    20: GGMLType("IQ4_NL", 32, 18, "declined", _NOT_IN_CANDLE),
    21: GGMLType("IQ3_S", 256, 110, "declined", _NOT_IN_CANDLE),
    22: GGMLType("IQ2_S", 256, 82, "declined", _NOT_IN_CANDLE),
    23: GGMLType("IQ4_XS", 256, 136, "declined", _NOT_IN_CANDLE),
    24: GGMLType("I8", 1, 1, "declined", _INTEGER_OR_F64),
    25: GGMLType("I16", 1, 2, "declined", _INTEGER_OR_F64),
    26: GGMLType("I32", 1, 4, "declined", _INTEGER_OR_F64),
    27: GGMLType("I64", 1, 8, "declined", _INTEGER_OR_F64),
    28: GGMLType("F64", 1, 8, "declined", _INTEGER_OR_F64),
    29: GGMLType("IQ1_M", 256, 56, "declined", _NOT_IN_CANDLE),
    30: GGMLType("BF16", 1, 2, "dense", "bfloat16"),
    31: GGMLType("Q4_0_4_4", None, None, "declined", _REMOVED_REPACK),
    32: GGMLType("Q4_0_4_8", None, None, "declined", _REMOVED_REPACK),
    33: GGMLType("Q4_0_8_8", None, None, "declined", _REMOVED_REPACK),
    34: GGMLType("TQ1_0", 256, 54, "declined", _NOT_IN_CANDLE),
    35: GGMLType("TQ2_0", 256, 66, "declined", _NOT_IN_CANDLE),
    36: GGMLType("IQ4_NL_4_4", None, None, "declined", _REMOVED_REPACK),
    37: GGMLType("IQ4_NL_4_8", None, None, "declined", _REMOVED_REPACK),
    38: GGMLType("IQ4_NL_8_8", None, None, "declined", _REMOVED_REPACK),
    39: GGMLType("MXFP4", 32, 17, "declined", _NOT_IN_CANDLE),
}


def ggml_type_name(type_id: int) -> str:
    t = GGML_TYPE_TABLE.get(type_id)
    return t.name if t else f"GGML type {type_id}"


def why_refused(type_id: int, tensor: str | None = None, as_tensor: bool = True):
    """The GGUFUnsupported to raise for a tensor of this type, or None when it
    is read. as_tensor=False asks about reading its raw bytes only, which the
    block formats without a kernel allow."""
    label = f"tensor {tensor!r}: " if tensor else ""
    t = GGML_TYPE_TABLE.get(type_id)
    if t is None:
        return GGUFUnsupported(f"{label}unknown GGML type id {type_id} -- declined rather than misread")
    if t.handling == "declined" or (t.handling == "bytes" and as_tensor):
        return GGUFUnsupported(f"{label}{t.name} {t.target}")
    return None


# metadata value type ids (gguf.md): scalars as numpy dtypes; 8 string, 9 array
_VALUE_DTYPES = {0: np.dtype("<u1"), 1: np.dtype("<i1"), 2: np.dtype("<u2"), 3: np.dtype("<i2"),
                 4: np.dtype("<u4"), 5: np.dtype("<i4"), 6: np.dtype("<f4"), 7: np.dtype("?"),
                 10: np.dtype("<u8"), 11: np.dtype("<i8"), 12: np.dtype("<f8")}
_T_STRING, _T_ARRAY = 8, 9
_MAX_RANK = 4
_ALIGN_DEFAULT = 32


class TensorSlot:
    """Where one tensor lives in the file. `extents` are GGUF's (fastest
    first); `shape` is torch order, their reverse -- a linear weight stored
    with extents [in, out] is (out, in), blocks running along `in`. `start`
    is the absolute file offset, `size` its byte count (None for a type whose
    geometry this loader does not know)."""

    __slots__ = ("name", "type_id", "extents", "shape", "start", "size", "count")

    def __init__(self, name, type_id, extents, start, size, count):
        self.name, self.type_id, self.extents = name, type_id, tuple(extents)
        self.shape = self.extents[::-1]
        self.start, self.size, self.count = start, size, count

    @property
    def type_name(self) -> str:
        return ggml_type_name(self.type_id)

    @property
    def handling(self) -> str:
        t = GGML_TYPE_TABLE.get(self.type_id)
        return t.handling if t else "declined"

    @property
    def block_format(self) -> str | None:
        t = GGML_TYPE_TABLE.get(self.type_id)
        return t.target if t and t.handling == "block" else None

    def __repr__(self):
        return f"TensorSlot({self.name!r}, {self.type_name}, shape={self.shape}, {self.size} bytes)"


def _scan(buf, path: str):
    """Parse the header, metadata and tensor table of the mapped file `buf`;
    returns (version, metadata, value types, alignment, data start, slots)."""
    end = len(buf)
    at = 0

    def span(n, what):
        nonlocal at
        if n < 0 or at + n > end:
            raise GGUFMalformed(f"{path}: the file ends inside {what} (needs {n} bytes at byte {at} of {end})")
        lo = at
        at += n
        return lo

    def scalar(dt, what):
        return np.frombuffer(buf, dt, 1, span(dt.itemsize, what))[0].item()

    def u32(what):
        return scalar(_VALUE_DTYPES[4], what)

    def u64(what):
        return scalar(_VALUE_DTYPES[10], what)

    def text(what):
        n = u64(f"the length of {what}")
        lo = span(n, what)
        # tokenizer pieces need not be valid UTF-8: keep their bytes round-trippable
        return bytes(buf[lo:lo + n]).decode("utf-8", "surrogateescape")

    def value(vtype, what, in_array=False):
        if vtype in _VALUE_DTYPES:
            return scalar(_VALUE_DTYPES[vtype], what)
        if vtype == _T_STRING:
            return text(what)
        if vtype != _T_ARRAY:
            raise GGUFMalformed(f"{path}: {what} has value type {vtype}, which the format does not define")
        if in_array:
            raise GGUFUnsupported(f"{path}: {what} is an array of arrays; not read")
        etype = u32(f"the element type of {what}")
        count = u64(f"the length of {what}")
        if count > end - at:  # every element takes at least a byte
            raise GGUFMalformed(f"{path}: {what} says it holds {count} elements but {end - at} bytes remain")
        if etype in _VALUE_DTYPES:
            dt = _VALUE_DTYPES[etype]
            items = np.frombuffer(buf, dt, count, span(dt.itemsize * count, what)).tolist()
        else:
            items = [value(etype, f"element {k} of {what}", True) for k in range(count)]
        return MetadataArray(items, etype)

    head = bytes(buf[span(4, "the magic number"):4])
    if head != b"GGUF":
        raise GGUFMalformed(f"{path}: starts with {head!r}; a GGUF file starts with b'GGUF'")
    version = u32("the format version")
    if version not in (2, 3):
        swapped = int.from_bytes(version.to_bytes(4, "little"), "big")
        if swapped in (1, 2, 3):
            raise GGUFUnsupported(f"{path}: written big-endian (version word {version:#010x}); this reader takes "
                                  "little-endian files")
        raise GGUFUnsupported(f"{path}: format version {version}; versions 2 and 3 are read")
    n_tensors = u64("the tensor count")
    n_meta = u64("the metadata count")
    if 8 * (n_tensors + n_meta) > end:
        raise GGUFMalformed(f"{path}: the header lists {n_meta} metadata entries and {n_tensors} tensors, more "
                            f"than {end} bytes can hold")
    meta, vtypes = {}, {}
    for k in range(n_meta):
        key = text(f"the key of metadata entry {k}")
        vtype = u32(f"the value type of metadata {key!r}")
        if key in meta:
            raise GGUFMalformed(f"{path}: metadata {key!r} is defined more than once")
        meta[key] = value(vtype, f"metadata {key!r}")
        vtypes[key] = vtype
    align = meta.get("general.alignment", _ALIGN_DEFAULT)
    if isinstance(align, bool) or not isinstance(align, int) or align <= 0 or align & (align - 1):
        raise GGUFMalformed(f"{path}: general.alignment is {align!r}, not a positive power of two")
    table = []
    for k in range(n_tensors):
        name = text(f"the name of tensor {k}")
        rank = u32(f"the rank of {name!r}")
        if not 1 <= rank <= _MAX_RANK:
            raise GGUFMalformed(f"{path}: {name!r} has rank {rank}; GGUF tensors have 1 to {_MAX_RANK} extents")
        extents = [u64(f"extent {d} of {name!r}") for d in range(rank)]
        tid = u32(f"the GGML type of {name!r}")
        rel = u64(f"the offset of {name!r}")
        table.append((name, extents, tid, rel))
    data_start = -(-at // align) * align
    slots = {}
    for name, extents, tid, rel in table:
        if name in slots:
            raise GGUFMalformed(f"{path}: two tensors are named {name!r}")
        if rel % align:
            raise GGUFMalformed(f"{path}: {name!r} starts at data offset {rel}, off the {align}-byte alignment")
        count = int(np.prod(extents, dtype=np.int64))
        t = GGML_TYPE_TABLE.get(tid)
        size = None
        if t is not None and t.block_elems is not None:
            if extents[0] % t.block_elems:
                raise GGUFMalformed(f"{path}: {name!r} is {t.name} but its first extent {extents[0]} does not "
                                    f"divide into blocks of {t.block_elems}")
            size = count // t.block_elems * t.block_bytes
            if data_start + rel + size > end:
                raise GGUFMalformed(f"{path}: {name!r} needs {size} bytes from byte {data_start + rel} and the "
                                    f"file ends at {end} (cut short)")
        slots[name] = TensorSlot(name, tid, extents, data_start + rel, size, count)
    return version, meta, vtypes, align, data_start, slots


class MetadataArray(list):
    """A metadata array value; `element_type` is its GGUF value type id."""

    def __init__(self, items, element_type):
        super().__init__(items)
        self.element_type = element_type


class GGUFContainer:
    """A GGUF file opened read-only through a memory map.

        with GGUFContainer(path) as g:
            g.metadata["general.architecture"]
            g.slot("blk.0.attn_q.weight")        # a TensorSlot
            g.bytes_of("blk.0.attn_q.weight")    # its stored bytes (a view)
    """

    def __init__(self, path):
        self.path = os.fspath(path)
        self._file = open(self.path, "rb")
        self._map = None
        try:
            if os.fstat(self._file.fileno()).st_size == 0:
                raise GGUFMalformed(f"{self.path}: zero bytes long, so not a GGUF file")
            self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
            (self.version, self.metadata, self.value_types, self.alignment, self.data_start,
             self.tensors) = _scan(memoryview(self._map), self.path)
        except BaseException:
            self.close()
            raise

    def slot(self, name: str) -> TensorSlot:
        if name not in self.tensors:
            raise KeyError(f"{self.path}: no tensor {name!r} in this file")
        return self.tensors[name]

    def bytes_of(self, name: str, strict: bool = True) -> memoryview:
        """The stored bytes of `name`, a view into the map. Types declined as
        tensors stay declined here unless strict=False; block formats without
        a kernel are readable."""
        sl = self.slot(name)
        if strict:
            err = why_refused(sl.type_id, name, as_tensor=False)
            if err is not None:
                raise err
        if sl.size is None:
            raise why_refused(sl.type_id, name) or GGUFUnsupported(f"tensor {name!r}: byte size unknown")
        return memoryview(self._map)[sl.start:sl.start + sl.size]

    def close(self):
        if self._map is not None:
            try:
                self._map.close()
            except BufferError:  # a caller still holds a view; the map goes with it
                pass
            self._map = None
        if self._file is not None:
            self._file.close()
            self._file = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __repr__(self):
        return f"GGUFContainer({self.path!r}, v{getattr(self, 'version', '?')}, {len(getattr(self, 'tensors', {}))} tensors)"


# ----------------------------------------------------------------- to the device

_STAGE_BYTES = 64 << 20


def _to_device(view: memoryview, device):
    """The bytes of `view` in a flat uint8 device tensor: copied from the map
    into a pinned staging buffer in pieces of at most 64 MB, each followed by
    an asynchronous host-to-device copy."""
    import numpy as np
    import torch

    n = len(view)
    out = torch.empty(n, dtype=torch.uint8, device=device)
    if n == 0:
        return out
    src = np.frombuffer(view, dtype=np.uint8)
    stage = torch.empty(min(n, _STAGE_BYTES), dtype=torch.uint8, pin_memory=True)
    host = stage.numpy()
    for p in range(0, n, _STAGE_BYTES):
        q = min(n, p + _STAGE_BYTES)
        if p:
            torch.cuda.current_stream(out.device).synchronize()  # the previous piece has left the buffer
        host[:q - p] = src[p:q]
        out[p:q].copy_(stage[:q - p], non_blocking=True)
    torch.cuda.current_stream(out.device).synchronize()
    return out


def _unpermute_rows(rows2d, n_head: int):
    """Reverse llama.cpp's rotary row order for q/k weights, on whole rows
    (a row is a contiguous run of blocks, so no block is touched): stored row
    (h, d, p) -> HF row (h, p, d), d < rows / n_head / 2, p in {0, 1}."""
    import torch

    n = rows2d.shape[0]
    if n_head <= 0 or n % (2 * n_head):
        raise GGUFUnsupported(f"cannot undo the llama.cpp q/k row order of {n} rows for {n_head} heads")
    dim = n // n_head // 2
    h = torch.arange(n_head).view(n_head, 1, 1)
    p = torch.arange(2).view(1, 2, 1)
    d = torch.arange(dim).view(1, 1, dim)
    src = (h * (2 * dim) + d * 2 + p).reshape(-1).to(rows2d.device)
    return rows2d.index_select(0, src)


def load_tensor(f: GGUFContainer, name: str, keep_blocks: bool = False, permute_heads: int | None = None,
                device="cuda"):
    """One tensor of `f` on `device` (reference: torchnative.gguf.load_tensor).

    F32 / F16 / BF16: a dense tensor of that dtype, bit for bit.
    Q4_0 / Q8_0 / Q4_K: with keep_blocks a QTensor holding the file's blocks
    unchanged, else their dequantisation as float32 (bit-exact, the reference's
    to_float). Other GGML types are refused by name.
    permute_heads (Llama's .attn_q. / .attn_k.): undo llama.cpp's rotary row
    order, by rows, so blocks stay byte-identical."""
    import torch

    from . import quant

    info = f.slot(name)
    why = why_refused(info.type_id, name)
    if why is not None:
        raise why
    dev = torch.device(device)
    data = _to_device(f.bytes_of(name), dev)
    if info.handling == "dense":
        t = data.view(getattr(torch, GGML_TYPE_TABLE[info.type_id].target)).reshape(info.shape)
        if permute_heads is not None:
            t = _unpermute_rows(t.reshape(info.shape[0], -1), permute_heads).reshape(info.shape)
        return t
    rows = info.shape[0] if len(info.shape) > 1 else 1
    if permute_heads is not None:
        data = _unpermute_rows(data.view(rows, -1), permute_heads).reshape(-1).contiguous()
    q = quant.QTensor(data, info.shape, info.block_format)
    return q if keep_blocks else quant._dequantize(q)


def quantized_linear(f: GGUFContainer, name: str, bias=None, device="cuda", permute_heads: int | None = None):
    """A QuantizedLinear whose weight is tensor `name`'s own blocks on the
    device (reference: torchnative.gguf.quantized_linear). The tensor must be
    a 2-D block tensor, (out_features, in_features) in torch order; blocks run
    along in_features, the contracted dimension, so nothing is repacked."""
    from . import quant

    info = f.slot(name)
    if info.handling != "block":
        why = why_refused(info.type_id, name)
        if why is not None:
            raise why
        raise GGUFUnsupported(f"tensor {name!r} is {info.type_name}, not a block-quantised type: build an "
                              "nn.Linear from load_tensor() instead")
    if len(info.shape) != 2:
        raise GGUFUnsupported(f"tensor {name!r} has shape {info.shape}; a linear weight is 2-D")
    out_features, in_features = info.shape
    qw = load_tensor(f, name, keep_blocks=True, permute_heads=permute_heads, device=device)
    return quant.QuantizedLinear(in_features, out_features, qw, bias, info.block_format)
