"""GGUF checkpoints straight to the device, keeping the file's own blocks.

Mirrors torchnative's `torchnative.gguf` (torchnative/python/torchnative/gguf/
__init__.py, reader.py): `GGUFFile` reads the container (header, typed
metadata, tensor descriptors, aligned tensor data) with `struct` and `mmap`
only; `load_tensor(f, name, keep_blocks=...)` turns one tensor into a device
tensor, and `quantized_linear(f, name)` into a `QuantizedLinear` whose weight
is the tensor's GGML blocks, byte for byte -- never decoded and re-encoded.

What differs from the reference is where the bytes land: the reference hands
them to candle's host QTensor (`torch._C._quantized_from_blob`); here they go
from the memory map through one pinned staging buffer to HBM
(`cudaMemcpyAsync` by torch), and the block formats that have B200 kernels
(Q4_0, Q8_0, Q4_K) become a `QTensor` on the device. Other GGML block formats are
listed and readable as raw bytes but refused by name when asked to become a
tensor, as are the types the reference refuses.

GGUF layout (little-endian): magic "GGUF", version (2 or 3), tensor count and
metadata count (u64); metadata entries (string key, u32 value type, value);
tensor descriptors (string name, u32 n_dims, n_dims u64 extents with the
fastest-varying first, u32 GGML type, u64 offset into the data section); the
data section starts at the next multiple of `general.alignment` (default 32).
"""

from __future__ import annotations

import mmap
import os
import struct

__all__ = ["GGML_TYPES", "GGUFFile", "GGUFFormatError", "GGUFTensorInfo", "UnsupportedGGUF", "load_tensor",
           "quantized_linear", "refusal", "type_name"]

_MAGIC = b"GGUF"
_DEFAULT_ALIGNMENT = 32
_MAX_DIMS = 4


class GGUFFormatError(ValueError):
    """Not a well-formed GGUF file: bad magic, truncation, inconsistent sizes."""


class UnsupportedGGUF(NotImplementedError):
    """A well-formed GGUF construct this loader refuses, by name."""


_ACT_SIDE = ("is a block format llama.cpp uses only for the activation operand inside its dot products, "
             "never as a stored weight")
_NO_KERNEL = ("is a GGML block format without a B200 kernel in this backend (Q4_0, Q8_0 and Q4_K have one); its "
              "bytes can be read with GGUFFile.raw, not turned into a tensor")
_NO_CANDLE = "has no candle GgmlDType in the reference, so neither side has storage or a kernel for it"
_NOT_WEIGHT = "is a plain numeric type no LLM checkpoint uses for weights; refused rather than guessed at"
_REPACKED = "is a repacked layout llama.cpp removed from the file format; files carrying it are not read"

# id -> (name, elements per block, bytes per block, kind, torch dtype / backend format / reason).
# kind: "dense" (read as that dtype), "block" (held as a device QTensor of that
# format), "raw" (a GGML block format this backend has no kernel for), or
# "refused". Block sizes are ggml's type_traits; the tests check them against
# the installed gguf-py's GGML_QUANT_SIZES.
GGML_TYPES = {
    0: ("F32", 1, 4, "dense", "float32"),
    1: ("F16", 1, 2, "dense", "float16"),
    2: ("Q4_0", 32, 18, "block", "q4_0"),
    3: ("Q4_1", 32, 20, "raw", _NO_KERNEL),
    6: ("Q5_0", 32, 22, "raw", _NO_KERNEL),
    7: ("Q5_1", 32, 24, "raw", _NO_KERNEL),
    8: ("Q8_0", 32, 34, "block", "q8_0"),
    9: ("Q8_1", 32, 36, "refused", _ACT_SIDE),
    10: ("Q2_K", 256, 84, "raw", _NO_KERNEL),
    11: ("Q3_K", 256, 110, "raw", _NO_KERNEL),
    12: ("Q4_K", 256, 144, "block", "q4_k"),
    13: ("Q5_K", 256, 176, "raw", _NO_KERNEL),
    14: ("Q6_K", 256, 210, "raw", _NO_KERNEL),
    15: ("Q8_K", 256, 292, "refused", _ACT_SIDE),
    16: ("IQ2_XXS", 256, 66, "refused", _NO_CANDLE),
    17: ("IQ2_XS", 256, 74, "refused", _NO_CANDLE),
    18: ("IQ3_XXS", 256, 98, "refused", _NO_CANDLE),
    19: ("IQ1_S", 256, 50, "refused", _NO_CANDLE),
    20: ("IQ4_NL", 32, 18, "refused", _NO_CANDLE),
    21: ("IQ3_S", 256, 110, "refused", _NO_CANDLE),
    22: ("IQ2_S", 256, 82, "refused", _NO_CANDLE),
    23: ("IQ4_XS", 256, 136, "refused", _NO_CANDLE),
    24: ("I8", 1, 1, "refused", _NOT_WEIGHT),
    25: ("I16", 1, 2, "refused", _NOT_WEIGHT),
    26: ("I32", 1, 4, "refused", _NOT_WEIGHT),
    27: ("I64", 1, 8, "refused", _NOT_WEIGHT),
    28: ("F64", 1, 8, "refused", _NOT_WEIGHT),
    29: ("IQ1_M", 256, 56, "refused", _NO_CANDLE),
    30: ("BF16", 1, 2, "dense", "bfloat16"),
    31: ("Q4_0_4_4", None, None, "refused", _REPACKED),
    32: ("Q4_0_4_8", None, None, "refused", _REPACKED),
    33: ("Q4_0_8_8", None, None, "refused", _REPACKED),
    34: ("TQ1_0", 256, 54, "refused", _NO_CANDLE),
    35: ("TQ2_0", 256, 66, "refused", _NO_CANDLE),
    36: ("IQ4_NL_4_4", None, None, "refused", _REPACKED),
    37: ("IQ4_NL_4_8", None, None, "refused", _REPACKED),
    38: ("IQ4_NL_8_8", None, None, "refused", _REPACKED),
    39: ("MXFP4", 32, 17, "refused", _NO_CANDLE),
}


def type_name(ggml_type: int) -> str:
    t = GGML_TYPES.get(ggml_type)
    return t[0] if t else f"<unknown GGML type id {ggml_type}>"


def refusal(ggml_type: int, tensor_name: str | None = None, for_tensor: bool = True):
    """The UnsupportedGGUF this loader raises for the type, or None.
    `for_tensor`: turning the bytes into a tensor (raw block formats refuse
    then, but their bytes stay readable)."""
    where = f" (tensor {tensor_name!r})" if tensor_name else ""
    t = GGML_TYPES.get(ggml_type)
    if t is None:
        return UnsupportedGGUF(f"GGML type id {ggml_type}{where} is not one this loader knows; refused rather "
                               "than read as something else")
    name, _, _, kind, why = t
    if kind == "refused" or (kind == "raw" and for_tensor):
        return UnsupportedGGUF(f"GGML type {name}{where} {why}")
    return None


# metadata value types: id -> struct format (scalars); 8 = string, 9 = array
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


class GGUFTensorInfo:
    """One descriptor. `shape` is torch order (the reverse of GGUF's extents,
    whose first is the fastest-varying): a linear weight stored with extents
    [in, out] is (out, in), nn.Linear's layout, and its blocks run along `in`."""

    __slots__ = ("name", "ggml_type", "ne", "shape", "offset", "nbytes", "n_elements")

    def __init__(self, name, ggml_type, ne, offset, nbytes, n_elements):
        self.name, self.ggml_type, self.ne = name, ggml_type, tuple(ne)
        self.shape = tuple(reversed(self.ne))
        self.offset, self.nbytes, self.n_elements = offset, nbytes, n_elements

    @property
    def type_name(self) -> str:
        return type_name(self.ggml_type)

    @property
    def kind(self) -> str:
        t = GGML_TYPES.get(self.ggml_type)
        return t[3] if t else "refused"

    @property
    def format(self) -> str | None:
        t = GGML_TYPES.get(self.ggml_type)
        return t[4] if t and t[3] == "block" else None

    def __repr__(self):
        return f"GGUFTensorInfo({self.name!r}, {self.type_name}, shape={self.shape}, nbytes={self.nbytes})"


class _Reader:
    def __init__(self, buf, size, path):
        self.buf, self.size, self.pos, self.path = buf, size, 0, path

    def _need(self, n, what):
        if n < 0 or self.pos + n > self.size:
            raise GGUFFormatError(f"{self.path}: truncated while reading {what} ({n} bytes at offset {self.pos}, "
                                  f"file is {self.size} bytes)")
        p = self.pos
        self.pos += n
        return p

    def unpack(self, fmt, what):
        n = struct.calcsize(fmt)
        return struct.unpack_from(fmt, self.buf, self._need(n, what))[0]

    def string(self, what):
        n = self.unpack("<Q", f"the length of {what}")
        p = self._need(n, what)
        # surrogateescape: tokenizer entries that are not UTF-8 round-trip
        return bytes(self.buf[p:p + n]).decode("utf-8", "surrogateescape")

    def value(self, vtype, what, nested=False):
        if vtype in _SCALAR:
            return self.unpack(_SCALAR[vtype], what)
        if vtype == _STRING:
            return self.string(what)
        if vtype == _ARRAY:
            if nested:
                raise UnsupportedGGUF(f"{self.path}: {what}: arrays of arrays are not read")
            etype = self.unpack("<I", f"the element type of {what}")
            count = self.unpack("<Q", f"the element count of {what}")
            if count > self.size - self.pos:  # every element is at least one byte
                raise GGUFFormatError(f"{self.path}: {what} claims {count} elements with "
                                      f"{self.size - self.pos} bytes left")
            if etype in _SCALAR:
                fmt = _SCALAR[etype]
                n = struct.calcsize(fmt) * count
                p = self._need(n, what)
                items = list(struct.unpack_from(f"<{count}{fmt[1]}", self.buf, p))
            else:
                items = [self.value(etype, f"{what}[{i}]", nested=True) for i in range(count)]
            return GGUFArray(etype, items)
        raise GGUFFormatError(f"{self.path}: {what}: unknown metadata value type {vtype}")


class GGUFArray(list):
    """A metadata array that remembers its element type."""

    def __init__(self, element_type, items):
        super().__init__(items)
        self.element_type = element_type


class GGUFFile:
    """A GGUF file, memory-mapped read-only.

        with GGUFFile(path) as f:
            f.metadata["general.architecture"]
            f.tensors["blk.0.attn_q.weight"]   # GGUFTensorInfo
            f.raw("blk.0.attn_q.weight")       # the stored bytes
    """

    def __init__(self, path):
        self.path = os.fspath(path)
        self._fh = open(self.path, "rb")
        self._mm = None
        try:
            self.size = os.fstat(self._fh.fileno()).st_size
            if self.size == 0:
                raise GGUFFormatError(f"{self.path}: empty file, not GGUF")
            self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ)
            self._parse()
        except BaseException:
            self.close()
            raise

    def close(self):
        if self._mm is not None:
            self._mm.close()
            self._mm = None
        if self._fh is not None:
            self._fh.close()
            self._fh = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _parse(self):
        r = _Reader(self._mm, self.size, self.path)
        magic = bytes(self._mm[r._need(4, "the magic"):4])
        if magic != _MAGIC:
            raise GGUFFormatError(f"{self.path}: not a GGUF file (magic {magic!r}, expected {_MAGIC!r})")
        version = r.unpack("<I", "the version")
        if version not in (2, 3):
            if struct.unpack(">I", struct.pack("<I", version))[0] in (1, 2, 3):
                raise UnsupportedGGUF(f"{self.path}: a big-endian GGUF file (version field {version:#x}); only "
                                      "little-endian files are read")
            raise UnsupportedGGUF(f"{self.path}: GGUF version {version} is not read (2 and 3 are)")
        self.version = version
        n_tensors = r.unpack("<Q", "the tensor count")
        n_kv = r.unpack("<Q", "the metadata count")
        if 8 * (n_tensors + n_kv) > self.size:
            raise GGUFFormatError(f"{self.path}: {n_kv} metadata entries and {n_tensors} tensors cannot fit in "
                                  f"{self.size} bytes")
        self.metadata, self.metadata_types = {}, {}
        for i in range(n_kv):
            key = r.string(f"metadata key #{i}")
            vtype = r.unpack("<I", f"the value type of {key!r}")
            if key in self.metadata:
                raise GGUFFormatError(f"{self.path}: metadata key {key!r} appears twice")
            self.metadata[key] = r.value(vtype, f"metadata {key!r}")
            self.metadata_types[key] = vtype
        align = self.metadata.get("general.alignment", _DEFAULT_ALIGNMENT)
        if isinstance(align, bool) or not isinstance(align, int) or align <= 0 or align & (align - 1):
            raise GGUFFormatError(f"{self.path}: general.alignment = {align!r} is not a power of two")
        self.alignment = align
        descs = []
        for i in range(n_tensors):
            name = r.string(f"tensor name #{i}")
            nd = r.unpack("<I", f"the dimension count of {name!r}")
            if not 1 <= nd <= _MAX_DIMS:
                raise GGUFFormatError(f"{self.path}: tensor {name!r} has {nd} dimensions (1..{_MAX_DIMS} allowed)")
            ne = [r.unpack("<Q", f"extent {d} of {name!r}") for d in range(nd)]
            gt = r.unpack("<I", f"the type of {name!r}")
            off = r.unpack("<Q", f"the data offset of {name!r}")
            descs.append((name, ne, gt, off))
        self.data_offset = (r.pos + align - 1) // align * align
        self.tensors = {}
        for name, ne, gt, off in descs:
            if name in self.tensors:
                raise GGUFFormatError(f"{self.path}: tensor {name!r} appears twice")
            if off % align:
                raise GGUFFormatError(f"{self.path}: tensor {name!r} at data offset {off}, not a multiple of "
                                      f"the alignment {align}")
            n = 1
            for e in ne:
                n *= e
            t = GGML_TYPES.get(gt)
            nbytes = None
            if t is not None and t[1] is not None:
                if ne[0] % t[1]:
                    raise GGUFFormatError(f"{self.path}: tensor {name!r} is {t[0]} with a first extent of {ne[0]}, "
                                          f"not a multiple of its block of {t[1]}")
                nbytes = n // t[1] * t[2]
                if self.data_offset + off + nbytes > self.size:
                    raise GGUFFormatError(f"{self.path}: tensor {name!r} runs past the end of the file "
                                          "(truncated)")
            self.tensors[name] = GGUFTensorInfo(name, gt, ne, self.data_offset + off, nbytes, n)

    def info(self, name) -> GGUFTensorInfo:
        try:
            return self.tensors[name]
        except KeyError:
            raise KeyError(f"{self.path} has no tensor named {name!r}") from None

    def raw(self, name, refuse=True) -> memoryview:
        """The stored bytes of `name` (GGML blocks or packed scalars), a view
        of the map. Types refused as tensors by the reference stay refused
        unless refuse=False; block formats without a kernel here are readable."""
        info = self.info(name)
        if refuse:
            why = refusal(info.ggml_type, name, for_tensor=False)
            if why is not None:
                raise why
        if info.nbytes is None:
            raise refusal(info.ggml_type, name) or UnsupportedGGUF(f"tensor {name!r}: no known byte size")
        return memoryview(self._mm)[info.offset:info.offset + info.nbytes]

    def __repr__(self):
        return f"GGUFFile({self.path!r}, version={getattr(self, 'version', '?')}, tensors={len(self.tensors)})"


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
        raise UnsupportedGGUF(f"cannot undo the llama.cpp q/k row order of {n} rows for {n_head} heads")
    dim = n // n_head // 2
    h = torch.arange(n_head).view(n_head, 1, 1)
    p = torch.arange(2).view(1, 2, 1)
    d = torch.arange(dim).view(1, 1, dim)
    src = (h * (2 * dim) + d * 2 + p).reshape(-1).to(rows2d.device)
    return rows2d.index_select(0, src)


def load_tensor(f: GGUFFile, name: str, keep_blocks: bool = False, permute_heads: int | None = None,
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

    info = f.info(name)
    why = refusal(info.ggml_type, name)
    if why is not None:
        raise why
    dev = torch.device(device)
    data = _to_device(f.raw(name), dev)
    if info.kind == "dense":
        t = data.view(getattr(torch, GGML_TYPES[info.ggml_type][4])).reshape(info.shape)
        if permute_heads is not None:
            t = _unpermute_rows(t.reshape(info.shape[0], -1), permute_heads).reshape(info.shape)
        return t
    rows = info.shape[0] if len(info.shape) > 1 else 1
    if permute_heads is not None:
        data = _unpermute_rows(data.view(rows, -1), permute_heads).reshape(-1).contiguous()
    q = quant.QTensor(data, info.shape, info.format)
    return q if keep_blocks else quant._dequantize(q)


def quantized_linear(f: GGUFFile, name: str, bias=None, device="cuda", permute_heads: int | None = None):
    """A QuantizedLinear whose weight is tensor `name`'s own blocks on the
    device (reference: torchnative.gguf.quantized_linear). The tensor must be
    a 2-D block tensor, (out_features, in_features) in torch order; blocks run
    along in_features, the contracted dimension, so nothing is repacked."""
    from . import quant

    info = f.info(name)
    if info.kind != "block":
        why = refusal(info.ggml_type, name)
        if why is not None:
            raise why
        raise UnsupportedGGUF(f"tensor {name!r} is {info.type_name}, not a block-quantised type: build an "
                              "nn.Linear from load_tensor() instead")
    if len(info.shape) != 2:
        raise UnsupportedGGUF(f"tensor {name!r} has shape {info.shape}; a linear weight is 2-D")
    out_features, in_features = info.shape
    qw = load_tensor(f, name, keep_blocks=True, permute_heads=permute_heads, device=device)
    return quant.QuantizedLinear(in_features, out_features, qw, bias, info.format)
