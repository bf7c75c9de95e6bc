"""The Q4_0 and Q8_0 operator family on a B200, mirroring torchnative's `torch._C`
quant entry points (torchnative/rust/torch_c/src/quant.rs) and its
`QuantizedLinear` module (torchnative/python/torchnative/quant/__init__.py).

Same names, argument meaning and errors as the reference; the compute goes
through the C ABI of libtorchnative_b200.so. There is no CPU path here: a CPU
tensor is refused by name (torchnative's own CPU kernels serve those).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N

Q4_0_BLOCK_ELEMS = 32
Q4_0_BLOCK_BYTES = 18
Q8_0_BLOCK_BYTES = 34
# format -> (elements per block, bytes per block); the formats that have B200
# kernels (quant.rs format_name spellings)
_FORMATS = {"q4_0": (Q4_0_BLOCK_ELEMS, Q4_0_BLOCK_BYTES), "q8_0": (Q4_0_BLOCK_ELEMS, Q8_0_BLOCK_BYTES),
            "q4_k": (256, 144)}
_LINEAR = {"q4_0": "tn_q4_0_linear", "q8_0": "tn_q8_0_linear", "q4_k": "tn_q4_k_linear"}
_DEQUANT = {"q4_0": "tn_q4_0_dequantize", "q8_0": "tn_q8_0_dequantize", "q4_k": "tn_q4_k_dequantize"}

_DTYPE_CODE = {torch.float32: N.TN_F32, torch.bfloat16: N.TN_BF16, torch.float16: N.TN_F16,
               torch.float64: N.TN_F64}


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


class QTensor:
    """A block-quantised weight: the GGML blob plus its logical shape.

    The reference keeps this as `Repr::Quantized(Arc<QTensor>)` inside a
    TensorBase (torch_c/src/tensor.rs:110, 970, 1297). Here the blob is a uint8
    torch tensor on the device, byte-identical to `_quantized_blob`.
    """

    __slots__ = ("blob", "shape", "format")

    def __init__(self, blob: torch.Tensor, shape, fmt: str = "q4_0"):
        if fmt not in _FORMATS:
            raise NotImplementedError(f"torch._C._quantize: format {fmt!r} is not implemented on this backend "
                                      f"(implemented: {sorted(_FORMATS)})")
        if blob.dtype != torch.uint8 or blob.dim() != 1:
            raise ValueError("QTensor blob must be a flat uint8 tensor")
        self.blob = blob
        self.shape = tuple(int(s) for s in shape)
        self.format = fmt

    @property
    def device(self) -> torch.device:
        return self.blob.device

    def nbytes(self) -> int:
        return self.blob.numel()

    def __repr__(self):
        return f"QTensor(shape={self.shape}, format={self.format}, device={self.device})"


def _expect_blob_size(op: str, shape, fmt: str, nbytes: int) -> None:
    elems, tbytes = _FORMATS[fmt]
    count = 1
    for s in shape:
        count *= int(s)
    want = count // elems * tbytes
    if count % elems != 0 or nbytes != want:
        raise ValueError(f"{op}: {fmt} stores {elems} elements in {tbytes} bytes, so a {list(shape)} tensor needs "
                         f"{want} bytes; got {nbytes}")


def _require_cuda(op: str, t: torch.Tensor) -> None:
    if t.device.type != "cuda":
        raise NotImplementedError(f"{op}: this is the CUDA arm (sm_100a); a {t.device.type} tensor belongs to "
                                  "torchnative's CPU path")


def _quantize(tensor: torch.Tensor, format: str = "q4_0") -> QTensor:
    """torch._C._quantize (quant.rs:124-172) on the device."""
    op = "torch._C._quantize"
    if format not in _FORMATS:
        raise NotImplementedError(f"{op}: format {format!r} is not implemented on this backend")
    _require_cuda(op, tensor)
    if format == "q4_k":
        raise NotImplementedError(f"{op}: the q4_k writer (llama.cpp's weighted make_qkx2_quants search) is not on "
                                  "this backend; q4_k weights come from GGUF files (torchnative_b200.gguf)")
    if tensor.dim() == 0:
        raise NotImplementedError(f"{op}: a 0-d tensor cannot be quantised")
    block = _FORMATS[format][0]
    last = tensor.shape[-1]
    if last % block != 0:
        raise NotImplementedError(f"{op}: {format} stores {block} elements per block, so it must have their last dim "
                                  f"divisible by block size -- got {last}, which is not a multiple of {block} "
                                  f"(shape {list(tensor.shape)})")
    src = tensor.detach().to(torch.float32).contiguous()
    cols = last
    rows = src.numel() // cols if cols else 0
    blob = torch.empty(src.numel() // block * _FORMATS[format][1], dtype=torch.uint8, device=src.device)
    if format == "q8_0":  # BlockQ8_0::from_float (k_quants.rs:676-706), the same writer as for activations
        N.check(N.lib().tn_q8_0_quantize(_ptr(src), N.TN_F32, cols, _ptr(blob), rows, cols, _stream(src.device)))
    else:
        N.check(N.lib().tn_q4_0_quantize(_ptr(src), _ptr(blob), rows, cols, _stream(src.device)))
    return QTensor(blob, tuple(tensor.shape), format)


def _dequantize(q: QTensor) -> torch.Tensor:
    """torch._C._dequantize (quant.rs:180-189): back to dense float32, bit-exact."""
    op = "torch._C._dequantize"
    if not isinstance(q, QTensor):
        raise TypeError(f"{op}: expected a quantised tensor")
    _require_cuda(op, q.blob)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    cols = q.shape[-1]
    rows = out.numel() // cols if cols else 0
    N.check(getattr(N.lib(), _DEQUANT[q.format])(_ptr(q.blob), _ptr(out), rows, cols, _stream(q.device)))
    return out


def _quantized_format(q: QTensor) -> str:
    return q.format


def _quantized_nbytes(q: QTensor) -> int:
    return q.nbytes()


def _quantized_blob(q: QTensor) -> bytes:
    """torch._C._quantized_blob (quant.rs:220-227): the raw GGML bytes."""
    return q.blob.cpu().numpy().tobytes()


def _quantized_from_blob(data: bytes, shape, format: str = "q4_0", device="cuda") -> QTensor:
    """torch._C._quantized_from_blob (quant.rs:235-262), placed on `device`."""
    op = "torch._C._quantized_from_blob"
    if format not in _FORMATS:
        raise NotImplementedError(f"{op}: format {format!r} is not implemented on this backend")
    _expect_blob_size(op, shape, format, len(data))
    host = torch.frombuffer(bytearray(data), dtype=torch.uint8)
    return QTensor(host.to(device), shape, format)


def _quantized_to(q: QTensor, device) -> QTensor:
    """torch._C._quantized_to (quant.rs:384-405): the same blocks on another
    device, byte for byte, never re-quantised; same device returns q itself."""
    device = torch.device(device)
    if q.device == device or (device.type == q.device.type and device.index is None):
        return q
    return QTensor(q.blob.to(device), q.shape, q.format)


def _quantized_linear(input: torch.Tensor, weight: QTensor, bias: torch.Tensor | None = None,
                      act_mode: int = N.TN_ACT_Q8_0) -> torch.Tensor:
    """torch._C._quantized_linear(input, weight, bias) (quant.rs:286-369):
    input @ dequant(weight).T + bias, with the reference's Q8_0 activation
    quantisation (k_quants.rs:2479-2510) by default.

    Accepts float32 activations as the reference does, and also bfloat16 and
    float16 (widened exactly inside the kernel, so nothing is spent that the
    caller cannot see); the result has the activation's dtype."""
    op = "torch._C._quantized_linear"
    if not isinstance(weight, QTensor):
        raise NotImplementedError(f"{op}: the weight must be a quantised tensor (torch._C._quantize), got "
                                  f"{type(weight).__name__}")
    if input.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise NotImplementedError(f"{op}: the activation must be float32 (or bfloat16/float16 on CUDA), got {input.dtype}")
    if input.device != weight.device:
        raise RuntimeError(f"{op}: Expected all tensors to be on the same device, but found at least two devices, "
                           f"{input.device} (the input) and {weight.device} (the quantised weight). Move the module "
                           "with `.to(device)`; QuantizedLinear moves its blocks byte for byte (torch._C._quantized_to).")
    _require_cuda(op, input)
    if len(weight.shape) != 2:
        raise RuntimeError(f"{op}: the quantised weight must be 2-D (out_features, in_features), got {weight.shape}")
    out_features, in_features = weight.shape
    if input.dim() == 0 or input.shape[-1] != in_features:
        raise RuntimeError(f"{op}: mat1 and mat2 shapes cannot be multiplied ({list(input.shape)} and "
                           f"{in_features}x{out_features})")
    if bias is not None:
        if bias.dtype != torch.float32:
            raise NotImplementedError(f"{op}: the bias must be float32, got {bias.dtype}")
        if tuple(bias.shape) != (out_features,):
            raise RuntimeError(f"{op}: bias shape {list(bias.shape)} does not match out_features {out_features}")
        if bias.device != input.device:
            raise RuntimeError(f"{op}: Expected all tensors to be on the same device (bias on {bias.device})")
        bias = bias.contiguous()
    lead = input.shape[:-1]
    x = input.reshape(-1, in_features)
    if x.stride(-1) != 1:
        x = x.contiguous()
    m = x.shape[0]
    y = torch.empty((m, out_features), dtype=input.dtype, device=input.device)
    if m and out_features:
        code = _DTYPE_CODE[input.dtype]
        lin = getattr(N.lib(), _LINEAR[weight.format])
        N.check(lin(_ptr(x), code, x.stride(0) if m > 1 else in_features, _ptr(weight.blob), _ptr(bias), _ptr(y),
                    code, m, out_features, in_features, int(act_mode), _stream(input.device)))
    return y.reshape(*lead, out_features)


def _q8_0_quantize(x: torch.Tensor) -> torch.Tensor:
    """The activation quantiser alone (BlockQ8_0::from_float, k_quants.rs:676-706):
    rows of x -> GGML Q8_0 blocks, as a flat uint8 tensor."""
    op = "torch._C._quantize"
    _require_cuda(op, x)
    if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise NotImplementedError(f"{op}: q8_0 activations must be float32, bfloat16 or float16, got {x.dtype}")
    cols = x.shape[-1]
    x2 = x.reshape(-1, cols)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    out = torch.empty(rows * (cols // 32) * 34, dtype=torch.uint8, device=x.device)
    N.check(N.lib().tn_q8_0_quantize(_ptr(x2), _DTYPE_CODE[x.dtype], x2.stride(0) if rows > 1 else cols, _ptr(out),
                                     rows, cols, _stream(x.device)))
    return out


class QuantizedLinear(torch.nn.Module):
    """`nn.Linear` with a Q4_0 weight on the device (quant/__init__.py:100-252
    of the reference): `qweight` is a plain attribute, not a Parameter; the bias
    stays dense float32; `.to(device)` moves the blocks byte for byte."""

    def __init__(self, in_features, out_features, qweight: QTensor | None, bias, fmt: str = "q4_0"):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.format = fmt
        self.qweight = qweight
        self.bias = bias

    @classmethod
    def from_linear(cls, mod: torch.nn.Linear, fmt: str = "q4_0"):
        out_features, in_features = mod.weight.shape
        return cls(in_features, out_features, _quantize(mod.weight, fmt), mod.bias, fmt)

    @classmethod
    def pending_from_linear(cls, mod: torch.nn.Linear, fmt: str = "q4_0", shard: tuple[int, int] | None = None):
        """The load-time swap (quant/__init__.py:154-181 of the reference): the
        layer is replaced before its weight exists (a meta tensor during
        `from_pretrained`), keeping the loader's `weight` entry registered until
        `adopt` receives the tensor. `shard = (rank, world)` makes this the
        tensor-parallel load point: the layer keeps only output rows
        [rank * out / world, (rank + 1) * out / world) of whatever arrives, the
        column shard of a Q4_0 linear (a row range of a GGML blob is a byte
        range, so nothing is re-quantised)."""
        out_features, in_features = mod.weight.shape
        if shard is not None:
            rank, world = shard
            if world < 1 or not 0 <= rank < world or out_features % world != 0:
                raise ValueError(f"cannot shard {out_features} output rows {world} ways (rank {rank})")
            out_features //= world
        bias = mod.bias
        if bias is not None and shard is not None and bias.device.type != "meta":
            bias = torch.nn.Parameter(bias.detach()[shard[0] * out_features:(shard[0] + 1) * out_features].clone(),
                                      requires_grad=False)
        self = cls(in_features, out_features, None, bias, fmt)
        self.shard = shard
        self.register_parameter("weight", mod.weight)
        return self

    def adopt(self, weight):
        """Take the arriving weight once (quant/__init__.py:183-237 of the
        reference): a dense tensor is quantised here (on its device, so the
        dense copy lives only for this call); an already block-quantised
        QTensor (a GGUF file's own blocks) is kept byte for byte. Under a
        tensor-parallel shard only this rank's rows are kept, sliced out of the
        dense rows before quantisation or out of the blob's rows as bytes."""
        if self.qweight is not None:
            raise ValueError(f"{type(self).__name__} already holds a quantised weight; adopt() is for the loading "
                             "placeholder and runs once.")
        if hasattr(weight, "qweight") and not isinstance(weight, QTensor):
            weight = weight.qweight
        shard = getattr(self, "shard", None)
        rows = self.out_features * (shard[1] if shard else 1)
        if isinstance(weight, QTensor):
            if tuple(weight.shape) != (rows, self.in_features):
                raise ValueError(f"pre-quantised weight shape {tuple(weight.shape)} does not match "
                                 f"({rows}, {self.in_features})")
            if shard is not None:
                row_bytes = weight.blob.numel() // rows
                r0 = shard[0] * self.out_features
                blob = weight.blob.view(rows, row_bytes)[r0:r0 + self.out_features].reshape(-1).contiguous()
                weight = QTensor(blob, (self.out_features, self.in_features), weight.format)
            self.qweight = weight
            self.format = weight.format
        else:
            if tuple(weight.shape) != (rows, self.in_features):
                raise ValueError(f"weight shape {tuple(weight.shape)} does not match ({rows}, {self.in_features})")
            if shard is not None:
                r0 = shard[0] * self.out_features
                weight = weight[r0:r0 + self.out_features]
            self.qweight = _quantize(weight, self.format)
        if "weight" in self._parameters:
            del self._parameters["weight"]
        # a bias the loader filled in full before the weight arrived: keep this
        # rank's slice of it too
        b = self.bias
        if shard is not None and b is not None and b.device.type != "meta" and b.numel() == rows:
            r0 = shard[0] * self.out_features
            self.bias = torch.nn.Parameter(b.detach()[r0:r0 + self.out_features].clone(), requires_grad=False)

    def _apply(self, fn, recurse=True):
        result = super()._apply(fn, recurse)
        if self.qweight is not None:
            target = fn(torch.empty(0)).device
            if self.qweight.device != target:
                self.qweight = _quantized_to(self.qweight, target)
        return result

    def forward(self, x):
        if self.qweight is None:
            raise RuntimeError("QuantizedLinear was asked to run before its weight arrived.")
        return _quantized_linear(x, self.qweight, self.bias)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, format={self.format}")


class QuantizeReport:
    """What `quantize_` replaced and what it skipped (with the reason), and the
    bytes on both sides (the reference's _Report, quant/__init__.py:255-298)."""

    def __init__(self, fmt: str):
        self.format = fmt
        self.replaced: list[str] = []
        self.skipped: list[tuple[str, str]] = []
        self.dense_bytes = 0
        self.quantized_bytes = 0

    @property
    def ratio(self) -> float:
        return self.quantized_bytes / self.dense_bytes if self.dense_bytes else float("nan")

    def __str__(self):
        return (f"quantize_({self.format}): {len(self.replaced)} linears replaced, {len(self.skipped)} skipped, "
                f"{self.dense_bytes} -> {self.quantized_bytes} bytes")


def quantize_(model: torch.nn.Module, format: str = "q4_0", predicate=None) -> QuantizeReport:
    """Swap every `nn.Linear` of `model` (on a CUDA device) for a
    `QuantizedLinear` in place, as the reference's `quantize_`
    (quant/__init__.py:300-365) does: `predicate(name, module)` narrows the
    choice, `lm_head` is not special-cased, a layer the format refuses is
    skipped with its reason, and a call that finds nothing to replace raises."""
    report = QuantizeReport(format)
    todo = []
    for name, module in model.named_modules():
        for child_name, child in module.named_children():
            if not isinstance(child, torch.nn.Linear):
                continue
            full = f"{name}.{child_name}" if name else child_name
            if predicate is not None and not predicate(full, child):
                report.skipped.append((full, "excluded by predicate"))
                continue
            todo.append((module, child_name, full, child))
    for parent, child_name, full, child in todo:
        try:
            q = QuantizedLinear.from_linear(child, format)
        except NotImplementedError as exc:
            report.skipped.append((full, str(exc).split(": ", 1)[-1]))
            continue
        setattr(parent, child_name, q)
        report.replaced.append(full)
        report.dense_bytes += child.weight.numel() * child.weight.element_size()
        report.quantized_bytes += q.qweight.nbytes()
    if not report.replaced and not report.skipped:
        if isinstance(model, torch.nn.Linear):
            raise ValueError("quantize_ replaces the children of the module it is given, not the module itself: "
                             "assign `parent.name = QuantizedLinear.from_linear(parent.name, fmt)` instead")
        raise ValueError(f"quantize_ found no nn.Linear to replace in {type(model).__name__}; nothing was quantised")
    return report
