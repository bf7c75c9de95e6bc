"""torchnative_b200 -- B200 (sm_100a) kernels for torchnative's two hot
operators, the GGML Q4_0 weight-only linear and scaled_dot_product_attention,
behind the C ABI in include/torchnative_b200.h.

The host mirror of the reference's operator interface:
  torchnative_b200.quant       -- torch._C._quantize / _dequantize / _quantized_* /
                                  _quantized_linear and QuantizedLinear
  torchnative_b200.attention   -- aten._scaled_dot_product_flash_attention_for_cpu
"""

from . import _native  # noqa: F401

__all__ = ["quant", "attention", "build"]
