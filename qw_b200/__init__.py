"""qw_b200 -- B200-native affine 4-bit group-quantized matmul for cr0sh/qw's
Qwen 27B linear layers (decode qmv, verify-batch qmm, tcgen05 prefill qmm,
tensor-parallel linear stack).

The compute lives in libqwqmm.so (C ABI in include/qw_qmm.h); this package is
the Python mirror of the reference's operator surface on torch tensors.
"""
from .ops import (QuantizedFusedLinear, QuantizedLinear, QuantizedMlp, compiled_moe_expert_forward, compiled_swiglu_activation, dequantize, device_status,
                  quantize_weights, quantized_linear_forward, quantized_linear_forward_global_scale, quantized_matmul,
                  quantized_matmul_argmax, quantized_matmul_chain, quantized_matmul_swiglu, quantized_matmul_topk,
                  swiglu_mlp, topk)

__all__ = [
    "QuantizedFusedLinear",
    "QuantizedLinear",
    "QuantizedMlp",
    "compiled_moe_expert_forward",
    "compiled_swiglu_activation",
    "dequantize",
    "device_status",
    "quantize_weights",
    "quantized_linear_forward",
    "quantized_linear_forward_global_scale",
    "quantized_matmul",
    "quantized_matmul_argmax",
    "quantized_matmul_chain",
    "quantized_matmul_swiglu",
    "quantized_matmul_topk",
    "swiglu_mlp",
    "topk",
]
