"""qw_b200 -- B200-native affine group-quantized matmul for cr0sh/qw's Qwen
27B linear layers: decode qmv, verify-batch qmm and tcgen05 prefill qmm (4-
and 8-bit codes), the fused SwiGLU MLP input, the greedy-token and top-k
candidate steps after the LM head, and the tensor-parallel linear stack with
its NVLink peer allreduce.

The compute lives in libqwqmm.so (C ABI in include/qw_qmm.h); this package is
the Python mirror of the reference's operator surface on torch tensors.
"""
from .ops import (QuantizedFusedLinear, QuantizedLinear, QuantizedMlp, compiled_moe_expert_forward,
                  compiled_swiglu_activation, decode_schedule, dequantize, device_status, quantize_weights,
                  quantized_linear_forward,
                  quantized_linear_forward_global_scale, quantized_matmul, quantized_matmul_argmax,
                  quantized_matmul_chain, quantized_matmul_swiglu, quantized_matmul_topk, swiglu_mlp, topk)

__all__ = [
    "QuantizedFusedLinear",
    "QuantizedLinear",
    "QuantizedMlp",
    "compiled_moe_expert_forward",
    "compiled_swiglu_activation",
    "decode_schedule",
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
