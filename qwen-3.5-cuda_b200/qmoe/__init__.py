"""qmoe -- B200 (sm_100a) MoE block for Qwen3.5-35B-A3B-shaped layers.

Host-side mirror of the reference's interfaces (quantized.hpp, matmul_q4.hpp,
layer_moe.hpp) over the C-ABI of include/qmoe.h.  The CUDA library is
required: there is no CPU fallback.
"""
from . import _lib
from ._lib import lib, check, status_string
from .quant import GgmlType, QuantTensor, ggml_type_block_size, ggml_type_size, calculate_tensor_bytes
from .matmul import matmul_type_supported, matmul_dispatch, dequantize_row
from .layer import ModelConfig, MoeLayer

__all__ = ["lib", "check", "status_string", "GgmlType", "QuantTensor", "ggml_type_block_size", "ggml_type_size",
           "calculate_tensor_bytes", "matmul_type_supported", "matmul_dispatch", "dequantize_row", "ModelConfig",
           "MoeLayer"]
