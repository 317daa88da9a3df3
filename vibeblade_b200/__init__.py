"""vibeblade_b200 -- B200-native (sm_100a) GGUF k-quant dequantize-and-multiply.

Drop-in device implementation of VibeBlade's quantized matmul path
(kevin046/VibeBlade cpp/src/dequant.cpp, cpp/include/dequant.h): Q4_K, Q6_K and Q8_0
weights -- and every other type the reference's dispatcher reads -- in the reference's
K x N block layout, dequantized and multiplied by hand-written CUDA kernels in
``libvbq.so`` behind the C ABI in ``include/vbq.h``.
"""
from . import formats
from .formats import (GGML_TYPE_BF16, GGML_TYPE_F16, GGML_TYPE_F32, GGML_TYPE_Q2_K, GGML_TYPE_Q3_K,
                      GGML_TYPE_Q4_0, GGML_TYPE_Q4_1, GGML_TYPE_Q4_K, GGML_TYPE_Q5_0, GGML_TYPE_Q5_1,
                      GGML_TYPE_Q5_K, GGML_TYPE_Q6_K, GGML_TYPE_Q8_0, GGML_TYPE_Q8_K, row_bytes,
                      tensor_nbytes)
from .dequant import (dequantize, dequantize_row, gemv_dequant, gemv_dequant_mt, gemv_fused,
                      gemv_scratch_bytes)
from .gguf import GGUFFile
from .gemm import gemm_dequant, gemm_swiglu, device_status
from .moe import gemm_grouped, moe_ffn, moe_route, moe_sort, moe_workspace_bytes
from ._lib import VbqError

__all__ = [
    "formats", "GGML_TYPE_Q4_K", "GGML_TYPE_Q6_K", "GGML_TYPE_Q8_0", "GGML_TYPE_F32",
    "GGML_TYPE_F16", "GGML_TYPE_BF16", "GGML_TYPE_Q4_0", "GGML_TYPE_Q4_1", "GGML_TYPE_Q5_0",
    "GGML_TYPE_Q5_1", "GGML_TYPE_Q2_K", "GGML_TYPE_Q3_K", "GGML_TYPE_Q5_K", "GGML_TYPE_Q8_K",
    "row_bytes", "GGUFFile",
    "tensor_nbytes", "dequantize", "dequantize_row", "gemv_dequant", "gemv_dequant_mt", "gemv_fused",
    "gemv_scratch_bytes", "gemm_dequant", "gemm_swiglu", "device_status", "gemm_grouped", "moe_ffn",
    "moe_route", "moe_sort", "moe_workspace_bytes",
    "VbqError",
]
