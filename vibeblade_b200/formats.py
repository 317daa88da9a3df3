"""GGUF block formats on the k-quant matmul path.

Type ids and block geometry follow the reference's ``ggml_type`` enum and size tables
(cpp/include/ggml_types.h:11-27, :31-71) and its packed block structs
(cpp/include/ggml_types.h:109-141).  A weight matrix is K rows of N values; each row is
a run of blocks along N and rows are ``row_bytes(type, N)`` apart, exactly the layout
``gemv_dequant`` reads (cpp/src/dequant.cpp:749-771).
"""
from __future__ import annotations

GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q4_0 = 2
GGML_TYPE_Q4_1 = 3
GGML_TYPE_Q5_0 = 6
GGML_TYPE_Q5_1 = 7
GGML_TYPE_Q8_0 = 8
GGML_TYPE_Q2_K = 10
GGML_TYPE_Q3_K = 11
GGML_TYPE_Q4_K = 12
GGML_TYPE_Q5_K = 13
GGML_TYPE_Q6_K = 14
GGML_TYPE_Q8_K = 15
GGML_TYPE_BF16 = 30

TYPE_NAMES = {GGML_TYPE_F32: "F32", GGML_TYPE_F16: "F16", GGML_TYPE_BF16: "BF16",
              GGML_TYPE_Q4_0: "Q4_0", GGML_TYPE_Q4_1: "Q4_1", GGML_TYPE_Q5_0: "Q5_0",
              GGML_TYPE_Q5_1: "Q5_1", GGML_TYPE_Q8_0: "Q8_0", GGML_TYPE_Q2_K: "Q2_K",
              GGML_TYPE_Q3_K: "Q3_K", GGML_TYPE_Q4_K: "Q4_K", GGML_TYPE_Q5_K: "Q5_K",
              GGML_TYPE_Q6_K: "Q6_K", GGML_TYPE_Q8_K: "Q8_K"}
NAME_TO_TYPE = {v: k for k, v in TYPE_NAMES.items()}

# values per block (cpp/include/ggml_types.h:31-50)
BLOCK_VALUES = {GGML_TYPE_F32: 1, GGML_TYPE_F16: 1, GGML_TYPE_BF16: 1,
                GGML_TYPE_Q4_0: 32, GGML_TYPE_Q4_1: 32, GGML_TYPE_Q5_0: 32, GGML_TYPE_Q5_1: 32,
                GGML_TYPE_Q8_0: 32, GGML_TYPE_Q2_K: 256, GGML_TYPE_Q3_K: 256,
                GGML_TYPE_Q4_K: 256, GGML_TYPE_Q5_K: 256, GGML_TYPE_Q6_K: 256,
                GGML_TYPE_Q8_K: 256}
# bytes per block (cpp/include/ggml_types.h:52-71); Q8_0 is the 34-byte GGUF block
BLOCK_BYTES = {GGML_TYPE_F32: 4, GGML_TYPE_F16: 2, GGML_TYPE_BF16: 2,
               GGML_TYPE_Q4_0: 18, GGML_TYPE_Q4_1: 20, GGML_TYPE_Q5_0: 22, GGML_TYPE_Q5_1: 24,
               GGML_TYPE_Q8_0: 34, GGML_TYPE_Q2_K: 84, GGML_TYPE_Q3_K: 110,
               GGML_TYPE_Q4_K: 144, GGML_TYPE_Q5_K: 176, GGML_TYPE_Q6_K: 210,
               GGML_TYPE_Q8_K: 292}
# the quantized types of the path (the tensor-core GEMM, MoE and the tiled GEMV kernels
# take these; F32 / F16 / BF16 weights -- small tensors such as the MoE router in GGUF
# files -- and the other block types take the generic GEMV)
QUANTIZED = (GGML_TYPE_Q8_0, GGML_TYPE_Q4_K, GGML_TYPE_Q6_K)
# the reference dispatcher's other block types (cpp/src/dequant.cpp:412-422): dequantize
# and the generic GEMV read them, each in the reference's reading of its block
OTHER_BLOCK_TYPES = (GGML_TYPE_Q4_0, GGML_TYPE_Q4_1, GGML_TYPE_Q5_0, GGML_TYPE_Q5_1,
                     GGML_TYPE_Q2_K, GGML_TYPE_Q3_K, GGML_TYPE_Q5_K, GGML_TYPE_Q8_K)

# byte offsets inside a block
Q4K_D, Q4K_DMIN, Q4K_SCALES, Q4K_QS = 0, 2, 4, 16          # block_q4_K :118-124
Q6K_QL, Q6K_QH, Q6K_SCALES, Q6K_D = 0, 128, 192, 208       # block_q6_K :135-141
Q80_D, Q80_QS = 0, 2                                       # GGUF Q8_0: fp16 d, int8 qs[32]

SUPPORTED = tuple(BLOCK_VALUES)


def parse_type(t) -> int:
    """Accept a ggml type id or its name ("Q4_K", "q6_k", ...)."""
    if isinstance(t, str):
        key = t.upper()
        if key not in NAME_TO_TYPE:
            raise RuntimeError(f"Unsupported dequant type: {t}")
        return NAME_TO_TYPE[key]
    t = int(t)
    if t not in BLOCK_VALUES:
        raise RuntimeError(f"Unsupported dequant type: {t}")
    return t


def bits_per_weight(t) -> float:
    t = parse_type(t)
    return 8.0 * BLOCK_BYTES[t] / BLOCK_VALUES[t]


def bytes_per_weight(t) -> float:
    t = parse_type(t)
    return BLOCK_BYTES[t] / BLOCK_VALUES[t]


def row_bytes(t, n: int) -> int:
    """Row stride of a K x N matrix: (N / block_values) * block_bytes, truncating like
    the reference (cpp/src/dequant.cpp:749-763)."""
    t = parse_type(t)
    return (int(n) // BLOCK_VALUES[t]) * BLOCK_BYTES[t]


def tensor_nbytes(t, n_values: int) -> int:
    """Bytes of n_values stored in blocks, rounding up (cpp/include/ggml_types.h:195-199)."""
    t = parse_type(t)
    bv = BLOCK_VALUES[t]
    return ((int(n_values) + bv - 1) // bv) * BLOCK_BYTES[t]


def matrix_nbytes(t, k: int, n: int) -> int:
    return int(k) * row_bytes(t, n)
