"""GGUF block formats on NexusLLM's GEMV path.

`DataType` keeps the numeric values of ``nexus::DataType``
(include/nexus_common.hpp:244-260) so that a value passed through the
reference's ``gemv_dispatch(const void* W, DataType dt, ...)``
(include/nexus_backend.hpp:55-62) means the same thing here and in the C ABI
(include/nexus_gpu.h).  Block sizes are the packed struct sizes of
include/quantization.hpp:8-47.

Weight bytes are the TRUE block byte counts (rows * cols / block_elems *
block_bytes).  The reference's ``TensorShape::total_bytes`` over-estimates
them (it counts Q4_0 as 5 bits and Q6_K as 7 bits per weight,
include/nexus_common.hpp:262-281), so it must not be used to size uploads.
"""
from __future__ import annotations

import enum


class DataType(enum.IntEnum):
    FP32 = 0
    FP16 = 1
    BF16 = 2
    FP8_E4M3 = 3
    INT8 = 4
    INT4_AWQ = 5
    INT4_GPTQ = 6
    GGUF_Q4_0 = 7
    GGUF_Q4_K = 8
    GGUF_Q8_0 = 9
    GGUF_Q5_0 = 10
    GGUF_Q5_K = 11
    GGUF_Q6_K = 12
    GGUF_Q2_K = 13
    GGUF_Q3_K = 14


# dtype -> (elements per block, bytes per block)
BLOCK = {
    DataType.FP16: (1, 2),
    DataType.GGUF_Q4_0: (32, 18),
    DataType.GGUF_Q8_0: (32, 34),
    DataType.GGUF_Q5_K: (256, 176),
    DataType.GGUF_Q6_K: (256, 210),
}

# short names used by the C ABI entry points (nexus_fused_gemv_<name>)
NAME = {
    DataType.FP16: "fp16",
    DataType.GGUF_Q4_0: "q4_0",
    DataType.GGUF_Q8_0: "q8_0",
    DataType.GGUF_Q5_K: "q5_k",
    DataType.GGUF_Q6_K: "q6_k",
}
BY_NAME = {v: k for k, v in NAME.items()}

GEMV_TYPES = tuple(BLOCK)


def parse(dtype) -> DataType:
    if isinstance(dtype, str):
        return BY_NAME[dtype.lower()]
    return DataType(int(dtype))


def check_shape(dtype, rows: int, cols: int) -> None:
    """Raise ValueError when `cols` does not hold whole blocks.

    The reference silently drops a remainder (``cols / 32``, ``cols / QK_K``,
    src/quantization.cpp:269,337,516,627); this library rejects it instead.
    """
    dt = parse(dtype)
    if dt not in BLOCK:
        raise ValueError(f"unsupported GEMV weight type {dt!r}")
    per, _ = BLOCK[dt]
    if rows < 0 or cols < 0 or cols % per:
        raise ValueError(f"{dt.name}: cols={cols} must be a multiple of {per}")


def row_bytes(dtype, cols: int) -> int:
    dt = parse(dtype)
    per, nbytes = BLOCK[dt]
    return cols // per * nbytes


def weight_bytes(dtype, rows: int, cols: int) -> int:
    return rows * row_bytes(dtype, cols)


def bytes_per_weight(dtype) -> float:
    per, nbytes = BLOCK[parse(dtype)]
    return nbytes / per
