"""Host-side mirror of ``nexus::QuantizationKernel`` (include/quantization.hpp:56-154).

Same names, argument meaning and error behaviour as the reference's static
GEMV and dequantization methods, executed on the GPU through the C ABI
(``nexus_fused_gemv_*`` / ``nexus_dequantize_gguf_*`` in include/nexus_gpu.h):

* ``fused_gemv_q4_0(W, x, y, rows, cols)`` writes ``y[:rows]`` in place, like
  the reference (src/quantization.cpp:264-330).  W is the raw block bytes
  (numpy uint8, or uint16 halves for FP16), x float32[cols], y float32[rows].
* ``dequantize_gguf_q4_0(blocks, output, num_blocks)`` fills ``output``.
* ``fp16_to_fp32(h)`` is the reference's non-IEEE decoder (pure Python; the
  GPU kernels use the same bit rule).

The calls are synchronous; weights are uploaded once per host buffer and kept
on the device (see nexus_gpu_weight_cache_invalidate).
"""
from __future__ import annotations

import struct

import numpy as np

from . import _native
from .formats import BLOCK, DataType


def _ptr(a: np.ndarray) -> int:
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("arrays must be C-contiguous")
    return a.ctypes.data


def _check_sizes(W: np.ndarray, x: np.ndarray, y: np.ndarray, dt: DataType, rows: int, cols: int) -> None:
    per, nbytes = BLOCK[dt]
    if W.nbytes < rows * (cols // per) * nbytes:
        raise ValueError("W holds fewer bytes than rows x cols blocks")
    if x.dtype != np.float32 or x.size < cols:
        raise ValueError("x must be float32 with at least cols elements")
    if y.dtype != np.float32 or y.size < rows:
        raise ValueError("y must be float32 with at least rows elements")


class QuantizationKernel:
    @staticmethod
    def fp16_to_fp32(h: int) -> float:
        """include/quantization.hpp:59-70 (exponent 0x1f -> +0.0; zero/subnormal
        halves decode as if normal: 0x0000 -> 2**-15)."""
        w = (h & 0x7FFF) << 13
        sign = (h & 0x8000) << 16
        if (h & 0x7C00) >> 10 == 0x1F:
            return 0.0
        return struct.unpack("<f", struct.pack("<I", sign | (w + (0x70 << 23))))[0]

    @staticmethod
    def _gemv(dt: DataType, W, x, y, rows: int, cols: int) -> None:
        _check_sizes(W, x, y, dt, rows, cols)
        getattr(_native.lib(), f"nexus_fused_gemv_{_NAME[dt]}")(_ptr(W), _ptr(x), _ptr(y), rows, cols)

    @staticmethod
    def fused_gemv_q4_0(W_q4, x, y, rows: int, cols: int) -> None:
        QuantizationKernel._gemv(DataType.GGUF_Q4_0, W_q4, x, y, rows, cols)

    @staticmethod
    def fused_gemv_q8_0(W_q8, x, y, rows: int, cols: int) -> None:
        QuantizationKernel._gemv(DataType.GGUF_Q8_0, W_q8, x, y, rows, cols)

    @staticmethod
    def fused_gemv_fp16(W_fp16, x, y, rows: int, cols: int) -> None:
        QuantizationKernel._gemv(DataType.FP16, W_fp16, x, y, rows, cols)

    @staticmethod
    def fused_gemv_q5_k(W_q5_k, x, y, rows: int, cols: int) -> None:
        QuantizationKernel._gemv(DataType.GGUF_Q5_K, W_q5_k, x, y, rows, cols)

    @staticmethod
    def fused_gemv_q6_k(W_q6_k, x, y, rows: int, cols: int) -> None:
        QuantizationKernel._gemv(DataType.GGUF_Q6_K, W_q6_k, x, y, rows, cols)

    @staticmethod
    def _deq(dt: DataType, blocks, output, num_blocks: int) -> None:
        per, nbytes = BLOCK[dt]
        if blocks.nbytes < num_blocks * nbytes or output.dtype != np.float32 or output.size < num_blocks * per:
            raise ValueError("buffer too small")
        getattr(_native.lib(), f"nexus_dequantize_gguf_{_NAME[dt]}")(_ptr(blocks), _ptr(output), num_blocks)

    @staticmethod
    def dequantize_gguf_q4_0(blocks, output, num_blocks: int) -> None:
        QuantizationKernel._deq(DataType.GGUF_Q4_0, blocks, output, num_blocks)

    @staticmethod
    def dequantize_gguf_q5_k(blocks, output, num_blocks: int) -> None:
        QuantizationKernel._deq(DataType.GGUF_Q5_K, blocks, output, num_blocks)

    @staticmethod
    def dequantize_gguf_q6_k(blocks, output, num_blocks: int) -> None:
        QuantizationKernel._deq(DataType.GGUF_Q6_K, blocks, output, num_blocks)


_NAME = {DataType.GGUF_Q4_0: "q4_0", DataType.GGUF_Q8_0: "q8_0", DataType.FP16: "fp16",
         DataType.GGUF_Q5_K: "q5_k", DataType.GGUF_Q6_K: "q6_k"}
