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

    # ---------------------------------------------- INT4-AWQ and FP8-E4M3
    @staticmethod
    def fused_gemv_int4(W_packed, x, scales, zeros, y, rows: int, cols: int, group_size: int) -> None:
        """src/quantization.cpp:102-200: W_packed uint32 [rows][cols/8] (column c
        = nibble c % 8 of word c / 8), scales / zeros float32
        [rows][cols/group_size] (zeros may be None), w = (q - zero) * scale."""
        ng = rows * (cols // group_size) if group_size else 0
        if W_packed.dtype != np.uint32 or W_packed.size < rows * (cols // 8):
            raise ValueError("W_packed must be uint32 with rows * cols/8 words")
        if scales.dtype != np.float32 or scales.size < ng or (zeros is not None and
                                                              (zeros.dtype != np.float32 or zeros.size < ng)):
            raise ValueError("scales/zeros must be float32 with rows * cols/group_size elements")
        if x.dtype != np.float32 or x.size < cols or y.dtype != np.float32 or y.size < rows:
            raise ValueError("x / y must be float32 of at least cols / rows elements")
        _native.lib().nexus_fused_gemv_int4(_ptr(W_packed), _ptr(x), _ptr(scales),
                                            None if zeros is None else _ptr(zeros), _ptr(y), rows, cols, group_size)

    @staticmethod
    def fused_gemv_fp8(W_fp8, x, y, rows: int, cols: int, scale: float) -> None:
        """src/quantization.cpp:202-262: one E4M3 byte per weight times scale."""
        if W_fp8.nbytes < rows * cols:
            raise ValueError("W_fp8 holds fewer than rows * cols bytes")
        if x.dtype != np.float32 or x.size < cols or y.dtype != np.float32 or y.size < rows:
            raise ValueError("x / y must be float32 of at least cols / rows elements")
        _native.lib().nexus_fused_gemv_fp8(_ptr(W_fp8), _ptr(x), _ptr(y), rows, cols, float(scale))

    @staticmethod
    def dequantize_int4_awq(packed, scales, zeros, output, count: int, group_size: int) -> None:
        """src/quantization.cpp:28-46."""
        if packed.dtype != np.uint32 or packed.size * 8 < count or output.dtype != np.float32 or output.size < count:
            raise ValueError("buffer too small")
        _native.lib().nexus_dequantize_int4_awq(_ptr(packed), _ptr(scales), None if zeros is None else _ptr(zeros),
                                                _ptr(output), count, group_size)

    @staticmethod
    def dequantize_fp8_e4m3(input, output, count: int, scale: float) -> None:
        """src/quantization.cpp:62-68."""
        if input.nbytes < count or output.dtype != np.float32 or output.size < count:
            raise ValueError("buffer too small")
        _native.lib().nexus_dequantize_fp8_e4m3(_ptr(input), _ptr(output), count, float(scale))


_NAME = {DataType.GGUF_Q4_0: "q4_0", DataType.GGUF_Q8_0: "q8_0", DataType.FP16: "fp16",
         DataType.GGUF_Q5_K: "q5_k", DataType.GGUF_Q6_K: "q6_k"}
