"""ctypes binding of libnexus_gpu.so (the C ABI in include/nexus_gpu.h).

The library is built in-tree (``nexusllm_b200/lib/libnexus_gpu.so``, see
nexusllm_b200/build.py).  There is no fallback: if the library is missing,
`lib()` raises, and every GPU entry point of this package fails with it.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libnexus_gpu.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "nexus_gpu.h")

_VP, _SZ, _I32, _U32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_uint32
_FP = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes)
SIGNATURES = {
    "nexus_fused_gemv_q4_0": (None, [_VP, _VP, _VP, _SZ, _SZ]),
    "nexus_fused_gemv_q8_0": (None, [_VP, _VP, _VP, _SZ, _SZ]),
    "nexus_fused_gemv_fp16": (None, [_VP, _VP, _VP, _SZ, _SZ]),
    "nexus_fused_gemv_q5_k": (None, [_VP, _VP, _VP, _SZ, _SZ]),
    "nexus_fused_gemv_q6_k": (None, [_VP, _VP, _VP, _SZ, _SZ]),
    "nexus_dequantize_gguf_q4_0": (None, [_VP, _VP, _SZ]),
    "nexus_dequantize_gguf_q5_k": (None, [_VP, _VP, _SZ]),
    "nexus_dequantize_gguf_q6_k": (None, [_VP, _VP, _SZ]),
    "nexus_fused_gemv_int4": (None, [_VP, _VP, _VP, _VP, _VP, _SZ, _SZ, _SZ]),
    "nexus_fused_gemv_fp8": (None, [_VP, _VP, _VP, _SZ, _SZ, ctypes.c_float]),
    "nexus_dequantize_int4_awq": (None, [_VP, _VP, _VP, _VP, _SZ, _SZ]),
    "nexus_dequantize_fp8_e4m3": (None, [_VP, _VP, _SZ, ctypes.c_float]),
    "nexus_gpu_gemv_int4_workspace_size": (_SZ, [_SZ]),
    "nexus_gpu_gemv_int4": (_I32, [_VP, _VP, _VP, _VP, _VP, _SZ, _SZ, _SZ, _VP, _SZ, _VP]),
    "nexus_gpu_gemv_fp8": (_I32, [_VP, _VP, _VP, _SZ, _SZ, ctypes.c_float, _VP]),
    "nexus_gpu_dequantize_int4_awq": (_I32, [_VP, _VP, _VP, _VP, _SZ, _SZ, _VP]),
    "nexus_gpu_dequantize_fp8_e4m3": (_I32, [_VP, _VP, _SZ, ctypes.c_float, _VP]),
    "nexus_gpu_gemv_dispatch": (_I32, [_VP, _U32, _VP, _VP, _SZ, _SZ]),
    "nexus_gpu_allocate_device_memory": (_VP, [_SZ]),
    "nexus_gpu_free_device_memory": (None, [_VP]),
    "nexus_gpu_copy_host_to_device_async": (_I32, [_VP, _VP, _SZ, _VP]),
    "nexus_gpu_copy_device_to_host_async": (_I32, [_VP, _VP, _SZ, _VP]),
    "nexus_gpu_synchronize": (_I32, [_VP]),
    "nexus_gpu_weight_cache_invalidate": (_I32, [_VP]),
    "nexus_gpu_weight_cache_bytes": (_SZ, []),
    "nexus_gpu_weight_bytes": (_SZ, [_U32, _SZ, _SZ]),
    "nexus_gpu_gemv": (_I32, [_VP, _U32, _VP, _U32, _VP, _SZ, _SZ, _SZ, _VP]),
    "nexus_gpu_gemv_workspace_size": (_SZ, [_U32, _SZ, _SZ, _SZ]),
    "nexus_gpu_gemv_ws": (_I32, [_VP, _U32, _VP, _U32, _VP, _SZ, _SZ, _SZ, _VP, _SZ, _VP]),
    "nexus_gpu_gemv_noalloc": (_I32, [_VP, _U32, _VP, _U32, _VP, _SZ, _SZ, _SZ, _VP]),
    "nexus_gpu_stack_create": (_I32, [_U32, _VP, _U32, ctypes.c_uint64, ctypes.POINTER(_VP)]),
    "nexus_gpu_stack_run": (_I32, [_VP, _VP, _VP]),
    "nexus_gpu_stack_destroy": (_I32, [_VP]),
    "nexus_gpu_stack_create_tokens": (_I32, [_U32, _VP, _U32, ctypes.c_uint64, _U32, ctypes.POINTER(_VP)]),
    "nexus_gpu_stack_create_ex": (_I32, [_U32, _VP, _U32, ctypes.c_uint64, _U32, _U32, ctypes.POINTER(_VP)]),
    "nexus_gpu_stack_create_sharded": (_I32, [_U32, _VP, _U32, ctypes.c_uint64, _U32, _U32, ctypes.POINTER(_VP)]),
    "nexus_gpu_stack_export": (_I32, [_VP, _VP, ctypes.POINTER(ctypes.c_uint64)]),
    "nexus_gpu_stack_connect": (_I32, [_VP, _VP, ctypes.c_uint64]),
    "nexus_gpu_stack_output": (_I32, [_VP, _U32, ctypes.POINTER(_VP)]),
    "nexus_gpu_stack_connect_local": (_I32, [_VP, _U32]),
    "nexus_gpu_stack_set_wait_limit": (_I32, [_VP, ctypes.c_uint64]),
    "nexus_gpu_stack_wait": (_I32, [_VP, _VP]),
    "nexus_gpu_dequantize": (_I32, [_VP, _U32, _VP, _SZ, _VP]),
    "nexus_gpu_last_error": (ctypes.c_char_p, []),
    "nexus_gpu_device_status": (_I32, [ctypes.POINTER(ctypes.c_uint32)]),
    "nexus_gpu_device_info": (_I32, [ctypes.c_char_p, _SZ, ctypes.POINTER(ctypes.c_int),
                                     ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "nexus_gpu_version": (ctypes.c_char_p, []),
    "nexus_gpu_gguf_open": (_I32, [ctypes.c_char_p, ctypes.POINTER(_VP)]),
    "nexus_gpu_gguf_close": (_I32, [_VP]),
    "nexus_gpu_gguf_model": (_I32, [_VP, _VP]),
    "nexus_gpu_gguf_tensor": (_I32, [_VP, ctypes.c_uint64, _VP]),
    "nexus_gpu_gguf_find": (_I32, [_VP, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]),
    "nexus_gpu_gguf_upload_size": (ctypes.c_uint64, [_VP, _VP, ctypes.c_uint64]),
    "nexus_gpu_gguf_upload": (_I32, [_VP, _VP, ctypes.c_uint64, _VP, ctypes.c_uint64, _VP, _VP]),
}

class StackTask(ctypes.Structure):
    """NexusGpuStackTask (include/nexus_gpu.h)."""
    _fields_ = [("W", _VP), ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64), ("y", _VP),
                ("x_source", ctypes.c_int32), ("after", ctypes.c_int32)]


class StackTaskEx(ctypes.Structure):
    """NexusGpuStackTaskEx (include/nexus_gpu.h): a stack task with fusions."""
    _fields_ = [("W", _VP), ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64), ("y", _VP),
                ("x_source", ctypes.c_int32), ("after", ctypes.c_int32), ("x_source2", ctypes.c_int32),
                ("residual_source", ctypes.c_int32), ("norm_weight", _VP), ("norm_eps", ctypes.c_float),
                ("W_up", _VP)]


class GgufModel(ctypes.Structure):
    """NexusGpuGgufModel (include/nexus_gpu.h)."""
    _fields_ = [("architecture", ctypes.c_char * 64), ("version", ctypes.c_uint32), ("alignment", ctypes.c_uint32),
                ("tensor_count", ctypes.c_uint64), ("skipped", ctypes.c_uint64), ("data_offset", ctypes.c_uint64),
                ("vocab_size", ctypes.c_uint32), ("hidden_size", ctypes.c_uint32),
                ("intermediate_size", ctypes.c_uint32), ("num_hidden_layers", ctypes.c_uint32),
                ("num_attention_heads", ctypes.c_uint32), ("num_key_value_heads", ctypes.c_uint32),
                ("max_position_embeddings", ctypes.c_uint32), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("is_moe", ctypes.c_uint32), ("num_experts", ctypes.c_uint32),
                ("num_experts_per_tok", ctypes.c_uint32)]


class GgufTensor(ctypes.Structure):
    """NexusGpuGgufTensor (include/nexus_gpu.h)."""
    _fields_ = [("name", ctypes.c_char * 128), ("ggml_type", ctypes.c_uint32), ("dtype", ctypes.c_int32),
                ("served", ctypes.c_uint32), ("n_dims", ctypes.c_uint32), ("dims", ctypes.c_uint64 * 4),
                ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64), ("file_offset", ctypes.c_uint64),
                ("bytes", ctypes.c_uint64)]


_lib = None


def header_symbols(path: str = HEADER) -> list[str]:
    """Every function the public header declares (NEXUS_GPU_API ... name(...))."""
    text = open(path).read()
    return re.findall(r"NEXUS_GPU_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class NexusGpuError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"status {status}: {message}")
        self.status = status


def check(status: int) -> None:
    if status != 0:
        raise NexusGpuError(status, lib().nexus_gpu_last_error().decode(errors="replace"))
