"""nexusllm_b200 -- B200-native (sm_100a) fused quantized GEMV for NexusLLM.

The product is the C-ABI library libnexus_gpu.so (include/nexus_gpu.h); this
package builds it, binds it with ctypes, and mirrors the reference's
``QuantizationKernel`` and ``INexusComputeBackend`` GEMV interfaces on top.
"""
from .formats import BLOCK, DataType, GEMV_TYPES, row_bytes, weight_bytes  # noqa: F401

__version__ = "0.1.0"
