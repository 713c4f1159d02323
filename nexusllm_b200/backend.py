"""The CUDA compute device behind NexusLLM's backend interface.

``CUDABackend`` mirrors the reference's ``INexusComputeBackend`` GEMV and
memory methods (include/nexus_backend.hpp:46-62) -- the methods that the
reference's CUDA stub forwards to the CPU (src/nexus_backend.cpp:239-367) run
on the GPU here, through the C ABI (include/nexus_gpu.h).  It also exposes the
device-pointer GEMV for callers that keep weights and activations in HBM
(``gemv``), taking torch CUDA tensors; torch only provides device memory and
streams.
"""
from __future__ import annotations

import numpy as np

from . import _native
from .formats import BLOCK, DataType, check_shape, parse, weight_bytes


class CUDABackend:
    """INexusComputeBackend for DEVICE_CUDA (ComputeDeviceType value 1)."""

    type = 1

    def __init__(self):
        self._lib = _native.lib()

    # -- reference-shaped methods (host pointers) -------------------------
    def gemv_dispatch(self, W: np.ndarray | None, dt, x: np.ndarray, y: np.ndarray, rows: int, cols: int) -> None:
        """INexusComputeBackend::gemv_dispatch (include/nexus_backend.hpp:55-62).

        W is None -> no-op (include/transformer_ops.hpp:158).  Raises
        NexusGpuError with the NexusStatus code on bad arguments."""
        if W is None:
            return
        dt = parse(dt)
        rc = self._lib.nexus_gpu_gemv_dispatch(W.ctypes.data, int(dt), x.ctypes.data, y.ctypes.data, rows, cols)
        _native.check(rc)

    def synchronize(self, stream: int = 0) -> None:
        _native.check(self._lib.nexus_gpu_synchronize(stream or None))

    def allocate_device_memory(self, nbytes: int) -> int:
        return self._lib.nexus_gpu_allocate_device_memory(nbytes) or 0

    def free_device_memory(self, ptr: int) -> None:
        self._lib.nexus_gpu_free_device_memory(ptr)

    def copy_host_to_device_async(self, dst: int, src: np.ndarray, nbytes: int, stream: int = 0) -> bool:
        return self._lib.nexus_gpu_copy_host_to_device_async(dst, src.ctypes.data, nbytes, stream or None) == 0

    def copy_device_to_host_async(self, dst: np.ndarray, src: int, nbytes: int, stream: int = 0) -> bool:
        return self._lib.nexus_gpu_copy_device_to_host_async(dst.ctypes.data, src, nbytes, stream or None) == 0

    def weight_cache_invalidate(self, W: np.ndarray | None = None) -> None:
        _native.check(self._lib.nexus_gpu_weight_cache_invalidate(W.ctypes.data if W is not None else None))

    def weight_cache_bytes(self) -> int:
        return self._lib.nexus_gpu_weight_cache_bytes()

    # -- device-resident API (torch CUDA tensors) --------------------------
    def gemv(self, W, dt, x, y=None, stream=None, workspace=None):
        """y[M, rows] = x[M, cols] . W[rows, cols]^T on the GPU.

        W: flat uint8 CUDA tensor of blocks; x: float32 or bfloat16 CUDA tensor
        [M, cols] or [cols]; y: optional float32 output.  Asynchronous on
        `stream` (default: torch's current stream)."""
        import torch

        dt = parse(dt)
        squeeze = x.dim() == 1
        x2 = x.reshape(1, -1) if squeeze else x
        M, cols = x2.shape
        per, nbytes = BLOCK[dt]
        rows = W.numel() * W.element_size() // (cols // per * nbytes) if cols else 0
        check_shape(dt, rows, cols)
        if W.numel() * W.element_size() != weight_bytes(dt, rows, cols):
            raise ValueError("W size does not match rows x cols")
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        xdt = {torch.float32: 0, torch.bfloat16: 2}[x2.dtype]
        if y is None:
            y = torch.empty((M, rows), dtype=torch.float32, device=x.device)
        st = (stream if stream is not None else torch.cuda.current_stream(x.device)).cuda_stream
        if workspace is None:
            rc = self._lib.nexus_gpu_gemv(W.data_ptr(), int(dt), x2.data_ptr(), xdt, y.data_ptr(), M, rows, cols, st)
        else:
            rc = self._lib.nexus_gpu_gemv_ws(W.data_ptr(), int(dt), x2.data_ptr(), xdt, y.data_ptr(), M, rows, cols,
                                             workspace.data_ptr(), workspace.numel() * workspace.element_size(), st)
        _native.check(rc)
        return y.reshape(-1) if squeeze else y

    def dequantize(self, W, dt, count: int, out=None, stream=None):
        import torch

        dt = parse(dt)
        if out is None:
            out = torch.empty(count, dtype=torch.float32, device=W.device)
        st = (stream if stream is not None else torch.cuda.current_stream(W.device)).cuda_stream
        _native.check(self._lib.nexus_gpu_dequantize(W.data_ptr(), int(dt), out.data_ptr(), count, st))
        return out

    def workspace_size(self, dt, M: int, rows: int, cols: int) -> int:
        return self._lib.nexus_gpu_gemv_workspace_size(int(parse(dt)), M, rows, cols)
