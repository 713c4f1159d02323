"""The C-ABI library loads, exports every symbol include/nexus_gpu.h declares,
and its argument validation works without a GPU (no compute calls here)."""
import ctypes

import pytest

from nexusllm_b200 import _native
from nexusllm_b200.formats import DataType, weight_bytes


@pytest.fixture(scope="module")
def L():
    return _native.lib()


def test_exports_every_declared_symbol(L):
    names = _native.header_symbols()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    # and the Python binding declares exactly those
    assert set(names) == set(_native.SIGNATURES)


def test_weight_bytes_match_block_layouts(L):
    for dt in (DataType.FP16, DataType.GGUF_Q4_0, DataType.GGUF_Q8_0, DataType.GGUF_Q5_K, DataType.GGUF_Q6_K):
        for rows, cols in [(4096, 4096), (11008, 4096), (4096, 11008), (3, 256)]:
            assert L.nexus_gpu_weight_bytes(int(dt), rows, cols) == weight_bytes(dt, rows, cols)
    assert L.nexus_gpu_weight_bytes(7, 4096, 4096) == 9_437_184  # config 1
    assert L.nexus_gpu_weight_bytes(12, 11008, 4096) == 36_986_880
    assert L.nexus_gpu_weight_bytes(12, 4096, 11008) == 4096 * 9030  # unaligned Q6_K rows
    assert L.nexus_gpu_weight_bytes(7, 1, 33) == 0
    assert L.nexus_gpu_weight_bytes(0, 1, 32) == 0


def test_workspace_size(L):
    assert L.nexus_gpu_gemv_workspace_size(1, 1, 4096, 4096) == 0  # FP16 needs none
    assert L.nexus_gpu_gemv_workspace_size(7, 1, 4096, 4096) == 128 * 64 + 128 * 16
    assert L.nexus_gpu_gemv_workspace_size(7, 4, 10, 4096) == 4 * 128 * 64 + 4 * 128 * 16


def test_argument_errors_need_no_device(L):
    x = (ctypes.c_float * 64)()
    y = (ctypes.c_float * 64)()
    w = (ctypes.c_uint8 * 4096)()
    # W == NULL is the reference's no-op (include/transformer_ops.hpp:158)
    assert L.nexus_gpu_gemv_dispatch(None, 7, x, y, 4, 64) == 0
    # FP32 / unknown weight types are not this library's
    assert L.nexus_gpu_gemv_dispatch(w, 0, x, y, 4, 64) == -3
    assert L.nexus_gpu_gemv_dispatch(w, 8, x, y, 4, 64) == -3
    # cols must hold whole blocks
    assert L.nexus_gpu_gemv_dispatch(w, 7, x, y, 4, 33) == -5
    assert L.nexus_gpu_gemv_dispatch(w, 11, x, y, 1, 128) == -5
    assert b"multiple" in L.nexus_gpu_last_error()
    # activation rows beyond the x quantizer's grid are refused before any size is computed
    huge = 1 << 40
    assert L.nexus_gpu_gemv_noalloc(w, 7, x, 0, y, huge, 4, 64, None) == -9
    assert b"activation rows" in L.nexus_gpu_last_error()
    assert L.nexus_gpu_gemv_ws(w, 7, x, 0, y, huge, 4, 64, None, 0, None) == -9
    assert L.nexus_gpu_gemv_workspace_size(7, huge, 4, 64) == 0


def test_device_api_rejects_null_or_reports_no_device(L):
    # valid shape, null device pointers: INVALID_ARGUMENT on a GPU box,
    # NO_DEVICE where there is no GPU -- never a launch
    rc = L.nexus_gpu_gemv(None, 7, None, 0, None, 1, 16, 64, None)
    assert rc in (-9, -101), rc


def test_stack_token_counts_checked_before_the_device(L):
    # 0 and > 64 tokens are refused as arguments on any machine; 5..15 tokens
    # (split into multi-token stacks of 2..4) get as far as the device: NO_DEVICE
    # without a GPU, never an argument error
    T = _native.StackTask
    arr = (T * 1)(T(16, 64, 64, None, -1, -1))
    h = ctypes.c_void_p()
    for tokens in (0, 65):
        assert L.nexus_gpu_stack_create_tokens(7, arr, 1, 64, tokens, ctypes.byref(h)) == -9
        assert b"tokens" in L.nexus_gpu_last_error()
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except ImportError:
        has_gpu = False
    if not has_gpu:
        for tokens in (5, 8, 15):
            assert L.nexus_gpu_stack_create_tokens(7, arr, 1, 64, tokens, ctypes.byref(h)) == -101
            assert h.value is None


def test_version(L):
    assert L.nexus_gpu_version().startswith(b"nexus_gpu")
