"""GPU parity through the C++ drop-in: NexusLLM's QuantizationKernel
entry points (mangled C++ symbols, host pointers, synchronous -- as
src/forward_pass.cpp calls them through matmul_vec_dispatch) and the
INexusComputeBackend device's virtual gemv_dispatch, both against the C
oracle: GEMV within 1e-3 L2-relative, dequantization bit-exact."""
import ctypes
import os

import numpy as np
import pytest

import oracle
from nexusllm_b200 import build as nb
from nexusllm_b200 import synth

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(nb.DROPIN_OUT), reason="drop-in not built")]
torch = pytest.importorskip("torch")

TOL = 1e-3
BLOCK = {7: "9BlockQ4_0", 9: "9BlockQ8_0", 11: "9BlockQ5_K", 12: "9BlockQ6_K"}
NAME = {7: "q4_0", 9: "q8_0", 11: "q5_k", 12: "q6_k", 1: "fp16"}
_P, _SZ = ctypes.c_void_p, ctypes.c_size_t


@pytest.fixture(scope="module")
def lib():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return ctypes.CDLL(nb.DROPIN_OUT)


def _gemv_fn(lib, dt):
    w = "PKt" if dt == 1 else f"PKNS_{BLOCK[dt]}E"  # const uint16_t* / const nexus::BlockX*
    fn = getattr(lib, f"_ZN5nexus18QuantizationKernel15fused_gemv_{NAME[dt]}E{w}PKfPfmm")
    fn.restype = None
    fn.argtypes = [_P, _P, _P, _SZ, _SZ]
    return fn


@pytest.mark.parametrize("dt", [7, 9, 11, 12, 1], ids=lambda d: NAME[d])
def test_quantization_kernel_symbols_run_on_the_gpu(lib, port, dt):
    rows, cols = 700, 4096
    W = synth.blocks_numpy(dt, rows, cols, 900 + dt)
    x = synth.activations_numpy(1, cols, 901)[0]
    y = np.full(rows, np.nan, np.float32)
    _gemv_fn(lib, dt)(W.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols)
    assert oracle.l2_rel(y, port.gemv(dt, W, x, rows, cols)) <= TOL


@pytest.mark.parametrize("dt", [7, 11, 12], ids=lambda d: NAME[d])
def test_quantization_kernel_dequantizers_bit_exact(lib, port, golden, dt):
    W = np.ascontiguousarray(golden[f"deq/{dt}/W"])
    per, nbytes = {7: (32, 18), 11: (256, 176), 12: (256, 210)}[dt]
    nb_ = W.size // nbytes
    fn = getattr(lib, f"_ZN5nexus18QuantizationKernel20dequantize_gguf_{NAME[dt]}EPKNS_{BLOCK[dt]}EPfm")
    fn.restype = None
    fn.argtypes = [_P, _P, _SZ]
    out = np.zeros(nb_ * per, np.float32)
    fn(W.ctypes.data, out.ctypes.data, nb_)
    want = port.dequantize(dt, W, nb_ * per)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_backend_gemv_dispatch_runs_on_the_gpu(lib, port):
    fn = lib.nexus_dropin_backend_gemv
    fn.restype = ctypes.c_int32
    fn.argtypes = [_P, ctypes.c_uint32, _P, _P, _SZ, _SZ]
    for dt in (7, 12):
        rows, cols = 512, 11008 if dt == 12 else 4096
        W = synth.blocks_numpy(dt, rows, cols, 950 + dt)
        x = synth.activations_numpy(1, cols, 951)[0]
        y = np.full(rows, np.nan, np.float32)
        assert fn(W.ctypes.data, dt, x.ctypes.data, y.ctypes.data, rows, cols) == 0
        assert oracle.l2_rel(y, port.gemv(dt, W, x, rows, cols)) <= TOL
    name = ctypes.create_string_buffer(256)
    kind = ctypes.c_uint32(0)
    lib.nexus_dropin_backend_name(name, 256, ctypes.byref(kind))
    assert b"B200" in name.value or b"NVIDIA" in name.value, name.value
