"""nexus_gpu_gemv_noalloc: the GEMV entry point that allocates nothing.

Some callers cannot call cudaMalloc -- engines that hand all device memory to
weights and KV cache at start-up, code that must not trigger the device-wide
synchronisation an allocation can cause, callers with no workspace of their
own.  For them the library keeps the quantized activations in a fixed 1 MiB
array of its own instead of a workspace.  These tests call the entry point
through the C ABI and check it against the ordinary entry point
(nexus_gpu_gemv) within the GEMV tolerance used everywhere (1e-3
L2-relative), on two calls in a row with different activations, so that a
stale scratch from the first call would show up in the second.  The file is
named to be collected last, and it needs no state from other tests.
"""
import ctypes

import numpy as np
import pytest

import oracle
from nexusllm_b200 import _native, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-3
SCRATCH_BYTES = 1 << 20


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


def _call(fn, W, dt, X, rows, cols):
    M = X.shape[0]
    y = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = fn(W.data_ptr(), dt, X.data_ptr(), 0, y.data_ptr(), M, rows, cols, st)
    return rc, y


@pytest.mark.parametrize("dt", [7, 9, 11, 12, 1], ids=["q4_0", "q8_0", "q5_k", "q6_k", "fp16"])
def test_noalloc_matches_the_allocating_entry_point_twice(L, dt):
    rows, cols = 1000, 4096
    W = synth.blocks_torch(dt, rows, cols, 500 + dt)
    for call, M in enumerate((1, 3)):
        X = torch.from_numpy(synth.activations_numpy(M, cols, 600 + 10 * dt + call)).cuda()
        rc_a, y_a = _call(L.nexus_gpu_gemv, W, dt, X, rows, cols)
        rc_b, y_b = _call(L.nexus_gpu_gemv_noalloc, W, dt, X, rows, cols)
        torch.cuda.synchronize()
        assert rc_a == 0 and rc_b == 0, L.nexus_gpu_last_error()
        assert torch.isfinite(y_b).all()
        assert oracle.l2_rel(y_b.cpu().numpy(), y_a.cpu().numpy()) <= TOL, (dt, call)


def test_noalloc_rejects_shapes_beyond_its_scratch(L):
    dt, rows = 7, 4
    cols = 32 * (SCRATCH_BYTES // 80 + 32)  # one activation row needs more than 1 MiB of scratch
    W = torch.zeros(rows * (cols // 32) * 18, dtype=torch.uint8, device="cuda")
    X = torch.zeros((1, cols), dtype=torch.float32, device="cuda")
    rc, y = _call(L.nexus_gpu_gemv_noalloc, W, dt, X, rows, cols)
    torch.cuda.synchronize()
    assert rc == -102
    assert b"1048576-byte" in L.nexus_gpu_last_error()
    assert torch.isnan(y).all()  # nothing was launched


def test_noalloc_leaves_no_expired_wait(L):
    bits = ctypes.c_uint32(99)
    assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0
    assert bits.value == 0
