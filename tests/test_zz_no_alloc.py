"""nexus_gpu_gemv_noalloc: the GEMV entry point that allocates nothing.

Some callers cannot call cudaMalloc -- engines that hand all device memory to
weights and KV cache at start-up, code that must not trigger the device-wide
synchronisation an allocation can cause, callers with no workspace of their
own.  For them the library keeps the quantized activations in a fixed 1 MiB
array of its own instead of a workspace.  These tests call the entry point
through the C ABI and check it against the ordinary entry point
(nexus_gpu_gemv) and against the CPU oracle within the GEMV tolerance used
everywhere (1e-3 L2-relative), on two calls in a row with different
activations, so that a stale scratch from the first call would show up in
the second.  A further test checks that the device's free memory does not
move across calls.  The file is named to be collected last, and it needs no
state from other tests.
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
    Wh = synth.blocks_numpy(dt, rows, cols, 500 + dt)
    W = torch.from_numpy(Wh.view(np.uint8)).cuda()
    port = oracle.port()
    for call, M in enumerate((1, 3)):
        Xh = synth.activations_numpy(M, cols, 600 + 10 * dt + call)
        X = torch.from_numpy(Xh).cuda()
        rc_a, y_a = _call(L.nexus_gpu_gemv, W, dt, X, rows, cols)
        rc_b, y_b = _call(L.nexus_gpu_gemv_noalloc, W, dt, X, rows, cols)
        torch.cuda.synchronize()
        assert rc_a == 0 and rc_b == 0, L.nexus_gpu_last_error()
        assert torch.isfinite(y_b).all()
        got = y_b.cpu().numpy()
        assert oracle.l2_rel(got, y_a.cpu().numpy()) <= TOL, (dt, call)
        want = port.gemv_batched(dt, Wh, Xh, rows, cols)
        assert oracle.l2_rel(got.reshape(-1), want.reshape(-1)) <= TOL, (dt, call)


def test_noalloc_calls_leave_device_memory_unchanged(L):
    """After the first call (which loads the module and resolves the scratch
    address), calls of several shapes change the device's free memory by
    nothing: no cudaMalloc, no allocating library routine."""
    rows, cols = 512, 4096
    W = synth.blocks_torch(7, rows, cols, 77)
    Xs = [torch.randn(M, cols, device="cuda") for M in (1, 2, 3)]
    ys = [torch.empty(M, rows, device="cuda") for M in (1, 2, 3)]
    st = torch.cuda.current_stream().cuda_stream
    assert L.nexus_gpu_gemv_noalloc(W.data_ptr(), 7, Xs[0].data_ptr(), 0, ys[0].data_ptr(), 1, rows, cols, st) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        for X, y in zip(Xs, ys):
            rc = L.nexus_gpu_gemv_noalloc(W.data_ptr(), 7, X.data_ptr(), 0, y.data_ptr(), X.shape[0], rows, cols, st)
            assert rc == 0, L.nexus_gpu_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


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
