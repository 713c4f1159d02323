"""A bounded wait that runs out: failure detection of the GEMV stack.

Rank 1 of a two-rank sharded stack is created and connected but never runs --
a rank that left between steps.  Both ranks live in this process on one GPU
(nexus_gpu_stack_connect_local), and only rank 0's kernel is launched, so no
two kernels wait on each other.  Rank 0's second task needs rows that only
rank 1 computes; its wait must give up after the stack's wait limit (set to
50 ms here), report NEXUS_GPU_ERROR_TIMEOUT (-103, the reference's status
convention, include/nexus_common.hpp:329-340) through nexus_gpu_stack_wait,
set the timeout bit of nexus_gpu_device_status, and leave the stack poisoned
(its next run fails the same way, at once).  A fresh stack then runs clean.
No fault, trap or endless loop is involved: every wait is bounded.
"""
import ctypes
import time

import pytest

import oracle
from nexusllm_b200 import _native, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

Q4_0, H = 7, 1024
TIMEOUT = -103


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


def _rank_stack(L, Ws, rank):
    r0, r1 = H * rank // 2, H * (rank + 1) // 2
    row_bytes = H // 32 * 18
    T = _native.StackTaskEx
    tasks = (T * 2)(T(Ws[0][r0 * row_bytes:r1 * row_bytes].data_ptr(), H, H, None, -1, -1, -1, -2, None, 0.0, None),
                    T(Ws[1][r0 * row_bytes:r1 * row_bytes].data_ptr(), H, H, None, 0, -1, -1, -2, None, 0.0, None))
    h = ctypes.c_void_p()
    assert L.nexus_gpu_stack_create_ex(Q4_0, tasks, 2, H, 2, rank, ctypes.byref(h)) == 0, L.nexus_gpu_last_error()
    return h


def test_wait_for_a_rank_that_never_runs_expires(L):
    Ws = [synth.blocks_torch(Q4_0, H, H, 31 + i) for i in range(2)]
    h0, h1 = _rank_stack(L, Ws, 0), _rank_stack(L, Ws, 1)
    x = torch.randn(H, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    bits = ctypes.c_uint32(0)
    try:
        assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0 and bits.value == 0
        pair = (ctypes.c_void_p * 2)(h0.value, h1.value)
        assert L.nexus_gpu_stack_connect_local(pair, 2) == 0, L.nexus_gpu_last_error()
        assert L.nexus_gpu_stack_connect_local(pair, 2) == -9  # connected once only
        assert L.nexus_gpu_stack_set_wait_limit(h0, 50_000_000) == 0
        t0 = time.perf_counter()
        assert L.nexus_gpu_stack_run(h0, x.data_ptr(), st) == 0
        rc = L.nexus_gpu_stack_wait(h0, st)
        took = time.perf_counter() - t0
        assert rc == TIMEOUT, (rc, L.nexus_gpu_last_error())
        assert b"expired" in L.nexus_gpu_last_error()
        assert took < 1.5, took
        assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0
        assert bits.value & 1, bits.value
        # poisoned: the next run fails too, without waiting out the limit again
        t0 = time.perf_counter()
        assert L.nexus_gpu_stack_run(h0, x.data_ptr(), st) == 0
        assert L.nexus_gpu_stack_wait(h0, st) == TIMEOUT
        assert time.perf_counter() - t0 < 1.0
        L.nexus_gpu_device_status(ctypes.byref(bits))
    finally:
        L.nexus_gpu_stack_destroy(h0)
        L.nexus_gpu_stack_destroy(h1)
    # a fresh (unsharded) stack runs clean afterwards, and matches the oracle
    y = [torch.empty(H, device="cuda") for _ in range(2)]
    T = _native.StackTask
    tasks = (T * 2)(T(Ws[0].data_ptr(), H, H, y[0].data_ptr(), -1, -1), T(Ws[1].data_ptr(), H, H, y[1].data_ptr(), 0, -1))
    h = ctypes.c_void_p()
    assert L.nexus_gpu_stack_create(Q4_0, tasks, 2, H, ctypes.byref(h)) == 0
    try:
        assert L.nexus_gpu_stack_run(h, x.data_ptr(), st) == 0
        assert L.nexus_gpu_stack_wait(h, st) == 0
        assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0 and bits.value == 0
        port = oracle.port()
        want = port.gemv(Q4_0, Ws[0].cpu().numpy(), x.cpu().numpy(), H, H)
        assert oracle.l2_rel(y[0].cpu().numpy(), want) <= 1e-3
    finally:
        L.nexus_gpu_stack_destroy(h)


def test_connect_local_checks_its_ranks(L):
    Ws = [synth.blocks_torch(Q4_0, H, H, 41 + i) for i in range(2)]
    h0, h1 = _rank_stack(L, Ws, 0), _rank_stack(L, Ws, 1)
    try:
        swapped = (ctypes.c_void_p * 2)(h1.value, h0.value)
        assert L.nexus_gpu_stack_connect_local(swapped, 2) == -9  # rank order
        one = (ctypes.c_void_p * 1)(h0.value)
        assert L.nexus_gpu_stack_connect_local(one, 1) == -9
        assert L.nexus_gpu_stack_set_wait_limit(None, 1) == -9
    finally:
        L.nexus_gpu_stack_destroy(h0)
        L.nexus_gpu_stack_destroy(h1)
