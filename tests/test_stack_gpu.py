"""GPU tests of GEMV stacks (nexus_gpu_stack_*): a decode step's GEMVs in one
persistent cooperative launch.

The stack must give, task by task, exactly the bits of the same GEMVs run one
at a time through nexus_gpu_gemv (same plan, same arithmetic) -- given the
input the stack hands a dependent task: its source's output with the lowest
mantissa bit cleared (the stack carries each run's parity there) -- and stay
within the 1e-3 L2-relative GEMV tolerance of the C oracle.
"""
import ctypes

import numpy as np
import pytest

import oracle
from nexusllm_b200 import _native, synth
from nexusllm_b200.formats import weight_bytes

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-3


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


def layer_tasks(hidden, kv, ffn, layers, head_rows):
    """(name, rows, cols, x_source, after) of a decode-step stack."""
    out = []
    last_down = -1
    for l in range(layers):
        base = len(out)
        out += [("q", hidden, hidden, -1, last_down), ("k", kv, hidden, -1, last_down),
                ("v", kv, hidden, -1, last_down), ("o", hidden, hidden, base + 0, -1),
                ("gate", ffn, hidden, base + 3, -1), ("up", ffn, hidden, base + 3, -1),
                ("down", hidden, ffn, base + 4, -1)]
        last_down = base + 6
    out.append(("head", head_rows, hidden, -1, last_down))
    return out


def build(L, dt, spec, seed):
    Ws, ys, arr = [], [], (_native.StackTask * len(spec))()
    for i, (name, rows, cols, src, after) in enumerate(spec):
        W = synth.blocks_torch(dt, rows, cols, seed + i)
        y = torch.full((rows,), float("nan"), device="cuda")
        Ws.append(W)
        ys.append(y)
        arr[i] = _native.StackTask(W.data_ptr(), rows, cols, y.data_ptr(), src, after)
    h = ctypes.c_void_p()
    rc = L.nexus_gpu_stack_create(dt, arr, len(spec), spec[0][2], ctypes.byref(h))
    assert rc == 0, L.nexus_gpu_last_error()
    return h, Ws, ys


def stack_input(y):
    """A task's output as a dependent task of the stack consumes it: the
    lowest mantissa bit cleared."""
    return (y.view(torch.int32) & ~1).view(torch.float32)


def chain_single(L, dt, spec, Ws, x):
    """The same GEMVs one call at a time through nexus_gpu_gemv."""
    outs = []
    st = torch.cuda.current_stream().cuda_stream
    for i, (name, rows, cols, src, after) in enumerate(spec):
        xi = x if src < 0 else stack_input(outs[src])
        y = torch.empty(rows, device="cuda")
        assert L.nexus_gpu_gemv(Ws[i].data_ptr(), dt, xi.data_ptr(), 0, y.data_ptr(), 1, rows, cols, st) == 0
        outs.append(y)
    return outs


@pytest.mark.parametrize("dt,hidden,kv,ffn", [(7, 2048, 512, 5632), (9, 2048, 512, 5632),
                                              (11, 2048, 512, 5632), (12, 2048, 512, 5632),
                                              (7, 4096, 1024, 14336)])
def test_stack_equals_single_gemvs_and_oracle(L, port, dt, hidden, kv, ffn):
    spec = layer_tasks(hidden, kv, ffn, layers=2, head_rows=3000)
    h, Ws, ys = build(L, dt, spec, 700 + dt)
    try:
        x = torch.from_numpy(synth.activations_numpy(1, hidden, 701)[0]).cuda()
        st = torch.cuda.current_stream().cuda_stream
        assert L.nexus_gpu_stack_run(h, x.data_ptr(), st) == 0, L.nexus_gpu_last_error()
        ref = chain_single(L, dt, spec, Ws, x)
        torch.cuda.synchronize()
        for i, (name, *_rest) in enumerate(spec):
            assert torch.equal(ys[i], ref[i]), (i, name)
        # oracle on a few tasks, each with the input the stack gave it
        for i in (0, 3, 6, 13, len(spec) - 1):
            name, rows, cols, src, _ = spec[i]
            xi = (x if src < 0 else stack_input(ys[src])).cpu().numpy()
            Wh = Ws[i].cpu().numpy()
            want = port.gemv(dt, Wh, xi, rows, cols)
            assert oracle.l2_rel(ys[i].cpu().numpy(), want) <= TOL, (i, name)
        # run again with another input: counters reset, no stale state
        x2 = torch.from_numpy(synth.activations_numpy(1, hidden, 702)[0]).cuda()
        assert L.nexus_gpu_stack_run(h, x2.data_ptr(), st) == 0
        ref2 = chain_single(L, dt, spec, Ws, x2)
        torch.cuda.synchronize()
        for i in range(len(spec)):
            assert torch.equal(ys[i], ref2[i]), i
    finally:
        L.nexus_gpu_stack_destroy(h)


def test_stack_in_a_cuda_graph(L):
    dt = 7
    spec = layer_tasks(2048, 512, 5632, layers=3, head_rows=4096)
    h, Ws, ys = build(L, dt, spec, 900)
    try:
        x = torch.from_numpy(synth.activations_numpy(1, 2048, 901)[0]).cuda()
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            assert L.nexus_gpu_stack_run(h, x.data_ptr(), s.cuda_stream) == 0  # warm (uncaptured)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                assert L.nexus_gpu_stack_run(h, x.data_ptr(), s.cuda_stream) == 0
        first = [y.clone() for y in ys]
        for y in ys:
            y.fill_(float("nan"))
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        for a, b in zip(first, ys):
            assert torch.equal(a, b)
        del g
    finally:
        L.nexus_gpu_stack_destroy(h)


def test_stack_rejects_bad_task_lists(L):
    W = torch.zeros(weight_bytes(7, 64, 64), dtype=torch.uint8, device="cuda")
    y = torch.zeros(64, device="cuda")
    h = ctypes.c_void_p()

    def make(*tasks):
        arr = (_native.StackTask * len(tasks))(*tasks)
        return L.nexus_gpu_stack_create(7, arr, len(tasks), 64, ctypes.byref(h))

    T = _native.StackTask
    assert make(T(W.data_ptr(), 64, 64, y.data_ptr(), 0, -1)) == -5      # x from itself
    assert make(T(W.data_ptr(), 64, 96, y.data_ptr(), -1, -1)) == -5     # input length mismatch
    assert make(T(W.data_ptr(), 64, 64, y.data_ptr(), -1, 3)) == -9      # `after` not earlier
    assert make(T(W.data_ptr() + 2, 64, 64, y.data_ptr(), -1, -1)) == -9  # misaligned W
    arr = (_native.StackTask * 1)(T(W.data_ptr(), 64, 64, y.data_ptr(), -1, -1))
    assert L.nexus_gpu_stack_create(1, arr, 1, 64, ctypes.byref(h)) == -3  # FP16 not a stack format
    bits = ctypes.c_uint32(99)
    assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0 and bits.value == 0
