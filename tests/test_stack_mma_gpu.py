"""GPU tests of the tensor-core GEMV stack (nexus_gpu_stack_create_tokens with
16..64 tokens): a decode step's Q4_0 GEMVs for many requests in one
persistent tcgen05 launch.

Every task of every token must stay within the 1e-3 L2-relative GEMV
tolerance of the C oracle, fed the input the stack gave that task, and match
the single tcgen05 GEMM (nexus_gpu_gemv with M rows) on that input within
SAME_TOL: the same x conversion rule and products, but the stack splits a
hop group's concatenated tiles (q, k and v together), so its stream-K
boundaries -- the grouping of the fp32 chunk sums -- differ from the single
GEMM's.  Runs repeat bit for
bit, also as CUDA-graph replays, with no stale rows after a run with other
inputs.  Shapes outside the path are refused with an error.
"""
import ctypes

import numpy as np
import pytest

import oracle
from nexusllm_b200 import _native, synth
from tests.test_stack_gpu import layer_tasks

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-3
SAME_TOL = 1e-5  # fp32 reassociation of the chunk sums only


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


def build(L, spec, seed, tokens):
    Ws, ys = [], []
    arr = (_native.StackTask * len(spec))()
    for i, (name, rows, cols, src, after) in enumerate(spec):
        W = synth.blocks_torch(7, rows, cols, seed + i)
        y = torch.full((tokens, rows), float("nan"), device="cuda")
        Ws.append(W)
        ys.append(y)
        arr[i] = _native.StackTask(W.data_ptr(), rows, cols, y.data_ptr(), src, after)
    h = ctypes.c_void_p()
    rc = L.nexus_gpu_stack_create_tokens(7, arr, len(spec), spec[0][2], tokens, ctypes.byref(h))
    assert rc == 0, L.nexus_gpu_last_error()
    return h, Ws, ys


def run(L, h, x):
    st = torch.cuda.current_stream().cuda_stream
    assert L.nexus_gpu_stack_run(h, x.data_ptr(), st) == 0, L.nexus_gpu_last_error()


def status_clean(L, h):
    st = torch.cuda.current_stream().cuda_stream
    assert L.nexus_gpu_stack_wait(h, st) == 0, L.nexus_gpu_last_error()
    s = ctypes.c_uint32()
    assert L.nexus_gpu_device_status(ctypes.byref(s)) == 0 and s.value == 0, s.value


def single_gemm(L, W, x, rows, cols):
    M = x.shape[0]
    y = torch.empty(M, rows, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.nexus_gpu_gemv(W.data_ptr(), 7, x.data_ptr(), 0, y.data_ptr(), M, rows, cols, st) == 0
    return y


@pytest.mark.parametrize("tokens,hidden,kv,ffn,head", [(16, 2048, 512, 5632, 3000), (64, 2048, 512, 5632, 3000),
                                                       (40, 4096, 1024, 14336, 1000), (17, 1024, 256, 2816, 200)])
def test_mma_stack_matches_oracle_and_single_gemm(L, port, tokens, hidden, kv, ffn, head):
    spec = layer_tasks(hidden, kv, ffn, layers=2, head_rows=head)
    h, Ws, ys = build(L, spec, 300 + tokens, tokens)
    try:
        X = torch.from_numpy(synth.activations_numpy(tokens, hidden, 301 + tokens)).cuda().contiguous()
        run(L, h, X)
        torch.cuda.synchronize()
        status_clean(L, h)
        for i, (name, rows, cols, src, _) in enumerate(spec):
            assert torch.isfinite(ys[i]).all(), (i, name)
            xin = X if src < 0 else ys[src]
            ref = single_gemm(L, Ws[i], xin.contiguous(), rows, cols)
            torch.cuda.synchronize()
            err = oracle.l2_rel(ys[i].cpu().numpy().reshape(-1), ref.cpu().numpy().reshape(-1))
            assert err <= SAME_TOL, (i, name, err)
        Wh = {i: Ws[i].cpu().numpy() for i in (0, 3, 6, len(spec) - 1)}
        for t in (0, tokens // 2, tokens - 1):
            for i in Wh:
                name, rows, cols, src, _ = spec[i]
                xi = (X[t] if src < 0 else ys[src][t]).cpu().numpy()
                want = port.gemv(7, Wh[i], xi, rows, cols)
                assert oracle.l2_rel(ys[i][t].cpu().numpy(), want) <= TOL, (t, i, name)
        first = [y.clone() for y in ys]
        X2 = torch.from_numpy(synth.activations_numpy(tokens, hidden, 977)).cuda().contiguous()
        run(L, h, X2)
        run(L, h, X)
        torch.cuda.synchronize()
        for i in range(len(spec)):
            assert torch.equal(ys[i], first[i]), i
        status_clean(L, h)
    finally:
        L.nexus_gpu_stack_destroy(h)


def test_mma_stack_graph_replays_bit_for_bit(L):
    spec = layer_tasks(2048, 512, 5632, layers=3, head_rows=1000)
    h, Ws, ys = build(L, spec, 350, 32)
    try:
        X = torch.from_numpy(synth.activations_numpy(32, 2048, 351)).cuda().contiguous()
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            run(L, h, X)
            torch.cuda.synchronize()
            want = [y.clone() for y in ys]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                run(L, h, X)
            for _ in range(5):
                g.replay()
        torch.cuda.synchronize()
        for i in range(len(spec)):
            assert torch.equal(ys[i], want[i]), i
        status_clean(L, h)
        del g
    finally:
        L.nexus_gpu_stack_destroy(h)


def test_mma_stack_refuses_shapes_outside_the_path(L):
    W = synth.blocks_torch(7, 256, 1024, 5)
    y = torch.empty(64 * 256, device="cuda")
    h = ctypes.c_void_p()
    arr = (_native.StackTask * 1)(_native.StackTask(W.data_ptr(), 256, 1024, y.data_ptr(), -1, -1))
    for tokens in (0, 65):
        assert L.nexus_gpu_stack_create_tokens(7, arr, 1, 1024, tokens, ctypes.byref(h)) != 0
    for tokens in (5, 15):  # below the tensor-core range: several CUDA-core stacks, not this path
        assert L.nexus_gpu_stack_create_tokens(7, arr, 1, 1024, tokens, ctypes.byref(h)) == 0, L.nexus_gpu_last_error()
        L.nexus_gpu_stack_destroy(h)
    W8 = synth.blocks_torch(9, 256, 1024, 6)
    arr8 = (_native.StackTask * 1)(_native.StackTask(W8.data_ptr(), 256, 1024, y.data_ptr(), -1, -1))
    assert L.nexus_gpu_stack_create_tokens(9, arr8, 1, 1024, 16, ctypes.byref(h)) != 0  # Q4_0 only
    Wr = synth.blocks_torch(7, 256, 1056, 7)
    arrr = (_native.StackTask * 1)(_native.StackTask(Wr.data_ptr(), 256, 1056, y.data_ptr(), -1, -1))
    assert L.nexus_gpu_stack_create_tokens(7, arrr, 1, 1056, 16, ctypes.byref(h)) != 0  # cols % 256
    assert L.nexus_gpu_stack_create_tokens(7, arr, 1, 1024, 16, ctypes.byref(h)) == 0
    L.nexus_gpu_stack_destroy(h)
