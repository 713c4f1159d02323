"""GPU tests of multi-token GEMV stacks (nexus_gpu_stack_create_tokens): a
decode step's GEMVs for 2-4 requests in one launch, every weight read once
(5-15 requests: several such stacks, one after another, in one run).

Per token, every task's output must stay within the 1e-3 L2-relative GEMV
tolerance of the C oracle (fed the input the stack gave that task) and agree
closely with the single-token stack run on that token alone (same integer
arithmetic, another fixed summation order).  Runs repeat bit for bit, also
as CUDA-graph replays, and a second run with new inputs leaves no stale rows.
"""
import ctypes

import pytest

import oracle
from nexusllm_b200 import _native, synth
from tests.test_stack_gpu import layer_tasks, stack_input

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-3


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


def build(L, dt, spec, seed, tokens):
    """The stack for `tokens` tokens and, over the same weights, the
    single-token stack (tokens = 1 through nexus_gpu_stack_create)."""
    Ws, ys, ys1 = [], [], []
    arr = (_native.StackTask * len(spec))()
    arr1 = (_native.StackTask * len(spec))()
    for i, (name, rows, cols, src, after) in enumerate(spec):
        W = synth.blocks_torch(dt, rows, cols, seed + i)
        y = torch.full((tokens, rows), float("nan"), device="cuda")
        y1 = torch.full((rows,), float("nan"), device="cuda")
        Ws.append(W)
        ys.append(y)
        ys1.append(y1)
        arr[i] = _native.StackTask(W.data_ptr(), rows, cols, y.data_ptr(), src, after)
        arr1[i] = _native.StackTask(W.data_ptr(), rows, cols, y1.data_ptr(), src, after)
    h, h1 = ctypes.c_void_p(), ctypes.c_void_p()
    rc = L.nexus_gpu_stack_create_tokens(dt, arr, len(spec), spec[0][2], tokens, ctypes.byref(h))
    assert rc == 0, L.nexus_gpu_last_error()
    rc = L.nexus_gpu_stack_create(dt, arr1, len(spec), spec[0][2], ctypes.byref(h1))
    assert rc == 0, L.nexus_gpu_last_error()
    return h, h1, Ws, ys, ys1


def run(L, h, x):
    st = torch.cuda.current_stream().cuda_stream
    assert L.nexus_gpu_stack_run(h, x.data_ptr(), st) == 0, L.nexus_gpu_last_error()


def status_clean(L):
    s = ctypes.c_uint32()
    assert L.nexus_gpu_device_status(ctypes.byref(s)) == 0 and s.value == 0, s.value


@pytest.mark.parametrize("dt,tokens,hidden,kv,ffn", [(7, 4, 4096, 1024, 14336), (7, 2, 2048, 512, 5632),
                                                     (7, 3, 2048, 512, 5632), (9, 4, 2048, 512, 5632),
                                                     (9, 2, 4096, 1024, 14336), (12, 4, 2048, 512, 5632),
                                                     (11, 2, 2048, 512, 5632), (7, 6, 2048, 512, 5632),
                                                     (7, 11, 2048, 512, 5632), (9, 15, 2048, 512, 5632)])
def test_tokens_stack_matches_oracle_and_single_token_stack(L, port, dt, tokens, hidden, kv, ffn):
    spec = layer_tasks(hidden, kv, ffn, layers=2, head_rows=3000)
    h, h1, Ws, ys, ys1 = build(L, dt, spec, 900 + dt, tokens)
    try:
        X = torch.from_numpy(synth.activations_numpy(tokens, hidden, 901 + tokens)).cuda().contiguous()
        run(L, h, X)
        torch.cuda.synchronize()
        status_clean(L)
        for i in range(len(spec)):
            assert torch.isfinite(ys[i]).all(), (i, spec[i][0])
        # oracle, per token, on a few tasks, each fed the input the stack gave it
        for t in range(tokens):
            for i in (0, 3, 6, 13, len(spec) - 1):
                name, rows, cols, src, _ = spec[i]
                xi = (X[t] if src < 0 else stack_input(ys[src][t])).cpu().numpy()
                want = port.gemv(dt, Ws[i].cpu().numpy(), xi, rows, cols)
                assert oracle.l2_rel(ys[i][t].cpu().numpy(), want) <= TOL, (t, i, name)
        # the single-token stack on each token: the whole chain stays close
        for t in range(tokens):
            run(L, h1, X[t].contiguous())
            torch.cuda.synchronize()
            for i, (name, *_r) in enumerate(spec):
                err = oracle.l2_rel(ys[i][t].cpu().numpy(), ys1[i].cpu().numpy())
                assert err <= 1e-4, (t, i, name, err)
        # a second run with other inputs: no stale rows; runs repeat bit for bit
        first = [y.clone() for y in ys]
        X2 = torch.from_numpy(synth.activations_numpy(tokens, hidden, 977)).cuda().contiguous()
        run(L, h, X2)
        run(L, h, X)
        torch.cuda.synchronize()
        for i in range(len(spec)):
            assert torch.equal(ys[i], first[i]), i
        status_clean(L)
    finally:
        L.nexus_gpu_stack_destroy(h)
        L.nexus_gpu_stack_destroy(h1)


def test_tokens_stack_graph_replays_bit_for_bit(L):
    spec = layer_tasks(2048, 512, 5632, layers=3, head_rows=1000)
    h, h1, Ws, ys, ys1 = build(L, 7, spec, 950, 4)
    try:
        X = torch.from_numpy(synth.activations_numpy(4, 2048, 951)).cuda().contiguous()
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
        status_clean(L)
        del g
    finally:
        L.nexus_gpu_stack_destroy(h)
        L.nexus_gpu_stack_destroy(h1)


def test_tokens_stack_refuses_bad_arguments(L):
    W = synth.blocks_torch(7, 64, 1024, 5)
    y = torch.empty(8 * 64, device="cuda")
    arr = (_native.StackTask * 1)(_native.StackTask(W.data_ptr(), 64, 1024, y.data_ptr(), -1, -1))
    h = ctypes.c_void_p()
    for tokens in (0, 65, 1 << 31):
        assert L.nexus_gpu_stack_create_tokens(7, arr, 1, 1024, tokens, ctypes.byref(h)) != 0
        assert b"tokens" in L.nexus_gpu_last_error()
    # tokens = 1 is the plain stack
    assert L.nexus_gpu_stack_create_tokens(7, arr, 1, 1024, 1, ctypes.byref(h)) == 0
    L.nexus_gpu_stack_destroy(h)
