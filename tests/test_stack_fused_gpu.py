"""GEMV stacks with the decode layer's operations fused in (nexus_gpu_stack_create_ex):
RMSNorm on a task's input, SwiGLU either from two source tasks or as the
epilogue of a gate+up pair, residual adds (src/forward_pass.cpp:504-562;
TransformerOps, include/transformer_ops.hpp).

A small two-layer decoder (attention stood in by q -> o, as in bench.py) runs
as one stack.  Every task's output is checked against the C oracle fed with
the GPU's own inputs to that task (the oracle's GEMV is bit-identical to the
reference build; RMSNorm and SwiGLU too), within the 1e-3 L2-relative GEMV
tolerance.  Runs repeat bit for bit."""
import ctypes

import numpy as np
import pytest

import oracle
from nexusllm_b200 import _native, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-3
Q4_0 = 7


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


def decoder_tasks(H, KV, F, V, layers, seed, paired=False):
    """(task dicts, norm weights) of a fused decode stack.  paired: gate and up
    as one gate+up task with the SwiGLU epilogue; else two tasks whose outputs
    the down task combines (x_source2)."""
    g = torch.Generator().manual_seed(seed)
    tasks, norms = [], {}
    prev = -1  # the stack input is layer 0's residual stream
    for l in range(layers):
        b = len(tasks)
        norms[f"attn{l}"] = (1.0 + 0.1 * torch.randn(H, generator=g)).cuda()
        norms[f"ffn{l}"] = (1.0 + 0.1 * torch.randn(H, generator=g)).cuda()
        tasks += [dict(name="q", rows=H, cols=H, src=prev, norm=f"attn{l}"),
                  dict(name="k", rows=KV, cols=H, src=prev, norm=f"attn{l}"),
                  dict(name="v", rows=KV, cols=H, src=prev, norm=f"attn{l}"),
                  dict(name="o", rows=H, cols=H, src=b + 0, res=prev)]
        if paired:
            tasks += [dict(name="gate_up", rows=F, cols=H, src=b + 3, norm=f"ffn{l}", pair=True),
                      dict(name="down", rows=H, cols=F, src=b + 4, res=b + 3)]
        else:
            tasks += [dict(name="gate", rows=F, cols=H, src=b + 3, norm=f"ffn{l}"),
                      dict(name="up", rows=F, cols=H, src=b + 3, norm=f"ffn{l}"),
                      dict(name="down", rows=H, cols=F, src=b + 4, src2=b + 5, res=b + 3)]
        prev = len(tasks) - 1
    norms["out"] = (1.0 + 0.1 * torch.randn(H, generator=g)).cuda()
    tasks.append(dict(name="head", rows=V, cols=H, src=prev, norm="out"))
    for i, t in enumerate(tasks):
        t["W"] = synth.blocks_torch(Q4_0, t["rows"], t["cols"], seed + 31 * i)
        if t.get("pair"):
            t["W_up"] = synth.blocks_torch(Q4_0, t["rows"], t["cols"], seed + 31 * i + 7)
        t["y"] = torch.empty(t["rows"], device="cuda")
    return tasks, norms


def make_stack(L, tasks, norms, hidden, eps=1e-5):
    arr = (_native.StackTaskEx * len(tasks))()
    for i, t in enumerate(tasks):
        arr[i] = _native.StackTaskEx(t["W"].data_ptr(), t["rows"], t["cols"], t["y"].data_ptr(), t["src"], -1,
                                     t.get("src2", -1), t.get("res", -2),
                                     norms[t["norm"]].data_ptr() if "norm" in t else None, eps,
                                     t["W_up"].data_ptr() if "W_up" in t else None)
    h = ctypes.c_void_p()
    rc = L.nexus_gpu_stack_create_ex(Q4_0, arr, len(tasks), hidden, 1, 0, ctypes.byref(h))
    assert rc == 0, L.nexus_gpu_last_error()
    return h


def expected(port, tasks, norms, i, x_in, eps=1e-5):
    """Oracle output of task i from the GPU's actual inputs to it."""
    t = tasks[i]
    out = lambda j: x_in if j < 0 else tasks[j]["y"].cpu().numpy()  # noqa: E731
    x = out(t["src"])
    if "src2" in t:
        x = port.swiglu(x, out(t["src2"]))
    if "norm" in t:
        x = port.rmsnorm(x, norms[t["norm"]].cpu().numpy(), eps)
    y = port.gemv(Q4_0, t["W"].cpu().numpy(), x, t["rows"], t["cols"])
    if "W_up" in t:  # the pair's SwiGLU epilogue
        y = port.swiglu(y, port.gemv(Q4_0, t["W_up"].cpu().numpy(), x, t["rows"], t["cols"]))
    if "res" in t and t["res"] != -2:
        y = (y + out(t["res"])).astype(np.float32)
    return y


@pytest.mark.parametrize("paired", [False, True])
@pytest.mark.parametrize("dims", [(1024, 256, 2048, 1000, 2), (4096, 1024, 14336, 4099, 1), (8192, 1024, 28672, 512, 1)])
def test_fused_decoder_stack_matches_oracle(L, port, dims, paired):
    H, KV, F, V, layers = dims
    tasks, norms = decoder_tasks(H, KV, F, V, layers, 700 + H, paired)
    h = make_stack(L, tasks, norms, H)
    x = torch.from_numpy(synth.activations_numpy(1, H, 5)[0]).cuda()
    st = torch.cuda.current_stream().cuda_stream
    assert L.nexus_gpu_stack_run(h, x.data_ptr(), st) == 0
    torch.cuda.synchronize()
    first = [t["y"].clone() for t in tasks]
    xin = x.cpu().numpy()
    for i, t in enumerate(tasks):
        got = t["y"].cpu().numpy()
        assert np.isfinite(got).all(), t["name"]
        err = oracle.l2_rel(got, expected(port, tasks, norms, i, xin))
        assert err <= TOL, (i, t["name"], err)
    # a second run repeats the first bit for bit
    assert L.nexus_gpu_stack_run(h, x.data_ptr(), st) == 0
    torch.cuda.synchronize()
    for t, f in zip(tasks, first):
        assert torch.equal(t["y"], f), t["name"]
    bits = ctypes.c_uint32(0)
    assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0 and bits.value == 0
    L.nexus_gpu_stack_destroy(h)


def test_fused_task_argument_checks(L):
    H = 1024
    W = synth.blocks_torch(Q4_0, H, H, 3)
    y0, y1 = torch.empty(H, device="cuda"), torch.empty(H, device="cuda")
    nw = torch.ones(H + 1, device="cuda")
    h = ctypes.c_void_p()

    def create(**kw):
        base = dict(src=-1, src2=-1, res=-2, norm=None, w_up=None)
        base.update(kw)
        arr = (_native.StackTaskEx * 2)()
        arr[0] = _native.StackTaskEx(W.data_ptr(), H, H, y0.data_ptr(), -1, -1, -1, -2, None, 0.0)
        arr[1] = _native.StackTaskEx(W.data_ptr(), H, H, y1.data_ptr(), base["src"], -1, base["src2"], base["res"],
                                     base["norm"], 1e-5, base["w_up"])
        return L.nexus_gpu_stack_create_ex(Q4_0, arr, 2, H, 1, 0, ctypes.byref(h))

    assert create(src=0, src2=1) == -5          # x_source2 must be an earlier task
    assert create(src=-1, src2=0) == -5         # SwiGLU needs a task x_source
    assert create(src=0, res=5) == -5           # residual source not earlier
    assert create(src=0, norm=nw.data_ptr() + 4) == -9  # misaligned norm weights
    assert create(src=0, w_up=W.data_ptr() + 8) == -9    # misaligned up matrix
    assert create(src=0, src2=0, res=0, norm=nw.data_ptr()) == 0
    L.nexus_gpu_stack_destroy(h)


@pytest.fixture(scope="module")
def port():
    return oracle.port()


def test_residual_from_a_task_off_the_input_chain(L, port):
    """The residual's task is waited for on its own: c = W_c . y_a + y_b, where
    nothing else orders b before c."""
    H = 2048
    tasks = [dict(name="a", rows=H, cols=H, src=-1), dict(name="b", rows=H, cols=H, src=-1, norm="n"),
             dict(name="c", rows=H, cols=H, src=0, res=1)]
    norms = {"n": (1.0 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(4))).cuda()}
    for i, t in enumerate(tasks):
        t["W"] = synth.blocks_torch(Q4_0, H, H, 900 + i)
        t["y"] = torch.empty(H, device="cuda")
    h = make_stack(L, tasks, norms, H)
    x = torch.from_numpy(synth.activations_numpy(1, H, 8)[0]).cuda()
    for _ in range(3):
        assert L.nexus_gpu_stack_run(h, x.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        xin = x.cpu().numpy()
        for i, t in enumerate(tasks):
            assert oracle.l2_rel(t["y"].cpu().numpy(), expected(port, tasks, norms, i, xin)) <= TOL, t["name"]
        x = x * 0.5
    L.nexus_gpu_stack_destroy(h)
