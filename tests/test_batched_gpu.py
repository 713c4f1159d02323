"""GPU tests of batched decode (M >= 16 activation rows) on the tcgen05 tensor
cores (GGUF Q4_0, nexusllm_b200/csrc/mma_kernels.cuh), reached through
nexus_gpu_gemv exactly like the batch-1 path.

Weights are dequantized to fp16 with one rounding of (q - 8) * d and x is
carried as two fp16 parts, so outputs are compared with the C oracle (the
reference's AVX2 arithmetic) within the 1e-3 L2-relative GEMV tolerance, not
bit for bit.  Shapes cover ragged row tiles, split K, several token groups and
bf16 activations.
"""
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


def run(L, W, x, rows, cols, x_dtype=0):
    M = x.shape[0]
    y = torch.full((M, rows), float("nan"), device="cuda")
    rc = L.nexus_gpu_gemv(W.data_ptr(), Q4_0, x.data_ptr(), x_dtype, y.data_ptr(), M, rows, cols,
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.nexus_gpu_last_error()
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("rows,cols,M", [(4096, 4096, 16), (1024, 4096, 17), (300, 4096, 33), (4096, 14336, 64),
                                         (128, 256, 16), (1000, 1024, 80)])
def test_batched_matches_oracle(L, port, rows, cols, M):
    W = synth.blocks_torch(Q4_0, rows, cols, 41 + rows)
    x = torch.from_numpy(synth.activations_numpy(M, cols, 42 + M)).cuda()
    y = run(L, W, x, rows, cols)
    assert torch.isfinite(y).all()
    Wh = W.cpu().numpy()
    xs = x.cpu().numpy()
    for t in sorted({0, M // 2, M - 1}):
        want = port.gemv(Q4_0, Wh, xs[t], rows, cols)
        err = oracle.l2_rel(y[t].cpu().numpy(), want)
        assert err <= TOL, (t, err)
    # every token against the batch-1 (CUDA-core) path
    y1 = torch.empty(rows, device="cuda")
    for t in range(M):
        assert L.nexus_gpu_gemv(W.data_ptr(), Q4_0, x[t].data_ptr(), 0, y1.data_ptr(), 1, rows, cols,
                                torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        e = (torch.linalg.vector_norm(y[t] - y1) / torch.linalg.vector_norm(y1)).item()
        assert e <= TOL, (t, e)


def test_batched_is_deterministic_and_bf16(L, port):
    rows, cols, M = 2048, 4096, 24
    W = synth.blocks_torch(Q4_0, rows, cols, 77)
    x = torch.from_numpy(synth.activations_numpy(M, cols, 78)).cuda()
    a, b = run(L, W, x, rows, cols), run(L, W, x, rows, cols)
    assert torch.equal(a, b)
    xb = x.to(torch.bfloat16)
    yb = run(L, W, xb, rows, cols, x_dtype=2)
    want = port.gemv(Q4_0, W.cpu().numpy(), xb[5].float().cpu().numpy(), rows, cols)
    assert oracle.l2_rel(yb[5].cpu().numpy(), want) <= TOL


def test_batched_scales_and_non_finite_tokens(L, port):
    rows, cols, M = 512, 2048, 16
    W = synth.blocks_torch(Q4_0, rows, cols, 90)
    x = torch.from_numpy(synth.activations_numpy(M, cols, 91)).cuda()
    x[1] *= 3.0e4      # large activations: the per-token power of two keeps fp16 in range
    x[2] *= 1.0e-6     # small ones keep their precision
    x[3, 7] = float("nan")
    y = run(L, W, x, rows, cols)
    Wh, xs = W.cpu().numpy(), x.cpu().numpy()
    for t in (0, 1, 2, 4):
        assert oracle.l2_rel(y[t].cpu().numpy(), port.gemv(Q4_0, Wh, xs[t], rows, cols)) <= TOL, t
    assert torch.isnan(y[3]).all()
    import ctypes
    st = ctypes.c_uint32(0)
    assert L.nexus_gpu_device_status(ctypes.byref(st)) == 0 and st.value == 0
