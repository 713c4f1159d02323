"""INT4-AWQ and FP8-E4M3 GEMV and dequantization on the GPU against the C
oracle (bit-identical to the reference build, tests/test_awq_fp8.py).

GEMV results agree within the 1e-3 L2-relative tolerance (INT4 carries x as
16-bit fixed point like the GGUF path; FP8 sums in another order);
dequantization is bit-exact.  Shapes cover the fast kernels (group sizes that
are multiples of 32, 16-byte rows) and the generic kernel (other group sizes,
ragged columns, unaligned weights, K beyond the shared-memory limit)."""
import ctypes

import numpy as np
import pytest

import oracle
from nexusllm_b200 import _native
from nexusllm_b200.quantization import QuantizationKernel

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-3


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


@pytest.fixture(scope="module")
def port():
    return oracle.port()


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _int4_case(rows, cols, gs, seed, with_zeros=True):
    r = np.random.default_rng(seed)
    W = r.integers(0, 2**32, size=rows * cols // 8, dtype=np.uint64).astype(np.uint32)
    ng = rows * cols // gs
    scales = r.uniform(0.001, 0.02, size=ng).astype(np.float32)
    zeros = r.integers(0, 16, size=ng).astype(np.float32) if with_zeros else None
    x = r.standard_normal(cols).astype(np.float32)
    return W, scales, zeros, x


def _gemv_int4(L, W, scales, zeros, x, rows, cols, gs, w_offset_bytes=0):
    if w_offset_bytes:
        raw = torch.zeros(W.nbytes + 64, dtype=torch.uint8, device="cuda")
        raw[w_offset_bytes:w_offset_bytes + W.nbytes] = _dev(W.view(np.uint8))
        dW = raw.data_ptr() + w_offset_bytes
    else:
        t = _dev(W)
        dW = t.data_ptr()
    dS, dX = _dev(scales), _dev(x)
    dZ = _dev(zeros) if zeros is not None else None
    y = torch.full((rows,), float("nan"), device="cuda")
    rc = L.nexus_gpu_gemv_int4(dW, dS.data_ptr(), None if dZ is None else dZ.data_ptr(), dX.data_ptr(), y.data_ptr(),
                               rows, cols, gs, None, 0, _stream())
    assert rc == 0, L.nexus_gpu_last_error()
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("rows,cols,gs,z", [(4096, 4096, 128, True), (1, 128, 128, True), (37, 256, 32, False),
                                            (300, 14336, 128, True), (64, 4096, 64, True), (129, 32768, 128, True),
                                            (16, 1000, 8, True), (9, 200, 40, True), (33, 96, 32, True),
                                            (5, 40960, 128, True)])
def test_int4_gemv_matches_oracle(L, port, rows, cols, gs, z):
    W, scales, zeros, x = _int4_case(rows, cols, gs, rows * 7 + cols, z)
    y = _gemv_int4(L, W, scales, zeros, x, rows, cols, gs)
    want = port.gemv_int4(W, x, scales, zeros, rows, cols, gs)
    assert np.isfinite(y).all()
    assert oracle.l2_rel(y, want) <= TOL


def test_int4_unaligned_weights_take_the_generic_kernel(L, port):
    rows, cols, gs = 70, 1024, 128
    W, scales, zeros, x = _int4_case(rows, cols, gs, 5)
    y = _gemv_int4(L, W, scales, zeros, x, rows, cols, gs, w_offset_bytes=4)
    assert oracle.l2_rel(y, port.gemv_int4(W, x, scales, zeros, rows, cols, gs)) <= TOL


def test_int4_workspace_checks(L):
    rows, cols, gs = 8, 256, 32
    W, scales, zeros, x = _int4_case(rows, cols, gs, 9)
    dW, dS, dZ, dX = _dev(W), _dev(scales), _dev(zeros), _dev(x)
    y = torch.empty(rows, device="cuda")
    need = L.nexus_gpu_gemv_int4_workspace_size(cols)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    args = (dW.data_ptr(), dS.data_ptr(), dZ.data_ptr(), dX.data_ptr(), y.data_ptr(), rows, cols, gs)
    assert L.nexus_gpu_gemv_int4(*args, ws.data_ptr(), need - 1, _stream()) == -102  # WORKSPACE
    assert L.nexus_gpu_gemv_int4(*args, ws.data_ptr(), need, _stream()) == 0
    torch.cuda.synchronize()


def _fp8_case(rows, cols, seed, nan_codes):
    r = np.random.default_rng(seed)
    if nan_codes:
        W = r.integers(0, 256, size=rows * cols, dtype=np.uint8)
    else:  # realistic weights: normal values encoded to E4M3
        W = torch.randn(rows * cols, generator=torch.Generator().manual_seed(seed)).mul(0.5).to(
            torch.float8_e4m3fn).view(torch.uint8).numpy()
    return W, r.standard_normal(cols).astype(np.float32)


@pytest.mark.parametrize("rows,cols,nan", [(4096, 4096, False), (4096, 4096, True), (1, 16, True), (37, 100, True),
                                           (300, 14336, False), (7, 16384, True), (5, 16400, True), (16, 33, False),
                                           (1000, 2048, True)])
def test_fp8_gemv_matches_oracle(L, port, rows, cols, nan):
    W, x = _fp8_case(rows, cols, rows + cols, nan)
    dW, dX = _dev(W), _dev(x)
    y = torch.full((rows,), float("nan"), device="cuda")
    assert L.nexus_gpu_gemv_fp8(dW.data_ptr(), dX.data_ptr(), y.data_ptr(), rows, cols, 0.0625, _stream()) == 0
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    want = port.gemv_fp8(W, x, rows, cols, 0.0625)
    assert np.isfinite(got).all()
    assert oracle.l2_rel(got, want) <= TOL


def test_fp8_every_code_through_the_gemv(L, port):
    """One row per code: the fast kernel's e4m3x2 conversion and NaN patch
    against the reference decoder, code by code (x = 1 on a single column)."""
    cols = 32
    W = np.zeros((256, cols), np.uint8)
    W[:, 5] = np.arange(256, dtype=np.uint8)
    x = np.zeros(cols, np.float32)
    x[5] = 1.0
    dW, dX = _dev(W), _dev(x)
    y = torch.empty(256, device="cuda")
    assert L.nexus_gpu_gemv_fp8(dW.data_ptr(), dX.data_ptr(), y.data_ptr(), 256, cols, 1.0, _stream()) == 0
    torch.cuda.synchronize()
    want = port.dequantize_fp8_e4m3(np.arange(256, dtype=np.uint8), 256, 1.0)
    np.testing.assert_array_equal(y.cpu().numpy(), want)


def test_dequant_bit_exact(L, port):
    r = np.random.default_rng(1)
    packed = r.integers(0, 2**32, size=4096, dtype=np.uint64).astype(np.uint32)
    for gs, with_z in ((32, True), (8, False), (128, True), (40, True)):
        count = 4096 * 8 - 3
        ng = (count + gs - 1) // gs
        s = r.uniform(-0.1, 0.1, ng).astype(np.float32)
        z = r.uniform(0, 15, ng).astype(np.float32) if with_z else None
        out = torch.empty(count, device="cuda")
        dP, dS = _dev(packed), _dev(s)
        dZ = _dev(z) if with_z else None
        assert L.nexus_gpu_dequantize_int4_awq(dP.data_ptr(), dS.data_ptr(), None if dZ is None else dZ.data_ptr(),
                                               out.data_ptr(), count, gs, _stream()) == 0
        torch.cuda.synchronize()
        want = port.dequantize_int4_awq(packed, s, z, count, gs)
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    codes = r.integers(0, 256, size=100003, dtype=np.uint8)
    out = torch.empty(codes.size, device="cuda")
    dC = _dev(codes)
    assert L.nexus_gpu_dequantize_fp8_e4m3(dC.data_ptr(), out.data_ptr(), codes.size, 0.37, _stream()) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32),
                                  port.dequantize_fp8_e4m3(codes, codes.size, 0.37).view(np.uint32))


def test_host_drop_ins_match_the_reference_interface(port):
    rows, cols, gs = 100, 1024, 128
    W, scales, zeros, x = _int4_case(rows, cols, gs, 21)
    y = np.zeros(rows, np.float32)
    QuantizationKernel.fused_gemv_int4(W, x, scales, zeros, y, rows, cols, gs)
    assert oracle.l2_rel(y, port.gemv_int4(W, x, scales, zeros, rows, cols, gs)) <= TOL
    QuantizationKernel.fused_gemv_int4(W, x, scales, None, y, rows, cols, gs)
    assert oracle.l2_rel(y, port.gemv_int4(W, x, scales, None, rows, cols, gs)) <= TOL
    W8, x8 = _fp8_case(rows, 1000, 22, True)
    QuantizationKernel.fused_gemv_fp8(W8, x8, y, rows, 1000, 0.25)
    assert oracle.l2_rel(y, port.gemv_fp8(W8, x8, rows, 1000, 0.25)) <= TOL
    out = np.zeros(rows * cols, np.float32)
    QuantizationKernel.dequantize_int4_awq(W, scales, zeros, out, rows * cols, gs)
    np.testing.assert_array_equal(out.view(np.uint32),
                                  port.dequantize_int4_awq(W, scales, zeros, rows * cols, gs).view(np.uint32))
    out8 = np.zeros(W8.size, np.float32)
    QuantizationKernel.dequantize_fp8_e4m3(W8, out8, W8.size, 0.25)
    np.testing.assert_array_equal(out8.view(np.uint32), port.dequantize_fp8_e4m3(W8, W8.size, 0.25).view(np.uint32))
    st = ctypes.c_uint32(0)
    assert _native.lib().nexus_gpu_device_status(ctypes.byref(st)) == 0 and st.value == 0
