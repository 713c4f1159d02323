"""GPU parity of the fused quantized GEMV and dequantization, through the C ABI.

Tolerance (north star): GEMV outputs within 1e-3 L2-relative
(||y - y_ref||_2 / ||y_ref||_2) of the reference's AVX2 path; dequantized
values bit-exact.  The reference here is (a) the golden vectors the
reference's own code produced (tests/golden/) and (b) the C oracle
(oracle/nexus_oracle.c, bit-identical to the reference on those vectors) on
seeded inputs with the benchmark configurations' distributions.
"""
import ctypes

import numpy as np
import pytest

import oracle
from nexusllm_b200 import _native, synth
from nexusllm_b200.formats import BLOCK, DataType, weight_bytes

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-3
FORMATS = [DataType.GGUF_Q4_0, DataType.GGUF_Q8_0, DataType.GGUF_Q5_K, DataType.GGUF_Q6_K, DataType.FP16]
NAME = {DataType.GGUF_Q4_0: "q4_0", DataType.GGUF_Q8_0: "q8_0", DataType.GGUF_Q5_K: "q5_k",
        DataType.GGUF_Q6_K: "q6_k", DataType.FP16: "fp16"}


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return _native.lib()


@pytest.fixture(scope="module")
def be(L):
    from nexusllm_b200.backend import CUDABackend

    return CUDABackend()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8) if a.dtype != np.float32 else a).cuda()


def gpu_gemv(be, dt, W, x, rows, cols, x_bf16=False):
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    if x_bf16:
        xt = xt.to(torch.bfloat16)
    y = be.gemv(dev(W), dt, xt)
    return y.cpu().numpy()


# ------------------------------------------------------------- golden vectors
def test_golden_gemv_through_host_abi(L, golden):
    keys = sorted({k.rsplit("/", 1)[0] for k in golden if k.startswith("gemv/")})
    for key in keys:
        dt = DataType(int(key.split("/")[1]))
        rows, cols = (int(v) for v in key.split("/")[2].replace("fixture", "").split("x"))
        W = np.ascontiguousarray(golden[key + "/W"])
        x = np.ascontiguousarray(golden[key + "/x"])
        y = np.full(rows, np.nan, np.float32)
        getattr(L, "nexus_fused_gemv_" + NAME[dt])(W.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols)
        err = oracle.l2_rel(y, golden[key + "/y"])
        assert err <= TOL, (key, err)


def test_golden_dequant_bit_exact(L, be, golden):
    for dt in (DataType.GGUF_Q4_0, DataType.GGUF_Q5_K, DataType.GGUF_Q6_K):
        W = np.ascontiguousarray(golden[f"deq/{int(dt)}/W"])
        want = golden[f"deq/{int(dt)}/out"]
        per, nb_ = BLOCK[dt]
        out = np.full(want.size, np.nan, np.float32)
        getattr(L, "nexus_dequantize_gguf_" + NAME[dt])(W.ctypes.data, out.ctypes.data, W.size // nb_)
        np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32), err_msg=dt.name)
    for dt in (DataType.GGUF_Q8_0, DataType.FP16, DataType.GGUF_Q4_0, DataType.GGUF_Q5_K, DataType.GGUF_Q6_K):
        W = golden[f"deq/{int(dt)}/W"]
        want = golden[f"deq/{int(dt)}/out"]
        out = be.dequantize(dev(W), dt, want.size).cpu().numpy()
        np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32), err_msg=dt.name)


# ------------------------------------------------------------ seeded parity
SHAPES = [(4096, 4096), (1024, 4096), (11008, 4096), (4096, 11008), (300, 14336), (1, 4096), (7, 256),
          (149, 512), (4097, 1024), (64, 28672), (300, 1056), (45, 3104)]


@pytest.mark.parametrize("dt", FORMATS, ids=lambda d: d.name)
def test_parity_vs_oracle(be, port, dt):
    for i, (rows, cols) in enumerate(SHAPES):
        if cols % BLOCK[dt][0]:
            continue  # odd block counts (ungrouped lanes) exist only for the 32-element formats
        W = synth.blocks_numpy(dt, rows, cols, 1000 * int(dt) + i)
        x = synth.activations_numpy(1, cols, 7000 + i)[0]
        want = port.gemv(int(dt), W, x, rows, cols)
        got = gpu_gemv(be, dt, W, x, rows, cols)
        err = oracle.l2_rel(got, want)
        assert err <= TOL, (dt.name, rows, cols, err)
        # every row, not only the norm, must be close
        scale = np.abs(want).max() + 1e-30
        assert np.abs(got - want).max() <= 2e-3 * scale, (dt.name, rows, cols)


@pytest.mark.parametrize("dt", FORMATS, ids=lambda d: d.name)
def test_bf16_activations(be, port, dt):
    rows, cols = 1024, 4096
    W = synth.blocks_numpy(dt, rows, cols, 77)
    x = synth.activations_numpy(1, cols, 78)[0]
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()  # what the kernel sees
    want = port.gemv(int(dt), W, xb, rows, cols)
    got = gpu_gemv(be, dt, W, x, rows, cols, x_bf16=True)
    assert oracle.l2_rel(got, want) <= TOL


@pytest.mark.parametrize("dt", FORMATS, ids=lambda d: d.name)
def test_batched_rows_equal_single_calls(be, port, dt):
    rows, cols, M = 512, 2048, 4
    W = synth.blocks_numpy(dt, rows, cols, 91)
    X = synth.activations_numpy(M, cols, 92)
    Wd = dev(W)
    Y = be.gemv(Wd, dt, torch.from_numpy(X).cuda()).cpu().numpy()
    for m in range(M):
        y1 = be.gemv(Wd, dt, torch.from_numpy(X[m].copy()).cuda()).cpu().numpy()
        np.testing.assert_array_equal(Y[m], y1)
        assert oracle.l2_rel(Y[m], port.gemv(int(dt), W, X[m], rows, cols)) <= TOL


@pytest.mark.parametrize("dt", FORMATS, ids=lambda d: d.name)
def test_misaligned_weight_pointer_uses_generic_kernel(be, port, dt):
    rows, cols = 96, 1024
    W = synth.blocks_numpy(dt, rows, cols, 5).view(np.uint8)
    buf = torch.zeros(W.size + 16, dtype=torch.uint8, device="cuda")
    buf[2:2 + W.size] = torch.from_numpy(W).cuda()
    x = synth.activations_numpy(1, cols, 6)[0]
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = be._lib.nexus_gpu_gemv(buf.data_ptr() + 2, int(dt), torch.from_numpy(x).cuda().data_ptr(), 0,
                                y.data_ptr(), 1, rows, cols, st)
    assert rc == 0
    assert oracle.l2_rel(y.cpu().numpy(), port.gemv(int(dt), W, x, rows, cols)) <= TOL


def test_fp16_ragged_cols(be, port):
    for rows, cols in [(37, 100), (16, 33), (5, 8), (3, 1)]:
        W = synth.blocks_numpy(DataType.FP16, rows, cols, 3)
        x = synth.activations_numpy(1, cols, 4)[0]
        got = gpu_gemv(be, DataType.FP16, W, x, rows, cols)
        assert oracle.l2_rel(got, port.gemv(1, W, x, rows, cols)) <= TOL


def test_activation_edge_cases(be, port):
    dt, rows, cols = DataType.GGUF_Q4_0, 256, 1024
    W = synth.blocks_numpy(dt, rows, cols, 11)
    x = synth.activations_numpy(1, cols, 12)[0]
    x[0:32] = 0.0                      # an all-zero block
    x[32:64] *= 1e-30                  # a tiny block (near subnormal)
    x[64] = 1e4                        # a block with a huge dynamic range
    got = gpu_gemv(be, dt, W, x, rows, cols)
    assert oracle.l2_rel(got, port.gemv(int(dt), W, x, rows, cols)) <= TOL
    x[100] = np.inf
    got = gpu_gemv(be, dt, W, x, rows, cols)
    assert not np.isfinite(got).any()  # every row touches the Inf, as in fp32
    x[100] = np.nan
    got = gpu_gemv(be, dt, W, x, rows, cols)
    assert np.isnan(got).all()


@pytest.mark.parametrize("dt", [DataType.GGUF_Q4_0, DataType.GGUF_Q8_0, DataType.GGUF_Q5_K, DataType.GGUF_Q6_K])
def test_weight_edge_blocks(be, port, golden, dt):
    # the golden edge blocks (special fp16 scales -- zero, subnormal, Inf, NaN,
    # the largest half, a subnormal Q5_K dmin -- and extreme codes) as one
    # matrix of 256-weight rows (the generic kernel) ...
    W = golden[f"deq/{int(dt)}/W"]
    per, nb_ = BLOCK[dt]
    rows = W.size // nb_ * per // 256
    cols = 256
    x = synth.activations_numpy(1, cols, 13)[0]
    got = gpu_gemv(be, dt, W, x, rows, cols)
    want = port.gemv(int(dt), W, x, rows, cols)
    assert oracle.l2_rel(got, want) <= TOL
    # ... and cycled through rows of 4096 weights, where the fast kernel runs
    blocks = W.reshape(-1, nb_)
    nb, per_row, rows = blocks.shape[0], 4096 // per, 24
    idx = (np.arange(rows)[:, None] * 7 + np.arange(per_row)[None, :]) % nb
    Wt = np.ascontiguousarray(blocks[idx.reshape(-1)]).reshape(-1)
    x = synth.activations_numpy(1, 4096, 14)[0]
    got = gpu_gemv(be, dt, Wt, x, rows, 4096)
    want = port.gemv(int(dt), Wt, x, rows, 4096)
    assert np.isfinite(want).all()
    assert oracle.l2_rel(got, want) <= TOL


def test_host_api_weight_cache(L, port):
    dt, rows, cols = DataType.GGUF_Q8_0, 512, 2048
    W = synth.blocks_numpy(dt, rows, cols, 21)
    x = synth.activations_numpy(1, cols, 22)[0]
    y1 = np.zeros(rows, np.float32)
    y2 = np.zeros(rows, np.float32)
    L.nexus_gpu_weight_cache_invalidate(None)
    assert L.nexus_gpu_gemv_dispatch(W.ctypes.data, int(dt), x.ctypes.data, y1.ctypes.data, rows, cols) == 0
    held = L.nexus_gpu_weight_cache_bytes()
    assert held >= weight_bytes(dt, rows, cols)
    assert L.nexus_gpu_gemv_dispatch(W.ctypes.data, int(dt), x.ctypes.data, y2.ctypes.data, rows, cols) == 0
    assert L.nexus_gpu_weight_cache_bytes() == held  # second call reused the upload
    np.testing.assert_array_equal(y1, y2)
    # the buffer now holds another tensor: the fingerprint notices the change
    W[:] = synth.blocks_numpy(dt, rows, cols, 23)
    assert L.nexus_gpu_gemv_dispatch(W.ctypes.data, int(dt), x.ctypes.data, y2.ctypes.data, rows, cols) == 0
    assert oracle.l2_rel(y2, port.gemv(int(dt), W, x, rows, cols)) <= TOL
    assert L.nexus_gpu_weight_cache_invalidate(W.ctypes.data) == 0
    assert L.nexus_gpu_weight_cache_bytes() == held - weight_bytes(dt, rows, cols) - (
        -weight_bytes(dt, rows, cols) % 256)


def test_host_api_full_weight_check(L, port, monkeypatch):
    """NEXUS_GPU_WEIGHT_CHECK=full: a change the sampled fingerprint does not
    look at (one block's scale, away from the 64 KiB probes) still re-uploads
    the weights, so the result follows the new bytes."""
    dt, rows, cols = DataType.GGUF_Q8_0, 4096, 4096  # 8.9 MB: many 64 KiB probes
    W = synth.blocks_numpy(dt, rows, cols, 31)
    x = synth.activations_numpy(1, cols, 32)[0]
    y = np.zeros(rows, np.float32)
    monkeypatch.setenv("NEXUS_GPU_WEIGHT_CHECK", "full")
    L.nexus_gpu_weight_cache_invalidate(None)
    try:
        assert L.nexus_gpu_gemv_dispatch(W.ctypes.data, int(dt), x.ctypes.data, y.ctypes.data, rows, cols) == 0
        raw = W.view(np.uint8).reshape(-1)
        off = 34 * 6100  # block 6100's fp16 scale, between two 64 KiB probes (34-byte blocks)
        assert 16 <= off % 65536 and off + 2 < raw.size - 64
        raw[off:off + 2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
        assert L.nexus_gpu_gemv_dispatch(W.ctypes.data, int(dt), x.ctypes.data, y.ctypes.data, rows, cols) == 0
        assert oracle.l2_rel(y, port.gemv(int(dt), W, x, rows, cols)) <= TOL
        r = off // (cols // 32 * 34)  # the changed row now matches the new scale
        want = port.gemv(int(dt), W, x, rows, cols)[r]
        assert abs(y[r] - want) <= 1e-3 * max(1.0, abs(want))
    finally:
        L.nexus_gpu_weight_cache_invalidate(None)


def test_full_size_lm_head_sampled_rows(be, port):
    """BASELINE config 4's largest matrix (LM head 128256 x 4096, Q4_0): the
    whole GEMV on the GPU, checked row-by-row against the oracle on 512
    sampled rows (the oracle on all 128256 rows would take minutes)."""
    dt, rows, cols = DataType.GGUF_Q4_0, 128256, 4096
    Wd = synth.blocks_torch(dt, rows, cols, 4004)
    x = synth.activations_numpy(1, cols, 4005)[0]
    y = be.gemv(Wd, dt, torch.from_numpy(x).cuda()).cpu().numpy()
    rng = np.random.default_rng(0)
    idx = np.sort(rng.choice(rows, 512, replace=False))
    rb = cols // 32 * 18
    Wh = Wd.view(rows, rb)[torch.from_numpy(idx).cuda()].cpu().numpy().reshape(-1)
    want = port.gemv(int(dt), Wh, x, len(idx), cols)
    assert oracle.l2_rel(y[idx], want) <= TOL
    assert np.isfinite(y).all()


def test_row_slices_are_bit_identical(be):
    """Row-sharding invariant: rows [a, b) computed from a sub-matrix equal the
    same rows of the full GEMV bit for bit (per-row arithmetic does not depend
    on how rows are spread over CTAs or GPUs)."""
    for dt in FORMATS:
        rows, cols = 2048, 4096
        Wd = synth.blocks_torch(dt, rows, cols, 55)
        x = torch.from_numpy(synth.activations_numpy(1, cols, 56)[0]).cuda()
        full = be.gemv(Wd, dt, x)
        rb = weight_bytes(dt, 1, cols)
        for a, b in [(0, 512), (512, 1024), (1000, 2048)]:
            if (a * rb) % 16:
                continue
            part = be.gemv(Wd[a * rb:b * rb], dt, x)
            assert torch.equal(part, full[a:b]), (dt.name, a, b)


def test_errors_and_status(L, be):
    x = torch.zeros(64, device="cuda")
    W = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    y = torch.zeros(64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.nexus_gpu_gemv(W.data_ptr(), 0, x.data_ptr(), 0, y.data_ptr(), 1, 4, 64, st) == -3
    assert L.nexus_gpu_gemv(W.data_ptr(), 7, x.data_ptr(), 0, y.data_ptr(), 1, 4, 48, st) == -5
    assert L.nexus_gpu_gemv(W.data_ptr(), 7, x.data_ptr(), 5, y.data_ptr(), 1, 4, 64, st) == -3
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    assert L.nexus_gpu_gemv_ws(W.data_ptr(), 7, x.data_ptr(), 0, y.data_ptr(), 1, 4, 64, ws.data_ptr(), 16, st) == -102
    bits = ctypes.c_uint32(99)
    assert L.nexus_gpu_device_status(ctypes.byref(bits)) == 0
    assert bits.value == 0, "a bounded device wait expired during the tests"


def test_fp16_special_halves_take_the_exact_decoder(be):
    """FP16 weights holding every kind of half the two kernel paths split on:
    zeros and subnormals (which the reference decodes as 2^-15 (1 + m/1024),
    served by the shifted hardware conversion), exponent 30 (|w| >= 32768)
    and Inf/NaN (decoded to 0), which send their 16-weight item to the
    bit-level decoder.  Rows mix both paths; compared with the C oracle."""
    port = oracle.port()
    rows, cols = 512, 4096
    r = np.random.default_rng(17)
    W = (r.standard_normal((rows, cols)) * 0.02).astype(np.float16).view(np.uint16)
    specials = np.array([0x0000, 0x8000, 0x0001, 0x83FF, 0x03FF, 0x7800, 0xF9FF, 0x7BFF, 0x7C00, 0xFC00, 0x7E00,
                         0xFFFF], np.uint16)
    for i in range(rows):  # most rows get a few special halves, some none
        k = r.integers(0, 4)
        W[i, r.integers(0, cols, size=k)] = r.choice(specials, size=k)
    W[0, :16] = 0x7C00  # a whole work item of Inf
    W[1, ::2] = 0x0000   # zeros everywhere in a row
    W = np.ascontiguousarray(W.reshape(-1))
    x = r.standard_normal(cols).astype(np.float32) * 0.01
    got = gpu_gemv(be, DataType.FP16, W, x, rows, cols)
    want = port.gemv(int(DataType.FP16), W, x, rows, cols)
    assert np.isfinite(got).all() and np.isfinite(want).all()
    assert oracle.l2_rel(got, want) <= TOL
    # row by row as well: the large values of exponent-30 halves must not hide a wrong row
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-3)
    assert np.median(rel) < 1e-4 and rel.max() < 1e-2
