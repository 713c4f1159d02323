"""INT4-AWQ and FP8-E4M3 on the CPU: the C oracle against the golden vectors
the reference's own quantization code produced (tests/golden/make_golden.py,
src/quantization.cpp:12-68,102-262), and the library's argument checks, which
run before any device is touched."""
import ctypes

import numpy as np
import pytest

import oracle
from nexusllm_b200 import _native


@pytest.fixture(scope="module")
def golden():
    import os
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


@pytest.fixture(scope="module")
def port():
    return oracle.port()


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_fp8_every_code(golden, port):
    codes = golden["fp8/codes"]
    for scale, key in ((1.0, "fp8/codes_x1"), (0.37, "fp8/codes_x037")):
        got = port.dequantize_fp8_e4m3(codes, 256, scale)
        np.testing.assert_array_equal(_bits(got), _bits(golden[key]))
    x1 = golden["fp8/codes_x1"]
    assert x1[0x7F] == 0 and x1[0xFF] == 0          # NaN codes decode to 0
    assert x1[0x7E] == 448.0 and x1[0x01] == 2.0 ** -9  # max normal, min subnormal
    assert np.signbit(x1[0x80]) and x1[0x80] == 0     # -0 keeps its sign


def test_int4_dequant(golden, port):
    p, s, z = golden["int4deq/packed"], golden["int4deq/scales"], golden["int4deq/zeros"]
    np.testing.assert_array_equal(_bits(port.dequantize_int4_awq(p, s, z, 1000, 32)), _bits(golden["int4deq/out_g32"]))
    np.testing.assert_array_equal(_bits(port.dequantize_int4_awq(p, golden["int4deq/scales_g8"], None, 1000, 8)),
                                  _bits(golden["int4deq/out_g8_nozero"]))


def _keys(golden, prefix):
    return sorted({k.rsplit("/", 1)[0] for k in golden.files if k.startswith(prefix)})


def test_int4_gemv_bit_exact(golden, port):
    keys = _keys(golden, "int4gemv/")
    assert len(keys) >= 7
    for key in keys:
        shape = key.split("/")[1]
        rows, rest = shape.split("x")
        cols, gs = rest.rstrip("z").split("g")
        rows, cols, gs = int(rows), int(cols), int(gs)
        zeros = golden[key + "/zeros"] if shape.endswith("z") else None
        y = port.gemv_int4(golden[key + "/W"], golden[key + "/x"], golden[key + "/scales"], zeros, rows, cols, gs)
        np.testing.assert_array_equal(_bits(y), _bits(golden[key + "/y"]), err_msg=key)


def test_fp8_gemv_bit_exact(golden, port):
    keys = _keys(golden, "fp8gemv/")
    assert len(keys) >= 6
    for key in keys:
        rows, cols = (int(v) for v in key.split("/")[1].split("x"))
        y = port.gemv_fp8(golden[key + "/W"], golden[key + "/x"], rows, cols, 0.0625)
        np.testing.assert_array_equal(_bits(y), _bits(golden[key + "/y"]), err_msg=key)


def test_oracle_flags_a_planted_int4_mistake(golden):
    """A wrong restatement must fail: shift every zero by one."""
    key = _keys(golden, "int4gemv/16x4096")[0]
    y = oracle.port().gemv_int4(golden[key + "/W"], golden[key + "/x"], golden[key + "/scales"],
                                golden[key + "/zeros"] + 1.0, 16, 4096, 128)
    assert oracle.l2_rel(y, golden[key + "/y"]) > 1e-3


@pytest.mark.skipif(not oracle.reference_available(), reason="reference build not present")
def test_port_matches_reference_on_random_shapes():
    P, R = oracle.port(), oracle.reference()
    rng = np.random.default_rng(3)
    for _ in range(60):
        rows, gs = int(rng.integers(1, 6)), int(rng.choice([8, 16, 32, 64, 128]))
        cols = gs * int(rng.integers(1, 9))
        W = rng.integers(0, 2**32, size=rows * cols // 8, dtype=np.uint64).astype(np.uint32)
        sc = rng.uniform(-0.05, 0.05, size=rows * cols // gs).astype(np.float32)
        z = rng.uniform(0, 15, size=sc.size).astype(np.float32)
        x = rng.standard_normal(cols).astype(np.float32)
        np.testing.assert_array_equal(_bits(P.gemv_int4(W, x, sc, z, rows, cols, gs)),
                                      _bits(R.gemv_int4(W, x, sc, z, rows, cols, gs)))
        c8 = int(rng.integers(1, 300))
        B = rng.integers(0, 256, size=rows * c8, dtype=np.uint8)
        x8 = rng.standard_normal(c8).astype(np.float32)
        np.testing.assert_array_equal(_bits(P.gemv_fp8(B, x8, rows, c8, 0.5)), _bits(R.gemv_fp8(B, x8, rows, c8, 0.5)))


def test_int4_argument_checks():
    L = _native.lib()
    bad_arg, bad_shape = -9, -5  # NEXUS_GPU_ERROR_INVALID_ARGUMENT, _SHAPE_MISMATCH
    f = L.nexus_gpu_gemv_int4
    assert f(None, None, None, None, None, 4, 256, 0, None, 0, None) == bad_arg      # group_size 0
    assert f(None, None, None, None, None, 4, 252, 4, None, 0, None) == bad_shape    # cols % 8
    assert f(None, None, None, None, None, 4, 256, 96, None, 0, None) == bad_shape   # cols % group_size
    assert L.nexus_gpu_gemv_int4_workspace_size(4096) >= 4096 // 32 * 80


def test_workspace_size_grows_with_cols():
    L = _native.lib()
    assert L.nexus_gpu_gemv_int4_workspace_size(8192) > L.nexus_gpu_gemv_int4_workspace_size(4096)
    assert isinstance(L.nexus_gpu_gemv_int4_workspace_size(0), int)
    _ = ctypes  # the entry points bind through _native.SIGNATURES


def test_layer_ops_bit_exact(golden, port):
    """RMSNorm and SwiGLU restated in the oracle against the reference build
    (TransformerOps, include/transformer_ops.hpp:23-44,86-95)."""
    for j in range(4):
        key = f"ops/rmsnorm/{j}"
        x, w, eps = golden[key + "/x"], golden[key + "/w"], float(golden[key + "/eps"][0])
        np.testing.assert_array_equal(_bits(port.rmsnorm(x, w, eps)), _bits(golden[key + "/out"]), err_msg=key)
        np.testing.assert_array_equal(_bits(port.rmsnorm(x, None, eps)), _bits(golden[key + "/out_now"]), err_msg=key)
    np.testing.assert_array_equal(_bits(port.swiglu(golden["ops/swiglu/g"], golden["ops/swiglu/u"])),
                                  _bits(golden["ops/swiglu/out"]))
