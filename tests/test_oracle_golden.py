"""The C oracle (oracle/nexus_oracle.c) against the golden vectors that the
reference's own quantization code produced (tests/golden/make_golden.py).

These pin the oracle: every later GPU parity test trusts it.  Dequantization
and fp16 decoding must be bit-exact; the GEMV restatement follows the
reference's AVX2 lane layout and fused operations and is expected to be
bit-exact as well.
"""
import hashlib

import numpy as np
import pytest

import oracle
from nexusllm_b200.formats import DataType


def test_fp16_known_answers(golden, port):
    for h, want in zip(golden["fp16/kat_in"], golden["fp16/kat_out"]):
        got = np.float32(port.fp16_to_fp32(int(h)))
        assert got.view(np.uint32) == want.view(np.uint32), hex(int(h))
    # the quirks the reference decoder has (include/quantization.hpp:59-70)
    assert port.fp16_to_fp32(0x0000) == pytest.approx(2.0 ** -15)
    assert port.fp16_to_fp32(0x7C00) == 0.0 and port.fp16_to_fp32(0x7E00) == 0.0


def test_fp16_full_table(golden, port):
    table = np.array([port.fp16_to_fp32(h) for h in range(65536)], np.float32)
    assert hashlib.sha256(table.tobytes()).digest() == golden["fp16/table_sha256"].tobytes()


@pytest.mark.parametrize("dt", [DataType.FP16, DataType.GGUF_Q4_0, DataType.GGUF_Q8_0,
                                DataType.GGUF_Q5_K, DataType.GGUF_Q6_K])
def test_dequant_bit_exact(golden, port, dt):
    W = golden[f"deq/{int(dt)}/W"]
    want = golden[f"deq/{int(dt)}/out"]
    got = port.dequantize(int(dt), W, want.size)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def _gemv_keys(golden):
    return sorted({k.rsplit("/", 1)[0] for k in golden if k.startswith("gemv/")})


def test_gemv_bit_exact(golden, port):
    keys = _gemv_keys(golden)
    assert len(keys) >= 25
    for key in keys:
        dt = int(key.split("/")[1])
        rows, cols = (int(v) for v in key.split("/")[2].replace("fixture", "").split("x"))
        y = port.gemv(dt, golden[key + "/W"], golden[key + "/x"], rows, cols)
        want = golden[key + "/y"]
        assert oracle.l2_rel(y, want) == 0.0, key
        np.testing.assert_array_equal(y.view(np.uint32), want.view(np.uint32), err_msg=key)


def test_oracle_flags_a_planted_mistake(golden):
    """A wrong restatement must fail the comparison: plant an off-by-one nibble
    bias into a copy of the golden input and check the output moves."""
    import oracle as o

    key = "gemv/7/37x96"
    W = golden[key + "/W"].copy().reshape(-1, 18)
    W[:, 2:] ^= 0x01  # flips every low nibble's least significant bit
    y = o.port().gemv(7, W.reshape(-1), golden[key + "/x"], 37, 96)
    assert o.l2_rel(y, golden[key + "/y"]) > 1e-2
