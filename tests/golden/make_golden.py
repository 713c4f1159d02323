"""Generate tests/golden/golden.npz from NexusLLM's own quantization code.

Run from the repository root, where oracle/_ref/libnexus_ref.so has been
built from the reference sources (``make -C oracle ref REF=<checkout>``):

    python tests/golden/make_golden.py

``python tests/golden/make_golden.py gguf`` writes tests/golden/gguf_ref.json
instead: what NexusLLM's own GGUF loader (oracle/_ref/libnexus_ref_gguf.so,
``make -C oracle ref-gguf``) reads from the synthetic files of
tests/gguf_cases.py -- metadata, which names resolve, each tensor's DataType,
dims, byte size and an FNV-1a hash of the bytes at its data pointer (over the
tensor's true size, as this library's parser reports it).

Every expected output in the fixture comes from the reference build
(src/quantization.cpp compiled unmodified with its build.sh flags, AVX2+FMA
branch).  The one exception is Q8_0 dequantization, which the reference only
does inline (``out = qs[j] * d``, src/forward_pass.cpp:379-384): its expected
values are the reference's own fp16 decoder output times the int8 value, one
float32 multiply, computed here with numpy.

Inputs are seeded (numpy PCG64) and include edge blocks: special fp16 scales
(zero, subnormal, max, Inf, NaN), extreme quant codes, every Q5_K 6-bit
scale/min code, negative Q6_K scales, and the constant blocks of the
reference's own GGUF fixture (tests/test_gguf_binary_mmap.py:62,81 in the
reference: Q8_0 d=0x3C00 with qs=1, Q4_0 d=0x3C00 with nibbles 0x11).
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from nexusllm_b200 import synth  # noqa: E402
from nexusllm_b200.formats import DataType  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden", "golden.npz")
OUT_GGUF = os.path.join(ROOT, "tests", "golden", "gguf_ref.json")

# fp16 bit patterns whose decoding the reference treats specially or that sit
# on the edges of the format
FP16_KAT = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x7C00, 0xFC00, 0x7E00,
            0xFFFF, 0x8001, 0x3555, 0xC000, 0x83FF, 0xFBFF]
D_SPECIAL = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x7C00, 0xFC00, 0x7E00, 0xBC00]

GEMV_SHAPES = {
    DataType.GGUF_Q4_0: [(1, 32), (37, 96), (40, 512), (67, 1024), (3, 4096)],
    DataType.GGUF_Q8_0: [(1, 32), (37, 96), (40, 512), (67, 1024), (3, 4096)],
    DataType.GGUF_Q5_K: [(1, 256), (37, 768), (19, 2048), (3, 4096)],
    DataType.GGUF_Q6_K: [(1, 256), (37, 768), (19, 2048), (3, 4096)],
    DataType.FP16: [(1, 8), (37, 100), (24, 520), (16, 33), (3, 4096)],
}


def _set_d(a: np.ndarray, off: int, vals) -> None:
    v = np.asarray(vals, np.uint16)
    a[: len(v), off] = (v & 0xFF).astype(np.uint8)
    a[: len(v), off + 1] = (v >> 8).astype(np.uint8)


def edge_blocks(dt: DataType, seed: int) -> np.ndarray:
    """Seeded random blocks with edge cases written into the first rows."""
    per = 32 if dt in (DataType.GGUF_Q4_0, DataType.GGUF_Q8_0) else 256
    nb = 64
    a = synth.blocks_numpy(dt, 1, nb * per, seed).reshape(nb, -1).copy()
    if dt == DataType.GGUF_Q4_0:
        _set_d(a, 0, D_SPECIAL)
        a[11, 2:] = 0x00
        a[12, 2:] = 0xFF
        a[13, 0:2] = [0x00, 0x3C]
        a[13, 2:] = 0x11  # the reference fixture's Q4_0 block (value -7)
        a[14, 2:] = np.arange(16, dtype=np.uint8) * 17
    elif dt == DataType.GGUF_Q8_0:
        _set_d(a, 0, D_SPECIAL)
        a[11, 2:] = np.uint8(127)
        a[12, 2:] = np.int8(-127).view(np.uint8)
        a[13, 2:] = np.int8(-128).view(np.uint8)
        a[14, 0:2] = [0x00, 0x3C]
        a[14, 2:] = 1  # the reference fixture's Q8_0 block
        a[15, 2:] = np.arange(-128, 128, 8).astype(np.int8).view(np.uint8)
    elif dt == DataType.GGUF_Q5_K:
        _set_d(a, 0, D_SPECIAL)          # d
        _set_d(a[11:], 2, D_SPECIAL)     # dmin
        a[22, 4:16] = 0xFF               # every scale and min = 63 with high bits
        a[23, 4:16] = 0x00
        a[24, 4:16] = [0x3F, 0x7F, 0xBF, 0xFF, 0x00, 0x40, 0x80, 0xC0, 0x0F, 0xF0, 0x5A, 0xA5]
        a[25, 16:48] = 0xFF
        a[26, 16:48] = 0x00
        a[27, 16:48] = 0xAA
        a[28, 16:48] = 0x55
        a[29, 48:] = 0xFF
        _set_d(a[30:], 2, [0x0001, 0x0200, 0x03FF, 0x8001])  # dmin subnormal
    else:  # Q6_K
        _set_d(a, 208, D_SPECIAL)
        a[11, 192:208] = np.int8(-128).view(np.uint8)
        a[12, 192:208] = np.uint8(127)
        a[13, 192:208] = np.int8(-1).view(np.uint8)
        a[14, 0:192] = 0xFF              # v = 31 everywhere
        a[15, 0:192] = 0x00              # v = -32 everywhere
        a[16, 128:192] = 0xAA
        a[17, 128:192] = 0x55
    return a.reshape(-1)


# INT4-AWQ GEMV cases (rows, cols, group_size, with zeros) and FP8 shapes.
INT4_SHAPES = [(1, 128, 128, True), (37, 256, 32, True), (16, 4096, 128, True), (5, 1000, 8, True),
               (3, 96, 32, False), (4, 200, 40, True), (2, 64, 64, False)]
FP8_SHAPES = [(1, 8), (37, 100), (24, 512), (16, 33), (3, 4096), (5, 16384)]


def int4_fp8(ref, g) -> None:
    """QuantizationKernel::fused_gemv_int4 / fused_gemv_fp8 and their
    dequantizers (src/quantization.cpp:12-68,102-262), from the reference build."""
    rng = np.random.default_rng(9500)
    codes = np.arange(256, dtype=np.uint8)
    g["fp8/codes"] = codes
    g["fp8/codes_x1"] = ref.dequantize_fp8_e4m3(codes, 256, 1.0)
    g["fp8/codes_x037"] = ref.dequantize_fp8_e4m3(codes, 256, 0.37)
    packed = rng.integers(0, 2**32, size=125, dtype=np.uint64).astype(np.uint32)
    sc = rng.uniform(0.001, 0.02, size=(1000 + 31) // 32).astype(np.float32)  # one scale per 32 elements
    zr = rng.integers(0, 16, size=sc.size).astype(np.float32)
    g["int4deq/packed"], g["int4deq/scales"], g["int4deq/zeros"] = packed, sc, zr
    g["int4deq/out_g32"] = ref.dequantize_int4_awq(packed, sc, zr, 1000, 32)
    s8 = np.random.default_rng(9501).uniform(-1, 1, 125).astype(np.float32)
    g["int4deq/scales_g8"] = s8
    g["int4deq/out_g8_nozero"] = ref.dequantize_int4_awq(packed, s8, None, 1000, 8)
    for j, (rows, cols, gs, with_z) in enumerate(INT4_SHAPES):
        r = np.random.default_rng(9600 + j)
        W = r.integers(0, 2**32, size=rows * cols // 8, dtype=np.uint64).astype(np.uint32)
        ng = rows * cols // gs
        scales = r.uniform(0.001, 0.02, size=ng).astype(np.float32)
        zeros = r.integers(0, 16, size=ng).astype(np.float32) if with_z else None
        x = synth.activations_numpy(1, cols, 9700 + j)[0]
        key = f"int4gemv/{rows}x{cols}g{gs}{'z' if with_z else ''}"
        g[key + "/W"], g[key + "/x"], g[key + "/scales"] = W, x, scales
        if with_z:
            g[key + "/zeros"] = zeros
        g[key + "/y"] = ref.gemv_int4(W, x, scales, zeros, rows, cols, gs)
    for j, (rows, cols) in enumerate(FP8_SHAPES):
        r = np.random.default_rng(9800 + j)
        W = r.integers(0, 256, size=rows * cols, dtype=np.uint8)  # every code, NaN codes included
        x = synth.activations_numpy(1, cols, 9900 + j)[0]
        key = f"fp8gemv/{rows}x{cols}"
        g[key + "/W"], g[key + "/x"] = W, x
        g[key + "/y"] = ref.gemv_fp8(W, x, rows, cols, 0.0625)


def layer_ops(ref, g) -> None:
    """TransformerOps::rmsnorm / swiglu (include/transformer_ops.hpp:23-44,86-95),
    the decode layer's ops around the GEMV, from the reference build."""
    r = np.random.default_rng(9990)
    for j, (n, scale, eps) in enumerate([(4096, 1.0, 1e-5), (512, 300.0, 1e-6), (33, 1e-3, 1e-5), (14336, 7.0, 1e-5)]):
        x = (r.standard_normal(n) * scale).astype(np.float32)
        w = (1.0 + 0.1 * r.standard_normal(n)).astype(np.float32)
        key = f"ops/rmsnorm/{j}"
        g[key + "/x"], g[key + "/w"], g[key + "/eps"] = x, w, np.array([eps], np.float32)
        g[key + "/out"] = ref.rmsnorm(x, w, eps)
        g[key + "/out_now"] = ref.rmsnorm(x, None, eps)
    gate = np.concatenate([(r.standard_normal(4000) * 6).astype(np.float32),
                           np.array([-100, -88, -87, 0, -0.0, 80, 100, 1e-30, -1e-30], np.float32)])
    up = r.standard_normal(gate.size).astype(np.float32)
    g["ops/swiglu/g"], g["ops/swiglu/u"] = gate, up
    g["ops/swiglu/out"] = ref.swiglu(gate, up)


def main() -> None:
    ref = oracle.reference()
    g = {}
    f16 = np.array(FP16_KAT, np.uint16)
    g["fp16/kat_in"] = f16
    g["fp16/kat_out"] = np.array([ref.fp16_to_fp32(int(h)) for h in FP16_KAT], np.float32)
    table = np.array([ref.fp16_to_fp32(h) for h in range(65536)], np.float32)
    g["fp16/table_sha256"] = np.frombuffer(hashlib.sha256(table.tobytes()).digest(), np.uint8)

    # dequantization
    for i, dt in enumerate([DataType.GGUF_Q4_0, DataType.GGUF_Q8_0, DataType.GGUF_Q5_K, DataType.GGUF_Q6_K]):
        W = edge_blocks(dt, 9000 + i)
        per = 32 if dt in (DataType.GGUF_Q4_0, DataType.GGUF_Q8_0) else 256
        nbytes = 18 if dt == DataType.GGUF_Q4_0 else 34 if dt == DataType.GGUF_Q8_0 else 176 if dt == DataType.GGUF_Q5_K else 210
        nb = W.size // nbytes
        if dt == DataType.GGUF_Q8_0:
            blk = W.reshape(nb, 34)
            d = np.array([ref.fp16_to_fp32(int(h)) for h in blk[:, 0:2].copy().view(np.uint16).reshape(-1)], np.float32)
            out = (blk[:, 2:].view(np.int8).astype(np.float32) * d[:, None]).astype(np.float32).reshape(-1)
        else:
            out = ref.dequantize(int(dt), W, nb * per)
        g[f"deq/{int(dt)}/W"] = W
        g[f"deq/{int(dt)}/out"] = out
    fp16_all = np.concatenate([np.array(FP16_KAT + D_SPECIAL, np.uint16),
                               synth.blocks_numpy(DataType.FP16, 1, 230, 9010)])
    g["deq/1/W"] = fp16_all
    g["deq/1/out"] = ref.dequantize(1, fp16_all, fp16_all.size)

    # GEMV
    for dt, shapes in GEMV_SHAPES.items():
        for j, (rows, cols) in enumerate(shapes):
            seed = 9100 + 10 * int(dt) + j
            W = synth.blocks_numpy(dt, rows, cols, seed)
            x = synth.activations_numpy(1, cols, seed + 5000)[0]
            y = ref.gemv(int(dt), W, x, rows, cols)
            key = f"gemv/{int(dt)}/{rows}x{cols}"
            g[key + "/W"] = W
            g[key + "/x"] = x
            g[key + "/y"] = y
    # the reference's own GGUF fixture blocks (constant), as whole matrices
    q8 = np.tile(np.concatenate([[0x00, 0x3C], np.ones(32, np.uint8)]).astype(np.uint8), 64 * 2)
    q4 = np.tile(np.concatenate([[0x00, 0x3C], np.full(16, 0x11, np.uint8)]).astype(np.uint8), 128 * 2)
    for dt, W, rows, cols in [(DataType.GGUF_Q8_0, q8, 64, 64), (DataType.GGUF_Q4_0, q4, 128, 64)]:
        x = synth.activations_numpy(1, cols, 9999)[0]
        key = f"gemv/{int(dt)}/fixture{rows}x{cols}"
        g[key + "/W"] = W
        g[key + "/x"] = x
        g[key + "/y"] = ref.gemv(int(dt), W, x, rows, cols)

    int4_fp8(ref, g)
    layer_ops(ref, g)
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: {len(g)} arrays, {os.path.getsize(OUT)} bytes")


def gguf_fixture() -> None:
    import json
    import tempfile

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import gguf_cases
    from nexusllm_b200 import gguf

    out = {}
    with tempfile.TemporaryDirectory() as d:
        for case, (path, tensors) in gguf_cases.build(d).items():
            names = [t[0] for t in tensors] + gguf_cases.ALIASES
            hb = []
            with gguf.GGUFFile(path) as f:  # our sizes; 0 where our parser has no such tensor
                for n in names:
                    try:
                        hb.append(f.tensors[f.find(n)]["bytes"])
                    except Exception:
                        hb.append(0)
            st, model, res = oracle.reference_gguf_load(path, names, hb)
            out[case] = {"status": st, "model": model, "names": names, "hash_bytes": hb, "tensors": res}
    with open(OUT_GGUF, "w") as fh:
        json.dump(out, fh, indent=1, sort_keys=True)
    print(f"wrote {OUT_GGUF}")


if __name__ == "__main__":
    if sys.argv[1:] == ["gguf"]:
        gguf_fixture()
    else:
        main()
