"""CPU check of gemv_m1_kernel's index arithmetic (nexusllm_b200/csrc/gemv_kernels.cuh).

Restates, in Python, how the kernel splits rows over CTAs, row groups and
K-chunks, which byte ranges the producer warp bulk-copies (and tail-copies)
from global memory into each shared-memory stage, and which shared-memory
bytes the consumer decoders read.  For every configuration shape and a set of
ragged ones it asserts that every global read stays inside the weight matrix,
every bulk copy is 16-byte aligned with a size that is a multiple of 16, every
shared-memory write and read stays inside its row slot and the dynamic
shared-memory allocation, and the decoders read exactly the bytes the copies
delivered.  The format constants are parsed from the kernel header, so the
check follows the kernel when they change.
"""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "nexusllm_b200", "csrc", "gemv_kernels.cuh")
SMS = 148
SMEM_OPTIN = 232448  # B200 max dynamic shared memory per block (227 KB)


def _fmt_constants():
    text = open(HDR).read()
    out = {}
    for name in ("FmtQ4_0", "FmtQ8_0", "FmtQ5_K", "FmtQ6_K", "FmtF16"):
        body = re.search(r"struct %s \{(.*?)\};" % name, text, re.S).group(1)
        vals = dict(re.findall(r"(k\w+) = (\w+)", body))
        out[name] = {k: (v == "true") if v in ("true", "false") else int(v) for k, v in vals.items()}
    return out


FMT = _fmt_constants()
CONSUMER_WARPS = 8


def c16(v):
    return (v + 15) // 16 * 16


def layout(f, K):
    rg = CONSUMER_WARPS * f["kRows"]
    chunk = f["kChunkWI"] // f["kWIPerBlock"] * f["kBlockBytes"]
    stride = c16(chunk + 32)
    stage = rg * stride
    xb = (K // 32) * 80 if f["kIntX"] else K * 4
    xb = (xb + 127) // 128 * 128
    smem = 128 + xb + f["kStages"] * stage + 128
    return rg, chunk, stride, stage, xb, smem


def reads(name, base, j):
    """(first, last) shared byte offsets a decoder touches for work item j
    whose data starts at `base` (block base for Q4_0/Q8_0/FP16, super-block
    base for the K-quants); plus the used byte range."""
    if name == "FmtQ4_0":
        q = base + 2
        return [(base, base + 1), (q & ~3, (q & ~3) + 19)], (base, base + 17)
    if name == "FmtQ8_0":
        q = base + 2
        return [(base, base + 1), (q & ~3, (q & ~3) + 35)], (base, base + 33)
    if name == "FmtQ5_K":
        sub = j & 7
        return [(base, base + 15), (base + 16 + 4 * sub, base + 19 + 4 * sub),
                (base + 48 + 16 * sub, base + 63 + 16 * sub)], (base, base + 175)
    if name == "FmtQ6_K":
        p = j & 7
        a, b = base + 16 * p, base + 128 + 8 * p
        return [((a & ~3), (a & ~3) + 19), ((b & ~3), (b & ~3) + 11), (base + 192 + 2 * p, base + 193 + 2 * p),
                (base + 208, base + 209)], (base, base + 209)
    return [((base & ~3), (base & ~3) + 35)], (base, base + 31)


def simulate(name, N, K, ctas=None):
    f = FMT[name]
    rg, chunk, stride, stage, xb, smem = layout(f, K)
    assert smem <= SMEM_OPTIN, (name, K, smem)
    per = 16 if name == "FmtF16" else 32
    nwi = K // per
    rb = {"FmtQ4_0": K // 32 * 18, "FmtQ8_0": K // 32 * 34, "FmtQ5_K": K // 256 * 176,
          "FmtQ6_K": K // 256 * 210, "FmtF16": K * 2}[name]
    total = N * rb
    floor16 = total & ~15
    G = min(SMS, N)
    nchunks = (nwi + f["kChunkWI"] - 1) // f["kChunkWI"]
    for c in (ctas if ctas is not None else range(G)):
        if c >= G:
            continue
        rb0, re0 = N * c // G, N * (c + 1) // G
        assert re0 > rb0
        ngroups = (re0 - rb0 + rg - 1) // rg
        for g in range(ngroups):
            r0 = rb0 + g * rg
            nr = min(rg, re0 - r0)
            reff = (nr + CONSUMER_WARPS - 1) // CONSUMER_WARPS
            assert reff <= f["kRows"]
            for ch in range(nchunks):
                nwi_c = min(f["kChunkWI"], nwi - ch * f["kChunkWI"])
                cbytes = nwi_c // f["kWIPerBlock"] * f["kBlockBytes"]
                coff = ch * chunk
                tx = 0
                for rl in range(nr):
                    start = (r0 + rl) * rb + coff
                    end = start + cbytes
                    assert end <= (r0 + rl + 1) * rb <= total
                    a = start & ~15
                    bend = min((end + 15) & ~15, floor16)
                    slot_lo, slot_hi = rl * stride, (rl + 1) * stride
                    if bend > a:
                        n = bend - a
                        assert a % 16 == 0 and n % 16 == 0 and 0 <= a and bend <= total
                        assert slot_lo + n <= slot_hi
                        tx += n
                    covered_hi = max(bend, a)
                    for pos in range(max(a, bend), end, 2):
                        assert pos % 2 == 0 and pos + 2 <= total
                        assert slot_lo + (pos - a) + 2 <= slot_hi
                        covered_hi = pos + 2
                    delivered = (slot_lo, slot_lo + (covered_hi - a))  # bytes present in smem
                    delta = start & 15
                    if name == "FmtQ5_K":
                        assert delta == 0
                    for j in range(nwi_c):
                        off = j * f["kBlockBytes"] if f["kWIPerBlock"] == 1 else (j // 8) * f["kBlockBytes"]
                        base = slot_lo + delta + off
                        rr, used = reads(name, base, j)
                        for lo, hi in rr:
                            assert slot_lo <= lo and hi < slot_hi, (name, N, K, c, g, ch, rl, j)
                        assert delivered[0] <= used[0] and used[1] < delivered[1], (name, N, K, rl, j)
                        if name == "FmtQ5_K":
                            assert (base + 48) % 16 == 0
                        gj = ch * f["kChunkWI"] + j
                        if f["kIntX"]:
                            assert gj * 64 + 63 < (K // 32) * 64
                            assert (K // 32) * 64 + gj * 16 + 15 < xb
                        else:
                            assert gj * 64 + 63 < xb
                assert tx < (1 << 20)
    return True


CONFIG_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (11008, 4096), (4096, 11008),
                 (8192, 8192), (1024, 8192), (28672, 8192), (8192, 28672), (128256, 4096), (128256, 8192)]
RAGGED = [(1, 256), (3, 512), (7, 768), (37, 1024), (149, 2048), (150, 256), (300, 4096), (4097, 4096),
          (513, 11008), (64, 2816)]


@pytest.mark.parametrize("name", sorted(FMT))
def test_config_shapes_in_bounds(name):
    for N, K in CONFIG_SHAPES:
        G = min(SMS, N)
        simulate(name, N, K, ctas=sorted({0, 1, G // 2, G - 2, G - 1}))


@pytest.mark.parametrize("name", sorted(FMT))
def test_ragged_shapes_in_bounds(name):
    for N, K in RAGGED:
        if name != "FmtF16" and K % 256 and name in ("FmtQ5_K", "FmtQ6_K"):
            continue
        simulate(name, N, K)


def test_q6_k_unaligned_rows_exercise_the_tail_copy():
    # K=256*3: rows of 630 bytes; with 3 rows the matrix is 1890 bytes, not a
    # multiple of 16, so the last row's last chunk needs the 2-byte tail path
    simulate("FmtQ6_K", 3, 768)
    simulate("FmtQ4_0", 1, 32)   # 18-byte matrix
    simulate("FmtQ8_0", 1, 96)   # 102-byte matrix
