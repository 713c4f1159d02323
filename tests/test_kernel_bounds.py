"""CPU check of gemv_m1_kernel's index arithmetic (nexusllm_b200/csrc/gemv_kernels.cuh)
and of the host plan that sizes it (plan_fast in nexusllm_b200/csrc/nexus_gpu.cu).

Restates, in Python, how the kernel splits rows over CTAs and stages, which
byte range the producer bulk-copies (and tail-copies) into each shared-memory
stage buffer, which shared bytes the consumer decoders read, and which x
slices and y rows each thread touches (including the plan's choice of K
segments, which may leave warps past the last row group idle).  For every configuration shape and a
set of ragged ones it asserts that every global read stays inside the weight
matrix and x, every bulk copy is 16-byte aligned with a size that is a
multiple of 16, every shared write and read stays inside its stage buffer and
the allocation, the decoders read only bytes the copies delivered, every row
slot and y index is in range, and every row gets exactly the warps of
its row group.  Constants are parsed from the kernel header so the check follows the
kernel when they change.
"""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "nexusllm_b200", "csrc", "gemv_kernels.cuh")
SMS = 148
SMEM_OPTIN = 232448  # B200 max dynamic shared memory per block (227 KB)


def _constants():
    text = open(HDR).read()
    glob = {k: int(v) for k, v in re.findall(r"constexpr int (k\w+) = (\d+);", text)}
    glob["kConsumers"] = glob["kConsumerWarps"] * 32
    glob["kSmemHeader"] = glob["kBarBytes"] + glob["kMaxSlots"] * 4 + glob["kMaxStages"] * glob["kMaxStageRows"] * 4
    fmts = {}
    for name in ("FmtQ4_0", "FmtQ8_0", "FmtQ5_K", "FmtQ6_K", "FmtF16"):
        body = re.search(r"struct %s \{(.*?)\};" % name, text, re.S).group(1)
        vals = dict(re.findall(r"(k\w+) = (\w+)", body))
        fmts[name] = {k: (v == "true") if v in ("true", "false") else int(v) for k, v in vals.items()}
    return glob, fmts


C, FMT = _constants()


def plan(name, K, rb):
    """Mirror of plan_fast<F> (nexus_gpu.cu); None when the generic kernel runs."""
    f = FMT[name]
    NW = K // f["kWIElems"]
    if NW < 32:
        return None
    W = C["kConsumerWarps"]
    Gp = f["kGroup"] if NW % f["kGroup"] == 0 else 1
    S, best = 0, None
    for c in range(1, C["kMaxSegments"] + 1):
        sw = -(-(-(-NW // c)) // Gp) * Gp
        j = -(-sw // (32 * Gp)) * Gp
        groups = W // c
        if j > C["kMaxJ"] or groups == 0:
            continue
        if groups * rb > C["kStageMaxBytes"] and c < C["kMaxSegments"]:
            continue
        cost = j / groups
        if best is None or cost < best - 1e-9:
            best, S, SW, J = cost, c, sw, j
    if S == 0:
        return None
    n_grp = W // S
    m = max(1, min(4, C["kStageTargetBytes"] // (n_grp * rb)))
    R = min(n_grp * m, C["kMaxStageRows"])
    sb = (R * rb + 32 + 15) // 16 * 16
    avail = SMEM_OPTIN - C["kSmemHeader"] - 128
    ns = min(C["kMaxStages"], avail // sb)
    while ns > 2 and ns * R * S > C["kMaxSlots"]:
        ns -= 1
    if ns < 2 or ns * R * S > C["kMaxSlots"]:
        return None
    return dict(NW=NW, S=S, SW=SW, J=J, G=Gp, R=R, sb=sb, ns=ns, smem=C["kSmemHeader"] + ns * sb)


def reads_group(name, base, wi):
    """Grouped decoders (dot_*_x2 / dot_*_x4): ranges read for the group that
    starts at work item wi, and the used byte range."""
    if name == "FmtQ4_0":
        b = base + 18 * wi
        assert b % 4 == 0
        return [(b, b + 35)], (b, b + 35)
    if name == "FmtQ8_0":
        b = base + 34 * wi
        assert b % 4 == 0
        return [(b, b + 67)], (b, b + 67)
    if name == "FmtQ5_K":
        o, h = base + 176 * (wi // 8), (wi >> 2) & 1
        assert o % 16 == 0 and wi % 4 == 0
        return [(o, o + 15), (o + 16 + 16 * h, o + 31 + 16 * h), (o + 48 + 64 * h, o + 111 + 64 * h)], (o, o + 175)
    o, h = base + 210 * (wi // 8), (wi >> 2) & 1
    assert wi % 4 == 0
    a, b, c = o + 64 * h, o + 128 + 32 * h, o + 192 + 8 * h
    return [(a & ~3, (a & ~3) + 67), (b & ~3, (b & ~3) + 35), (c & ~3, (c & ~3) + 11), (o + 208, o + 209)], \
        (o, o + 209)


def reads(name, base, wi):
    """Shared byte ranges (inclusive) a decoder touches for work item wi of a
    row whose data starts at `base`, and the used byte range."""
    if name == "FmtQ4_0":
        b = base + 18 * wi
        q = b + 2
        return [(b, b + 1), (q & ~3, (q & ~3) + 19)], (b, b + 17)
    if name == "FmtQ8_0":
        b = base + 34 * wi
        q = b + 2
        return [(b, b + 1), (q & ~3, (q & ~3) + 35)], (b, b + 33)
    if name == "FmtQ5_K":
        o, sub = base + 176 * (wi // 8), wi & 7
        assert o % 16 == 0
        return [(o, o + 15), (o + 16 + 4 * sub, o + 19 + 4 * sub), (o + 48 + 16 * sub, o + 63 + 16 * sub)], \
            (o, o + 175)
    if name == "FmtQ6_K":
        o, pr = base + 210 * (wi // 8), wi & 7
        a, b = o + 16 * pr, o + 128 + 8 * pr
        return [(a & ~3, (a & ~3) + 19), (b & ~3, (b & ~3) + 11), (o + 192 + 2 * pr, o + 193 + 2 * pr),
                (o + 208, o + 209)], (o, o + 209)
    b = base + 32 * wi
    return [(b & ~3, (b & ~3) + 35)], (b, b + 31)


ROW_BYTES = {"FmtQ4_0": lambda K: K // 32 * 18, "FmtQ8_0": lambda K: K // 32 * 34,
             "FmtQ5_K": lambda K: K // 256 * 176, "FmtQ6_K": lambda K: K // 256 * 210,
             "FmtF16": lambda K: K * 2}


def simulate(name, N, K, ctas=None):
    f = FMT[name]
    rb = ROW_BYTES[name](K)
    pl = plan(name, K, rb)
    if pl is None:
        return False
    W15 = C["kConsumerWarps"]
    assert pl["smem"] <= SMEM_OPTIN
    NW, S, SW, J, Gp, R, sb, ns = pl["NW"], pl["S"], pl["SW"], pl["J"], pl["G"], pl["R"], pl["sb"], pl["ns"]
    n_grp = W15 // S
    assert 1 <= n_grp and n_grp * S <= W15  # warps past the last row group idle
    total = N * rb
    floor16 = total & ~15
    G = min(SMS, N)
    # (segment, lane, j) -> work item: every work item of a row covered exactly once
    cover = set()
    starts = set()   # first work item of each lane group
    for sg in range(S):
        for lane in range(32):
            for j in range(C["kMaxJ"]):
                o = Gp * (lane + 32 * (j // Gp)) + (j % Gp)
                wi = sg * SW + o
                if j < J and o < SW and wi < NW:
                    assert wi not in cover
                    cover.add(wi)
                    if j % Gp == 0:
                        starts.add(wi)
                        # a group is whole whenever its first item is valid
                        assert all(o + t < SW and wi + t < NW for t in range(Gp))
                    if f["kIntX"]:
                        assert wi * 64 + 63 < (K // 32) * 64 and wi < K // 32
                    else:
                        assert wi * 16 + 15 < K
    assert cover == set(range(NW))
    if Gp > 1 and name in ("FmtQ4_0", "FmtQ8_0"):
        assert rb % 4 == 0  # block pairs start 4-byte aligned
    for c in (ctas if ctas is not None else range(G)):
        if c >= G:
            continue
        rb0, re0 = N * c // G, N * (c + 1) // G
        assert re0 > rb0
        n_st = (re0 - rb0 + R - 1) // R
        for i in range(n_st):
            r0 = rb0 + i * R
            nr = min(R, re0 - r0)
            start, end = r0 * rb, r0 * rb + nr * rb
            a = start & ~15
            bend = min((end + 15) & ~15, floor16)
            n = bend - a if bend > a else 0
            assert a % 16 == 0 and n % 16 == 0 and n <= sb and bend <= total and n < (1 << 20)
            hi = a + n
            for pos in range(max(a, bend), end, 2):
                assert pos + 2 <= total and (pos - a) + 2 <= sb
                hi = pos + 2
            delivered = hi - a
            delta = start & 15
            if name == "FmtQ5_K":
                assert delta == 0
            # every row of the stage goes to exactly one row group, the one
            # q % n_grp of its CTA-local index q; slot and counter indices in range
            seen = []
            for grp in range(n_grp):
                rl = grp - (i * R) % n_grp
                if rl < 0:
                    rl += n_grp
                while rl < nr:
                    assert (i * R + rl) % n_grp == grp
                    seen.append(rl)
                    st = i % ns
                    assert (st * R + rl) * S + (S - 1) < C["kMaxSlots"]
                    assert st * R + rl < C["kMaxStages"] * C["kMaxStageRows"]
                    assert r0 + rl < re0
                    rl += n_grp
            assert sorted(seen) == list(range(nr))
            for rl in range(nr):
                rowbase = delta + rl * rb
                for wi in (sorted(starts) if Gp > 1 else range(NW)):
                    rr, used = reads_group(name, rowbase, wi) if Gp > 1 else reads(name, rowbase, wi)
                    for lo, hi2 in rr:
                        assert 0 <= lo and hi2 < sb, (name, N, K, c, i, rl, wi)
                    assert used[1] < delivered, (name, N, K, c, i, rl, wi)
    return True


CONFIG_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (11008, 4096), (4096, 11008),
                 (8192, 8192), (1024, 8192), (28672, 8192), (8192, 28672), (128256, 4096), (128256, 8192)]
RAGGED = [(1, 1024), (3, 1024), (37, 1024), (149, 2048), (150, 4096), (300, 4096), (4097, 4096),
          (513, 11008), (64, 2816), (5, 28672), (7, 1056), (9, 3104)]


@pytest.mark.parametrize("name", sorted(FMT))
def test_config_shapes_in_bounds(name):
    ran = 0
    for N, K in CONFIG_SHAPES:
        G = min(SMS, N)
        ran += simulate(name, N, K, ctas=sorted({0, 1, G // 2, G - 2, G - 1}))
    assert ran >= 8


@pytest.mark.parametrize("name", sorted(FMT))
def test_ragged_shapes_in_bounds(name):
    for N, K in RAGGED:
        if name in ("FmtQ5_K", "FmtQ6_K") and K % 256:
            continue
        G = min(SMS, N)
        simulate(name, N, K, ctas=sorted({0, G // 2, G - 1}))


def test_fast_path_covers_the_configurations():
    for name in ("FmtQ4_0", "FmtQ8_0", "FmtQ5_K", "FmtQ6_K"):
        for N, K in CONFIG_SHAPES:
            assert plan(name, K, ROW_BYTES[name](K)) is not None, (name, K)


def test_unaligned_totals_exercise_the_tail_copy():
    # Q6_K K=1024*... rows of 840 B; N=3 -> 2520 B total, not a multiple of 16
    assert simulate("FmtQ6_K", 3, 1024)
    assert simulate("FmtQ8_0", 1, 1024)   # 1088-byte matrix
    assert simulate("FmtQ4_0", 3, 1024)   # 1728 = 108*16 -> no tail; still in bounds
