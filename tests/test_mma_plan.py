"""CPU checks of the batched tensor-core path's index arithmetic
(nexusllm_b200/csrc/mma_kernels.cuh, run_gemm_tc in nexus_gpu.cu), restated in
Python before any GPU run:

* the weight order q4_unit_f16 writes into an A stage, decoded here from the
  raw bytes exactly as the kernel's word selection and nibble masks do, is the
  permutation q4_perm_src that mma_xprep_kernel applies to x, so A . B equals
  W . x term for term;
* the stream-K split covers every (tile, chunk) once, gives each CTA at most
  two shared tiles, and the fix-up reads exactly the partial-sum slots the
  sharing CTAs wrote;
* shared-memory offsets, alignments and the copy sizes fit the hardware limits.
"""
import numpy as np
import pytest

# ---- constants of mma_kernels.cuh
ROWS, RAW_K, RAW_ROW_BYTES, UNIT_K = 128, 256, 144, 64
RAW_STAGES, A_STAGES, MAX_B_STAGES, MAX_TOKENS = 5, 3, 12, 64
ACC_COLS, A_STAGE_COLS, TMEM_COLS, B_RING_BYTES = MAX_TOKENS, 128, 512, 96 * 1024
SMEM_B = 0
SMEM_RAW = SMEM_B + B_RING_BYTES
SMEM_BAR = SMEM_RAW + RAW_STAGES * ROWS * RAW_ROW_BYTES
BAR_COUNT = 2 * RAW_STAGES + 2 * A_STAGES + 2 * MAX_B_STAGES + 5
SMEM_BYTES = SMEM_BAR + 8 * BAR_COUNT + 16 + 1024


def perm_src(p, odd):
    """q4_perm_src: element of a 32-weight block stored at K position p."""
    i, m = p >> 3, p & 7
    sel = ((m >> 2) & 1) + 2 * (m & 1)
    if odd:
        byte = 4 * i + sel
    else:
        byte = (sel if sel < 2 else 12 + sel) if i == 0 else 4 * i - 2 + sel
    return byte + (16 if m & 2 else 0)


def perm_dst(s, odd):
    """q4_perm_dst: K position of element s of a block."""
    hi, byte = s >> 4, s & 15
    if odd:
        i, sel = byte >> 2, byte & 3
    elif byte < 2 or byte > 13:
        i, sel = 0, (byte if byte < 2 else byte - 12)
    else:
        i, sel = (byte + 2) >> 2, (byte + 2) & 3
    return 8 * i + ((sel >> 1) | (hi << 1) | ((sel & 1) << 2))


def test_perm_is_a_bijection_and_dst_inverts_it():
    for odd in (0, 1):
        assert sorted(perm_src(p, odd) for p in range(32)) == list(range(32))
        for p in range(32):
            assert perm_dst(perm_src(p, odd), odd) == p


def scale_bits(h):
    """q4_scale_h2's fp16 bits of a Q4_0 scale (one half)."""
    e, m = h & 0x7C00, h & 0x3FF
    sub = (h & 0x8000) | (512 + (m >> 1) + (m & (m >> 1) & 1))
    return 0 if e == 0x7C00 else (sub if e == 0 else h)


def test_scale_decode_matches_reference_decoder_rounded_to_fp16():
    # NexusLLM's decoder: ((h & 0x7fff) << 13) + (0x70 << 23), sign kept, exponent 0x1f -> +0
    for h in range(1 << 16):
        if (h & 0x7C00) == 0x7C00:
            want = np.float16(0.0)
        else:
            bits = (((h & 0x7FFF) << 13) + (0x70 << 23)) | ((h & 0x8000) << 16)
            want = np.float32(np.array([bits], dtype=np.uint32).view(np.float32)[0]).astype(np.float16)
        got = np.array([scale_bits(h)], dtype=np.uint16).view(np.float16)[0]
        assert got.tobytes() == np.float16(want).tobytes(), hex(h)


def _decode_word(w):
    """q4_word_f16's element order: the 8 nibbles of w as (code, byte, high)."""
    b = [(w >> (8 * k)) & 0xFF for k in range(4)]
    lo = lambda k: (b[k] & 15, k, 0)  # noqa: E731
    hi = lambda k: (b[k] >> 4, k, 1)  # noqa: E731
    return [lo(0), lo(2), hi(0), hi(2), lo(1), lo(3), hi(1), hi(3)]


def _unit_codes(row, U):
    """Codes of unit U of one 144-byte raw row in A order, decoded the way
    q4_unit_f16 selects words: g = 12 little-endian words of bytes 32U..32U+47."""
    g = [int.from_bytes(bytes(row[32 * U + 4 * k: 32 * U + 4 * k + 4]), "little") for k in range(12)]
    w0 = ((g[U] >> 16) & 0xFFFF) | ((g[U + 4] & 0xFFFF) << 16)  # __byte_perm(g[U], g[U+4], 0x5432)
    words = [w0, g[U + 1], g[U + 2], g[U + 3]] + [g[U + 5 + i] for i in range(4)]
    scales = [g[U] & 0xFFFF, g[U + 4] >> 16]
    out = []
    for j, w in enumerate(words):
        for code, _byte, _hi in _decode_word(w):
            out.append((code, scales[j // 4]))
    return out


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_unit_decode_matches_x_permutation(seed):
    rng = np.random.default_rng(seed)
    row = rng.integers(0, 256, RAW_ROW_BYTES, dtype=np.uint8)  # 8 Q4_0 blocks
    # reference meaning of the row: element e of block b has code
    # lo/hi nibble of qs[e % 16], scale bytes 0..1 of the block
    blocks = [row[18 * b: 18 * b + 18] for b in range(8)]
    for U in range(4):
        got = _unit_codes(row, U)
        assert len(got) == UNIT_K
        for p in range(UNIT_K):
            blk = 2 * U + (p >> 5)
            e = perm_src(p & 31, blk & 1)  # the x element mma_xprep_kernel puts at this K position
            qs = blocks[blk][2:]
            want_code = (qs[e] & 15) if e < 16 else (qs[e - 16] >> 4)
            want_scale = int(blocks[blk][0]) | (int(blocks[blk][1]) << 8)
            assert got[p] == (want_code, want_scale), (U, p)


def test_unit_reads_stay_in_row_and_are_conflict_free():
    for U in range(4):
        lo, hi = 32 * U, 32 * U + 48
        assert lo % 16 == 0 and hi <= RAW_ROW_BYTES
    # 16-byte loads of 8 consecutive rows at a 144-byte pitch: a quarter warp
    # covers 32 distinct banks
    for U in range(4):
        banks = set()
        for r in range(8):
            base = (r * RAW_ROW_BYTES + 32 * U) // 4
            banks |= {(base + k) % 32 for k in range(4)}
        assert len(banks) == 32


def test_tensor_memory_columns():
    assert ACC_COLS + A_STAGE_COLS * A_STAGES <= TMEM_COLS
    for sa in range(A_STAGES):
        for U in range(4):
            col = ACC_COLS + A_STAGE_COLS * sa + 32 * U
            assert col + 32 <= ACC_COLS + A_STAGE_COLS * (sa + 1)  # two 16-column stores stay in the stage
            for ks in range(UNIT_K // 16):
                assert col + 8 * ks + 8 <= col + 32  # each MMA reads 8 columns of the unit
    assert ACC_COLS + A_STAGE_COLS * A_STAGES <= TMEM_COLS


class Ring:
    """RingPos of mma_kernels.cuh."""

    def __init__(self, n):
        self.n, self.stage, self.phase = n, 0, 0

    def next(self):
        self.stage += 1
        if self.stage == self.n:
            self.stage, self.phase = 0, self.phase ^ 1


@pytest.mark.parametrize("n", [3, 5, 12, 7])
def test_ring_positions_match_division(n):
    r = Ring(n)
    for i in range(200):
        assert (r.stage, r.phase) == (i % n, (i // n) & 1)
        if i >= n:  # the wait for the previous use of the stage
            assert r.phase ^ 1 == ((i // n) - 1) & 1
        r.next()


def sk_lo(total, G, b):
    return b * total // G


def sk_owner(total, G, L):
    b = L * G // total
    while b + 1 < G and sk_lo(total, G, b + 1) <= L:
        b += 1
    while b > 0 and sk_lo(total, G, b) > L:
        b -= 1
    return b


def tc_ctas(sms, tiles, n_chunks):
    """Mirror of tc_ctas: a tile-aligned split (s CTAs a tile, s dividing the
    chunks, >= 2 chunks each) when it keeps >= 85 % of the SMs busy, else
    stream-K over every SM with >= 2 chunks a CTA."""
    for s in range(n_chunks // 2, 0, -1):
        if n_chunks % s == 0 and tiles * s <= sms:
            if tiles * s * 100 >= 85 * sms:
                return tiles * s
            break
    return max(1, min(sms, tiles * n_chunks // 2))


def plan(sms, rows, cols):
    n_chunks = cols // RAW_K
    tiles = (rows + ROWS - 1) // ROWS
    total = tiles * n_chunks
    G = tc_ctas(sms, tiles, n_chunks)
    return tiles, n_chunks, total, G


@pytest.mark.parametrize("rows,cols", [(128256, 4096), (14336, 4096), (4096, 14336), (1024, 4096), (4096, 4096),
                                       (128, 256), (300, 4096), (1000, 1024), (28672, 8192), (8192, 28672),
                                       (129, 512), (4096, 1024)])
@pytest.mark.parametrize("sms", [148, 132, 7])
def test_stream_k_partition(rows, cols, sms):
    tiles, nc, total, G = plan(sms, rows, cols)
    assert 1 <= G <= sms and G <= total
    seen = np.zeros((tiles, nc), dtype=np.int32)
    writers = {}  # tile -> [(cta, slot)]
    for b in range(G):
        lo, hi = sk_lo(total, G, b), sk_lo(total, G, b + 1)
        assert hi > lo  # every CTA has work
        assert total // G <= hi - lo <= -(-total // G)
        t0, t1 = lo // nc, (hi - 1) // nc
        shared = 0
        for t in range(t0, t1 + 1):
            c0 = lo - t * nc if t == t0 else 0
            c1 = hi - t * nc if t == t1 else nc
            assert 0 <= c0 < c1 <= nc
            seen[t, c0:c1] += 1
            if not (c0 == 0 and c1 == nc):
                shared += 1
                writers.setdefault(t, []).append((b, 2 * b + (0 if t == t0 else 1)))
        assert shared <= 2
    assert (seen == 1).all()
    slots = [s for w in writers.values() for _, s in w]
    assert len(slots) == len(set(slots)) and max(slots, default=0) < 2 * G
    for t, w in writers.items():
        bf, bl = sk_owner(total, G, t * nc), sk_owner(total, G, (t + 1) * nc - 1)
        assert [b for b, _ in w] == list(range(bf, bl + 1))  # contiguous CTAs, in order
        # the fix-up's slot formula
        for b, s in w:
            tb0 = sk_lo(total, G, b) // nc
            assert s == 2 * b + (0 if t == tb0 else 1)
        assert len(w) >= 2  # a shared tile has at least two writers; the last arrival sees bl - bf
    # tiles nobody shares are written directly by their one CTA
    for t in range(tiles):
        if t not in writers:
            assert sk_owner(total, G, t * nc) == sk_owner(total, G, (t + 1) * nc - 1)


def b_stages(NB):
    return min(MAX_B_STAGES, B_RING_BYTES // (NB * 512))


def test_shared_memory_layout():
    assert SMEM_BYTES <= 227 * 1024
    for off in (SMEM_B, SMEM_RAW):
        assert off % 1024 == 0  # swizzle atoms and TMA destinations
    assert (ROWS * RAW_ROW_BYTES) % 128 == 0
    for NB in (16, 32, 48, 64):
        n = b_stages(NB)
        assert 2 <= n <= MAX_B_STAGES and n * NB * 512 <= B_RING_BYTES
        assert (NB * 128) % 1024 == 0  # every x tile starts on a swizzle atom
        # 4 unit tiles per chunk stage; descriptor start field (address / 16) stays in 14 bits
        assert (SMEM_B + n * NB * 512 + 1024 * 64) // 16 < (1 << 14)
    assert SMEM_BAR % 8 == 0
    # transaction counts fit the mbarrier's tx field
    assert ROWS * RAW_ROW_BYTES < (1 << 20) and 4 * MAX_TOKENS * 128 < (1 << 20)
    # raw chunk x coordinates are whole 144-byte multiples: 16-byte aligned
    assert RAW_ROW_BYTES % 16 == 0


@pytest.mark.parametrize("NB", [16, 32, 48, 64])
def test_fixup_covers_tile_once(NB):
    n4 = NB * (ROWS // 4)
    seen = np.zeros((NB, ROWS), dtype=np.int32)
    for tid in range(256):
        for f in range(tid, n4, 256):
            tok = f // (ROWS // 4)
            for e in range(4):
                seen[tok, 4 * (f % (ROWS // 4)) + e] += 1
    assert (seen == 1).all()
    # partial slots are float4-aligned: slot * NB * 128 floats
    assert (NB * ROWS * 4) % 16 == 0


@pytest.mark.parametrize("M", [16, 17, 33, 64, 80, 128])
def test_token_groups(M):
    groups = [min(MAX_TOKENS, M - g0) for g0 in range(0, M, MAX_TOKENS)]
    for Mg in groups:
        NB = (Mg + 15) // 16 * 16
        assert NB % 16 == 0 and 16 <= NB <= MAX_TOKENS  # UMMA N for M = 128
        tcols = 32 if NB <= 32 else 64
        assert NB <= tcols
        assert (NB // 2) % 4 == 0  # each dequant group reads its half of the columns 4 at a time
