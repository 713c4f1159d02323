// mma_kernels.cuh -- batched decode (M >= 16 activation rows) on the sm_100a
// tcgen05 tensor cores, GGUF Q4_0 weights.
//
// Y[M][N] = X[M][K] . W[N][K]^T.  At M >= 16 the GEMV becomes a contraction
// with enough reuse of every weight for the tensor cores; weights still
// stream once from HBM.
//  * Work is tiles of 128 weight rows (the UMMA M) x chunks of 256 weights
//    (144 bytes a row).  A persistent grid of one CTA per SM splits the
//    tiles x chunks sequence into equal contiguous ranges (stream-K): a CTA
//    finishes whole tiles and starts or ends at most two partial ones.  The
//    CTAs sharing a tile store partial sums; the last of them to arrive (a
//    per-tile counter) adds them in CTA order, so results are deterministic,
//    all in one launch.
//  * Warp 0 streams raw Q4_0 chunks (128 rows x 144 bytes) with 2-D TMA
//    tensor copies and the matching x tiles (fp16, 128-byte swizzle,
//    straight into the UMMA operand layout) into a deeper ring of their own.
//  * Warps 2..17 dequantize: four groups of four warps, group g owning the
//    64-weight unit g of every chunk, a thread per weight row.  A thread reads
//    its row's unit (two blocks, 36 bytes) with three conflict-free 16-byte
//    shared loads and decodes the nibbles with lop3 into the fp16 "1024 + q"
//    form: exact q - 8 by one subtraction (low nibbles) or one fma with 1/16
//    (high nibbles, read as 16 q), then one fp16 rounding of (q - 8) * d.  The
//    nibbles come out in a fixed permuted order inside each block; the x
//    preparation kernel applies the same permutation to K, so the contraction
//    is unchanged.  The decode is the kernel's critical path (latency-bound
//    ALU work), hence sixteen warps.
//  * The A operand lives in tensor memory: a thread writes its row (its TMEM
//    lane) of an A stage with tcgen05.st, and the MMA reads A from there, so
//    shared memory carries only raw weights and x tiles.
//  * Warp 1 owns the tensor memory: it allocates it (accumulator and A
//    stages) and one of its threads issues tcgen05.mma (kind::f16: fp16 x
//    fp16 -> fp32, A from tensor memory, B from shared memory) for every 16
//    weights of K, releasing each operand stage with tcgen05.commit.
//  * x is carried in fp16, x * 2^-e with a per-token power of two that keeps
//    the token inside fp16 range (relative error 2^-11 per element); y = acc *
//    2^e.  Weights carry one fp16 rounding of (q - 8) * d.  Together about
//    3e-4 L2-relative on y.
//  * The dequantizing warps read the accumulator (tcgen05.ld) and write y or
//    the partial sums.
// Every mbarrier wait is bounded; a failed wait stops the CTA's work, the
// producers drain their copies in flight, and the tensor memory is freed on
// every path.  No cluster multicast anywhere.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "gemv_kernels.cuh"

namespace nexus_gpu {

constexpr int kMmaRows = 128;         // weight rows per tile (UMMA M)
constexpr int kRawK = 256;            // weights per row in one raw chunk
constexpr int kRawRowBytes = 144;     // 8 Q4_0 blocks
constexpr int kRawChunkBytes = kMmaRows * kRawRowBytes;
constexpr int kUnitK = 64;            // K per operand stage: one 128-byte swizzle row of fp16
constexpr int kUnitsPerChunk = kRawK / kUnitK;
constexpr int kRawStages = 5;
constexpr int kMaxTokens = 64;        // activation rows per launch (B columns <= 64)
// Tensor memory (512 columns x 128 lanes, the whole SM's): the fp32
// accumulator in columns [0, 64), then kAStages A stages of one chunk each
// (128 columns: 256 fp16 weights of every row, unit u in columns 32u..32u+31).
constexpr int kAccCols = kMaxTokens;
constexpr int kAStageCols = 32 * kUnitsPerChunk;
constexpr int kAStages = 3;
constexpr int kTmemCols = 512;
static_assert(kAccCols + kAStageCols * kAStages <= kTmemCols, "A stages exceed tensor memory");
// x tiles: a ring of chunk stages (4 unit tiles of NB x 128 bytes) in a fixed
// byte budget, so few tokens get a deep ring (x tiles arrive ~1 us after
// their copies are issued).
constexpr int kBRingBytes = 96 * 1024;
constexpr int kMaxBStages = 12;
// Warp 0: raw-weight and x-tile copies; warp 1: tensor memory and MMA;
// warps 2..17: dequantization and epilogue, four groups of four warps (group
// g owns unit g of every chunk; warp w may touch only tensor-memory lanes
// 32 (w % 4) .. 32 (w % 4) + 31, so each group covers the four quarters).
constexpr int kDequantWarps = 16;
constexpr int kMmaThreads = (2 + kDequantWarps) * 32;
constexpr int kDequantThreads = kDequantWarps * 32;
constexpr int kMmaSmemB = 0;
constexpr int kMmaSmemRaw = kMmaSmemB + kBRingBytes;
constexpr int kMmaSmemBar = kMmaSmemRaw + kRawStages * kRawChunkBytes;
constexpr int kMmaBarCount = 2 * kRawStages + 2 * kAStages + 2 * kMaxBStages + 5;
constexpr int kMmaSmemBytes = kMmaSmemBar + 8 * kMmaBarCount + 16 + 1024;  // + TMEM address, flags, alignment slack

struct MmaParams {
    int N, K;             // weight rows, cols
    int M, NB;            // tokens; tokens rounded up to 16 (the UMMA N)
    int tiles, n_chunks;  // row tiles; 256-weight chunks per row
    long long total;      // tiles * n_chunks
    int G;                // CTAs (gridDim.x)
    int b_stages;         // x-tile ring depth in chunks: min(kMaxBStages, kBRingBytes / (NB * 512))
    float* y;             // [M][N]
    float* partial;       // [2 G][NB][128]: partial sums of the tiles a CTA shares
    unsigned* arrivals;   // [tiles]: CTAs done with a shared tile (zeroed by mma_xprep_kernel)
    const float* xscale;  // [NB]: 2^e per token
};

// Stream-K split: CTA b owns chunks [lo(b), lo(b+1)) of the tile-major
// sequence of tiles x n_chunks.
__host__ __device__ __forceinline__ long long sk_lo(long long total, int G, int b) {
    return (long long)b * total / G;
}
// The CTA whose range holds linear chunk L (ranges are non-empty: G <= total).
__host__ __device__ __forceinline__ int sk_owner(long long total, int G, long long L) {
    int b = (int)(L * G / total);
    while (b + 1 < G && sk_lo(total, G, b + 1) <= L) ++b;
    while (b > 0 && sk_lo(total, G, b) > L) --b;
    return b;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), start address in 16-byte units.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3fffu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}
// Same with A read from tensor memory (128 lanes = rows, 8 columns = 16
// fp16 weights of K per row).
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                                uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 4 consecutive accumulator columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
    uint32_t r0, r1, r2, r3;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(taddr)
                 : "memory");
    v[0] = __uint_as_float(r0);
    v[1] = __uint_as_float(r1);
    v[2] = __uint_as_float(r2);
    v[3] = __uint_as_float(r3);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive columns of this warp's 32 lanes (one register per column).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// fp16x2 (d, d) of a Q4_0 scale with NexusLLM's decoder: normal halves are
// exact, Inf/NaN decode to +0, zero and subnormal halves (mantissa m) to
// 2^-15 (1 + m/1024), which is the fp16 subnormal 512 + m/2 ulps, rounded to
// nearest even here in integer arithmetic (m = 1023 rounds up to 2^-14).
__device__ __forceinline__ uint32_t q4_scale_h2(uint32_t h) {
    h &= 0xffffu;
    const uint32_t e = h & 0x7c00u, m = h & 0x3ffu;
    const uint32_t sub = (h & 0x8000u) | (512u + (m >> 1) + (m & (m >> 1) & 1u));
    const uint32_t b = e == 0x7c00u ? 0u : (e == 0u ? sub : h);
    return b | (b << 16);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// One 32-bit word of Q4_0 codes (bytes b0..b3, each a low and a high nibble)
// -> 8 fp16 weights (q - 8) * d in the order
//   lo(b0) lo(b2) hi(b0) hi(b2) lo(b1) lo(b3) hi(b1) hi(b3).
// "1024 + q" is an exact fp16 (0x6400 | q); the high nibbles are read in place
// as 16 q (0x6400 | 16 q = 1024 + 16 q), so q - 8 = v / 16 - 72 exactly.
__device__ __forceinline__ uint4 q4_word_f16(uint32_t w, uint32_t d2) {
    const __half2 k1032 = bits_h2(0x64086408u), kSixteenth = bits_h2(0x2c002c00u), kM72 = bits_h2(0xd480d480u);
    const __half2 d = bits_h2(d2);
    const uint32_t w8 = w >> 8;
    const __half2 l0 = __hsub2(bits_h2((w & 0x000f000fu) | 0x64006400u), k1032);
    const __half2 h0 = __hfma2(bits_h2((w & 0x00f000f0u) | 0x64006400u), kSixteenth, kM72);
    const __half2 l1 = __hsub2(bits_h2((w8 & 0x000f000fu) | 0x64006400u), k1032);
    const __half2 h1 = __hfma2(bits_h2((w8 & 0x00f000f0u) | 0x64006400u), kSixteenth, kM72);
    return make_uint4(h2_bits(__hmul2(l0, d)), h2_bits(__hmul2(h0, d)), h2_bits(__hmul2(l1, d)),
                      h2_bits(__hmul2(h1, d)));
}

// Unit U (blocks 2U and 2U+1, bytes 36U .. 36U+35) of one 144-byte raw row,
// given as the 12 words g of bytes 32U .. 32U+47 (the unit at word offset U)
// -> 32 tensor-memory columns of the row's lane (64 fp16 weights: block 2U in
// columns 0..15, block 2U+1 in 16..31).  Block 2U: scale in the low half of
// word U, codes q0 q1 in its high half, q2..q13 in words U+1..U+3, q14 q15 in
// the low half of word U+4.  Block 2U+1: scale in the high half of word U+4,
// codes in words U+5..U+8.
template <int U>
__device__ __forceinline__ void q4_unit_decode(const uint32_t (&g)[12], uint32_t (&wa)[16], uint32_t (&wb)[16]) {
    const uint32_t dA = q4_scale_h2(g[U]), dB = q4_scale_h2(g[U + 4] >> 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 o = q4_word_f16(i == 0 ? __byte_perm(g[U], g[U + 4], 0x5432) : g[U + i], dA);
        wa[4 * i] = o.x;
        wa[4 * i + 1] = o.y;
        wa[4 * i + 2] = o.z;
        wa[4 * i + 3] = o.w;
        const uint4 e = q4_word_f16(g[U + 5 + i], dB);
        wb[4 * i] = e.x;
        wb[4 * i + 1] = e.y;
        wb[4 * i + 2] = e.z;
        wb[4 * i + 3] = e.w;
    }
}

// Unit U of one row: three 16-byte shared loads of bytes 32U .. 32U+47, the
// decode, and two 16-column tensor-memory stores at columns ta + 32U.
template <int U>
__device__ __forceinline__ void q4_unit_tmem(uint32_t raw_row, uint32_t ta) {
    uint32_t g[12];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const uint4 v = lds128(raw_row + 32 * U + 16 * k);
        g[4 * k] = v.x;
        g[4 * k + 1] = v.y;
        g[4 * k + 2] = v.z;
        g[4 * k + 3] = v.w;
    }
    uint32_t wa[16], wb[16];
    q4_unit_decode<U>(g, wa, wb);
    tmem_st16(ta + 32 * U, wa);
    tmem_st16(ta + 32 * U + 16, wb);
}
// The same, one block at a time: block 2U's 16 columns are stored before block
// 2U+1 is decoded (fewer live registers, for kernels with more warps).
template <int U>
__device__ __forceinline__ void q4_unit_tmem_lean(uint32_t raw_row, uint32_t ta) {
    uint32_t g[12];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const uint4 v = lds128(raw_row + 32 * U + 16 * k);
        g[4 * k] = v.x;
        g[4 * k + 1] = v.y;
        g[4 * k + 2] = v.z;
        g[4 * k + 3] = v.w;
    }
    uint32_t w[16];
    const uint32_t dA = q4_scale_h2(g[U]), dB = q4_scale_h2(g[U + 4] >> 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 o = q4_word_f16(i == 0 ? __byte_perm(g[U], g[U + 4], 0x5432) : g[U + i], dA);
        w[4 * i] = o.x;
        w[4 * i + 1] = o.y;
        w[4 * i + 2] = o.z;
        w[4 * i + 3] = o.w;
    }
    tmem_st16(ta + 32 * U, w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 e = q4_word_f16(g[U + 5 + i], dB);
        w[4 * i] = e.x;
        w[4 * i + 1] = e.y;
        w[4 * i + 2] = e.z;
        w[4 * i + 3] = e.w;
    }
    tmem_st16(ta + 32 * U + 16, w);
}

// Element of a 32-weight block stored at K position p (0..31) of the block by
// q4_unit_decode: word i = p / 8 covers code bytes beta_i (block parity `odd`),
// and position m = p % 8 of the word takes byte beta_i[((m >> 2) & 1) + 2 (m & 1)],
// high nibble (element + 16) when m & 2.
__host__ __device__ __forceinline__ int q4_perm_src(int p, int odd) {
    const int i = p >> 3, m = p & 7;
    const int sel = ((m >> 2) & 1) + 2 * (m & 1);
    int byte;
    if (odd)
        byte = 4 * i + sel;
    else
        byte = i == 0 ? (sel < 2 ? sel : 12 + sel) : 4 * i - 2 + sel;
    return byte + ((m & 2) ? 16 : 0);
}

// Inverse of q4_perm_src: the K position of element s (0..31) of a block.
__host__ __device__ __forceinline__ int q4_perm_dst(int s, int odd) {
    const int hi = s >> 4, byte = s & 15;
    int i, sel;
    if (odd) {
        i = byte >> 2;
        sel = byte & 3;
    } else if (byte < 2 || byte > 13) {
        i = 0;
        sel = byte < 2 ? byte : byte - 12;
    } else {
        i = (byte + 2) >> 2;
        sel = (byte + 2) & 3;
    }
    return 8 * i + ((sel >> 1) | (hi << 1) | ((sel & 1) << 2));
}

// Bounded wait that also gives up once another thread of the CTA has.  The
// thread sleeps in try_wait (woken when the phase completes) rather than
// spinning, so waiting warps leave their schedulers to the working ones.
__device__ __forceinline__ bool mma_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_device_status, kStatusWaitTimeout);
            *abort = 1;
            return false;
        }
    }
}

// One lane of the (converged) warp: true in exactly one lane.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b32 l;\n\t"
        "elect.sync l|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// mma_wait by every lane of a warp, with one warp-wide verdict (lanes never
// part ways at the warp-synchronous steps that follow).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    const bool ok = mma_wait(bar, parity, abort);
    return __all_sync(0xffffffffu, ok);
}

// The segments of CTA b: tiles t0..t1, chunks [c0, c1) of each.
struct MmaSeg {
    int tile, c0, c1;
};
struct MmaRange {
    long long lo, hi;
    int t0, t1;
    __device__ MmaSeg seg(int t, int nc) const {
        MmaSeg s;
        s.tile = t;
        s.c0 = t == t0 ? (int)(lo - (long long)t * nc) : 0;
        s.c1 = t == t1 ? (int)(hi - (long long)t * nc) : nc;
        return s;
    }
};

// A ring position: stage index and the parity of its current use.
struct RingPos {
    uint32_t stage = 0, phase = 0;
    __device__ __forceinline__ void next(uint32_t n) {
        if (++stage == n) {
            stage = 0;
            phase ^= 1u;
        }
    }
};

__global__ void __launch_bounds__(kMmaThreads, 1)
    gemm_q4_0_mma_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                         const MmaParams P) {
    extern __shared__ uint8_t mma_smem_raw[];
    const uint32_t sraw = smem_u32(mma_smem_raw);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;  // 1024-byte aligned: swizzle atoms
    uint8_t* smem = mma_smem_raw + (sbase - sraw);
    const uint32_t bar0 = sbase + kMmaSmemBar;
    const uint32_t raw_full = bar0, raw_empty = raw_full + 8 * kRawStages;
    const uint32_t a_full = raw_empty + 8 * kRawStages, a_empty = a_full + 8 * kAStages;
    const uint32_t b_full = a_empty + 8 * kAStages, b_empty = b_full + 8 * kMaxBStages;
    const uint32_t acc_full = b_empty + 8 * kMaxBStages, acc_empty = acc_full + 8, drain = acc_empty + 8;
    const uint32_t part_done = drain + 8, decided = part_done + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMmaSmemBar + 8 * kMmaBarCount);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = P.n_chunks, NB = P.NB;
    const uint32_t nbs = (uint32_t)P.b_stages, b_unit = (uint32_t)NB * 128u, b_stage = 4u * b_unit;
    MmaRange R;
    R.lo = sk_lo(P.total, P.G, blockIdx.x);
    R.hi = sk_lo(P.total, P.G, blockIdx.x + 1);
    R.t0 = (int)(R.lo / nc);
    R.t1 = (int)((R.hi - 1) / nc);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRawStages; ++s) {
            mbar_init(raw_full + 8 * s, 1);
            mbar_init(raw_empty + 8 * s, 1);  // the MMA commit of the chunk: its dequant is done
        }
        for (int s = 0; s < kAStages; ++s) {
            mbar_init(a_full + 8 * s, kDequantWarps);  // every dequant warp, once per chunk
            mbar_init(a_empty + 8 * s, 1);
        }
        for (int s = 0; s < kMaxBStages; ++s) {
            mbar_init(b_full + 8 * s, 1);
            mbar_init(b_empty + 8 * s, 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kDequantWarps);
        mbar_init(drain, 1);
        mbar_init(part_done, kDequantWarps);
        mbar_init(decided, 1);
        *abort = 0;
        *last_flag = 0;
        fence_mbar_init();
    }
    // warp 1 allocates all of tensor memory: accumulator and A stages
    const uint32_t tcols = kTmemCols;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = __shfl_sync(0xffffffffu, *reinterpret_cast<volatile uint32_t*>(tmem_slot), 0);
    // launched with programmatic stream serialization: the prologue above
    // overlaps the x preparation; its outputs (x tiles, scales, arrival
    // counters) are read only after this wait
    pdl_wait();
    pdl_launch_dependents();

    // Warps 0 and 1 run their loops with all 32 lanes (warp-uniform values,
    // so the copy and MMA operands stay in uniform registers) and one elected
    // lane issues each copy, MMA and commit.
    if (warp == 0) {
        // ------------------------- raw weight chunks and x tiles, per chunk
        const bool leader = elect_one();
        RingPos rp, bp;
        uint32_t issued = 0;
        bool ok = true;
        for (int t = R.t0; t <= R.t1 && ok; ++t) {
            const MmaSeg S = R.seg(t, nc);
            for (int c = S.c0; c < S.c1; ++c, ++issued, rp.next(kRawStages), bp.next(nbs)) {
                if ((issued >= kRawStages && !warp_wait(raw_empty + 8 * rp.stage, rp.phase ^ 1u, abort)) ||
                    (issued >= nbs && !warp_wait(b_empty + 8 * bp.stage, bp.phase ^ 1u, abort))) {
                    ok = false;
                    break;
                }
                if (leader) {
                    mbar_arrive_expect_tx(raw_full + 8 * rp.stage, kRawChunkBytes);
                    tma_load_2d(sbase + kMmaSmemRaw + rp.stage * kRawChunkBytes, &tmW, c * kRawRowBytes,
                                t * kMmaRows, raw_full + 8 * rp.stage);
                    const uint32_t dst = sbase + kMmaSmemB + bp.stage * b_stage, bar = b_full + 8 * bp.stage;
                    mbar_arrive_expect_tx(bar, b_stage);
                    tma_load_2d(dst, &tmX, c * kRawK, 0, bar);
                    tma_load_2d(dst + b_unit, &tmX, c * kRawK + kUnitK, 0, bar);
                    tma_load_2d(dst + 2 * b_unit, &tmX, c * kRawK + 2 * kUnitK, 0, bar);
                    tma_load_2d(dst + 3 * b_unit, &tmX, c * kRawK + 3 * kUnitK, 0, bar);
                }
                __syncwarp();
            }
        }
        if (leader && *abort)  // leave no copy in flight
            for (uint32_t k = 0; k < issued && (k < kRawStages || k < nbs); ++k) {
                const uint32_t j = issued - 1 - k;
                if (k < kRawStages) mbar_wait_bounded(raw_full + 8 * (j % kRawStages), (j / kRawStages) & 1);
                if (k < nbs) mbar_wait_bounded(b_full + 8 * (j % nbs), (j / nbs) & 1);
            }
        __syncwarp();
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA
        // kind::f16: fp32 accumulator (bit 4), fp16 A and B, both K-major,
        // N = NB (bits 17..22, N/8), M = 128 (bits 24..28, M/16)
        const uint32_t idesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(kMmaRows >> 4) << 24);
        const uint32_t b_unit16 = b_unit >> 4;  // one unit tile in descriptor address units
        const bool leader = elect_one();         // the same lane issues every MMA and commit
        RingPos ap, bp, rp;
        bool ok = true;
        for (int t = R.t0, k = 0; t <= R.t1 && ok; ++t, ++k) {
            const MmaSeg S = R.seg(t, nc);
            // the previous segment's accumulator has been read out
            if (k > 0 && !warp_wait(acc_empty, (k - 1) & 1, abort)) break;
            tc_fence_after();
            for (int c = S.c0; c < S.c1; ++c, ap.next(kAStages), bp.next(nbs), rp.next(kRawStages)) {
                if (!warp_wait(a_full + 8 * ap.stage, ap.phase, abort) ||
                    !warp_wait(b_full + 8 * bp.stage, bp.phase, abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = tmem_d + kAccCols + kAStageCols * ap.stage;
                const uint64_t b0 = umma_desc_sw128(sbase + kMmaSmemB + bp.stage * b_stage);
                if (leader) {
                    // unit u: A columns 32u.., B tile u; K steps of 16: 8 A columns, 32 bytes of B
#pragma unroll
                    for (int u = 0; u < kUnitsPerChunk; ++u) {
                        const uint64_t bu = b0 + (uint64_t)(u * b_unit16);
                        umma_f16_tmem_a(tmem_d, a0 + 32 * u, bu, idesc, (c > S.c0 || u > 0) ? 1u : 0u);
                        umma_f16_tmem_a(tmem_d, a0 + 32 * u + 8, bu + 2, idesc, 1u);
                        umma_f16_tmem_a(tmem_d, a0 + 32 * u + 16, bu + 4, idesc, 1u);
                        umma_f16_tmem_a(tmem_d, a0 + 32 * u + 24, bu + 6, idesc, 1u);
                    }
                    // free the stages once these MMAs are done (every dequant warp
                    // arrived on a_full, so the raw chunk has been read too)
                    umma_commit(a_empty + 8 * ap.stage);
                    umma_commit(b_empty + 8 * bp.stage);
                    umma_commit(raw_empty + 8 * rp.stage);
                }
                __syncwarp();
            }
            if (ok && leader) umma_commit(acc_full);
            __syncwarp();
        }
        // no MMA may still read shared memory or write the accumulator when
        // the CTA tears down
        if (leader) {
            umma_commit(drain);
            mbar_wait_bounded(drain, 0);
        }
        __syncwarp();
    } else {
        // ----------------------------------------- dequantize, epilogue, fix-up
        const int dw = warp - 2, grp = dw >> 2, quarter = warp & 3;
        const int r = quarter * 32 + lane;  // accumulator lane = weight row of the tile
        const uint32_t lane_base = tmem_d + ((uint32_t)(quarter * 32) << 16);
        const bool leader = dw == 0 && lane == 0;
        constexpr int kTokSlice = kMaxTokens / 4;  // accumulator columns a group reads at most
        const int tok_lo = grp * (NB / 4), tok_hi = tok_lo + NB / 4;
        RingPos rp, ap;
        uint32_t chunks = 0, n_part = 0;
        bool ok = true;
        for (int t = R.t0, k = 0; t <= R.t1 && ok; ++t, ++k) {
            const MmaSeg S = R.seg(t, nc);
            for (int c = S.c0; c < S.c1; ++c, ++chunks, rp.next(kRawStages), ap.next(kAStages)) {
                if (!warp_wait(raw_full + 8 * rp.stage, rp.phase, abort) ||
                    (chunks >= kAStages && !warp_wait(a_empty + 8 * ap.stage, ap.phase ^ 1u, abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();  // the MMAs that read this A stage before are done
                const uint32_t raw_row = sbase + kMmaSmemRaw + rp.stage * kRawChunkBytes + (uint32_t)r * kRawRowBytes;
                const uint32_t ta = lane_base + kAccCols + kAStageCols * ap.stage;
                switch (grp) {
                    case 0: q4_unit_tmem<0>(raw_row, ta); break;
                    case 1: q4_unit_tmem<1>(raw_row, ta); break;
                    case 2: q4_unit_tmem<2>(raw_row, ta); break;
                    default: q4_unit_tmem<3>(raw_row, ta); break;
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full + 8 * ap.stage);
            }
            if (!ok || !warp_wait(acc_full, k & 1, abort)) {
                ok = false;
                break;
            }
            // epilogue: this warp's 32 accumulator lanes, this group's quarter of the tokens
            tc_fence_after();
            float v[kTokSlice];
#pragma unroll
            for (int j = 0; j < kTokSlice; j += 4)
                if (j < NB / 4) tmem_ld4(lane_base + (uint32_t)(tok_lo + j), v + j);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
            const int row = t * kMmaRows + r;
            if (S.c0 == 0 && S.c1 == nc) {
#pragma unroll
                for (int j = 0; j < kTokSlice; ++j) {
                    const int tok = tok_lo + j;
                    if (tok < tok_hi && tok < P.M && row < P.N)
                        P.y[(size_t)tok * P.N + row] = v[j] * __ldg(P.xscale + tok);
                }
                continue;
            }
            // a tile shared with other CTAs: store this CTA's partial sums
            const int slot = 2 * (int)blockIdx.x + (t == R.t0 ? 0 : 1);
            float* mine = P.partial + (size_t)slot * NB * kMmaRows;
#pragma unroll
            for (int j = 0; j < kTokSlice; ++j) {
                const int tok = tok_lo + j;
                if (tok < tok_hi) mine[(size_t)tok * kMmaRows + r] = v[j];
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) mbar_arrive(part_done);
            if (leader) {
                bool last = false;
                if (mma_wait(part_done, n_part & 1, abort)) {
                    const int bf = sk_owner(P.total, P.G, (long long)t * nc);
                    const int bl = sk_owner(P.total, P.G, (long long)(t + 1) * nc - 1);
                    last = atomicAdd(P.arrivals + t, 1u) == (unsigned)(bl - bf);
                    __threadfence();
                }
                *last_flag = last ? 1 : 0;
                mbar_arrive(decided);
            }
            if (!warp_wait(decided, n_part & 1, abort)) {
                ok = false;
                break;
            }
            ++n_part;
            if (*last_flag && !*abort) {
                // the last CTA to finish the tile adds every partial in CTA
                // order: the dequant threads over the tile's NB x 128 sums as
                // float4s; up to kFixBatch CTAs' slots are loaded before any
                // is added
                __threadfence();
                const int bf = sk_owner(P.total, P.G, (long long)t * nc);
                const int bl = sk_owner(P.total, P.G, (long long)(t + 1) * nc - 1);
                const int tid = (int)threadIdx.x - (kMmaThreads - kDequantThreads), n4 = NB * (kMmaRows / 4);
                constexpr int kFixBatch = 4;
                for (int f = tid; f < n4; f += kDequantThreads) {
                    const int tok = f / (kMmaRows / 4);
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int b0 = bf; b0 <= bl; b0 += kFixBatch) {
                        float4 p[kFixBatch];
#pragma unroll
                        for (int i = 0; i < kFixBatch; ++i) {
                            const int b = b0 + i;
                            if (b <= bl) {
                                const int sl = 2 * b + (t == (int)(sk_lo(P.total, P.G, b) / nc) ? 0 : 1);
                                p[i] = __ldcg(reinterpret_cast<const float4*>(P.partial + (size_t)sl * NB * kMmaRows) + f);
                            }
                        }
#pragma unroll
                        for (int i = 0; i < kFixBatch; ++i)
                            if (b0 + i <= bl) {
                                acc.x += p[i].x;
                                acc.y += p[i].y;
                                acc.z += p[i].z;
                                acc.w += p[i].w;
                            }
                    }
                    if (tok >= P.M) continue;
                    const float sc = __ldg(P.xscale + tok), a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int rr = t * kMmaRows + 4 * (f % (kMmaRows / 4)) + e;
                        if (rr < P.N) P.y[(size_t)tok * P.N + rr] = a4[e] * sc;
                    }
                }
            }
        }
        if (!ok) *abort = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(tcols) : "memory");
    }
}

// Four consecutive elements x[e .. e+3] of fp32 or bf16 activations; `vec`
// when the row start is 16-byte (fp32) or 8-byte (bf16) aligned.
__device__ __forceinline__ void xprep_load4(const void* x, int bf16, int vec, size_t e, float (&o)[4]) {
    if (bf16) {
        const uint16_t* p = static_cast<const uint16_t*>(x) + e;
        uint32_t w0, w1;
        if (vec) {
            const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
            w0 = u.x;
            w1 = u.y;
        } else {
            w0 = (uint32_t)__ldg(p) | ((uint32_t)__ldg(p + 1) << 16);
            w1 = (uint32_t)__ldg(p + 2) | ((uint32_t)__ldg(p + 3) << 16);
        }
        o[0] = __uint_as_float(w0 << 16);
        o[1] = __uint_as_float(w0 & 0xffff0000u);
        o[2] = __uint_as_float(w1 << 16);
        o[3] = __uint_as_float(w1 & 0xffff0000u);
    } else {
        const float* p = static_cast<const float*>(x) + e;
        if (vec) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(p));
            o[0] = f.x;
            o[1] = f.y;
            o[2] = f.z;
            o[3] = f.w;
        } else {
            for (int k = 0; k < 4; ++k) o[k] = __ldg(p + k);
        }
    }
}

// x [M][K] (fp32 or bf16) -> the B operand [NB][K] in fp16, x * 2^-e with K
// permuted inside every 32-weight block as q4_unit_decode orders the weights
// (element s of a block goes to position q4_perm_dst(s)), and the per-token
// scale 2^e.  One CTA per padded token row t < NB (rows >= M are zero); the
// first 16 K elements a thread reads stay in registers between the amax and
// the conversion (one pass over x for K <= 16384).  CTA 0 also zeroes the
// per-tile arrival counters of the GEMM.
__global__ void __launch_bounds__(256) mma_xprep_kernel(const void* __restrict__ x, int x_bf16, int vec, int M,
                                                        int NB, int K, __half* __restrict__ xp,
                                                        float* __restrict__ xscale, unsigned* __restrict__ arrivals,
                                                        int tiles) {
    constexpr int kHeld = 16;
    const int t = blockIdx.x, tid = threadIdx.x;
    __shared__ uint32_t s_max[8];
    pdl_wait();  // x may be the previous kernel's output; the previous GEMM still reads the counters
    pdl_launch_dependents();
    if (t == 0)
        for (int i = tid; i < tiles; i += blockDim.x) arrivals[i] = 0u;
    const bool real = t < M;
    const size_t row = (size_t)t * K;
    float v[kHeld][4];
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < kHeld; ++i) {
        const int e = 4 * (tid + 256 * i);
        if (real && e < K) {
            xprep_load4(x, x_bf16, vec, row + e, v[i]);
        } else {
            v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) m = max(m, __float_as_uint(v[i][k]) & 0x7fffffffu);
    }
    if (real)
        for (int e = 4 * (tid + 256 * kHeld); e < K; e += 1024) {
            float o[4];
            xprep_load4(x, x_bf16, vec, row + e, o);
            for (int k = 0; k < 4; ++k) m = max(m, __float_as_uint(o[k]) & 0x7fffffffu);
        }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((tid & 31) == 0) s_max[tid >> 5] = m;
    __syncthreads();
    uint32_t amax = 0;
    for (int w = 0; w < 8; ++w) amax = max(amax, s_max[w]);
    // 2^e with amax * 2^-e in [2^13, 2^14): full fp16 precision, no overflow
    int ex = 0;
    if (amax != 0 && amax < 0x7f800000u) ex = max((int)((amax >> 23) & 0xff) - 127 - 13, -110);  // tiny x: 2^110 max
    const float down = ldexpf(1.0f, -ex);
    auto put = [&](int e, const float (&o)[4]) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int s = e + k, blk = s >> 5;
            xp[row + 32 * blk + q4_perm_dst(s & 31, blk & 1)] = __float2half_rn(o[k] * down);
        }
    };
#pragma unroll
    for (int i = 0; i < kHeld; ++i) {
        const int e = 4 * (tid + 256 * i);
        if (e < K) put(e, v[i]);
    }
    for (int e = 4 * (tid + 256 * kHeld); e < K; e += 1024) {
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        if (real) xprep_load4(x, x_bf16, vec, row + e, o);
        put(e, o);
    }
    if (tid == 0) xscale[t] = real ? ldexpf(1.0f, ex) : 0.0f;
}

}  // namespace nexus_gpu
