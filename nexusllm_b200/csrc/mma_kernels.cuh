// mma_kernels.cuh -- batched decode (M >= 16 activation rows) on the sm_100a
// tcgen05 tensor cores, GGUF Q4_0 weights.
//
// Y[M][N] = X[M][K] . W[N][K]^T.  At M >= 16 the GEMV becomes a contraction
// with enough reuse of every weight for the tensor cores; weights still
// stream once from HBM.
//  * A CTA owns a tile of 128 weight rows (the UMMA M) and a range of K
//    (split-K when the matrix has few row tiles; partial sums are then added
//    by a second kernel in a fixed order, so results are deterministic).
//  * Warp 0 streams raw Q4_0 chunks of 128 rows x 256 weights (144 bytes a
//    row) with 2-D TMA tensor copies; warp 2 streams the matching x tiles
//    (fp16, 128-byte swizzle, straight into the UMMA operand layout).
//  * Warps 4..11 dequantize: (q - 8) * d computed in fp16 from the exact
//    integer q - 8 with one rounding, written into the K-major 128-byte-swizzle
//    A layout, 64 weights of a row per stage.
//  * Warp 1 owns the tensor memory: it allocates the fp32 accumulator and one
//    of its threads issues tcgen05.mma (kind::f16: fp16 x fp16 -> fp32) for
//    every 16 weights of K, releasing each operand stage with tcgen05.commit.
//  * x is split into two fp16 parts, hi = fp16(x * 2^-e) and lo =
//    fp16(x * 2^-e - hi), with a per-token power of two 2^e that keeps the
//    token inside fp16 range; both parts are B columns, so the accumulator
//    holds sum(w * hi) and sum(w * lo) and y = (hi_sum + lo_sum) * 2^e.  The x
//    representation error is about 2^-22 relative; the weights carry one fp16
//    rounding of (q - 8) * d (2^-12 relative), about 2e-4 L2-relative on y.
//  * Warps 4..11 then read the accumulator (tcgen05.ld) and write y.
// Every mbarrier wait is bounded; a failed wait stops the CTA's work, the
// producers drain their copies in flight, and the tensor memory is freed on
// every path.  No cluster multicast anywhere.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "gemv_kernels.cuh"

namespace nexus_gpu {

constexpr int kMmaRows = 128;        // weight rows per tile (UMMA M)
constexpr int kRawK = 256;           // weights per row in one raw chunk
constexpr int kRawRowBytes = 144;    // 8 Q4_0 blocks
constexpr int kRawChunkBytes = kMmaRows * kRawRowBytes;
constexpr int kUnitK = 64;           // K per operand stage: one 128-byte swizzle row of fp16
constexpr int kRawStages = 4;
constexpr int kAbStages = 3;
constexpr int kMaxTokens = 64;       // activation rows per launch (hi + lo columns <= 128)
constexpr int kMmaThreads = 12 * 32; // 0 raw TMA, 1 MMA + TMEM, 2 x TMA, 3 idle, 4..11 dequant + epilogue
constexpr int kATileBytes = kMmaRows * 128;
constexpr int kBTileBytes = 2 * kMaxTokens * 128;
constexpr int kMmaSmemA = 0;
constexpr int kMmaSmemB = kMmaSmemA + kAbStages * kATileBytes;
constexpr int kMmaSmemRaw = kMmaSmemB + kAbStages * kBTileBytes;
constexpr int kMmaSmemBar = kMmaSmemRaw + kRawStages * kRawChunkBytes;
constexpr int kMmaSmemBytes = kMmaSmemBar + 256 + 1024;  // barriers, TMEM address, 1024-byte alignment slack

struct MmaParams {
    int N, K;             // weight rows, cols
    int M, MP;            // tokens; tokens rounded up to 8 (B has 2*MP columns: hi, then lo)
    int chunks_per_split; // raw chunks (256 weights) per CTA
    int n_chunks;         // K / 256
    int splits;
    float* out;           // splits == 1: y [M][N]; else partial [splits][M][N]
    const float* xscale;  // [MP]: 2^e per token
};

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
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 4 consecutive accumulator columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
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

// fp16x2 (lo, hi) of two weights: (q - 8) * d with q the 4-bit codes in the
// low nibbles of the two 16-bit halves of t: exact q - 8 via the 1024 + q
// trick, then one fp16 rounding of the product.
__device__ __forceinline__ uint32_t q4_pair_f16(uint32_t t, __half2 d2) {
    const uint32_t h = (t & 0x000F000Fu) | 0x64006400u;  // fp16 1024 + q in each half
    __half2 v = *reinterpret_cast<const __half2*>(&h);
    v = __hsub2(v, __float2half2_rn(1032.0f));            // q - 8, exact
    v = __hmul2(v, d2);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Bounded wait that also gives up once another thread of the CTA has.
__device__ __forceinline__ bool mma_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t k = 1;; ++k) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((k & 63u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&g_device_status, kStatusWaitTimeout);
                *abort = 1;
                return false;
            }
        }
    }
}

__global__ void __launch_bounds__(kMmaThreads, 1)
    gemm_q4_0_mma_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                         const MmaParams P) {
    extern __shared__ uint8_t mma_smem_raw[];
    const uint32_t sraw = smem_u32(mma_smem_raw);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;  // 1024-byte aligned: swizzle atoms
    uint8_t* smem = mma_smem_raw + (sbase - sraw);
    const uint32_t bar0 = sbase + kMmaSmemBar;
    const uint32_t raw_full = bar0, raw_empty = bar0 + 8 * kRawStages;
    const uint32_t a_full = raw_empty + 8 * kRawStages, b_full = a_full + 8 * kAbStages;
    const uint32_t ab_empty = b_full + 8 * kAbStages, acc_full = ab_empty + 8 * kAbStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMmaSmemBar + 8 * (2 * kRawStages + 3 * kAbStages + 1));
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x / P.splits, split = blockIdx.x % P.splits;
    const int c_begin = split * P.chunks_per_split;
    const int n_my = min(P.chunks_per_split, P.n_chunks - c_begin);  // >= 1 by the host's split choice
    const int n_units = 4 * n_my;
    const int NB = 2 * P.MP;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRawStages; ++s) {
            mbar_init(raw_full + 8 * s, 1);
            mbar_init(raw_empty + 8 * s, 8);
        }
        for (int s = 0; s < kAbStages; ++s) {
            mbar_init(a_full + 8 * s, 8);
            mbar_init(b_full + 8 * s, 1);
            mbar_init(ab_empty + 8 * s, 1);
        }
        mbar_init(acc_full, 1);
        *abort = 0;
        fence_mbar_init();
    }
    // warp 1 allocates the accumulator: NB fp32 columns, a power of two >= 32
    const uint32_t tcols = NB <= 32 ? 32u : (NB <= 64 ? 64u : 128u);
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    if (warp == 0) {
        // ---------------------------------------------------- raw weight chunks
        if (lane == 0) {
            int issued = 0;
            for (int c = 0; c < n_my; ++c) {
                const int s = c % kRawStages;
                if (c >= kRawStages && !mma_wait(raw_empty + 8 * s, ((c / kRawStages) - 1) & 1, abort)) break;
                mbar_arrive_expect_tx(raw_full + 8 * s, kRawChunkBytes);
                tma_load_2d(sbase + kMmaSmemRaw + s * kRawChunkBytes, &tmW, (c_begin + c) * kRawRowBytes,
                            tile * kMmaRows, raw_full + 8 * s);
                ++issued;
            }
            if (*abort)  // leave no copy in flight
                for (int k = 0; k < kRawStages && k < issued; ++k) {
                    const int j = issued - 1 - k;
                    mbar_wait_bounded(raw_full + 8 * (j % kRawStages), (j / kRawStages) & 1);
                }
        }
    } else if (warp == 2) {
        // ----------------------------------------------------------- x tiles
        if (lane == 0) {
            int issued = 0;
            for (int u = 0; u < n_units; ++u) {
                const int s = u % kAbStages;
                if (u >= kAbStages && !mma_wait(ab_empty + 8 * s, ((u / kAbStages) - 1) & 1, abort)) break;
                mbar_arrive_expect_tx(b_full + 8 * s, (uint32_t)NB * 128u);
                tma_load_2d(sbase + kMmaSmemB + s * kBTileBytes, &tmX, c_begin * kRawK + u * kUnitK, 0,
                            b_full + 8 * s);
                ++issued;
            }
            if (*abort)
                for (int k = 0; k < kAbStages && k < issued; ++k) {
                    const int j = issued - 1 - k;
                    mbar_wait_bounded(b_full + 8 * (j % kAbStages), (j / kAbStages) & 1);
                }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA
        if (lane == 0) {
            // kind::f16: fp32 accumulator (bit 4), fp16 A and B, both K-major,
            // N = NB (bits 17..22, N/8), M = 128 (bits 24..28, M/16)
            const uint32_t idesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(kMmaRows >> 4) << 24);
            int done = 0;
            for (int u = 0; u < n_units; ++u) {
                const int s = u % kAbStages;
                const uint32_t par = (u / kAbStages) & 1;
                if (!mma_wait(a_full + 8 * s, par, abort) || !mma_wait(b_full + 8 * s, par, abort)) break;
                tc_fence_after();
                const uint32_t a0 = sbase + kMmaSmemA + s * kATileBytes, b0 = sbase + kMmaSmemB + s * kBTileBytes;
#pragma unroll
                for (int ks = 0; ks < kUnitK / 16; ++ks)
                    umma_f16(tmem_d, umma_desc_sw128(a0 + 32 * ks), umma_desc_sw128(b0 + 32 * ks), idesc,
                             (u > 0 || ks > 0) ? 1u : 0u);
                umma_commit(ab_empty + 8 * s);  // frees the A and B stage once these MMAs are done
                ++done;
            }
            umma_commit(acc_full);  // every MMA issued so far has completed when this arrives
            // no MMA may still read shared memory or write the accumulator when
            // the CTA tears down (the epilogue waits for it too)
            mbar_wait_bounded(acc_full, 0);
            (void)done;
        }
    } else if (warp >= 4) {
        // ----------------------------------------------- dequantize, epilogue
        const int d_tid = threadIdx.x - 128;  // 0..255
        const int r = d_tid & 127, h = d_tid >> 7;
        bool ok = true;
        for (int c = 0; c < n_my && ok; ++c) {
            const int rs = c % kRawStages;
            if (!mma_wait(raw_full + 8 * rs, (c / kRawStages) & 1, abort)) {
                ok = false;
                break;
            }
            const uint32_t raw_row = sbase + kMmaSmemRaw + rs * kRawChunkBytes + r * kRawRowBytes;
            for (int u = 0; u < 4; ++u) {
                const int iu = 4 * c + u, s = iu % kAbStages;
                if (iu >= kAbStages && !mma_wait(ab_empty + 8 * s, ((iu / kAbStages) - 1) & 1, abort)) {
                    ok = false;
                    break;
                }
                // block 2u + h of the chunk: elements 32h .. 32h+31 of this 64-weight unit
                const uint32_t blk = raw_row + (uint32_t)((2 * u + h) * 18);
                uint32_t q[4];
                lds_words_2a<4>(blk + 2, q);
                const __half2 d2 = __float2half2_rn(nexus_fp16(lds16(blk)));
                uint32_t H[16];  // fp16 pairs of elements (2i, 2i+1)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t t01 = __byte_perm(q[j], 0, 0x4140), t23 = __byte_perm(q[j], 0, 0x4342);
                    H[2 * j] = q4_pair_f16(t01, d2);
                    H[2 * j + 1] = q4_pair_f16(t23, d2);
                    H[8 + 2 * j] = q4_pair_f16(t01 >> 4, d2);
                    H[9 + 2 * j] = q4_pair_f16(t23 >> 4, d2);
                }
                const uint32_t arow = sbase + kMmaSmemA + s * kATileBytes + (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const uint32_t chunk = (uint32_t)((4 * h + jj) ^ (r & 7));
                    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(arow + 16 * chunk), "r"(H[4 * jj]),
                                 "r"(H[4 * jj + 1]), "r"(H[4 * jj + 2]), "r"(H[4 * jj + 3])
                                 : "memory");
                }
                fence_async_shared();  // generic-proxy stores -> visible to the tensor core's async proxy
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full + 8 * s);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(raw_empty + 8 * rs);
        }
        // epilogue: warp (w % 4) reads accumulator lanes 32*(w%4) ..; the two
        // warps of a lane quarter split the tokens
        if (ok && mma_wait(acc_full, 0, abort)) {
            tc_fence_after();
            const int quarter = warp & 3, half = (warp - 4) >> 2;
            const int row = tile * kMmaRows + quarter * 32 + lane;
            const int t_lo = half * (P.MP / 2), t_hi = (half + 1) * (P.MP / 2);
            float* out = P.out + (size_t)split * P.M * P.N;
            for (int t0 = t_lo; t0 < t_hi; t0 += 4) {
                float vh[4], vl[4];
                const uint32_t lane_base = tmem_d + ((uint32_t)(quarter * 32) << 16);
                tmem_ld4(lane_base + (uint32_t)t0, vh);
                tmem_ld4(lane_base + (uint32_t)(P.MP + t0), vl);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int t = t0 + k;
                    if (t < P.M && t < t_hi && row < P.N) out[(size_t)t * P.N + row] = (vh[k] + vl[k]) * __ldg(P.xscale + t);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(tcols) : "memory");
    }
}

// x [M][K] (fp32 or bf16) -> hi/lo fp16 rows of the B operand [2*MP][K] and
// the per-token scale 2^e.  One CTA per padded token row t < MP.
__global__ void __launch_bounds__(256) mma_xprep_kernel(const void* __restrict__ x, int x_bf16, int M, int MP, int K,
                                                        __half* __restrict__ xp, float* __restrict__ xscale) {
    const int t = blockIdx.x;
    __shared__ uint32_t s_max[8];
    const bool real = t < M;
    auto load = [&](int k) -> float {
        if (!real) return 0.0f;
        const size_t e = (size_t)t * K + k;
        return x_bf16 ? __uint_as_float((uint32_t) static_cast<const uint16_t*>(x)[e] << 16)
                      : static_cast<const float*>(x)[e];
    };
    uint32_t m = 0;
    for (int k = threadIdx.x; k < K; k += blockDim.x) m = max(m, __float_as_uint(load(k)) & 0x7fffffffu);
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = m;
    __syncthreads();
    uint32_t amax = 0;
    for (int w = 0; w < 8; ++w) amax = max(amax, s_max[w]);
    // 2^e with amax * 2^-e in [2^13, 2^14): hi keeps fp16's full precision, no overflow
    int e = 0;
    if (amax != 0 && amax < 0x7f800000u) e = max((int)((amax >> 23) & 0xff) - 127 - 13, -110);  // tiny x: 2^110 max
    const float down = ldexpf(1.0f, -e);
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = load(k) * down;
        const __half hi = __float2half_rn(v);
        const __half lo = __float2half_rn(v - __half2float(hi));
        xp[(size_t)t * K + k] = hi;
        xp[(size_t)(MP + t) * K + k] = lo;
    }
    if (threadIdx.x == 0) xscale[t] = real ? ldexpf(1.0f, e) : 0.0f;
}

// y[t][n] = sum over splits of partial[s][t][n], in split order.
__global__ void mma_splitk_reduce_kernel(const float* __restrict__ partial, float* __restrict__ y, int splits,
                                         size_t count) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float acc = partial[i];
    for (int s = 1; s < splits; ++s) acc += partial[(size_t)s * count + i];
    y[i] = acc;
}

}  // namespace nexus_gpu
