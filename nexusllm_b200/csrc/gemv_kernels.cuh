// gemv_kernels.cuh -- batch-1 fused quantized GEMV for sm_100a.
//
// y[N] = W[N, K] . x[K] straight from GGUF blocks (NexusLLM
// QuantizationKernel::fused_gemv_{q4_0,q8_0,q5_k,q6_k,fp16},
// src/quantization.cpp:264-722).
//
// Data path (one CTA per SM, 8 consumer warps + 1 producer warp):
//  * The CTA owns a contiguous range of rows.  Rows are processed in groups
//    of up to 8*R rows (R rows per consumer warp) and, inside a group, in
//    K-chunks of 32 "work items" (a work item = 32 weights; 16 for FP16).
//  * The producer warp streams each (row group, K-chunk) tile from HBM into a
//    ring of shared-memory stages with 1-D bulk copies (cp.async.bulk on the
//    TMA engine), one copy per row segment, completing on a "full" mbarrier.
//    Row segments start on 16-byte boundaries rounded down from the true
//    start, so blocks of any size (18, 34, 176, 210 bytes) land at a known
//    2-byte offset and are realigned with byte permutes in registers.
//  * Consumer lane l takes work item l of each row segment, loads that work
//    item's slice of x once and reuses it for the warp's R rows, dequantizes
//    in registers and accumulates.  The stage is released on an "empty"
//    mbarrier; at the end of a row group each warp reduces its R partial
//    sums with shuffles and writes y.
//
// Arithmetic.  For the integer formats the activation is first turned into
// a 16-bit fixed-point vector by xquant_kernel (per 32-element block: scale
// s = amax/32639 and X = rint(x/s) split into two signed 8-bit limbs
// X = 256*Xh + Xl, plus the block sums of X).  Each block's dot product is
// then exact int32 dp4a arithmetic over (weight code, limb) pairs, scaled once
// per block by the block's fp16 scale(s) (as the reference does,
// src/quantization.cpp:325,374) and by s.  The only rounding beyond fp32
// accumulation is the fixed-point representation of x: |x - X*s| <= s/2 with
// s <= amax/32639, about 2e-5 relative L2 error on the GEMV, well inside the
// 1e-3 parity tolerance.  FP16 weights use fp32 FMA on fp32 x directly.
// Weight decoding follows the reference's block layouts and its own (not
// ggml's) Q5_K / Q6_K bit orders (src/quantization.cpp:418-509).
#pragma once

#include "device_common.cuh"

namespace nexus_gpu {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kXQLimbBytes = 64;   // Xh[32] then Xl[32], int8
constexpr int kXQMetaBytes = 16;   // {float s, int sum X[0:16), int sum X[16:32), pad}
constexpr float kXQMax = 32639.0f;  // largest |X| whose high limb fits int8

struct GemvParams {
    const uint8_t* W;        // weight blocks, 16-byte aligned
    uint64_t total_bytes;    // N * row_bytes
    uint64_t row_bytes;
    int N, K;
    int nwi;                 // work items per row
    const uint8_t* xq_limbs; // [K/32][64]      (integer formats)
    const int4* xq_meta;     // [K/32]          (integer formats)
    const void* x;           // fp32 or bf16 [K] (FP16 weights)
    int x_bf16;
    float* y;
};

// ------------------------------------------------------------------ formats
struct FmtQ4_0 {
    static constexpr int kBlockBytes = 18, kWIPerBlock = 1, kWIElems = 32;
    static constexpr int kRows = 4, kChunkWI = 32, kStages = 6;
    static constexpr bool kIntX = true;
};
struct FmtQ8_0 {
    static constexpr int kBlockBytes = 34, kWIPerBlock = 1, kWIElems = 32;
    static constexpr int kRows = 2, kChunkWI = 32, kStages = 6;
    static constexpr bool kIntX = true;
};
struct FmtQ5_K {
    static constexpr int kBlockBytes = 176, kWIPerBlock = 8, kWIElems = 32;
    static constexpr int kRows = 4, kChunkWI = 32, kStages = 5;
    static constexpr bool kIntX = true;
};
struct FmtQ6_K {
    static constexpr int kBlockBytes = 210, kWIPerBlock = 8, kWIElems = 32;
    static constexpr int kRows = 2, kChunkWI = 32, kStages = 7;
    static constexpr bool kIntX = true;
};
struct FmtF16 {
    static constexpr int kBlockBytes = 32, kWIPerBlock = 1, kWIElems = 16;  // 16 halves per work item
    static constexpr int kRows = 2, kChunkWI = 32, kStages = 6;
    static constexpr bool kIntX = false;
};

template <class F>
struct Layout {
    static constexpr int kRG = kConsumerWarps * F::kRows;                         // rows per group
    static constexpr int kChunkBytes = F::kChunkWI / F::kWIPerBlock * F::kBlockBytes;
    static constexpr int kRowStride = (kChunkBytes + 32 + 15) / 16 * 16;           // room for 16-B rounding
    static constexpr int kStageBytes = kRG * kRowStride;
    static constexpr int kBarBytes = 128;
    __host__ __device__ static size_t x_bytes(int K) {
        size_t b = F::kIntX ? (size_t)(K / 32) * (kXQLimbBytes + kXQMetaBytes) : (size_t)K * 4;
        return (b + 127) / 128 * 128;
    }
    __host__ __device__ static size_t smem_bytes(int K) { return kBarBytes + x_bytes(K) + (size_t)F::kStages * kStageBytes + 128; }
};

// x slice of one work item, integer formats
struct XInt {
    uint32_t h[8], l[8];
    float s;
    int sa, sb;
};

__device__ __forceinline__ void load_xint(uint32_t limbs, uint32_t meta, int gj, XInt& X) {
    const uint32_t a = limbs + gj * kXQLimbBytes;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        uint4 v = lds128(a + 16 * q);
        X.h[4 * q + 0] = v.x; X.h[4 * q + 1] = v.y; X.h[4 * q + 2] = v.z; X.h[4 * q + 3] = v.w;
        uint4 u = lds128(a + 32 + 16 * q);
        X.l[4 * q + 0] = u.x; X.l[4 * q + 1] = u.y; X.l[4 * q + 2] = u.z; X.l[4 * q + 3] = u.w;
    }
    uint4 m = lds128(meta + gj * kXQMetaBytes);
    X.s = __uint_as_float(m.x);
    X.sa = (int)m.y;
    X.sb = (int)m.z;
}

// Q4_0 (include/quantization.hpp:8-11; src/quantization.cpp:264-330).
// p: shared address of the 18-byte block (2-byte aligned).
__device__ __forceinline__ float dot_q4_0(uint32_t p, const XInt& X) {
    uint32_t q[4];
    lds_words_2a<4>(p + 2, q);
    const float d = nexus_fp16(lds16(p));
    int shl = 0, shh = 0, sll = 0, slh = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t lo = q[k] & 0x0F0F0F0Fu;  // weights 4k..4k+3
        const uint32_t hi = q[k] & 0xF0F0F0F0u;  // 16 * weights 16+4k..
        shl = dp4a_us(lo, X.h[k], shl);
        shh = dp4a_us(hi, X.h[4 + k], shh);
        sll = dp4a_us(lo, X.l[k], sll);
        slh = dp4a_us(hi, X.l[4 + k], slh);
    }
    // 16 * sum((q - 8) * X), exact in int32
    const int t16 = ((shl * 16 + shh) << 8) + sll * 16 + slh - 128 * (X.sa + X.sb);
    return (d * X.s) * (0.0625f * (float)t16);
}

// Q8_0 (include/quantization.hpp:14-17; src/quantization.cpp:332-379).
__device__ __forceinline__ float dot_q8_0(uint32_t p, const XInt& X) {
    uint32_t q[8];
    lds_words_2a<8>(p + 2, q);
    const float d = nexus_fp16(lds16(p));
    int sh = 0, sl = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        sh = dp4a_ss(q[k], X.h[k], sh);
        sl = dp4a_ss(q[k], X.l[k], sl);
    }
    return (d * X.s) * (float)((sh << 8) + sl);
}

// Q5_K sub-block `sub` (32 weights) of the 176-byte super-block at o
// (16-byte aligned).  Scales: src/quantization.cpp:418-430; bit layout
// :456-470 (qh bit 2(i%4) of qh[4sub+i/4] for element i, bit 2(i%4)+1 for
// element 16+i); w = v*(d*sc) - dmin*m.
__device__ __forceinline__ float dot_q5_k(uint32_t o, int sub, const XInt& X) {
    const uint32_t dd = lds32(o);
    const float d = nexus_fp16(dd & 0xffffu);
    const float dmin = nexus_fp16(dd >> 16);
    const uint32_t s0 = lds32(o + 4), s1 = lds32(o + 8), s2 = lds32(o + 12);
    const int i = sub & 3;
    const uint32_t b0 = __byte_perm(s0, 0, 0x4440 + i);  // s[i]
    const uint32_t b1 = __byte_perm(s1, 0, 0x4440 + i);  // s[i+4]
    const uint32_t b2 = __byte_perm(s2, 0, 0x4440 + i);  // s[i+8]
    const uint32_t sc = sub < 4 ? (b0 & 63u) : ((b2 & 15u) | ((b0 >> 6) << 4));
    const uint32_t mn = sub < 4 ? (b1 & 63u) : ((b2 >> 4) | ((b1 >> 6) << 4));
    const uint32_t qhw = lds32(o + 16 + 4 * sub);
    const uint4 qv = lds128(o + 48 + 16 * sub);
    const uint32_t qs[4] = {qv.x, qv.y, qv.z, qv.w};
    int sh = 0, sl = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t hb = (qhw >> (8 * k)) & 0xffu;  // qh byte k: elements 4k..4k+3 and 16+4k..
        // spread bits 0,2,4,6 (resp. 1,3,5,7) to bit 4 of bytes 0..3
        const uint32_t he = ((hb & 0x55u) * 0x00410410u) & 0x10101010u;
        const uint32_t ho = (((hb >> 1) & 0x55u) * 0x00410410u) & 0x10101010u;
        const uint32_t ulo = (qs[k] & 0x0F0F0F0Fu) | he;
        const uint32_t uhi = ((qs[k] >> 4) & 0x0F0F0F0Fu) | ho;
        sh = dp4a_us(ulo, X.h[k], sh);
        sh = dp4a_us(uhi, X.h[4 + k], sh);
        sl = dp4a_us(ulo, X.l[k], sl);
        sl = dp4a_us(uhi, X.l[4 + k], sl);
    }
    const float scale = d * (float)sc;
    const float minv = dmin * (float)mn;
    return X.s * (scale * (float)((sh << 8) + sl) - minv * (float)(X.sa + X.sb));
}

// Q6_K sub-blocks 2*pair and 2*pair+1 (16 weights each) of the 210-byte
// super-block at o (2-byte aligned).  Bit layout: src/quantization.cpp:487-506
// (element i<8 of sub-block sb: low nibble of ql[8sb+i] and bits (i%2)*4+{0,1}
// of qh[4sb+i/2]; element 8+i: high nibble and bits (i%2)*4+{2,3}); v-32.
__device__ __forceinline__ float dot_q6_k(uint32_t o, int pair, const XInt& X) {
    uint32_t L[4], H[2];
    lds_words_2a<4>(o + 16 * pair, L);
    lds_words_2a<2>(o + 128 + 8 * pair, H);
    const uint32_t scw = lds16(o + 192 + 2 * pair);
    const float d = nexus_fp16(lds16(o + 208));
    float r = 0.0f;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const uint32_t pa = __byte_perm(H[t], 0, 0x1100);  // qh bytes 0,0,1,1
        const uint32_t pb = __byte_perm(H[t], 0, 0x3322);  // qh bytes 2,2,3,3
        const uint32_t h0a = ((pa << 4) & 0x00300030u) | (pa & 0x30003000u);
        const uint32_t h0b = ((pb << 4) & 0x00300030u) | (pb & 0x30003000u);
        const uint32_t h1a = ((pa << 2) & 0x00300030u) | ((pa >> 2) & 0x30003000u);
        const uint32_t h1b = ((pb << 2) & 0x00300030u) | ((pb >> 2) & 0x30003000u);
        const uint32_t l0 = L[2 * t], l1 = L[2 * t + 1];
        const uint32_t u0 = (l0 & 0x0F0F0F0Fu) | h0a;         // elements 0..3
        const uint32_t u1 = (l1 & 0x0F0F0F0Fu) | h0b;         // 4..7
        const uint32_t u2 = ((l0 >> 4) & 0x0F0F0F0Fu) | h1a;  // 8..11
        const uint32_t u3 = ((l1 >> 4) & 0x0F0F0F0Fu) | h1b;  // 12..15
        int sh = dp4a_us(u0, X.h[4 * t + 0], 0);
        sh = dp4a_us(u1, X.h[4 * t + 1], sh);
        sh = dp4a_us(u2, X.h[4 * t + 2], sh);
        sh = dp4a_us(u3, X.h[4 * t + 3], sh);
        int sl = dp4a_us(u0, X.l[4 * t + 0], 0);
        sl = dp4a_us(u1, X.l[4 * t + 1], sl);
        sl = dp4a_us(u2, X.l[4 * t + 2], sl);
        sl = dp4a_us(u3, X.l[4 * t + 3], sl);
        const int sx = t == 0 ? X.sa : X.sb;
        const int sc = (int)(int8_t)((scw >> (8 * t)) & 0xffu);
        const float scale = d * (float)sc;
        r = fmaf(scale, (float)((sh << 8) + sl - 32 * sx), r);
    }
    return X.s * r;
}

// FP16: 16 halves at p (2-byte aligned) against fp32 x at xs (16-B aligned).
__device__ __forceinline__ float dot_f16(uint32_t p, uint32_t xs) {
    uint32_t w[8];
    lds_words_2a<8>(p, w);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 xv = lds128f(xs + 16 * q);
        a0 = fmaf(nexus_fp16(w[2 * q] & 0xffffu), xv.x, a0);
        a1 = fmaf(nexus_fp16_hi(w[2 * q]), xv.y, a1);
        a0 = fmaf(nexus_fp16(w[2 * q + 1] & 0xffffu), xv.z, a0);
        a1 = fmaf(nexus_fp16_hi(w[2 * q + 1]), xv.w, a1);
    }
    return a0 + a1;
}

template <class F>
__device__ __forceinline__ uint32_t wi_offset(int j) {
    if constexpr (F::kWIPerBlock == 1) return (uint32_t)j * F::kBlockBytes;
    else return (uint32_t)(j / F::kWIPerBlock) * F::kBlockBytes;
}

// ------------------------------------------------------------------- kernel
template <class F>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_m1_kernel(const GemvParams p) {
    using L = Layout<F>;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full_bar = sbase;                          // kStages x 8 B
    const uint32_t empty_bar = sbase + 8 * F::kStages;        // kStages x 8 B
    const uint32_t xs = sbase + L::kBarBytes;                 // x region
    const uint32_t stage0 = xs + (uint32_t)L::x_bytes(p.K);  // stage ring

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int row_begin = (int)((int64_t)p.N * c / G);
    const int row_end = (int)((int64_t)p.N * (c + 1) / G);
    const int n_groups = (row_end - row_begin + L::kRG - 1) / L::kRG;
    const int n_chunks = (p.nwi + F::kChunkWI - 1) / F::kChunkWI;

    if (threadIdx.x == 0) {
        for (int s = 0; s < F::kStages; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------- producer
        if (lane != 0) return;
        const uint64_t floor16 = p.total_bytes & ~(uint64_t)15;
        int it = 0;
        bool ok = true;
        for (int g = 0; g < n_groups && ok; ++g) {
            const int r0 = row_begin + g * L::kRG;
            const int nr = min(L::kRG, row_end - r0);
            for (int ch = 0; ch < n_chunks; ++ch, ++it) {
                const int s = it % F::kStages, use = it / F::kStages;
                if (use > 0 && !mbar_wait_bounded(empty_bar + 8 * s, (use - 1) & 1)) { ok = false; break; }
                const int nwi_c = min(F::kChunkWI, p.nwi - ch * F::kChunkWI);
                const uint64_t cbytes = (uint64_t)(nwi_c / F::kWIPerBlock) * F::kBlockBytes;
                const uint64_t coff = (uint64_t)ch * L::kChunkBytes;
                const uint32_t dst0 = stage0 + (uint32_t)s * L::kStageBytes;
                uint32_t tx = 0;
                bool tail = false;
                for (int rl = 0; rl < nr; ++rl) {
                    const uint64_t start = (uint64_t)(r0 + rl) * p.row_bytes + coff;
                    const uint64_t end = start + cbytes;
                    const uint64_t a = start & ~(uint64_t)15;
                    const uint64_t bend = min((end + 15) & ~(uint64_t)15, floor16);
                    if (bend > a) tx += (uint32_t)(bend - a);
                    // bytes past the last 16-byte boundary of the matrix
                    for (uint64_t pos = (bend > a ? bend : a); pos < end; pos += 2) {
                        const uint16_t v = *reinterpret_cast<const uint16_t*>(p.W + pos);
                        sts16(dst0 + rl * L::kRowStride + (uint32_t)(pos - a), v);
                        tail = true;
                    }
                }
                if (tail) fence_proxy_async_smem();
                mbar_arrive_expect_tx(full_bar + 8 * s, tx);
                for (int rl = 0; rl < nr; ++rl) {
                    const uint64_t start = (uint64_t)(r0 + rl) * p.row_bytes + coff;
                    const uint64_t end = start + cbytes;
                    const uint64_t a = start & ~(uint64_t)15;
                    const uint64_t bend = min((end + 15) & ~(uint64_t)15, floor16);
                    if (bend > a) bulk_g2s(dst0 + rl * L::kRowStride, p.W + a, (uint32_t)(bend - a), full_bar + 8 * s);
                }
            }
        }
        // Leave no copy in flight: wait (bounded) for every stage issued but
        // not consumed when something went wrong.
        if (!ok) {
            for (int k = 0; k < F::kStages && k < it; ++k) {
                const int j = it - 1 - k, s = j % F::kStages;
                mbar_wait_bounded(full_bar + 8 * s, (j / F::kStages) & 1);
            }
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    // x depends on the previous kernel in the stream (x quantization or the
    // GEMV that produced x); weights do not, so the producer never waits.
    pdl_wait();
    if constexpr (F::kIntX) {
        const int nxb = p.K / 32;
        const int4* lsrc = reinterpret_cast<const int4*>(p.xq_limbs);
        for (int i = threadIdx.x; i < nxb * (kXQLimbBytes / 16); i += kConsumerWarps * 32) {
            const int4 v = __ldg(lsrc + i);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(xs + 16 * i), "r"(v.x), "r"(v.y), "r"(v.z),
                         "r"(v.w)
                         : "memory");
        }
        const uint32_t ms = xs + nxb * kXQLimbBytes;
        for (int i = threadIdx.x; i < nxb; i += kConsumerWarps * 32) {
            const int4 v = __ldg(p.xq_meta + i);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(ms + 16 * i), "r"(v.x), "r"(v.y), "r"(v.z),
                         "r"(v.w)
                         : "memory");
        }
    } else {
        if (p.x_bf16) {
            const uint16_t* xb = static_cast<const uint16_t*>(p.x);
            for (int i = threadIdx.x; i < p.K; i += kConsumerWarps * 32) {
                const float v = __uint_as_float((uint32_t)xb[i] << 16);
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(xs + 4 * i), "f"(v) : "memory");
            }
        } else {
            const float* xf = static_cast<const float*>(p.x);
            for (int i = threadIdx.x; i < p.K; i += kConsumerWarps * 32)
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(xs + 4 * i), "f"(__ldg(xf + i)) : "memory");
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");

    const uint32_t xlimbs = xs;
    const uint32_t xmeta = xs + (uint32_t)(p.K / 32) * kXQLimbBytes;
    int it = 0;
    bool ok = true;
    for (int g = 0; g < n_groups && ok; ++g) {
        const int r0 = row_begin + g * L::kRG;
        const int nr = min(L::kRG, row_end - r0);
        const int reff = (nr + kConsumerWarps - 1) / kConsumerWarps;
        const int my0 = warp * reff;
        const int mynr = max(0, min(reff, nr - my0));
        float acc[F::kRows];
#pragma unroll
        for (int r = 0; r < F::kRows; ++r) acc[r] = 0.f;
        for (int ch = 0; ch < n_chunks; ++ch, ++it) {
            const int s = it % F::kStages, use = it / F::kStages;
            if (!mbar_wait_bounded(full_bar + 8 * s, use & 1)) { ok = false; break; }
            const int nwi_c = min(F::kChunkWI, p.nwi - ch * F::kChunkWI);
            const uint32_t st = stage0 + (uint32_t)s * L::kStageBytes;
            const uint64_t coff = (uint64_t)ch * L::kChunkBytes;
            for (int j = lane; j < nwi_c; j += 32) {
                const int gj = ch * F::kChunkWI + j;  // global work item = x block
                if constexpr (F::kIntX) {
                    XInt X;
                    load_xint(xlimbs, xmeta, gj, X);
#pragma unroll
                    for (int r = 0; r < F::kRows; ++r) {
                        if (r < mynr) {
                            const int rl = my0 + r;
                            const uint32_t delta =
                                (uint32_t)(((uint64_t)(r0 + rl) * p.row_bytes + coff) & 15);
                            const uint32_t base = st + rl * L::kRowStride + delta + wi_offset<F>(j);
                            if constexpr (F::kBlockBytes == 18) acc[r] += dot_q4_0(base, X);
                            else if constexpr (F::kBlockBytes == 34) acc[r] += dot_q8_0(base, X);
                            else if constexpr (F::kBlockBytes == 176) acc[r] += dot_q5_k(base, j & 7, X);
                            else acc[r] += dot_q6_k(base, j & 7, X);
                        }
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < F::kRows; ++r) {
                        if (r < mynr) {
                            const int rl = my0 + r;
                            const uint32_t delta =
                                (uint32_t)(((uint64_t)(r0 + rl) * p.row_bytes + coff) & 15);
                            const uint32_t base = st + rl * L::kRowStride + delta + wi_offset<F>(j);
                            acc[r] += dot_f16(base, xs + 64u * gj);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar + 8 * s);
        }
        if (!ok) break;
#pragma unroll
        for (int r = 0; r < F::kRows; ++r) {
            float v = acc[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && r < mynr) p.y[r0 + my0 + r] = v;
        }
    }
}

// -------------------------------------------------------- x quantization
// One warp per 32-element block of x (row m of M).  Writes limbs [M][K/32][64]
// and meta [M][K/32].  Non-finite blocks get s = amax (Inf/NaN) and X = 0, so
// every row that touches them comes out non-finite, as in fp32 arithmetic.
__global__ void __launch_bounds__(256) xquant_kernel(const void* __restrict__ x, int x_bf16, int K, int ldx,
                                                     uint8_t* __restrict__ limbs, int4* __restrict__ meta) {
    pdl_launch_dependents();
    const int nxb = K / 32;
    const int xb = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int m = blockIdx.y;
    pdl_wait();
    if (xb >= nxb) return;
    const size_t e = (size_t)m * ldx + (size_t)xb * 32 + lane;
    const float v = x_bf16 ? __uint_as_float((uint32_t)static_cast<const uint16_t*>(x)[e] << 16)
                           : static_cast<const float*>(x)[e];
    const uint32_t abits = __float_as_uint(v) & 0x7fffffffu;
    const uint32_t mbits = __reduce_max_sync(0xffffffffu, abits);
    const float amax = __uint_as_float(mbits);
    int X = 0;
    float s = 0.0f;
    if (mbits >= 0x7f800000u) {
        s = amax;  // Inf or NaN
    } else if (mbits != 0) {
        X = __float2int_rn(__fmul_rn(__fdiv_rn(v, amax), kXQMax));
        X = max(-32639, min(32639, X));
        s = __fdiv_rn(amax, kXQMax);
    }
    const int xh = (X + 128) >> 8;
    const int xl = X - (xh << 8);
    const size_t bidx = (size_t)m * nxb + xb;
    limbs[bidx * kXQLimbBytes + lane] = (uint8_t)(int8_t)xh;
    limbs[bidx * kXQLimbBytes + 32 + lane] = (uint8_t)(int8_t)xl;
    const int sa = __reduce_add_sync(0xffffffffu, lane < 16 ? X : 0);
    const int sb = __reduce_add_sync(0xffffffffu, lane < 16 ? 0 : X);
    if (lane == 0) meta[bidx] = make_int4((int)__float_as_uint(s), sa, sb, 0);
}

// ------------------------------------------------------ generic fallback
// Any shape, any 2-byte alignment: one warp per row, fp32 arithmetic straight
// from global memory with the reference's dequantization rules.  Used only for
// shapes outside the fast kernel's limits (FP16 with K % 16 != 0, K too large
// for x to stay in shared memory, or a weight pointer not 16-byte aligned).
__device__ __forceinline__ float deq_elem(int dtype, const uint8_t* row, uint64_t e) {
    switch (dtype) {
        case 1: {
            const uint16_t h = *reinterpret_cast<const uint16_t*>(row + 2 * e);
            return nexus_fp16(h);
        }
        case 7: {
            const uint8_t* b = row + (e / 32) * 18;
            const float d = nexus_fp16(*reinterpret_cast<const uint16_t*>(b));
            const int i = (int)(e % 32);
            const uint8_t v = b[2 + (i & 15)];
            const int q = (i < 16 ? (v & 15) : (v >> 4)) - 8;
            return (float)q * d;
        }
        case 9: {
            const uint8_t* b = row + (e / 32) * 34;
            const float d = nexus_fp16(*reinterpret_cast<const uint16_t*>(b));
            return (float)(int8_t)b[2 + e % 32] * d;
        }
        case 11: {
            const uint8_t* b = row + (e / 256) * 176;
            const int i = (int)(e % 256), sb = i / 32, t = i % 32, ii = t & 15;
            const float d = nexus_fp16(*reinterpret_cast<const uint16_t*>(b));
            const float dmin = nexus_fp16(*reinterpret_cast<const uint16_t*>(b + 2));
            const uint8_t* s = b + 4;
            const int k = sb & 3;
            const uint32_t sc = sb < 4 ? (s[k] & 63u) : ((s[k + 8] & 15u) | ((uint32_t)(s[k] >> 6) << 4));
            const uint32_t mn = sb < 4 ? (s[k + 4] & 63u) : ((uint32_t)(s[k + 8] >> 4) | ((uint32_t)(s[k + 4] >> 6) << 4));
            const uint8_t q = b[48 + sb * 16 + ii];
            const uint8_t h = b[16 + sb * 4 + ii / 4];
            const int sl = (ii % 4) * 2 + (t >= 16 ? 1 : 0);
            const uint32_t v = (t < 16 ? (q & 15u) : (uint32_t)(q >> 4)) | (((h >> sl) & 1u) << 4);
            return __fsub_rn(__fmul_rn((float)v, __fmul_rn(d, (float)sc)), __fmul_rn(dmin, (float)mn));
        }
        default: {  // 12: Q6_K
            const uint8_t* b = row + (e / 256) * 210;
            const int i = (int)(e % 256), sb = i / 16, t = i % 16, ii = t & 7;
            const float d = nexus_fp16(*reinterpret_cast<const uint16_t*>(b + 208));
            const uint8_t l = b[sb * 8 + ii];
            const uint8_t h = b[128 + sb * 4 + ii / 2];
            const int sh = (ii % 2) * 4 + (t >= 8 ? 2 : 0);
            const int v = (int)((t < 8 ? (l & 15u) : (uint32_t)(l >> 4)) | (((h >> sh) & 3u) << 4)) - 32;
            const int8_t sc = (int8_t)b[192 + sb];
            return __fmul_rn((float)v, __fmul_rn(d, (float)sc));
        }
    }
}

__global__ void __launch_bounds__(256) gemv_generic_kernel(int dtype, const uint8_t* __restrict__ W,
                                                           uint64_t row_bytes, int N, int K, const void* x,
                                                           int x_bf16, float* __restrict__ y) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (warp >= N) return;
    const uint8_t* row = W + (uint64_t)warp * row_bytes;
    float acc = 0.f;
    for (int e = lane; e < K; e += 32) {
        const float xv = x_bf16 ? __uint_as_float((uint32_t)static_cast<const uint16_t*>(x)[e] << 16)
                                : static_cast<const float*>(x)[e];
        acc = fmaf(deq_elem(dtype, row, (uint64_t)e), xv, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[warp] = acc;
}

}  // namespace nexus_gpu
