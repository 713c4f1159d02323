// gemv_kernels.cuh -- batch-1 fused quantized GEMV for sm_100a.
//
// y[N] = W[N, K] . x[K] straight from GGUF blocks (NexusLLM
// QuantizationKernel::fused_gemv_{q4_0,q8_0,q5_k,q6_k,fp16},
// src/quantization.cpp:264-722).
//
// Data path (one CTA per SM: 15 consumer warps + 1 producer warp):
//  * The CTA owns a contiguous range of rows.  Consecutive rows of a GGUF
//    matrix are contiguous in memory, so the CTA's weights are one contiguous
//    byte range, streamed in stages of R whole rows (about 16 KB).  Each stage
//    is ONE 1-D bulk copy (cp.async.bulk on the TMA engine) into a ring of
//    shared-memory buffers, completing on a "full" mbarrier; consumers release
//    it on an "empty" mbarrier.  One large copy per stage matters: the cost of
//    a bulk copy is dominated by its issue, not by its size.
//  * The copy starts on the 16-byte boundary at or below the first row, so
//    blocks of any size (18, 34, 176, 210 bytes) land at a known 2-byte offset
//    and are realigned in registers with byte permutes.
//  * x is stationary: a row is cut into S K-segments (S in {1, 3, 5, 15}),
//    each owned by one warp whose lanes keep that segment's slice of x in
//    registers (up to 4 work items of 32 weights -- 16 for FP16 -- per lane).
//    The warps form 15/S row groups; rows are dealt to the groups
//    round-robin, so each stage is worked on by several warps at once.
//  * A warp reduces its row partial with shuffles.  With S == 1 it writes y
//    directly; otherwise the S partials meet in shared slots and the last
//    warp to arrive (shared atomic counter) sums them in segment order.
//    Results are deterministic and do not depend on how rows are spread over
//    CTAs or GPUs.
//
// Arithmetic.  For the integer formats the activation is first turned into
// a 16-bit fixed-point vector by xquant_kernel (per 32-element block: scale
// s = amax/32639 and int16 X = rint(x/s), plus the block sums of X).  Each
// block's dot product is then exact int32 dp2a arithmetic (16-bit X against
// 8-bit weight codes, two products per instruction), scaled once
// per block by the block's fp16 scale(s) (as the reference does,
// src/quantization.cpp:325,374) and by s.  The only rounding beyond fp32
// accumulation is the fixed-point representation of x: |x - X*s| <= s/2 with
// s <= amax/32639, about 2e-5 relative L2 error on the GEMV, well inside the
// 1e-3 parity tolerance.  FP16 weights use fp32 FMA on fp32 x directly.
// Weight decoding follows the reference's block layouts and its own (not
// ggml's) Q5_K / Q6_K bit orders (src/quantization.cpp:418-509).
#pragma once

#include <cuda_fp16.h>

#include <type_traits>

#include "device_common.cuh"

namespace nexus_gpu {

constexpr int kConsumerWarps = 15;   // + 1 producer warp = 16 warps: 128 registers per thread
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumers + 32;
constexpr int kXQLimbBytes = 64;     // X[32], int16
constexpr int kXQMetaBytes = 16;     // {float s, int sum X[0:16), int sum X[16:32), int sum X[0:32)}
constexpr float kXQMax = 32639.0f;   // largest |X|
constexpr int kMaxJ = 4;             // work items (x slices in registers) per lane
constexpr int kMaxSegments = 15;     // K segments per row (one warp each)
constexpr int kMaxStageRows = 64;
constexpr int kMaxStages = 12;
constexpr int kMaxSlots = 1024;      // n_stages * stage_rows * segments partial sums
constexpr int kBarBytes = 256;       // 2 x kMaxStages mbarriers
constexpr int kSmemHeader = kBarBytes + kMaxSlots * 4 + kMaxStages * kMaxStageRows * 4;  // + slots + counters
constexpr int kStageTargetBytes = 32768;
// A stack's stages hold two rows per warp where they fit (its consumer warps
// work on two rows at once, sharing the x slices and one reduction).
constexpr int kStackStageTargetBytes = 73728;
constexpr int kStageMaxBytes = 73728;

struct GemvParams {
    const uint8_t* W;        // weight blocks, 16-byte aligned
    uint64_t total_bytes;    // N * row_bytes
    uint64_t row_bytes;
    int N, K;
    int nwi;                 // work items per row
    int segments;            // S: K segments per row, one warp each (divides kConsumerWarps)
    int seg_wi;              // work items per segment
    int wi_per_lane;         // J: work items per lane (a multiple of group)
    int group;               // consecutive work items per lane (1 or the format's kGroup)
    int stage_rows;          // R
    int stage_bytes;         // shared bytes per stage buffer (multiple of 16)
    int n_stages;
    const uint8_t* xq_limbs; // [K/32][64]      (integer formats)
    const int4* xq_meta;     // [K/32]          (integer formats)
    const void* x;           // fp32 or bf16 [K] (FP16 weights)
    int x_bf16;
    float* y;
};

// ------------------------------------------------------------------ formats
// kBlockBytes: bytes of one storage block; kWIPerBlock: work items per block;
// kWIElems: weights per work item.
// kGroup: consecutive work items one lane decodes together when the shape
// allows (a block pair for Q4_0/Q8_0, half a super-block for Q5_K/Q6_K), so
// that block headers are decoded and bytes realigned once per group.
struct FmtQ4_0 {
    static constexpr int kBlockBytes = 18, kWIPerBlock = 1, kWIElems = 32, kGroup = 2;
    static constexpr bool kIntX = true;
};
struct FmtQ8_0 {
    static constexpr int kBlockBytes = 34, kWIPerBlock = 1, kWIElems = 32, kGroup = 2;
    static constexpr bool kIntX = true;
};
struct FmtQ5_K {
    static constexpr int kBlockBytes = 176, kWIPerBlock = 8, kWIElems = 32, kGroup = 4;
    static constexpr bool kIntX = true;
};
struct FmtQ6_K {
    static constexpr int kBlockBytes = 210, kWIPerBlock = 8, kWIElems = 32, kGroup = 4;
    static constexpr bool kIntX = true;
};
struct FmtF16 {
    static constexpr int kBlockBytes = 32, kWIPerBlock = 1, kWIElems = 16, kGroup = 1;  // 16 halves per work item
    static constexpr bool kIntX = false;
};

// x slice of one work item, integer formats: the 32 X values as int16 pairs
// (v[j] = X[2j] | X[2j+1] << 16), the block scale and the block sums.
struct XInt {
    uint32_t v[16];
    float s;
    int sa, sb, sx;  // sums of X over [0,16), [16,32), [0,32)
};

// kCoherent: read through L2 (ld.global.cg) -- needed when the quantized x was
// written by other CTAs of the same kernel; otherwise the read-only path.
template <bool kCoherent = false>
__device__ __forceinline__ void load_xint(const uint8_t* limbs, const int4* meta, int gj, XInt& X) {
    const int4* a = reinterpret_cast<const int4*>(limbs + (size_t)gj * kXQLimbBytes);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int4 v = kCoherent ? __ldcg(a + q) : __ldg(a + q);
        X.v[4 * q + 0] = v.x; X.v[4 * q + 1] = v.y; X.v[4 * q + 2] = v.z; X.v[4 * q + 3] = v.w;
    }
    const int4 m = kCoherent ? __ldcg(meta + gj) : __ldg(meta + gj);
    X.s = __int_as_float(m.x);
    X.sa = m.y;
    X.sb = m.z;
    X.sx = m.w;
}

struct XF16 {
    float v[16];
};

__device__ __forceinline__ void load_xf16(const void* x, int x_bf16, int gj, XF16& X) {
    if (x_bf16) {
        const uint4* a = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + (size_t)gj * 16);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint4 w = __ldg(a + q);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                X.v[8 * q + 2 * k] = __uint_as_float(ws[k] << 16);
                X.v[8 * q + 2 * k + 1] = __uint_as_float(ws[k] & 0xffff0000u);
            }
        }
    } else {
        const float4* a = reinterpret_cast<const float4*>(static_cast<const float*>(x) + (size_t)gj * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 f = __ldg(a + q);
            X.v[4 * q] = f.x; X.v[4 * q + 1] = f.y; X.v[4 * q + 2] = f.z; X.v[4 * q + 3] = f.w;
        }
    }
}

// Q4_0 (include/quantization.hpp:8-11; src/quantization.cpp:264-330).
// p: shared address of the 18-byte block (2-byte aligned).
__device__ __forceinline__ float dot_q4_0(uint32_t p, const XInt& X) {
    uint32_t q[4];
    lds_words_2a<4>(p + 2, q);
    const float d = nexus_fp16(lds16(p));
    int al = 0, ah = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t lo = q[k] & 0x0F0F0F0Fu;  // weights 4k..4k+3
        const uint32_t hi = q[k] & 0xF0F0F0F0u;  // 16 * weights 16+4k..
        al = dpx_u(lo, X.v[2 * k], X.v[2 * k + 1], al);
        ah = dpx_u(hi, X.v[8 + 2 * k], X.v[9 + 2 * k], ah);
    }
    // sum((q - 8) * X), exact in int32 (ah carries a factor 16)
    const int t = al + (ah >> 4) - 8 * X.sx;
    return (d * X.s) * (float)t;
}

// Q8_0 (include/quantization.hpp:14-17; src/quantization.cpp:332-379).
__device__ __forceinline__ float dot_q8_0(uint32_t p, const XInt& X) {
    uint32_t q[8];
    lds_words_2a<8>(p + 2, q);
    const float d = nexus_fp16(lds16(p));
    int a0 = 0, a1 = 0;
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
        a0 = dpx_s(q[k], X.v[2 * k], X.v[2 * k + 1], a0);
        a1 = dpx_s(q[k + 1], X.v[2 * k + 2], X.v[2 * k + 3], a1);
    }
    return (d * X.s) * (float)(a0 + a1);
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
        sh = dpx_u(ulo, X.v[2 * k], X.v[2 * k + 1], sh);
        sl = dpx_u(uhi, X.v[8 + 2 * k], X.v[9 + 2 * k], sl);
    }
    const float scale = d * (float)sc;
    const float minv = dmin * (float)mn;
    return X.s * (scale * (float)(sh + sl) - minv * (float)X.sx);
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
        const uint32_t* v = X.v + 8 * t;  // elements 16t .. 16t+15
        int sh = dpx_u(u0, v[0], v[1], 0);
        int sl = dpx_u(u1, v[2], v[3], 0);
        sh = dpx_u(u2, v[4], v[5], sh);
        sl = dpx_u(u3, v[6], v[7], sl);
        const int sx = t == 0 ? X.sa : X.sb;
        const int sc = (int)(int8_t)((scw >> (8 * t)) & 0xffu);
        const float scale = d * (float)sc;
        r = fmaf(scale, (float)(sh + sl - 32 * sx), r);
    }
    return X.s * r;
}

// ------------------------------------------------------- grouped decoders
// 32 Q4_0 weights already in registers (4 words of nibble pairs) against x.
__device__ __forceinline__ float q4_0_block(float d, const uint32_t (&q)[4], const XInt& X) {
    int al = 0, ah = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t lo = q[k] & 0x0F0F0F0Fu;  // weights 4k..4k+3
        const uint32_t hi = q[k] & 0xF0F0F0F0u;  // 16 * weights 16+4k..
        al = dpx_u(lo, X.v[2 * k], X.v[2 * k + 1], al);
        ah = dpx_u(hi, X.v[8 + 2 * k], X.v[9 + 2 * k], ah);
    }
    // sum((q - 8) * X), exact: the high-nibble sum carries a factor 16
    const int t = al + (ah >> 4) - 8 * X.sx;
    return (d * X.s) * (float)t;
}

// Two consecutive Q4_0 blocks (36 bytes) at a 4-byte-aligned shared address.
__device__ __forceinline__ float dot_q4_0_x2(uint32_t p, const XInt& X0, const XInt& X1) {
    uint32_t w[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) w[k] = lds32(p + 4 * k);
    uint32_t q0[4], q1[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        q0[k] = __byte_perm(w[k], w[k + 1], 0x5432);  // bytes 2..17
        q1[k] = w[5 + k];                             // bytes 20..35
    }
    return q4_0_block(nexus_fp16(w[0] & 0xffffu), q0, X0) + q4_0_block(nexus_fp16_hi(w[4]), q1, X1);
}

__device__ __forceinline__ float q8_0_block(float d, const uint32_t (&q)[8], const XInt& X) {
    int a0 = 0, a1 = 0;
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
        a0 = dpx_s(q[k], X.v[2 * k], X.v[2 * k + 1], a0);
        a1 = dpx_s(q[k + 1], X.v[2 * k + 2], X.v[2 * k + 3], a1);
    }
    return (d * X.s) * (float)(a0 + a1);
}

// Two consecutive Q8_0 blocks (68 bytes) at a 4-byte-aligned shared address.
__device__ __forceinline__ float dot_q8_0_x2(uint32_t p, const XInt& X0, const XInt& X1) {
    uint32_t w[17];
#pragma unroll
    for (int k = 0; k < 17; ++k) w[k] = lds32(p + 4 * k);
    uint32_t q0[8], q1[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        q0[k] = __byte_perm(w[k], w[k + 1], 0x5432);  // bytes 2..33
        q1[k] = w[9 + k];                             // bytes 36..67
    }
    return q8_0_block(nexus_fp16(w[0] & 0xffffu), q0, X0) + q8_0_block(nexus_fp16_hi(w[8]), q1, X1);
}

// Q5_K sub-block: 16 qs bytes (4 words), its qh word, against x.
__device__ __forceinline__ int q5_k_sub(const uint4& qv, uint32_t qhw, const XInt& X) {
    const uint32_t qs[4] = {qv.x, qv.y, qv.z, qv.w};
    int sh = 0, sl = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t hb = (qhw >> (8 * k)) & 0xffu;
        const uint32_t he = ((hb & 0x55u) * 0x00410410u) & 0x10101010u;
        const uint32_t ho = (((hb >> 1) & 0x55u) * 0x00410410u) & 0x10101010u;
        const uint32_t ulo = (qs[k] & 0x0F0F0F0Fu) | he;
        const uint32_t uhi = ((qs[k] >> 4) & 0x0F0F0F0Fu) | ho;
        sh = dpx_u(ulo, X.v[2 * k], X.v[2 * k + 1], sh);
        sl = dpx_u(uhi, X.v[8 + 2 * k], X.v[9 + 2 * k], sl);
    }
    return sh + sl;
}

// Sub-blocks 4h..4h+3 (half h of the 176-byte super-block at 16-byte-aligned
// o).  Scales and mins of the four sub-blocks come out of the 12 packed bytes
// four at a time (src/quantization.cpp:418-430).
__device__ __forceinline__ float dot_q5_k_x4(uint32_t o, int h, const XInt (&X)[4]) {
    const uint32_t dd = lds32(o);
    const float d = nexus_fp16(dd & 0xffffu);
    const float dmin = nexus_fp16_hi(dd);
    const uint32_t s0 = lds32(o + 4), s1 = lds32(o + 8), s2 = lds32(o + 12);
    const uint32_t scw = h ? ((s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u)) : (s0 & 0x3F3F3F3Fu);
    const uint32_t mnw = h ? (((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u)) : (s1 & 0x3F3F3F3Fu);
    const uint4 qh = lds128(o + 16 + 16 * h);
    const uint32_t qhw[4] = {qh.x, qh.y, qh.z, qh.w};
    float r = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint4 qv = lds128(o + 48 + 64 * h + 16 * t);
        const int u = q5_k_sub(qv, qhw[t], X[t]);
        const float scale = d * (float)((scw >> (8 * t)) & 0xffu);
        const float minv = dmin * (float)((mnw >> (8 * t)) & 0xffu);
        r = fmaf(X[t].s, scale * (float)u - minv * (float)X[t].sx, r);
    }
    return r;
}

// Q6_K: 16 weights of one sub-block from 2 ql words and 1 qh word.
// v: the 8 int16 x pairs of the sub-block's 16 elements.
__device__ __forceinline__ int q6_k_sub(uint32_t l0, uint32_t l1, uint32_t hw, const uint32_t* v) {
    const uint32_t pa = __byte_perm(hw, 0, 0x1100);  // qh bytes 0,0,1,1
    const uint32_t pb = __byte_perm(hw, 0, 0x3322);  // qh bytes 2,2,3,3
    const uint32_t u0 = (l0 & 0x0F0F0F0Fu) | (((pa << 4) & 0x00300030u) | (pa & 0x30003000u));
    const uint32_t u1 = (l1 & 0x0F0F0F0Fu) | (((pb << 4) & 0x00300030u) | (pb & 0x30003000u));
    const uint32_t u2 = ((l0 >> 4) & 0x0F0F0F0Fu) | (((pa << 2) & 0x00300030u) | ((pa >> 2) & 0x30003000u));
    const uint32_t u3 = ((l1 >> 4) & 0x0F0F0F0Fu) | (((pb << 2) & 0x00300030u) | ((pb >> 2) & 0x30003000u));
    int sh = dpx_u(u0, v[0], v[1], 0);
    int sl = dpx_u(u1, v[2], v[3], 0);
    sh = dpx_u(u2, v[4], v[5], sh);
    sl = dpx_u(u3, v[6], v[7], sl);
    return sh + sl;
}

// Work items 4h..4h+3 (sub-blocks 8h..8h+7) of the 210-byte super-block at
// 2-byte-aligned o.
__device__ __forceinline__ float dot_q6_k_x4(uint32_t o, int h, const XInt (&X)[4]) {
    uint32_t L[16], H[8], SC[2];
    lds_words_2a<16>(o + 64 * h, L);
    lds_words_2a<8>(o + 128 + 32 * h, H);
    lds_words_2a<2>(o + 192 + 8 * h, SC);
    const float d = nexus_fp16(lds16(o + 208));
    float r = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int sc0 = (int)(int8_t)((SC[t >> 1] >> (16 * (t & 1))) & 0xffu);
        const int sc1 = (int)(int8_t)((SC[t >> 1] >> (16 * (t & 1) + 8)) & 0xffu);
        const int v0 = q6_k_sub(L[4 * t], L[4 * t + 1], H[2 * t], X[t].v) - 32 * X[t].sa;
        const int v1 = q6_k_sub(L[4 * t + 2], L[4 * t + 3], H[2 * t + 1], X[t].v + 8) - 32 * X[t].sb;
        r = fmaf(X[t].s, d * ((float)sc0 * (float)v0 + (float)sc1 * (float)v1), r);
    }
    return r;
}

// FP16: 16 halves at p against x held in registers.  FP16 rows are whole
// 32-byte work items (K % 16 == 0) and the staging keeps them 16-byte
// aligned, so two 128-bit shared loads fetch them.
// The reference's decoder rebiases the exponent without special-casing zero
// and subnormal halves (0x0000 -> 2^-15).  For every half whose exponent
// field is at most 29 that equals half the IEEE value of h + 0x0400 (exponent
// one higher), so the hardware conversion serves: one add per word, one
// conversion per half, and the sum is halved at the end (exact: the partial
// sums are all exactly doubled).  One SWAR test per word finds exponents 30
// and 31 (|w| >= 32768, Inf, NaN), for which the bit-level decoder runs.
__device__ __forceinline__ float dot_f16(uint32_t p, const XF16& X) {
    const uint4 lo = lds128(p), hi = lds128(p + 16);
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint32_t big = 0;  // bit 15 of a half set when its exponent field is 30 or 31
#pragma unroll
    for (int q = 0; q < 8; ++q) big |= (w[q] & 0x7c007c00u) + 0x08000800u;
    float a0 = 0.f, a1 = 0.f;
    if ((big & 0x80008000u) == 0u) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const uint32_t v = w[q] + 0x04000400u;  // no carry between the halves: both exponents <= 29
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v));
            a0 = fmaf(f.x, X.v[2 * q], a0);
            a1 = fmaf(f.y, X.v[2 * q + 1], a1);
        }
        return (a0 + a1) * 0.5f;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        a0 = fmaf(nexus_fp16(w[q] & 0xffffu), X.v[2 * q], a0);
        a1 = fmaf(nexus_fp16_hi(w[q]), X.v[2 * q + 1], a1);
    }
    return a0 + a1;
}

template <class F>
__device__ __forceinline__ uint32_t wi_offset(int j) {
    if constexpr (F::kWIPerBlock == 1) return (uint32_t)j * F::kBlockBytes;
    else return (uint32_t)(j / F::kWIPerBlock) * F::kBlockBytes;
}

template <class F, class X>
__device__ __forceinline__ float dot_wi(uint32_t row, int wi, const X& x) {
    const uint32_t b = row + wi_offset<F>(wi);
    if constexpr (F::kIntX) {
        if constexpr (F::kBlockBytes == 18) return dot_q4_0(b, x);
        else if constexpr (F::kBlockBytes == 34) return dot_q8_0(b, x);
        else if constexpr (F::kBlockBytes == 176) return dot_q5_k(b, wi & 7, x);
        else return dot_q6_k(b, wi & 7, x);
    } else {
        return dot_f16(b, x);
    }
}

// This lane's partial dot product of one row (shared address `row`) over its
// work items; G consecutive items per lane when grouped.  Groups are whole:
// the host only picks G > 1 when segments and rows hold whole groups.
template <class F, int G, class XT>
__device__ __forceinline__ float row_partial(uint32_t row, const int (&wi)[kMaxJ], const bool (&has)[kMaxJ],
                                             const XT (&X)[kMaxJ]) {
    float acc = 0.f;
    if constexpr (G == 1) {
#pragma unroll
        for (int j = 0; j < kMaxJ; ++j)
            if (has[j]) acc += dot_wi<F>(row, wi[j], X[j]);
    } else {
#pragma unroll
        for (int jj = 0; jj < kMaxJ / G; ++jj) {
            const int j = jj * G;
            if (!has[j]) continue;
            const uint32_t b = row + wi_offset<F>(wi[j]);
            if constexpr (F::kBlockBytes == 18) acc += dot_q4_0_x2(b, X[j], X[j + 1]);
            else if constexpr (F::kBlockBytes == 34) acc += dot_q8_0_x2(b, X[j], X[j + 1]);
            else if constexpr (F::kBlockBytes == 176)
                acc += dot_q5_k_x4(b, (wi[j] >> 2) & 1, *reinterpret_cast<const XInt(*)[4]>(&X[j]));
            else
                acc += dot_q6_k_x4(b, (wi[j] >> 2) & 1, *reinterpret_cast<const XInt(*)[4]>(&X[j]));
        }
    }
    return acc;
}

// Lane -> work items of segment sg: G consecutive items per lane per round of
// 32*G; has[j] is false past the segment or the row.
template <int G>
__device__ __forceinline__ void lane_items(int lane, int sg, int SW, int J, int NW, int (&wi)[kMaxJ],
                                           bool (&has)[kMaxJ]) {
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
        const int o = G * (lane + 32 * (j / G)) + (j % G);
        wi[j] = sg * SW + o;
        has[j] = j < J && o < SW && wi[j] < NW;
    }
}

// ------------------------------------------------------------------- kernel
// Warp w of the 15 consumer warps owns K segment (w % S) and row group
// (w / S), S in 1..15; the CTA's rows are dealt to the n_grp = 15/S row
// groups round-robin (row q of the CTA -> group q % n_grp), and the
// 15 - S*n_grp warps past the last group idle.  A warp keeps the x slices of its
// segment in registers (J work items per lane), so per row it only reads
// weights from shared memory.  With S == 1 a warp covers whole rows and writes
// y itself; with S > 1 each warp leaves its row partial in a shared slot and
// bumps the row's arrival counter, and the last of the S warps sums the slots
// in segment order and writes y -- deterministic, no CTA-wide barrier.
template <class F, int G>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_m1_kernel(const GemvParams p) {
    using XT = typename std::conditional<F::kIntX, XInt, XF16>::type;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full_bar = sbase;                     // kMaxStages x 8 B
    const uint32_t empty_bar = sbase + 8 * kMaxStages;  // kMaxStages x 8 B
    float* slots = reinterpret_cast<float*>(smem + kBarBytes);            // [n_stages][R][S]
    int* counters = reinterpret_cast<int*>(smem + kBarBytes + kMaxSlots * 4);  // [n_stages][R]
    const uint32_t stage0 = sbase + kSmemHeader;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_cta = gridDim.x, c = blockIdx.x;
    const int row_begin = (int)((int64_t)p.N * c / n_cta);
    const int row_end = (int)((int64_t)p.N * (c + 1) / n_cta);
    const int R = p.stage_rows;
    const int n_st = (row_end - row_begin + R - 1) / R;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.n_stages; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, kConsumerWarps);
        }
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < p.n_stages * R; i += blockDim.x) counters[i] = 0;
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------- producer
        if (lane != 0) return;
        const uint64_t floor16 = p.total_bytes & ~(uint64_t)15;
        const uint64_t stage_span = (uint64_t)R * p.row_bytes;
        uint64_t start = (uint64_t)row_begin * p.row_bytes;
        const uint64_t cta_end = (uint64_t)row_end * p.row_bytes;
        bool ok = true;
        int i = 0, s = 0;
        uint32_t phase = 0;  // parity of the empty-barrier phase to wait for
        for (; i < n_st; ++i) {
            if (i >= p.n_stages && !mbar_wait_bounded(empty_bar + 8 * s, phase)) {
                ok = false;
                break;
            }
            const uint64_t end = min(start + stage_span, cta_end);
            const uint64_t a = start & ~(uint64_t)15;
            const uint64_t bend = min((end + 15) & ~(uint64_t)15, floor16);
            const uint32_t dst = stage0 + (uint32_t)(s * p.stage_bytes);
            // bytes past the last 16-byte boundary of the matrix: plain copies
            if (bend < end) {
                for (uint64_t pos = (bend > a ? bend : a); pos < end; pos += 2)
                    sts16(dst + (uint32_t)(pos - a), *reinterpret_cast<const uint16_t*>(p.W + pos));
                fence_proxy_async_smem();
            }
            const uint32_t n = bend > a ? (uint32_t)(bend - a) : 0u;
            mbar_arrive_expect_tx(full_bar + 8 * s, n);
            if (n) bulk_g2s(dst, p.W + a, n, full_bar + 8 * s);
            start = end;
            if (++s == p.n_stages) {
                s = 0;
                if (i >= p.n_stages) phase ^= 1;  // passes 1, 2, ... wait parities 0, 1, ...
            }
        }
        // leave no copy in flight, also when consumers stopped after a failed wait
        (void)ok;
        for (int k = 0; k < p.n_stages && k < i; ++k) {
            const int j = i - 1 - k;
            mbar_wait_bounded(full_bar + 8 * (j % p.n_stages), (j / p.n_stages) & 1);
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int S = p.segments, NW = p.nwi, SW = p.seg_wi, J = p.wi_per_lane;
    const int sg = warp % S, grp = warp / S, n_grp = kConsumerWarps / S;
    int wi[kMaxJ];
    bool has[kMaxJ];
    lane_items<G>(lane, sg, SW, J, NW, wi, has);

    // x depends on the previous kernel in the stream (x quantization or the
    // GEMV that produced x); the weights do not, so the producer never waits.
    pdl_wait();
    XT X[kMaxJ];
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
        if (has[j]) {
            if constexpr (F::kIntX) load_xint(p.xq_limbs, p.xq_meta, wi[j], X[j]);
            else load_xf16(p.x, p.x_bf16, wi[j], X[j]);
        }
    }

    int s = 0, rot = 0;  // stage buffer, (i * R) % n_grp
    uint32_t phase = 0;  // parity of the full-barrier phase to wait for
    for (int i = 0; i < n_st; ++i) {
        const int r0 = row_begin + i * R;
        const int nr = min(R, row_end - r0);
        if (!mbar_wait_bounded(full_bar + 8 * s, phase)) break;
        const uint32_t base = stage0 + (uint32_t)(s * p.stage_bytes) + (uint32_t)(((uint64_t)r0 * p.row_bytes) & 15);
        // first local row of this warp's group in this stage
        int rl = grp - rot;
        if (rl < 0) rl += n_grp;
        if (grp >= n_grp) rl = nr;  // the 15 - S*n_grp warps past the last row group idle
        for (; rl < nr; rl += n_grp) {
            const uint32_t row = base + (uint32_t)(rl * p.row_bytes);
            float acc = row_partial<F, G>(row, wi, has, X);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (S == 1) {
                if (lane == 0) p.y[r0 + rl] = acc;
            } else if (lane == 0) {
                float* sl = slots + (s * R + rl) * S;
                sl[sg] = acc;
                __threadfence_block();
                const int prev = atomicAdd(&counters[s * R + rl], 1);
                if (prev == S - 1) {  // last segment of this row: sum in segment order
                    __threadfence_block();
                    float y = 0.f;
                    for (int k = 0; k < S; ++k) y += *(volatile float*)(sl + k);
                    p.y[r0 + rl] = y;
                    counters[s * R + rl] = 0;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar + 8 * s);
        if (++s == p.n_stages) {
            s = 0;
            phase ^= 1;
        }
        rot += R % n_grp;
        if (rot >= n_grp) rot -= n_grp;
    }
}

// -------------------------------------------------------- x quantization
// Element rule shared by every x quantizer (so all paths give the same bits):
// X = rint(x * (32639 / amax)), one IEEE division per block.  Blocks whose
// amax is below 2^-100 (where 32639 / amax could overflow) divide element by
// element instead: X = rint((x / amax) * 32639).  Called for finite amax > 0.
constexpr float kXQTiny = 0x1p-100f;
__device__ __forceinline__ float xq_inv(float amax) { return __fdiv_rn(kXQMax, amax); }
__device__ __forceinline__ int xq_clamp(float q) { return max(-32639, min(32639, __float2int_rn(q))); }
__device__ __forceinline__ int xq_elem_fast(float v, float inv) { return xq_clamp(__fmul_rn(v, inv)); }  // amax >= kXQTiny
__device__ __forceinline__ int xq_elem_tiny(float v, float amax) { return xq_clamp(__fmul_rn(__fdiv_rn(v, amax), kXQMax)); }
__device__ __forceinline__ int xq_elem(float v, float amax, float inv) {
    return amax >= kXQTiny ? xq_elem_fast(v, inv) : xq_elem_tiny(v, amax);
}

// One 32-element block of x, one element per lane: writes X (xq_elem) as
// int16, s = amax / 32639, and {s, sum X[0:16), sum X[16:32), sum X}.
// Non-finite blocks get s = amax (Inf/NaN) and X = 0.
__device__ __forceinline__ void quantize_x_block(float v, int lane, uint8_t* limbs, int4* meta) {
    const uint32_t abits = __float_as_uint(v) & 0x7fffffffu;
    const uint32_t mbits = __reduce_max_sync(0xffffffffu, abits);
    const float amax = __uint_as_float(mbits);
    int X = 0;
    float s = 0.0f;
    if (mbits >= 0x7f800000u) {
        s = amax;  // Inf or NaN
    } else if (mbits != 0) {
        X = xq_elem(v, amax, xq_inv(amax));
        s = __fdiv_rn(amax, kXQMax);
    }
    reinterpret_cast<int16_t*>(limbs)[lane] = (int16_t)X;
    const int sa = __reduce_add_sync(0xffffffffu, lane < 16 ? X : 0);
    const int sb = __reduce_add_sync(0xffffffffu, lane < 16 ? 0 : X);
    if (lane == 0) *meta = make_int4((int)__float_as_uint(s), sa, sb, sa + sb);
}

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
    const size_t bidx = (size_t)m * nxb + xb;
    quantize_x_block(v, lane, limbs + bidx * kXQLimbBytes, meta + bidx);
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
