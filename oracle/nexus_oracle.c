/*
 * nexus_oracle.c -- CPU ORACLE (TEST INFRASTRUCTURE ONLY).
 *
 * This file restates, in plain C, the arithmetic of NexusLLM's quantized GEMV
 * and dequantization path so that the CUDA product can be checked against it.
 * It is never linked into the product library and is never on a measured path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it,
 * and only as the checker (or as the timed CPU "port" baseline).
 *
 * Every function names the reference lines it follows.  The GEMV loops
 * reproduce the reference's AVX2+FMA branch (the branch selected by
 * NEXUS_HAVE_AVX2 on x86-64, include/nexus_common.hpp:63-71): the same 8-lane
 * accumulator layout, the same fused multiply-adds and the same left-to-right
 * horizontal sums, so that on identical inputs the result is expected to be
 * bit-identical to the reference build, not merely close.  Build flags:
 * -O2 -mfma -ffp-contract=off; every fused operation is an explicit fmaf().
 *
 * Parity is pinned: tests/golden/ holds vectors produced by the reference's
 * own src/quantization.cpp compiled unmodified (oracle/Makefile, target "ref"),
 * and tests/test_oracle_golden.py checks this file against them.
 *
 * Block byte layouts (little-endian, packed, alignof == 2):
 *   Q4_0 18 B : d u16 @0, qs[16] @2           (include/quantization.hpp:8-11)
 *   Q8_0 34 B : d u16 @0, qs[32] s8 @2        (include/quantization.hpp:14-17)
 *   Q5_K 176 B: d @0, dmin @2, scales[12] @4, qh[32] @16, qs[128] @48
 *                                             (include/quantization.hpp:31-37)
 *   Q6_K 210 B: ql[128] @0, qh[64] @128, scales[16] s8 @192, d @208
 *                                             (include/quantization.hpp:42-47)
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define Q4_0_BYTES 18
#define Q8_0_BYTES 34
#define Q5_K_BYTES 176
#define Q6_K_BYTES 210
#define QK 256

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* include/quantization.hpp:59-70.  Non-IEEE decoder: exponent 0x1f gives +0.0
 * (Inf/NaN dropped, sign discarded); zero and subnormal halves are NOT special
 * cased, so 0x0000 decodes to 2^-15 and 0x8000 to -2^-15. */
float oracle_fp16_to_fp32(uint16_t h) {
    uint32_t w = (uint32_t)(h & 0x7fffu) << 13;
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (uint32_t)(h & 0x7c00u) >> 10;
    if (e == 0x1fu) return 0.0f;
    uint32_t v = sign | (w + (0x70u << 23));
    float f;
    memcpy(&f, &v, 4);
    return f;
}

/* Left-to-right horizontal sum of an 8-lane accumulator, as written in the
 * reference: arr[0] + arr[1] + ... + arr[7] (quantization.cpp:302,360,402,572,676). */
static inline float hsum8(const float a[8]) {
    float s = a[0] + a[1];
    s = s + a[2];
    s = s + a[3];
    s = s + a[4];
    s = s + a[5];
    s = s + a[6];
    s = s + a[7];
    return s;
}

/* ---------------------------------------------------------------- dequant */

/* src/quantization.cpp:48-82 (x86 scalar branch :73-79): out = int8(q-8) * d. */
void oracle_dequantize_q4_0(const uint8_t* blocks, float* out, size_t num_blocks) {
    for (size_t b = 0; b < num_blocks; ++b) {
        const uint8_t* blk = blocks + b * Q4_0_BYTES;
        float d = oracle_fp16_to_fp32(rd16(blk));
        for (int i = 0; i < 16; ++i) {
            uint8_t v = blk[2 + i];
            int8_t v0 = (int8_t)((v & 0x0F) - 8);
            int8_t v1 = (int8_t)((v >> 4) - 8);
            out[b * 32 + i] = (float)v0 * d;
            out[b * 32 + 16 + i] = (float)v1 * d;
        }
    }
}

/* Q8_0 has no named dequantizer; the reference dequantizes inline with
 * out = qs[j] * d (src/forward_pass.cpp:379-384, transformer_engine.cpp:228-234). */
void oracle_dequantize_q8_0(const uint8_t* blocks, float* out, size_t num_blocks) {
    for (size_t b = 0; b < num_blocks; ++b) {
        const uint8_t* blk = blocks + b * Q8_0_BYTES;
        float d = oracle_fp16_to_fp32(rd16(blk));
        for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
    }
}

/* FP16 weights dequantize element-wise through the same decoder
 * (src/forward_pass.cpp:366-370). */
void oracle_dequantize_fp16(const uint16_t* w, float* out, size_t count) {
    for (size_t i = 0; i < count; ++i) out[i] = oracle_fp16_to_fp32(w[i]);
}

/* src/quantization.cpp:418-430 -- 8 (scale, min) 6-bit pairs from 12 bytes. */
static void unpack_q5_k_scales(const uint8_t* s, uint8_t* sc, uint8_t* m) {
    for (int i = 0; i < 4; ++i) {
        sc[i] = s[i] & 0x3F;
        m[i] = s[i + 4] & 0x3F;
        sc[i + 4] = (uint8_t)((s[i + 8] & 0x0F) | ((s[i] >> 6) << 4));
        m[i + 4] = (uint8_t)((s[i + 8] >> 4) | ((s[i + 4] >> 6) << 4));
    }
}

/* src/quantization.cpp:432-473.  NexusLLM's own intra-block bit layout (not
 * ggml's): for sub-block sb and i < 16, low nibble of qs[16sb+i] with qh bit
 * 2(i%4) of qh[4sb+i/4] gives element 32sb+i; the high nibble with bit
 * 2(i%4)+1 gives element 32sb+16+i.  Two roundings: (v*scale) then -min. */
void oracle_dequantize_q5_k(const uint8_t* blocks, float* out, size_t num_blocks) {
    for (size_t b = 0; b < num_blocks; ++b) {
        const uint8_t* blk = blocks + b * Q5_K_BYTES;
        const float d = oracle_fp16_to_fp32(rd16(blk));
        const float dmin = oracle_fp16_to_fp32(rd16(blk + 2));
        uint8_t sc[8], m[8];
        unpack_q5_k_scales(blk + 4, sc, m);
        const uint8_t* qh = blk + 16;
        const uint8_t* qs = blk + 48;
        for (int sb = 0; sb < 8; ++sb) {
            const float scale = d * (float)sc[sb];
            const float min_val = dmin * (float)m[sb];
            for (int i = 0; i < 16; ++i) {
                uint8_t q = qs[sb * 16 + i];
                uint8_t h = qh[sb * 4 + i / 4];
                int sl = (i % 4) * 2;
                uint8_t h0 = (h >> sl) & 1, h1 = (h >> (sl + 1)) & 1;
                uint8_t v0 = (uint8_t)((q & 0x0F) | (h0 << 4));
                uint8_t v1 = (uint8_t)((q >> 4) | (h1 << 4));
                float p0 = (float)v0 * scale;
                float p1 = (float)v1 * scale;
                out[b * QK + sb * 32 + i] = p0 - min_val;
                out[b * QK + sb * 32 + 16 + i] = p1 - min_val;
            }
        }
    }
}

/* src/quantization.cpp:475-509.  For sub-block sb (16 elements) and i < 8:
 * low nibble of ql[8sb+i] with bits (i%2)*4+{0,1} of qh[4sb+i/2] gives element
 * 16sb+i; the high nibble with bits (i%2)*4+{2,3} gives 16sb+8+i; value-32. */
void oracle_dequantize_q6_k(const uint8_t* blocks, float* out, size_t num_blocks) {
    for (size_t b = 0; b < num_blocks; ++b) {
        const uint8_t* blk = blocks + b * Q6_K_BYTES;
        const float d = oracle_fp16_to_fp32(rd16(blk + 208));
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        for (int sb = 0; sb < 16; ++sb) {
            const float scale = d * (float)sc[sb];
            for (int i = 0; i < 8; ++i) {
                uint8_t l = ql[sb * 8 + i];
                uint8_t h = qh[sb * 4 + i / 2];
                int s = (i % 2) * 4;
                uint8_t h0 = (h >> s) & 3, h1 = (h >> (s + 2)) & 3;
                int8_t v0 = (int8_t)((int8_t)((l & 0x0F) | (h0 << 4)) - 32);
                int8_t v1 = (int8_t)((int8_t)((l >> 4) | (h1 << 4)) - 32);
                out[b * QK + sb * 16 + i] = (float)v0 * scale;
                out[b * QK + sb * 16 + 8 + i] = (float)v1 * scale;
            }
        }
    }
}

/* ------------------------------------------------------------------- GEMV */

/* src/quantization.cpp:264-330, AVX2 branch :281-302.  Two 8-lane
 * accumulators: acc0 over (low nibbles 0-7, 8-15) x x[0:16), acc1 over (high
 * nibbles 0-7, 8-15) x x[16:32); block_sum = hsum(acc0 + acc1);
 * total += d * block_sum (:325).  The reference build (g++ -O3 -mfma, C++
 * mode, default -ffp-contract=fast) compiles that statement as one fused
 * multiply-add, so it is fmaf() here; the golden vectors confirm it. */
void oracle_gemv_q4_0(const uint8_t* W, const float* x, float* y, size_t rows, size_t cols) {
    const size_t nb = cols / 32;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t* row = W + r * nb * Q4_0_BYTES;
        float total = 0.0f;
        for (size_t b = 0; b < nb; ++b) {
            const uint8_t* blk = row + b * Q4_0_BYTES;
            const float d = oracle_fp16_to_fp32(rd16(blk));
            const float* xb = x + b * 32;
            float wl[16], wh[16], acc[8];
            for (int i = 0; i < 16; ++i) {
                uint8_t v = blk[2 + i];
                wl[i] = (float)((v & 0x0F) - 8);
                wh[i] = (float)((v >> 4) - 8);
            }
            for (int l = 0; l < 8; ++l) {
                float a0 = fmaf(wl[l], xb[l], 0.0f);
                a0 = fmaf(wl[8 + l], xb[8 + l], a0);
                float a1 = fmaf(wh[l], xb[16 + l], 0.0f);
                a1 = fmaf(wh[8 + l], xb[24 + l], a1);
                acc[l] = a0 + a1;
            }
            const float block_sum = hsum8(acc);
            total = fmaf(d, block_sum, total);
        }
        y[r] = total;
    }
}

/* src/quantization.cpp:332-379, AVX2 branch :349-360.  One 8-lane accumulator
 * over the four 8-element chunks; total += d * block_sum (:374), fused by the
 * reference build exactly as in the Q4_0 GEMV above. */
void oracle_gemv_q8_0(const uint8_t* W, const float* x, float* y, size_t rows, size_t cols) {
    const size_t nb = cols / 32;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t* row = W + r * nb * Q8_0_BYTES;
        float total = 0.0f;
        for (size_t b = 0; b < nb; ++b) {
            const uint8_t* blk = row + b * Q8_0_BYTES;
            const float d = oracle_fp16_to_fp32(rd16(blk));
            const int8_t* qs = (const int8_t*)(blk + 2);
            const float* xb = x + b * 32;
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int i = 0; i < 32; i += 8)
                for (int l = 0; l < 8; ++l) acc[l] = fmaf((float)qs[i + l], xb[i + l], acc[l]);
            const float block_sum = hsum8(acc);
            total = fmaf(d, block_sum, total);
        }
        y[r] = total;
    }
}

/* src/quantization.cpp:381-410.  8-lane FMA accumulator over full 8-element
 * chunks, horizontal sum, then a scalar tail (:405-407) for cols % 8 whose
 * sum += w * x the reference build also fuses into one multiply-add. */
void oracle_gemv_fp16(const uint16_t* W, const float* x, float* y, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r) {
        const uint16_t* row = W + r * cols;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        size_t c = 0;
        for (; c + 8 <= cols; c += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(oracle_fp16_to_fp32(row[c + l]), x[c + l], acc[l]);
        float sum = hsum8(acc);
        for (; c < cols; ++c) sum = fmaf(oracle_fp16_to_fp32(row[c]), x[c], sum);
        y[r] = sum;
    }
}

/* src/quantization.cpp:511-620, AVX2 branch :545-572.  Per 32-element
 * sub-block: w = fmsub(v, scale, min) (one rounding), acc = fma(w, x, acc)
 * over four 8-lane chunks, total += hsum(acc). */
void oracle_gemv_q5_k(const uint8_t* W, const float* x, float* y, size_t rows, size_t cols) {
    const size_t nb = cols / QK;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t* row = W + r * nb * Q5_K_BYTES;
        float total = 0.0f;
        for (size_t b = 0; b < nb; ++b) {
            const uint8_t* blk = row + b * Q5_K_BYTES;
            const float d = oracle_fp16_to_fp32(rd16(blk));
            const float dmin = oracle_fp16_to_fp32(rd16(blk + 2));
            uint8_t sc[8], m[8];
            unpack_q5_k_scales(blk + 4, sc, m);
            const uint8_t* qh = blk + 16;
            const uint8_t* qs = blk + 48;
            const float* xb = x + b * QK;
            for (int sb = 0; sb < 8; ++sb) {
                const float scale = d * (float)sc[sb];
                const float min_val = dmin * (float)m[sb];
                const float* xs = xb + sb * 32;
                float w[32], acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int i = 0; i < 16; ++i) {
                    uint8_t q = qs[sb * 16 + i];
                    uint8_t h = qh[sb * 4 + i / 4];
                    int sl = (i % 4) * 2;
                    w[i] = (float)((q & 0x0F) | (((h >> sl) & 1) << 4));
                    w[i + 16] = (float)((q >> 4) | (((h >> (sl + 1)) & 1) << 4));
                }
                for (int vi = 0; vi < 32; vi += 8)
                    for (int l = 0; l < 8; ++l) {
                        float vw = fmaf(w[vi + l], scale, -min_val);
                        acc[l] = fmaf(vw, xs[vi + l], acc[l]);
                    }
                total = total + hsum8(acc);
            }
        }
        y[r] = total;
    }
}

/* src/quantization.cpp:622-722, AVX2 branch :650-676.  Per 16-element
 * sub-block: vw = v * scale (separate multiply), acc = fma(vw0, x[0:8), 0),
 * acc = fma(vw1, x[8:16), acc), total += hsum(acc). */
void oracle_gemv_q6_k(const uint8_t* W, const float* x, float* y, size_t rows, size_t cols) {
    const size_t nb = cols / QK;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t* row = W + r * nb * Q6_K_BYTES;
        float total = 0.0f;
        for (size_t b = 0; b < nb; ++b) {
            const uint8_t* blk = row + b * Q6_K_BYTES;
            const float d = oracle_fp16_to_fp32(rd16(blk + 208));
            const uint8_t* ql = blk;
            const uint8_t* qh = blk + 128;
            const int8_t* sc = (const int8_t*)(blk + 192);
            const float* xb = x + b * QK;
            for (int sb = 0; sb < 16; ++sb) {
                const float scale = d * (float)sc[sb];
                const float* xs = xb + sb * 16;
                float w[16], acc[8];
                for (int i = 0; i < 8; ++i) {
                    uint8_t l = ql[sb * 8 + i];
                    uint8_t h = qh[sb * 4 + i / 2];
                    int s = (i % 2) * 4;
                    int8_t v0 = (int8_t)((int8_t)((l & 0x0F) | (((h >> s) & 3) << 4)) - 32);
                    int8_t v1 = (int8_t)((int8_t)((l >> 4) | (((h >> (s + 2)) & 3) << 4)) - 32);
                    w[i] = (float)v0;
                    w[i + 8] = (float)v1;
                }
                for (int l = 0; l < 8; ++l) {
                    float a = fmaf(w[l] * scale, xs[l], 0.0f);
                    acc[l] = fmaf(w[8 + l] * scale, xs[8 + l], a);
                }
                total = total + hsum8(acc);
            }
        }
        y[r] = total;
    }
}

/* ------------------------------------------------ INT4-AWQ and FP8-E4M3 */

/* src/quantization.cpp:12-26 (fp8_e4m3_to_fp32): sign, 4-bit exponent (bias
 * 7), 3-bit mantissa; exponent 0 is subnormal mant * 2^-9; 0x7F and 0xFF
 * (the E4M3 NaNs) decode to +0. */
float oracle_fp8_e4m3_to_fp32(uint8_t v) {
    if (v == 0x7F || v == 0xFF) return 0.0f;
    const int sign = (v >> 7) & 1, exp = (v >> 3) & 0xF, mant = v & 0x7;
    const float r = exp == 0 ? ldexpf((float)mant, -9) : ldexpf(1.0f + (float)mant / 8.0f, exp - 7);
    return sign ? -r : r;
}

/* src/quantization.cpp:28-46 (dequantize_int4_awq): element i is nibble i % 8
 * of word i / 8; w = ((float)q - zero) * scale (two roundings) with the group
 * i / group_size; zeros may be NULL (zero 0). */
void oracle_dequantize_int4_awq(const uint32_t* packed, const float* scales, const float* zeros, float* out,
                                size_t count, size_t group_size) {
    for (size_t i = 0; i < count; ++i) {
        const size_t g = i / group_size;
        const float scale = scales[g], zero = zeros ? zeros[g] : 0.0f;
        const uint32_t q = (packed[i / 8] >> ((i % 8) * 4)) & 0x0Fu;
        out[i] = ((float)q - zero) * scale;
    }
}

/* src/quantization.cpp:62-68 (dequantize_fp8_e4m3): decoded value * scale. */
void oracle_dequantize_fp8_e4m3(const uint8_t* in, float* out, size_t count, float scale) {
    for (size_t i = 0; i < count; ++i) out[i] = oracle_fp8_e4m3_to_fp32(in[i]) * scale;
}

/* src/quantization.cpp:102-200, AVX2 branch :146-180.  Per 8-column step c
 * (c + 8 <= cols): the group of column c supplies scale and zero for all 8
 * columns (:149-151), w = ((float)q - zero) * scale, acc[k] = fma(w, x, acc[k]);
 * horizontal sum; scalar tail with the group of each column, where the
 * reference build keeps sum += w * x as a separate multiply and add (unlike
 * the GGUF tails; checked against the reference build).  Row r reads words
 * [r*(cols/8), ...) and groups [r*(cols/group_size), ...). */
void oracle_gemv_int4(const uint32_t* W, const float* x, const float* scales, const float* zeros, float* y,
                      size_t rows, size_t cols, size_t group_size) {
    const size_t packed_cols = cols / 8;
    for (size_t r = 0; r < rows; ++r) {
        const uint32_t* row = W + r * packed_cols;
        const size_t g_base = r * (cols / group_size);
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        size_t c = 0;
        for (; c + 8 <= cols; c += 8) {
            const size_t g = g_base + c / group_size;
            const float scale = scales[g], zero = zeros ? zeros[g] : 0.0f;
            const uint32_t word = row[c / 8];
            for (int k = 0; k < 8; ++k) {
                const float w = ((float)((word >> (k * 4)) & 0x0Fu) - zero) * scale;
                acc[k] = fmaf(w, x[c + k], acc[k]);
            }
        }
        float sum = hsum8(acc);
        for (; c < cols; ++c) {
            const size_t g = g_base + c / group_size;
            const float scale = scales[g], zero = zeros ? zeros[g] : 0.0f;
            const float w = ((float)((row[c / 8] >> ((c % 8) * 4)) & 0x0Fu) - zero) * scale;
            const float p = w * x[c];
            sum = sum + p;
        }
        y[r] = sum;
    }
}

/* src/quantization.cpp:202-262, AVX2 branch :229-249: w = fp8(W) * scale,
 * 8-lane fma accumulator, horizontal sum, scalar tail as a separate multiply
 * and add (as the reference build compiles it). */
void oracle_gemv_fp8(const uint8_t* W, const float* x, float* y, size_t rows, size_t cols, float scale) {
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t* row = W + r * cols;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        size_t c = 0;
        for (; c + 8 <= cols; c += 8)
            for (int k = 0; k < 8; ++k) acc[k] = fmaf(oracle_fp8_e4m3_to_fp32(row[c + k]) * scale, x[c + k], acc[k]);
        float sum = hsum8(acc);
        for (; c < cols; ++c) {
            const float p = (oracle_fp8_e4m3_to_fp32(row[c]) * scale) * x[c];
            sum = sum + p;
        }
        y[r] = sum;
    }
}

/* ------------------------------------------- decode-layer ops beside the GEMV */

/* TransformerOps::rmsnorm (include/transformer_ops.hpp:23-44), fp32 weights or
 * none: sum_sq += x*x left to right (a separate multiply and add in the
 * reference build, checked against it), inv_rms = 1 / sqrt(sum_sq / dim +
 * eps), out = x * inv_rms * w. */
void oracle_rmsnorm(const float* x, const float* w, float* out, size_t dim, float eps) {
    float sum_sq = 0.0f;
    for (size_t i = 0; i < dim; ++i) {
        const float p = x[i] * x[i];
        sum_sq = sum_sq + p;
    }
    const float inv_rms = 1.0f / sqrtf((sum_sq / (float)dim) + eps);
    for (size_t i = 0; i < dim; ++i) {
        const float t = x[i] * inv_rms;
        out[i] = w ? t * w[i] : t;
    }
}

/* TransformerOps::silu / swiglu (include/transformer_ops.hpp:86-95):
 * out = (g / (1 + exp(-g))) * u. */
void oracle_swiglu(const float* g, const float* u, float* out, size_t dim) {
    for (size_t i = 0; i < dim; ++i) {
        const float s = g[i] / (1.0f + expf(-g[i]));
        out[i] = s * u[i];
    }
}

/* Dispatch by NexusLLM DataType value (include/nexus_common.hpp:244-260), as
 * TransformerOps::matmul_vec_dispatch does (include/transformer_ops.hpp:157-173).
 * Returns 0 on success, -3 (ERROR_FORMAT_UNSUPPORTED) for other types. */
int oracle_gemv_dispatch(const void* W, unsigned dtype, const float* x, float* y, size_t rows, size_t cols) {
    switch (dtype) {
        case 1: oracle_gemv_fp16((const uint16_t*)W, x, y, rows, cols); return 0;
        case 7: oracle_gemv_q4_0((const uint8_t*)W, x, y, rows, cols); return 0;
        case 9: oracle_gemv_q8_0((const uint8_t*)W, x, y, rows, cols); return 0;
        case 11: oracle_gemv_q5_k((const uint8_t*)W, x, y, rows, cols); return 0;
        case 12: oracle_gemv_q6_k((const uint8_t*)W, x, y, rows, cols); return 0;
        default: return -3;
    }
}
