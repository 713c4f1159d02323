// awq_fp8_kernels.cuh -- INT4-AWQ and FP8-E4M3 GEMV (batch 1) and
// dequantization, the reference's QuantizationKernel::fused_gemv_int4 /
// fused_gemv_fp8 / dequantize_int4_awq / dequantize_fp8_e4m3
// (src/quantization.cpp:12-68,102-262).
//
// Formats (row-major, row r at r * row_bytes):
//  * INT4-AWQ: uint32 words, column c of a row is nibble c % 8 of word c / 8;
//    scales and zeros are separate float32 arrays [rows][cols / group_size];
//    w = (q - zero) * scale, zeros may be absent (zero 0).
//  * FP8-E4M3: one byte per weight (bias 7, subnormal mant * 2^-9, the NaN
//    codes 0x7F / 0xFF decode to 0), one float32 scale for the matrix.
//
// GEMV kernels: a warp owns 1 or 2 rows at a time (2 when there are enough
// rows to keep every SM's warps busy); lane l streams their
// 16-byte chunks l, l + 32, ... with non-allocating 16-byte loads, the rows'
// loads of one chunk index in flight together and the chunk's x read from
// shared memory once for all of them.  The x vector is
// staged once per CTA in shared memory, transposed so that the 32 lanes'
// chunk reads are conflict-free (16-byte piece q of chunk c at (q * NC + c) *
// 16).
//  * INT4: x as the library's 16-bit fixed-point blocks (xquant_kernel, the
//    same quantization as the GGUF path), re-paired per 8 columns so that the
//    low and high nibbles of a word meet their x values in one dp2a each:
//    sum(q * X) is exact in int32, then per 32-column chunk
//    scale * s_x * (sum(q X) - zero * sum(X)).
//  * FP8: x in fp32; two weights per hardware e4m3x2 -> f16x2 conversion
//    (exact), fp32 fma; the matrix scale is applied once per row.  Words
//    holding a NaN code are patched to 0 first (a branch that real FP8
//    weights never take).
// Shapes outside the fast kernels' limits (column counts, group sizes, K too
// large for shared memory, unaligned pointers) take a generic kernel with the
// reference's per-element arithmetic.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "gemv_kernels.cuh"

namespace nexus_gpu {

constexpr int kRowsThreads = 256;          // 8 warps per CTA
constexpr int kRowsPerWarpMax = 2;  // rows a warp streams together (1 when rows are few)
constexpr int kInt4MaxCols = 32768;        // shared x: 72 bytes per 32 columns
constexpr int kFp8MaxCols = 16384;         // shared x: 4 bytes per column

// --------------------------------------------------------------- decoders
// fp8_e4m3_to_fp32 (src/quantization.cpp:12-26), exact.
__device__ __forceinline__ float fp8_e4m3_ref(uint32_t v) {
    v &= 0xffu;
    if ((v & 0x7fu) == 0x7fu) return 0.0f;
    const uint32_t e = (v >> 3) & 0xfu, m = v & 0x7u;
    const float mag = e == 0 ? (float)m * 0x1p-9f : __uint_as_float(((e + 120u) << 23) | (m << 20));
    return (v & 0x80u) ? -mag : mag;
}

// ------------------------------------------------------------ dequantize
// dequantize_int4_awq (src/quantization.cpp:28-46): ((float)q - zero) * scale,
// two roundings (no contraction), bit-exact.
__global__ void __launch_bounds__(256) dequant_int4_awq_kernel(const uint32_t* __restrict__ packed,
                                                               const float* __restrict__ scales,
                                                               const float* __restrict__ zeros,
                                                               float* __restrict__ out, uint64_t count,
                                                               uint64_t group_size) {
    pdl_wait();
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t g = i / group_size;
        const float scale = __ldg(scales + g), zero = zeros ? __ldg(zeros + g) : 0.0f;
        const uint32_t q = (__ldg(packed + i / 8) >> ((i % 8) * 4)) & 0x0fu;
        out[i] = __fmul_rn(__fsub_rn((float)q, zero), scale);
    }
}

// dequantize_fp8_e4m3 (src/quantization.cpp:62-68): decoded * scale, bit-exact.
__global__ void __launch_bounds__(256) dequant_fp8_kernel(const uint8_t* __restrict__ in, float* __restrict__ out,
                                                          uint64_t count, float scale) {
    pdl_wait();
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn(fp8_e4m3_ref(__ldg(in + i)), scale);
}

// ------------------------------------------------------------ helpers
// Plain (non-volatile) read-only loads: the compiler may issue the loads of
// several chunks and rows before the first is used.
__device__ __forceinline__ uint4 ldg_stream(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ----------------------------------------------------------- INT4 GEMV
struct Int4Params {
    const uint32_t* W;      // [rows][cols / 8]
    const float* scales;    // [rows][cols / group_size]
    const float* zeros;     // same, or null
    const uint8_t* limbs;   // x as 16-bit fixed point, [cols / 32][64 B] (xquant_kernel)
    const int4* meta;       // [cols / 32] {scale, sum X[0:16), sum X[16:32), sum X}
    float* y;
    int rows, cols, group_size;
};

// Words per 32-column chunk: 4.  Shared x per chunk: 4 pieces of 16 bytes,
// piece q = {(X0,X2), (X4,X6), (X1,X3), (X5,X7)} of columns 8q .. 8q+7, then
// {s_x, sum X} as a float2 after all pieces.
template <int kRowsPerWarp>
__global__ void __launch_bounds__(kRowsThreads) gemv_int4_kernel(const Int4Params p) {
    extern __shared__ __align__(16) uint8_t rows_smem[];
    const int NC = p.cols / 32;
    const uint32_t sx = smem_u32(rows_smem);
    const uint32_t smeta = sx + 64u * (uint32_t)NC;
    pdl_wait();  // the quantized x comes from the preceding kernel
    for (int c = threadIdx.x; c < NC; c += blockDim.x) {
        const int4* lv = reinterpret_cast<const int4*>(p.limbs + (size_t)c * kXQLimbBytes);
        const int4 m = __ldg(p.meta + c);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int4 v = __ldg(lv + q);  // pairs (X[8q], X[8q+1]) .. (X[8q+6], X[8q+7])
            const uint32_t a0 = __byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x5410);
            const uint32_t a1 = __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x5410);
            const uint32_t b0 = __byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x7632);
            const uint32_t b1 = __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x7632);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(sx + 16u * (uint32_t)(q * NC + c)), "r"(a0),
                         "r"(a1), "r"(b0), "r"(b1)
                         : "memory");
        }
        asm volatile("st.shared.v2.f32 [%0], {%1,%2};" ::"r"(smeta + 8u * (uint32_t)c), "f"(__int_as_float(m.x)),
                     "f"((float)m.w)
                     : "memory");
    }
    __syncthreads();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kRowsThreads / 32);
    const int ng = p.cols / p.group_size;
    const uint4* xs = reinterpret_cast<const uint4*>(rows_smem);
    const float2* xm = reinterpret_cast<const float2*>(rows_smem + 64 * NC);
    for (int row0 = (blockIdx.x * (kRowsThreads / 32) + (threadIdx.x >> 5)) * kRowsPerWarp; row0 < p.rows;
         row0 += warps * kRowsPerWarp) {
        float acc[kRowsPerWarp];
        const uint32_t* wrow[kRowsPerWarp];
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            acc[k] = 0.0f;
            wrow[k] = p.W + (size_t)min(row0 + k, p.rows - 1) * (p.cols / 8);  // clamped: extra rows are not stored
        }
#pragma unroll 4
        for (int c = lane; c < NC; c += 32) {
            uint4 w[kRowsPerWarp];
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) w[k] = ldg_stream(wrow[k] + 4 * c);
            uint4 xv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) xv[q] = xs[q * NC + c];
            const float2 mt = xm[c];
            const int g = (32 * c) / p.group_size;
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) {
                const size_t gi = (size_t)min(row0 + k, p.rows - 1) * ng + g;
                const float scale = __ldg(p.scales + gi), zero = p.zeros ? __ldg(p.zeros + gi) : 0.0f;
                const uint32_t ws[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
                int dot = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t lo = ws[q] & 0x0f0f0f0fu, hi = (ws[q] >> 4) & 0x0f0f0f0fu;
                    dot = dpx_u(lo, xv[q].x, xv[q].y, dot);  // columns 8q, 8q+2, 8q+4, 8q+6
                    dot = dpx_u(hi, xv[q].z, xv[q].w, dot);  // columns 8q+1, 8q+3, 8q+5, 8q+7
                }
                acc[k] = fmaf(scale * mt.x, fmaf(-zero, mt.y, (float)dot), acc[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            const float v = warp_sum(acc[k]);
            if (lane == 0 && row0 + k < p.rows) p.y[row0 + k] = v;
        }
    }
}

// ------------------------------------------------------------ FP8 GEMV
struct Fp8Params {
    const uint8_t* W;  // [rows][cols]
    const float* x;    // [cols]
    float* y;
    int rows, cols;
    float scale;
};

// Zero the bytes of w that hold a NaN code (0x7F or 0xFF).
__device__ __forceinline__ uint32_t fp8_clear_nan(uint32_t w) {
    const uint32_t n = ((w & 0x7f7f7f7fu) + 0x01010101u) & 0x80808080u;
    return w & ~((n << 1) - (n >> 7));
}

__device__ __forceinline__ float2 fp8x2_f32(uint32_t two) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two & 0xffffu), __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Chunk = 16 weights; shared x piece q of chunk c = x[16c + 4q .. 16c + 4q + 3].
template <int kRowsPerWarp>
__global__ void __launch_bounds__(kRowsThreads) gemv_fp8_kernel(const Fp8Params p) {
    extern __shared__ __align__(16) uint8_t rows_smem[];
    const int NC = p.cols / 16;
    const uint32_t sx = smem_u32(rows_smem);
    pdl_wait();
    for (int i = threadIdx.x; i < 4 * NC; i += blockDim.x) {
        const int c = i >> 2, q = i & 3;
        const float4 v = __ldg(reinterpret_cast<const float4*>(p.x) + i);
        asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(sx + 16u * (uint32_t)(q * NC + c)), "f"(v.x),
                     "f"(v.y), "f"(v.z), "f"(v.w)
                     : "memory");
    }
    __syncthreads();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kRowsThreads / 32);
    const float4* xs = reinterpret_cast<const float4*>(rows_smem);
    for (int row0 = (blockIdx.x * (kRowsThreads / 32) + (threadIdx.x >> 5)) * kRowsPerWarp; row0 < p.rows;
         row0 += warps * kRowsPerWarp) {
        float acc0[kRowsPerWarp], acc1[kRowsPerWarp];
        const uint8_t* wrow[kRowsPerWarp];
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            acc0[k] = acc1[k] = 0.0f;
            wrow[k] = p.W + (size_t)min(row0 + k, p.rows - 1) * p.cols;  // clamped: extra rows are not stored
        }
#pragma unroll 4
        for (int c = lane; c < NC; c += 32) {
            uint4 w[kRowsPerWarp];
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) w[k] = ldg_stream(wrow[k] + 16 * c);
            float4 xv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) xv[q] = xs[q * NC + c];
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) {
                // a NaN code in any byte: 0x7F/0xFF make bit 7 of (b & 0x7F) + 1 set
                const uint32_t any =
                    (((w[k].x & 0x7f7f7f7fu) + 0x01010101u) | ((w[k].y & 0x7f7f7f7fu) + 0x01010101u) |
                     ((w[k].z & 0x7f7f7f7fu) + 0x01010101u) | ((w[k].w & 0x7f7f7f7fu) + 0x01010101u)) &
                    0x80808080u;
                if (any) {
                    w[k].x = fp8_clear_nan(w[k].x);
                    w[k].y = fp8_clear_nan(w[k].y);
                    w[k].z = fp8_clear_nan(w[k].z);
                    w[k].w = fp8_clear_nan(w[k].w);
                }
                const uint32_t ws[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 a = fp8x2_f32(ws[q]), b = fp8x2_f32(ws[q] >> 16);
                    acc0[k] = fmaf(a.x, xv[q].x, acc0[k]);
                    acc1[k] = fmaf(a.y, xv[q].y, acc1[k]);
                    acc0[k] = fmaf(b.x, xv[q].z, acc0[k]);
                    acc1[k] = fmaf(b.y, xv[q].w, acc1[k]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            const float v = warp_sum(acc0[k] + acc1[k]);
            if (lane == 0 && row0 + k < p.rows) p.y[row0 + k] = v * p.scale;
        }
    }
}

// --------------------------------------------------------- generic GEMVs
// Any shape: a warp per row, the reference's per-element arithmetic in fp32.
__global__ void __launch_bounds__(256) gemv_int4_generic_kernel(const uint32_t* __restrict__ W,
                                                                const float* __restrict__ scales,
                                                                const float* __restrict__ zeros,
                                                                const float* __restrict__ x, float* __restrict__ y,
                                                                int rows, int cols, int group_size) {
    pdl_wait();
    const int lane = threadIdx.x & 31, warps = gridDim.x * 8;
    const int ng = cols / group_size;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += warps) {
        const uint32_t* wrow = W + (size_t)row * (cols / 8);
        float acc = 0.0f;
        for (int c = lane; c < cols; c += 32) {
            const size_t g = (size_t)row * ng + c / group_size;
            const float zero = zeros ? __ldg(zeros + g) : 0.0f;
            const float w = __fmul_rn(__fsub_rn((float)((__ldg(wrow + c / 8) >> ((c % 8) * 4)) & 0x0fu), zero),
                                      __ldg(scales + g));
            acc = fmaf(w, __ldg(x + c), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[row] = acc;
    }
}

__global__ void __launch_bounds__(256) gemv_fp8_generic_kernel(const uint8_t* __restrict__ W,
                                                               const float* __restrict__ x, float* __restrict__ y,
                                                               int rows, int cols, float scale) {
    pdl_wait();
    const int lane = threadIdx.x & 31, warps = gridDim.x * 8;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += warps) {
        const uint8_t* wrow = W + (size_t)row * cols;
        float acc = 0.0f;
        for (int c = lane; c < cols; c += 32) acc = fmaf(__fmul_rn(fp8_e4m3_ref(__ldg(wrow + c)), scale), __ldg(x + c), acc);
        acc = warp_sum(acc);
        if (lane == 0) y[row] = acc;
    }
}

}  // namespace nexus_gpu
