// ref_driver.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A thin extern "C" shim around NexusLLM's own, unmodified
// nexus::QuantizationKernel (include/quantization.hpp:56-154, implemented in
// src/quantization.cpp).  oracle/Makefile compiles this file together with the
// reference's src/quantization.cpp, straight from the reference checkout and
// with the reference's own build.sh flags (-O3 -std=c++20 -mavx2 -mfma
// -fopenmp), into oracle/_ref/libnexus_ref.so.  Nothing here re-implements the
// reference: every compute call lands in the reference's code.  The library is
// used (a) to generate and check the golden vectors under tests/golden/ and
// (b) as the timed CPU baseline ("kind": "reference") in bench.py.
//
// All C++ symbols are hidden (-fvisibility=hidden); only the ref_* functions
// below are exported, so this library never interposes on the product's
// symbols when both are loaded into one process.
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

#include "quantization.hpp"
#include "transformer_ops.hpp"

#if defined(_OPENMP)
#include <omp.h>
#endif

#define REF_API extern "C" __attribute__((visibility("default")))

using nexus::BlockQ4_0;
using nexus::BlockQ5_K;
using nexus::BlockQ6_K;
using nexus::BlockQ8_0;
using nexus::QuantizationKernel;

REF_API float ref_fp16_to_fp32(uint16_t h) { return QuantizationKernel::fp16_to_fp32(h); }

REF_API int ref_have_avx2(void) {
#if defined(NEXUS_HAVE_AVX2)
    return 1;
#else
    return 0;
#endif
}

REF_API int ref_max_threads(void) {
#if defined(_OPENMP)
    return omp_get_max_threads();
#else
    return 1;
#endif
}

REF_API void ref_set_omp_threads(int n) {
#if defined(_OPENMP)
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

REF_API void ref_dequantize_q4_0(const void* b, float* out, size_t nb) {
    QuantizationKernel::dequantize_gguf_q4_0(static_cast<const BlockQ4_0*>(b), out, nb);
}
REF_API void ref_dequantize_q5_k(const void* b, float* out, size_t nb) {
    QuantizationKernel::dequantize_gguf_q5_k(static_cast<const BlockQ5_K*>(b), out, nb);
}
REF_API void ref_dequantize_q6_k(const void* b, float* out, size_t nb) {
    QuantizationKernel::dequantize_gguf_q6_k(static_cast<const BlockQ6_K*>(b), out, nb);
}

REF_API void ref_fused_gemv_q4_0(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    QuantizationKernel::fused_gemv_q4_0(static_cast<const BlockQ4_0*>(W), x, y, rows, cols);
}
REF_API void ref_fused_gemv_q8_0(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    QuantizationKernel::fused_gemv_q8_0(static_cast<const BlockQ8_0*>(W), x, y, rows, cols);
}
REF_API void ref_fused_gemv_fp16(const uint16_t* W, const float* x, float* y, size_t rows, size_t cols) {
    QuantizationKernel::fused_gemv_fp16(W, x, y, rows, cols);
}
REF_API void ref_fused_gemv_q5_k(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    QuantizationKernel::fused_gemv_q5_k(static_cast<const BlockQ5_K*>(W), x, y, rows, cols);
}
REF_API void ref_fused_gemv_q6_k(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    QuantizationKernel::fused_gemv_q6_k(static_cast<const BlockQ6_K*>(W), x, y, rows, cols);
}

REF_API void ref_fused_gemv_int4(const uint32_t* W, const float* x, const float* scales, const float* zeros,
                                 float* y, size_t rows, size_t cols, size_t group_size) {
    QuantizationKernel::fused_gemv_int4(W, x, scales, zeros, y, rows, cols, group_size);
}
REF_API void ref_fused_gemv_fp8(const uint8_t* W, const float* x, float* y, size_t rows, size_t cols, float scale) {
    QuantizationKernel::fused_gemv_fp8(W, x, y, rows, cols, scale);
}
REF_API void ref_dequantize_int4_awq(const uint32_t* packed, const float* scales, const float* zeros, float* out,
                                     size_t count, size_t group_size) {
    QuantizationKernel::dequantize_int4_awq(packed, scales, zeros, out, count, group_size);
}
REF_API void ref_dequantize_fp8_e4m3(const uint8_t* in, float* out, size_t count, float scale) {
    QuantizationKernel::dequantize_fp8_e4m3(in, out, count, scale);
}

// TransformerOps (include/transformer_ops.hpp:23-44,86-95): the decode
// layer's RMSNorm and SwiGLU, header-only in the reference.
REF_API void ref_rmsnorm(const float* x, const float* w, float* out, size_t dim, float eps) {
    nexus::TransformerOps::rmsnorm(x, w, out, dim, eps);
}
REF_API void ref_swiglu(const float* g, const float* u, float* out, size_t dim) {
    nexus::TransformerOps::swiglu(g, u, out, dim);
}

// Bytes of one weight row for a NexusLLM DataType value (nexus_common.hpp:244-260).
static size_t row_bytes(unsigned dtype, size_t cols) {
    switch (dtype) {
        case 1: return cols * 2;
        case 7: return cols / 32 * sizeof(BlockQ4_0);
        case 9: return cols / 32 * sizeof(BlockQ8_0);
        case 11: return cols / nexus::QK_K * sizeof(BlockQ5_K);
        case 12: return cols / nexus::QK_K * sizeof(BlockQ6_K);
        default: return 0;
    }
}

static void call_rows(unsigned dtype, const uint8_t* W, const float* x, float* y, size_t rows, size_t cols) {
    switch (dtype) {
        case 1: ref_fused_gemv_fp16(reinterpret_cast<const uint16_t*>(W), x, y, rows, cols); break;
        case 7: ref_fused_gemv_q4_0(W, x, y, rows, cols); break;
        case 9: ref_fused_gemv_q8_0(W, x, y, rows, cols); break;
        case 11: ref_fused_gemv_q5_k(W, x, y, rows, cols); break;
        case 12: ref_fused_gemv_q6_k(W, x, y, rows, cols); break;
        default: break;
    }
}

// The reference's GEMV for one DataType, using up to `threads` host threads.
// Q5_K/Q6_K parallelise rows with their own OpenMP pragma
// (src/quantization.cpp:519,630), so they are called once with `threads`
// OpenMP threads.  Q4_0/Q8_0/FP16 have no pragma (single-threaded by design,
// src/quantization.cpp:264-410); to give the CPU baseline every core, the rows
// are split into `threads` contiguous slices and the unmodified reference
// function is called on each slice from its own std::thread.  Rows are
// independent, so the result is identical to a single call.
// Returns 0, or -3 for an unsupported dtype.
REF_API int ref_fused_gemv_threaded(unsigned dtype, const void* W, const float* x, float* y, size_t rows,
                                    size_t cols, int threads) {
    const size_t rb = row_bytes(dtype, cols);
    if (rb == 0) return -3;
    if (threads < 1) threads = 1;
    const uint8_t* Wb = static_cast<const uint8_t*>(W);
    if (dtype == 11 || dtype == 12 || threads == 1 || rows < 2) {
        ref_set_omp_threads(threads);
        call_rows(dtype, Wb, x, y, rows, cols);
        return 0;
    }
    const size_t nt = std::min<size_t>(static_cast<size_t>(threads), rows);
    std::vector<std::thread> pool;
    pool.reserve(nt);
    for (size_t t = 0; t < nt; ++t) {
        const size_t r0 = rows * t / nt, r1 = rows * (t + 1) / nt;
        pool.emplace_back([=] { call_rows(dtype, Wb + r0 * rb, x, y + r0, r1 - r0, cols); });
    }
    for (auto& th : pool) th.join();
    return 0;
}
