// dropin.cpp -- the C++ drop-in: NexusLLM's own GEMV entry points, defined on
// top of libnexus_gpu.
//
// This translation unit is compiled against NexusLLM's unmodified headers
// (include/quantization.hpp, include/nexus_backend.hpp; -I<NexusLLM>/include)
// and linked to libnexus_gpu.so.  It is what a NexusLLM maintainer adds to the
// engine's build in place of the GGUF bodies in src/quantization.cpp:264-722
// and of the forwarding CUDABackend in src/nexus_backend.cpp:239-367:
//
//  * nexus::QuantizationKernel::fused_gemv_{q4_0,q8_0,q5_k,q6_k,fp16} and
//    dequantize_gguf_{q4_0,q5_k,q6_k} with the exact signatures of
//    include/quantization.hpp:80-153 (same mangled symbols), forwarding to the
//    host-pointer C ABI (nexus_fused_gemv_*, nexus_dequantize_gguf_*):
//    synchronous, void, host pointers, weights cached on the device;
//  * nexus::CudaGemvBackend, an INexusComputeBackend
//    (include/nexus_backend.hpp:37-91) whose gemv_dispatch, memory and copy
//    calls run on the GPU through the library, and whose other kernels
//    (attention, RMSNorm, SwiGLU) go to a fallback backend -- the pattern of
//    the reference's CUDABackend, which holds a CPUBackend fallback for every
//    call (src/nexus_backend.cpp:280-282).  A DataType the library does not
//    serve (FP32 ...) also takes the fallback.
//
// Two extern "C" hooks let a test reach the C++ path without a C++ caller:
// nexus_dropin_backend_gemv (a GEMV through the backend's virtual
// gemv_dispatch) and nexus_dropin_backend_name.
#include <cstdint>
#include <cstdio>
#include <memory>
#include <string>

#include "nexus_backend.hpp"
#include "quantization.hpp"

#include "../../include/nexus_gpu.h"

#define DROPIN_API extern "C" __attribute__((visibility("default")))

namespace nexus {

// ------------------------------------------ QuantizationKernel (GGUF formats)
void QuantizationKernel::fused_gemv_q4_0(const BlockQ4_0* W_q4, const float* x, float* y, size_t rows, size_t cols) {
    nexus_fused_gemv_q4_0(W_q4, x, y, rows, cols);
}
void QuantizationKernel::fused_gemv_q8_0(const BlockQ8_0* W_q8, const float* x, float* y, size_t rows, size_t cols) {
    nexus_fused_gemv_q8_0(W_q8, x, y, rows, cols);
}
void QuantizationKernel::fused_gemv_fp16(const uint16_t* W_fp16, const float* x, float* y, size_t rows,
                                         size_t cols) {
    nexus_fused_gemv_fp16(W_fp16, x, y, rows, cols);
}
void QuantizationKernel::fused_gemv_q5_k(const BlockQ5_K* W_q5_k, const float* x, float* y, size_t rows,
                                         size_t cols) {
    nexus_fused_gemv_q5_k(W_q5_k, x, y, rows, cols);
}
void QuantizationKernel::fused_gemv_q6_k(const BlockQ6_K* W_q6_k, const float* x, float* y, size_t rows,
                                         size_t cols) {
    nexus_fused_gemv_q6_k(W_q6_k, x, y, rows, cols);
}
void QuantizationKernel::dequantize_gguf_q4_0(const BlockQ4_0* blocks, float* output, size_t num_blocks) {
    nexus_dequantize_gguf_q4_0(blocks, output, num_blocks);
}
void QuantizationKernel::dequantize_gguf_q5_k(const BlockQ5_K* blocks, float* output, size_t num_blocks) {
    nexus_dequantize_gguf_q5_k(blocks, output, num_blocks);
}
void QuantizationKernel::dequantize_gguf_q6_k(const BlockQ6_K* blocks, float* output, size_t num_blocks) {
    nexus_dequantize_gguf_q6_k(blocks, output, num_blocks);
}

// ------------------------------------------------- the CUDA compute device
class CudaGemvBackend final : public INexusComputeBackend {
public:
    explicit CudaGemvBackend(std::shared_ptr<INexusComputeBackend> fallback) : fallback_(std::move(fallback)) {
        caps_.type = ComputeDeviceType::DEVICE_CUDA;
        caps_.vendor = "NVIDIA Corporation";
        caps_.architecture = "Blackwell (sm_100a)";
        caps_.is_unified_memory = false;
        caps_.supports_fp16 = true;
        caps_.supports_int4 = true;
        caps_.supports_async_dma = true;
        caps_.api_version = "libnexus_gpu C ABI";
        char name[256] = {0};
        int sms = 0, major = 0, minor = 0;
        if (nexus_gpu_device_info(name, sizeof(name), &sms, &major, &minor) == NEXUS_GPU_SUCCESS) {
            caps_.device_name = name;
            caps_.description = std::to_string(sms) + " SMs, compute capability " + std::to_string(major) + "." +
                                std::to_string(minor);
        } else {
            caps_.device_name = "no CUDA device";
        }
        caps_.driver_version = nexus_gpu_version();
    }

    ComputeDeviceType get_type() const override { return ComputeDeviceType::DEVICE_CUDA; }
    const DeviceCapabilities& get_capabilities() const override { return caps_; }
    bool initialize() override { return true; }
    void shutdown() override {}
    void synchronize() override { nexus_gpu_synchronize(nullptr); }

    void* allocate_device_memory(size_t bytes) override { return nexus_gpu_allocate_device_memory(bytes); }
    void free_device_memory(void* ptr) override { nexus_gpu_free_device_memory(ptr); }
    bool copy_host_to_device_async(void* dst, const void* src, size_t bytes) override {
        return nexus_gpu_copy_host_to_device_async(dst, src, bytes, nullptr) == NEXUS_GPU_SUCCESS;
    }
    bool copy_device_to_host_async(void* dst, const void* src, size_t bytes) override {
        return nexus_gpu_copy_device_to_host_async(dst, src, bytes, nullptr) == NEXUS_GPU_SUCCESS;
    }

    // matmul_vec_dispatch's contract (include/transformer_ops.hpp:157-173):
    // W == nullptr is a no-op; host pointers; y written before return.
    void gemv_dispatch(const void* W, DataType dt, const float* x, float* y, size_t rows, size_t cols) override {
        const int32_t rc = nexus_gpu_gemv_dispatch(W, static_cast<uint32_t>(dt), x, y, rows, cols);
        if (rc == NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED && fallback_) {
            fallback_->gemv_dispatch(W, dt, x, y, rows, cols);
        } else if (rc != NEXUS_GPU_SUCCESS) {
            std::fprintf(stderr, "CudaGemvBackend::gemv_dispatch: status %d: %s\n", rc, nexus_gpu_last_error());
        }
        last_status_ = rc;
    }

    void paged_attention_decode(const float* q, const std::vector<int32_t>& block_table, PagedKVCacheManager& kv_mgr,
                                size_t layer_idx, size_t position, size_t num_heads, size_t num_kv_heads,
                                size_t head_dim, float* out) override {
        if (fallback_)
            fallback_->paged_attention_decode(q, block_table, kv_mgr, layer_idx, position, num_heads, num_kv_heads,
                                              head_dim, out);
    }
    void rmsnorm(const float* x, const void* weight, DataType dt, float* out, size_t dim, float eps) override {
        if (fallback_) fallback_->rmsnorm(x, weight, dt, out, dim, eps);
    }
    void swiglu(const float* gate, const float* up, float* out, size_t dim) override {
        if (fallback_) fallback_->swiglu(gate, up, out, dim);
    }

    int32_t last_status() const { return last_status_; }

private:
    DeviceCapabilities caps_;
    std::shared_ptr<INexusComputeBackend> fallback_;
    int32_t last_status_ = NEXUS_GPU_SUCCESS;
};

}  // namespace nexus

// A GEMV through the backend interface's virtual gemv_dispatch (host pointers),
// as TransformerEngine::forward_token calls it (src/transformer_engine.cpp:367-375).
// Returns the library status of the call.
DROPIN_API int32_t nexus_dropin_backend_gemv(const void* W, uint32_t dtype, const float* x, float* y, size_t rows,
                                             size_t cols) {
    static nexus::CudaGemvBackend device(nullptr);
    nexus::INexusComputeBackend& be = device;
    be.gemv_dispatch(W, static_cast<nexus::DataType>(dtype), x, y, rows, cols);
    return device.last_status();
}

// The backend's reported device name and type (capabilities as the reference
// reports them, include/nexus_backend.hpp:20-34).
DROPIN_API int32_t nexus_dropin_backend_name(char* out, size_t len, uint32_t* type) {
    static nexus::CudaGemvBackend device(nullptr);
    const nexus::DeviceCapabilities& c = device.get_capabilities();
    if (type) *type = static_cast<uint32_t>(c.type);
    if (out && len) std::snprintf(out, len, "%s", c.device_name.c_str());
    return 0;
}
