// nexus_gpu.cu -- host side of libnexus_gpu.so: the C ABI declared in
// include/nexus_gpu.h, per-device contexts (stream, workspace, weight cache)
// and kernel launchers.  Device code lives in gemv_kernels.cuh.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/nexus_gpu.h"
#include "gemv_kernels.cuh"
#include "stack_kernels.cuh"
#include "stack_mt_kernels.cuh"
#include "awq_fp8_kernels.cuh"
#include "mma_kernels.cuh"
#include "mma_stack_kernels.cuh"
#include "gguf_file.cuh"

namespace nexus_gpu {

// Fixed scratch of the no-allocation GEMV entry point (see nexus_gpu_gemv_noalloc).
static __device__ __align__(256) uint8_t g_noalloc_scratch[size_t(1) << 20];

namespace {

thread_local std::string t_last_error;

int32_t fail(int32_t code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

#define CUDA_TRY(expr)                                                                               \
    do {                                                                                             \
        cudaError_t e_ = (expr);                                                                     \
        if (e_ != cudaSuccess)                                                                       \
            return fail(e_ == cudaErrorMemoryAllocation ? NEXUS_GPU_ERROR_OUT_OF_TIER0_MEMORY       \
                                                        : NEXUS_GPU_ERROR_CUDA,                     \
                        "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

// ---------------------------------------------------------------- formats
struct FormatInfo {
    int elems;      // elements per block
    int bytes;      // bytes per block
};

bool format_info(uint32_t dtype, FormatInfo& f) {
    switch (dtype) {
        case NEXUS_GPU_FP16: f = {1, 2}; return true;
        case NEXUS_GPU_GGUF_Q4_0: f = {32, 18}; return true;
        case NEXUS_GPU_GGUF_Q8_0: f = {32, 34}; return true;
        case NEXUS_GPU_GGUF_Q5_K: f = {256, 176}; return true;
        case NEXUS_GPU_GGUF_Q6_K: f = {256, 210}; return true;
        default: return false;
    }
}

int32_t check_shape(uint32_t dtype, size_t rows, size_t cols, FormatInfo& f) {
    if (!format_info(dtype, f)) return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "unsupported weight dtype %u", dtype);
    if (cols % (size_t)f.elems != 0)
        return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "cols=%zu is not a multiple of the block size %d", cols, f.elems);
    if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "rows/cols exceed 2^31-1");
    return NEXUS_GPU_SUCCESS;
}

size_t row_bytes_of(const FormatInfo& f, size_t cols) { return cols / (size_t)f.elems * (size_t)f.bytes; }

bool is_int_format(uint32_t dtype) { return dtype != NEXUS_GPU_FP16; }

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// workspace: xq limbs [M][K/32][64] then meta [M][K/32][16 B]
size_t xq_bytes(uint32_t dtype, size_t M, size_t cols) {
    if (!is_int_format(dtype)) return 0;
    const size_t nxb = cols / 32;
    return align256(M * nxb * kXQLimbBytes) + align256(M * nxb * kXQMetaBytes);
}

// ---------------------------------------------------- batched (tensor cores)
// Batched decode runs on the tcgen05 tensor cores for GGUF Q4_0 with
// M >= kTcMinTokens activation rows and K a multiple of 256 (rows of whole
// 144-byte chunks for the 2-D tensor copies), in groups of <= 64 tokens.
constexpr size_t kTcMinTokens = 16;

bool tc_eligible(uint32_t dtype, size_t M, size_t cols) {
    return dtype == NEXUS_GPU_GGUF_Q4_0 && M >= kTcMinTokens && cols % kRawK == 0 && cols <= (size_t)INT32_MAX;
}

struct TcPlan {
    int tiles, n_chunks, G;
    long long total;
};
// CTAs of a tensor-core GEMM.  A tile-aligned split -- s CTAs a tile, s
// dividing the tile's chunks, at least 2 chunks each -- when it keeps at least
// 85 % of the SMs busy: every CTA then works on one tile, and a shared tile
// has one fix-up.  Otherwise stream-K over every SM (at least 2 chunks a CTA),
// where the CTAs whose range crosses a tile boundary carry two epilogues and
// often a fix-up.
int tc_ctas(int sms, int tiles, int n_chunks) {
    const long long total = (long long)tiles * n_chunks;
    for (int s = n_chunks / 2; s >= 1; --s)
        if (n_chunks % s == 0 && (long long)tiles * s <= sms) {
            if ((long long)tiles * s * 100 >= 85LL * sms) return tiles * s;
            break;
        }
    return (int)std::max<long long>(1, std::min<long long>(sms, total / 2));
}
// At most one persistent CTA per SM over the tiles x chunks sequence.
TcPlan tc_plan(int sms, size_t rows, size_t cols) {
    TcPlan p;
    p.n_chunks = (int)(cols / kRawK);
    p.tiles = (int)((rows + kMmaRows - 1) / kMmaRows);
    p.total = (long long)p.tiles * p.n_chunks;
    p.G = tc_ctas(sms, p.tiles, p.n_chunks);
    return p;
}
// Workspace of one token group (<= kMaxTokens): the B operand (fp16 rows),
// the per-token scales, the per-tile arrival counters and the partial sums of
// shared tiles (two slots a CTA).
struct TcLayout {
    size_t xscale, arrivals, partial, total;
};
TcLayout tc_layout(int sms, size_t rows, size_t cols) {
    const TcPlan pl = tc_plan(sms, rows, cols);
    TcLayout l;
    l.xscale = align256((size_t)kMaxTokens * cols * sizeof(__half));
    l.arrivals = l.xscale + align256(kMaxTokens * sizeof(float));
    l.partial = l.arrivals + align256((size_t)pl.tiles * sizeof(unsigned));
    l.total = l.partial + align256((size_t)2 * pl.G * kMaxTokens * kMmaRows * sizeof(float));
    return l;
}
size_t tc_group_bytes(int sms, size_t rows, size_t cols) { return tc_layout(sms, rows, cols).total; }

// --------------------------------------------------------------- contexts
struct CachedWeight {
    void* dptr = nullptr;
    size_t bytes = 0;
    uint64_t fingerprint = 0;
};

struct Workspace {
    void* ptr = nullptr;
    size_t bytes = 0;
};

struct Device {
    int id = -1;
    int sms = 0;
    int smem_optin = 0;
    cudaStream_t stream = nullptr;  // stream of the synchronous host-pointer API
    std::mutex mu;
    std::unordered_map<std::string, CachedWeight> cache;
    size_t cache_bytes = 0;
    std::unordered_map<cudaStream_t, Workspace> ws;
    void* dx = nullptr;
    size_t dx_cap = 0;
    void* dy = nullptr;
    size_t dy_cap = 0;
    bool smem_attr_set = false;
};

std::mutex g_devices_mu;
std::vector<std::unique_ptr<Device>> g_devices;

int32_t get_device(Device** out) {
    int id = 0;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(NEXUS_GPU_ERROR_NO_DEVICE, "no CUDA device");
    }
    CUDA_TRY(cudaGetDevice(&id));
    std::lock_guard<std::mutex> lk(g_devices_mu);
    if ((int)g_devices.size() < n) g_devices.resize(n);
    if (!g_devices[id]) {
        auto d = std::make_unique<Device>();
        d->id = id;
        CUDA_TRY(cudaDeviceGetAttribute(&d->sms, cudaDevAttrMultiProcessorCount, id));
        CUDA_TRY(cudaDeviceGetAttribute(&d->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, id));
        CUDA_TRY(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
        g_devices[id] = std::move(d);
    }
    *out = g_devices[id].get();
    return NEXUS_GPU_SUCCESS;
}

template <class F>
int32_t set_smem_attr(int bytes) {
    CUDA_TRY(cudaFuncSetAttribute(gemv_m1_kernel<F, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    if (F::kGroup > 1)
        CUDA_TRY(cudaFuncSetAttribute(gemv_m1_kernel<F, F::kGroup>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      bytes));
    return NEXUS_GPU_SUCCESS;
}

int32_t ensure_attrs(Device& d) {
    if (d.smem_attr_set) return NEXUS_GPU_SUCCESS;
    int32_t rc;
    if ((rc = set_smem_attr<FmtQ4_0>(d.smem_optin))) return rc;
    if ((rc = set_smem_attr<FmtQ8_0>(d.smem_optin))) return rc;
    if ((rc = set_smem_attr<FmtQ5_K>(d.smem_optin))) return rc;
    if ((rc = set_smem_attr<FmtQ6_K>(d.smem_optin))) return rc;
    if ((rc = set_smem_attr<FmtF16>(d.smem_optin))) return rc;
    d.smem_attr_set = true;
    return NEXUS_GPU_SUCCESS;
}

// ---------------------------------------------------------------- launches
template <class Kern, class... Args>
int32_t launch(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, args...));
    return NEXUS_GPU_SUCCESS;
}

// Fast-path geometry for a weight format and shape (see gemv_kernels.cuh).
// Returns false when the shape is outside the fast kernel's limits.
// max_j: the most work items a lane may hold (kMaxJ; 4 / tokens for the
// multi-token stack, whose lanes hold every token's slices); grouped: whether
// a lane may take a format's kGroup consecutive items together.
template <class F>
bool plan_fast(const Device& d, int N, int K, uint64_t row_bytes, GemvParams& p, size_t& smem,
               uint64_t stage_target = kStageTargetBytes, int max_j = kMaxJ, bool grouped = true) {
    const int NW = K / F::kWIElems;
    if (NW < 32) return false;
    // K segments S (1..15): S warps share a row, n_grp = 15/S row groups work
    // in parallel (15 - S*n_grp warps idle).  A lane holds J x slices, J =
    // its share of the SW = NW/S work items of a segment, so a row costs
    // about J/n_grp lane-rounds: pick the S that minimises it (ties: fewer
    // segments, less partial-sum traffic), with J <= kMaxJ and a stage that
    // holds one row per group within kStageMaxBytes.  Segment boundaries fall
    // on whole lane groups.
    const int Gp = (grouped && NW % F::kGroup == 0) ? F::kGroup : 1;
    int S = 0, SW = 0, J = 0;
    double best = 1e30;
    for (int cand = 1; cand <= kMaxSegments; ++cand) {
        const int sw = ((NW + cand - 1) / cand + Gp - 1) / Gp * Gp;
        const int j = (sw + 32 * Gp - 1) / (32 * Gp) * Gp;
        const int groups = kConsumerWarps / cand;
        if (j > max_j || groups == 0) continue;
        if ((uint64_t)groups * row_bytes > (uint64_t)kStageMaxBytes && cand < kMaxSegments) continue;
        const double cost = (double)j / groups;
        if (cost < best - 1e-9) {
            best = cost;
            S = cand;
            SW = sw;
            J = j;
        }
    }
    if (S == 0) return false;
    p.group = Gp;
    const int n_grp = kConsumerWarps / S;
    const uint64_t grp_bytes = (uint64_t)n_grp * row_bytes;
    const int m = (int)std::max<uint64_t>(1, std::min<uint64_t>(4, stage_target / grp_bytes));
    const int R = std::min(n_grp * m, kMaxStageRows);
    const uint64_t sb = (R * row_bytes + 32 + 15) / 16 * 16;
    const uint64_t avail = (uint64_t)d.smem_optin - kSmemHeader - 128;
    int ns = (int)std::min<uint64_t>(kMaxStages, avail / sb);
    while (ns > 2 && ns * R * S > kMaxSlots) --ns;
    if (ns < 2 || ns * R * S > kMaxSlots) return false;
    p.nwi = NW;
    p.segments = S;
    p.seg_wi = SW;
    p.wi_per_lane = J;
    p.stage_rows = R;
    p.stage_bytes = (int)sb;
    p.n_stages = ns;
    smem = kSmemHeader + (size_t)ns * sb;
    (void)N;
    return true;
}

template <class F>
int32_t launch_fast(Device& d, const GemvParams& p, size_t smem, cudaStream_t st) {
    const int grid = std::min(d.sms, p.N);
    if (F::kGroup > 1 && p.group == F::kGroup)
        return launch(gemv_m1_kernel<F, F::kGroup>, dim3(grid), dim3(kGemvThreads), smem, st, p);
    return launch(gemv_m1_kernel<F, 1>, dim3(grid), dim3(kGemvThreads), smem, st, p);
}

bool plan_for(uint32_t dtype, const Device& d, int N, int K, uint64_t rb, GemvParams& p, size_t& smem,
              uint64_t stage_target = kStageTargetBytes, int max_j = kMaxJ, bool grouped = true) {
    switch (dtype) {
        case NEXUS_GPU_GGUF_Q4_0: return plan_fast<FmtQ4_0>(d, N, K, rb, p, smem, stage_target, max_j, grouped);
        case NEXUS_GPU_GGUF_Q8_0: return plan_fast<FmtQ8_0>(d, N, K, rb, p, smem, stage_target, max_j, grouped);
        case NEXUS_GPU_GGUF_Q5_K: return plan_fast<FmtQ5_K>(d, N, K, rb, p, smem, stage_target, max_j, grouped);
        case NEXUS_GPU_GGUF_Q6_K: return plan_fast<FmtQ6_K>(d, N, K, rb, p, smem, stage_target, max_j, grouped);
        default: return (K % 16 == 0) && plan_fast<FmtF16>(d, N, K, rb, p, smem, stage_target);
    }
}

int32_t run_gemm_tc(Device& d, const void* dW, const void* dX, int xbf, float* dY, size_t M, size_t rows, size_t cols,
                    uint8_t* ws, cudaStream_t st);

// Workspace bytes of one GEMV call (gemv_ws_bytes with the tensor path allowed).
// Activation rows one GEMV call accepts: the x quantizer's grid has one row
// of CTAs per token (gridDim.y <= 65535).
constexpr size_t kMaxActivationRows = 65535;

size_t gemv_ws_bytes(int sms, uint32_t dtype, size_t M, size_t rows, size_t cols, bool allow_tc) {
    if (M > kMaxActivationRows) return 0;  // refused by every entry point before any size matters
    if (allow_tc && tc_eligible(dtype, M, cols)) return tc_group_bytes(sms, rows, cols);
    return xq_bytes(dtype, M, cols);
}

// One GEMV of M rows of x.  `ws` holds at least gemv_ws_bytes(d.sms, ...,
// allow_tc).  Batched Q4_0 (M >= 16) goes to the tensor cores when allowed.
int32_t run_gemv(Device& d, const void* dW, uint32_t dtype, const void* dX, uint32_t x_dtype, float* dY, size_t M,
                 size_t rows, size_t cols, uint8_t* ws, cudaStream_t st, bool allow_tc = true) {
    FormatInfo f;
    int32_t rc = check_shape(dtype, rows, cols, f);
    if (rc) return rc;
    if (x_dtype != NEXUS_GPU_FP32 && x_dtype != NEXUS_GPU_BF16)
        return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "unsupported activation dtype %u", x_dtype);
    if (M > kMaxActivationRows)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "M=%zu activation rows, at most %zu", M, kMaxActivationRows);
    if (M == 0 || rows == 0) return NEXUS_GPU_SUCCESS;
    if (cols == 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "cols == 0");
    if (!dW || !dX || !dY) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null device pointer");
    if ((rc = ensure_attrs(d))) return rc;
    const int K = (int)cols, N = (int)rows;
    const size_t rb = row_bytes_of(f, cols);
    const bool w16 = ((uintptr_t)dW & 15) == 0;
    const int xbf = x_dtype == NEXUS_GPU_BF16;
    if (allow_tc && w16 && tc_eligible(dtype, M, cols)) return run_gemm_tc(d, dW, dX, xbf, dY, M, rows, cols, ws, st);
    const size_t xes = xbf ? 2 : 4;
    const size_t nxb = cols / 32;
    uint8_t* limbs = ws;
    int4* meta = is_int_format(dtype) ? reinterpret_cast<int4*>(ws + align256(M * nxb * kXQLimbBytes)) : nullptr;

    GemvParams plan{};
    size_t smem = 0;
    const bool fast = w16 && plan_for(dtype, d, N, K, rb, plan, smem);
    if (fast && is_int_format(dtype)) {
        dim3 g((unsigned)((nxb + 7) / 8), (unsigned)M);
        if ((rc = launch(xquant_kernel, g, dim3(256), 0, st, dX, xbf, K, K, limbs, meta))) return rc;
    }
    for (size_t m = 0; m < M; ++m) {
        const uint8_t* xm = static_cast<const uint8_t*>(dX) + m * cols * xes;
        float* ym = dY + m * rows;
        if (!fast) {
            const int blocks = (N + 7) / 8;
            if ((rc = launch(gemv_generic_kernel, dim3(blocks), dim3(256), 0, st, (int)dtype,
                             static_cast<const uint8_t*>(dW), (uint64_t)rb, N, K, (const void*)xm, xbf, ym)))
                return rc;
            continue;
        }
        GemvParams p = plan;
        p.W = static_cast<const uint8_t*>(dW);
        p.total_bytes = (uint64_t)rb * rows;
        p.row_bytes = rb;
        p.N = N;
        p.K = K;
        p.y = ym;
        p.x = xm;
        p.x_bf16 = xbf;
        p.xq_limbs = limbs + m * nxb * kXQLimbBytes;
        p.xq_meta = meta ? meta + m * nxb : nullptr;
        switch (dtype) {
            case NEXUS_GPU_GGUF_Q4_0: rc = launch_fast<FmtQ4_0>(d, p, smem, st); break;
            case NEXUS_GPU_GGUF_Q8_0: rc = launch_fast<FmtQ8_0>(d, p, smem, st); break;
            case NEXUS_GPU_GGUF_Q5_K: rc = launch_fast<FmtQ5_K>(d, p, smem, st); break;
            case NEXUS_GPU_GGUF_Q6_K: rc = launch_fast<FmtQ6_K>(d, p, smem, st); break;
            default: rc = launch_fast<FmtF16>(d, p, smem, st); break;
        }
        if (rc) return rc;
    }
    return NEXUS_GPU_SUCCESS;
}

// ------------------------------------------------------------ tensor path
using TensorMapEncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                          const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                          CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                          CUtensorMapFloatOOBfill);

TensorMapEncodeTiled tensor_map_encoder() {
    static std::once_flag once;
    static TensorMapEncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<TensorMapEncodeTiled>(p);
        cudaGetLastError();
    });
    return fn;
}

int32_t mma_attrs(Device& d) {
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lk(mu);
    if (std::find(done.begin(), done.end(), d.id) != done.end()) return NEXUS_GPU_SUCCESS;
    if (d.smem_optin < kMmaSmemBytes)
        return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "batched path needs %d bytes of shared memory", kMmaSmemBytes);
    CUDA_TRY(cudaFuncSetAttribute(gemm_q4_0_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaSmemBytes));
    // both kernels of a batched GEMV on the same shared-memory carveout: no
    // reconfiguration of the SMs between the x preparation and the GEMM
    CUDA_TRY(cudaFuncSetAttribute(gemm_q4_0_mma_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    CUDA_TRY(cudaFuncSetAttribute(mma_xprep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    done.push_back(d.id);
    return NEXUS_GPU_SUCCESS;
}

// Batched Q4_0: token groups of <= 64, each one launch of x preparation and
// one of the persistent tensor-core GEMM.
int32_t run_gemm_tc(Device& d, const void* dW, const void* dX, int xbf, float* dY, size_t M, size_t rows, size_t cols,
                    uint8_t* ws, cudaStream_t st) {
    int32_t rc = mma_attrs(d);
    if (rc) return rc;
    TensorMapEncodeTiled encode = tensor_map_encoder();
    if (!encode) return fail(NEXUS_GPU_ERROR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const TcPlan pl = tc_plan(d.sms, rows, cols);
    const TcLayout lay = tc_layout(d.sms, rows, cols);
    const size_t rb = cols / 32 * 18;
    const size_t xes = xbf ? 2 : 4;
    __half* xp = reinterpret_cast<__half*>(ws);
    float* xscale = reinterpret_cast<float*>(ws + lay.xscale);
    unsigned* arrivals = reinterpret_cast<unsigned*>(ws + lay.arrivals);
    float* partial = reinterpret_cast<float*>(ws + lay.partial);
    for (size_t g0 = 0; g0 < M; g0 += kMaxTokens) {
        const int Mg = (int)std::min<size_t>(kMaxTokens, M - g0);
        const int NB = (Mg + 15) / 16 * 16;
        CUtensorMap tmW, tmX;
        {
            const cuuint64_t dims[2] = {(cuuint64_t)rb, (cuuint64_t)rows};
            const cuuint64_t strides[1] = {(cuuint64_t)rb};
            const cuuint32_t box[2] = {(cuuint32_t)kRawRowBytes, (cuuint32_t)kMmaRows};
            const cuuint32_t estr[2] = {1, 1};
            if (encode(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(dW), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return fail(NEXUS_GPU_ERROR_CUDA, "weight tensor map rejected (%zu x %zu bytes)", rows, rb);
        }
        {
            const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)NB};
            const cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(__half)};
            const cuuint32_t box[2] = {(cuuint32_t)kUnitK, (cuuint32_t)NB};
            const cuuint32_t estr[2] = {1, 1};
            if (encode(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xp, dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return fail(NEXUS_GPU_ERROR_CUDA, "activation tensor map rejected (%d x %zu)", NB, cols);
        }
        const uint8_t* xg = static_cast<const uint8_t*>(dX) + g0 * cols * xes;
        const int vec = ((uintptr_t)xg % (xbf ? 8 : 16)) == 0;  // rows start every cols * xes bytes: 1 KB multiples
        if ((rc = launch(mma_xprep_kernel, dim3(NB), dim3(256), 0, st, (const void*)xg, xbf, vec, Mg, NB, (int)cols,
                         xp, xscale, arrivals, pl.tiles)))
            return rc;
        MmaParams P;
        P.N = (int)rows;
        P.K = (int)cols;
        P.M = Mg;
        P.NB = NB;
        P.tiles = pl.tiles;
        P.n_chunks = pl.n_chunks;
        P.total = pl.total;
        P.G = pl.G;
        P.b_stages = std::min(kMaxBStages, kBRingBytes / (NB * 512));
        P.y = dY + g0 * rows;
        P.partial = partial;
        P.arrivals = arrivals;
        P.xscale = xscale;
        if ((rc = launch(gemm_q4_0_mma_kernel, dim3((unsigned)pl.G), dim3(kMmaThreads), kMmaSmemBytes, st, tmW, tmX,
                         P)))
            return rc;
    }
    return NEXUS_GPU_SUCCESS;
}

// ----------------------------------------------------------- dequantization
__global__ void dequant_kernel(int dtype, const uint8_t* __restrict__ W, float* __restrict__ out, uint64_t count) {
    const uint64_t i0 = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i0 >= count) return;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = (i0 + k < count) ? deq_elem(dtype, W, i0 + k) : 0.f;
    if (i0 + 4 <= count && ((uintptr_t)(out + i0) & 15) == 0) {
        *reinterpret_cast<float4*>(out + i0) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        for (int k = 0; k < 4 && i0 + k < count; ++k) out[i0 + k] = v[k];
    }
}

int32_t run_dequant(const void* dW, uint32_t dtype, float* dOut, size_t count, cudaStream_t st) {
    FormatInfo f;
    if (!format_info(dtype, f)) return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "unsupported dtype %u", dtype);
    if (count % (size_t)f.elems) return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "count not a whole number of blocks");
    if (count == 0) return NEXUS_GPU_SUCCESS;
    if (!dW || !dOut) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    const uint64_t threads = (count + 3) / 4;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    dequant_kernel<<<blocks, 256, 0, st>>>((int)dtype, static_cast<const uint8_t*>(dW), dOut, (uint64_t)count);
    CUDA_TRY(cudaGetLastError());
    return NEXUS_GPU_SUCCESS;
}

// ------------------------------------------------------------ workspace
int32_t get_workspace(Device& d, cudaStream_t st, size_t need, uint8_t** out) {
    if (need == 0) {
        *out = nullptr;
        return NEXUS_GPU_SUCCESS;
    }
    std::lock_guard<std::mutex> lk(d.mu);
    Workspace& w = d.ws[st];
    if (w.bytes < need) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        CUDA_TRY(cudaStreamIsCapturing(st, &cs));
        if (cs != cudaStreamCaptureStatusNone)
            return fail(NEXUS_GPU_ERROR_WORKSPACE,
                        "workspace of %zu bytes needed while the stream is capturing; make one uncaptured call "
                        "with these shapes first or pass a workspace to nexus_gpu_gemv_ws",
                        need);
        if (w.ptr) {
            CUDA_TRY(cudaStreamSynchronize(st));
            CUDA_TRY(cudaFree(w.ptr));
            w.ptr = nullptr;
            w.bytes = 0;
        }
        const size_t sz = align256(need + need / 4);
        CUDA_TRY(cudaMalloc(&w.ptr, sz));
        w.bytes = sz;
    }
    *out = static_cast<uint8_t*>(w.ptr);
    return NEXUS_GPU_SUCCESS;
}

// ------------------------------------------------- INT4-AWQ and FP8-E4M3
bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int32_t check_int4(size_t rows, size_t cols, size_t group_size) {
    if (group_size == 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "group_size is 0");
    if (cols % 8) return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "cols %zu not a multiple of 8 (whole packed words)", cols);
    if (cols % group_size)
        return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "cols %zu not a multiple of group_size %zu", cols, group_size);
    if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX)
        return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "rows or cols beyond 2^31");
    return NEXUS_GPU_SUCCESS;
}

// Workspace of an INT4 GEMV: x quantized to 16-bit fixed point.
size_t int4_ws_bytes(size_t cols) {
    const size_t nxb = cols / 32;
    return align256(nxb * kXQLimbBytes) + align256(nxb * kXQMetaBytes);
}

// Rows a warp streams together: 2 once every SM has at least 16 warps'
// worth of 2-row tasks, else 1 (more warps busy on small matrices).
int rows_per_warp(const Device& d, size_t rows) { return rows >= (size_t)d.sms * 16 * 2 ? 2 : 1; }

int rows_grid(const Device& d, size_t rows, int rpw) {
    const size_t per_cta = (kRowsThreads / 32) * (size_t)rpw;
    return (int)std::max<size_t>(1, std::min<size_t>((size_t)d.sms * 4, (rows + per_cta - 1) / per_cta));
}

int32_t rows_attrs(Device& d) {
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lk(mu);
    if (std::find(done.begin(), done.end(), d.id) != done.end()) return NEXUS_GPU_SUCCESS;
    const int need = std::max(kInt4MaxCols / 32 * 72, kFp8MaxCols * 4);
    if (d.smem_optin < need) return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "needs %d bytes of shared memory", need);
    CUDA_TRY(cudaFuncSetAttribute(gemv_int4_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, need));
    CUDA_TRY(cudaFuncSetAttribute(gemv_int4_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, need));
    CUDA_TRY(cudaFuncSetAttribute(gemv_fp8_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, need));
    CUDA_TRY(cudaFuncSetAttribute(gemv_fp8_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, need));
    done.push_back(d.id);
    return NEXUS_GPU_SUCCESS;
}

// y[rows] = W . x for INT4-AWQ weights (QuantizationKernel::fused_gemv_int4).
// ws holds int4_ws_bytes(cols) (fast path only).
int32_t run_gemv_int4(Device& d, const uint32_t* dW, const float* dS, const float* dZ, const float* dX, float* dY,
                      size_t rows, size_t cols, size_t gs, uint8_t* ws, cudaStream_t st) {
    int32_t rc = check_int4(rows, cols, gs);
    if (rc) return rc;
    if (rows == 0 || cols == 0) return NEXUS_GPU_SUCCESS;
    if (!dW || !dS || !dX || !dY) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    if ((rc = rows_attrs(d))) return rc;
    const int rpw = rows_per_warp(d, rows), grid = rows_grid(d, rows, rpw);
    if (cols % 32 == 0 && gs % 32 == 0 && cols <= (size_t)kInt4MaxCols && aligned16(dW) && ws) {
        uint8_t* limbs = ws;
        int4* meta = reinterpret_cast<int4*>(ws + align256(cols / 32 * kXQLimbBytes));
        dim3 g((unsigned)((cols / 32 + 7) / 8), 1);
        if ((rc = launch(xquant_kernel, g, dim3(256), 0, st, (const void*)dX, 0, (int)cols, (int)cols, limbs, meta)))
            return rc;
        Int4Params p;
        p.W = dW;
        p.scales = dS;
        p.zeros = dZ;
        p.limbs = limbs;
        p.meta = meta;
        p.y = dY;
        p.rows = (int)rows;
        p.cols = (int)cols;
        p.group_size = (int)gs;
        return rpw == 2 ? launch(gemv_int4_kernel<2>, dim3(grid), dim3(kRowsThreads), cols / 32 * 72, st, p)
                        : launch(gemv_int4_kernel<1>, dim3(grid), dim3(kRowsThreads), cols / 32 * 72, st, p);
    }
    return launch(gemv_int4_generic_kernel, dim3(rows_grid(d, rows, 1)), dim3(256), 0, st, dW, dS, dZ, dX, dY,
                  (int)rows, (int)cols, (int)gs);
}

// y[rows] = W . x for FP8-E4M3 weights (QuantizationKernel::fused_gemv_fp8).
int32_t run_gemv_fp8(Device& d, const uint8_t* dW, const float* dX, float* dY, size_t rows, size_t cols, float scale,
                     cudaStream_t st) {
    if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX)
        return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "rows or cols beyond 2^31");
    if (rows == 0) return NEXUS_GPU_SUCCESS;
    if (!dW || !dX || !dY) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    int32_t rc = rows_attrs(d);
    if (rc) return rc;
    const int rpw = rows_per_warp(d, rows), grid = rows_grid(d, rows, rpw);
    if (cols % 16 == 0 && cols > 0 && cols <= (size_t)kFp8MaxCols && aligned16(dW) && aligned16(dX)) {
        Fp8Params p;
        p.W = dW;
        p.x = dX;
        p.y = dY;
        p.rows = (int)rows;
        p.cols = (int)cols;
        p.scale = scale;
        return rpw == 2 ? launch(gemv_fp8_kernel<2>, dim3(grid), dim3(kRowsThreads), cols * 4, st, p)
                        : launch(gemv_fp8_kernel<1>, dim3(grid), dim3(kRowsThreads), cols * 4, st, p);
    }
    return launch(gemv_fp8_generic_kernel, dim3(rows_grid(d, rows, 1)), dim3(256), 0, st, dW, dX, dY, (int)rows,
                  (int)cols, scale);
}

int32_t run_dequant_int4(const uint32_t* dP, const float* dS, const float* dZ, float* dOut, size_t count, size_t gs,
                         cudaStream_t st) {
    if (gs == 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "group_size is 0");
    if (count == 0) return NEXUS_GPU_SUCCESS;
    if (!dP || !dS || !dOut) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    const unsigned grid = (unsigned)std::min<uint64_t>((count + 255) / 256, 1u << 20);
    return launch(dequant_int4_awq_kernel, dim3(grid), dim3(256), 0, st, dP, dS, dZ, dOut, (uint64_t)count,
                  (uint64_t)gs);
}

int32_t run_dequant_fp8(const uint8_t* dIn, float* dOut, size_t count, float scale, cudaStream_t st) {
    if (count == 0) return NEXUS_GPU_SUCCESS;
    if (!dIn || !dOut) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    const unsigned grid = (unsigned)std::min<uint64_t>((count + 255) / 256, 1u << 20);
    return launch(dequant_fp8_kernel, dim3(grid), dim3(256), 0, st, dIn, dOut, (uint64_t)count, scale);
}

// ---------------------------------------------------------- weight cache
uint64_t fnv1a(uint64_t h, const uint8_t* p, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 0x100000001b3ull;
    }
    return h;
}

// 64-bit mix of 8-byte words (a multiply-xorshift hash; not cryptographic).
inline uint64_t mix_words(uint64_t h, const uint8_t* p, size_t n) {
    for (size_t i = 0; i + 8 <= n; i += 8) {
        uint64_t w;
        memcpy(&w, p + i, 8);
        h = (h ^ w) * 0x9e3779b97f4a7c15ull;
        h ^= h >> 29;
    }
    return fnv1a(h, p + (n & ~(size_t)7), n & 7);
}

// Fingerprint of a host weight buffer, checked at every host-pointer GEMV to
// detect a buffer that now holds another tensor.  Default: the first and last
// 64 bytes and 16 bytes of every 64 KiB in between (about 150 probes for a
// 4096 x 4096 Q4_0 matrix, cheap next to the GEMV).  NEXUS_GPU_WEIGHT_CHECK=full
// hashes every byte instead (about 1 ms per 10 MB of weights on one host
// thread): then any change is detected, up to 64-bit hash collisions.
constexpr size_t kFingerprintStride = 64 * 1024;
bool full_weight_check() {
    const char* v = getenv("NEXUS_GPU_WEIGHT_CHECK");
    return v != nullptr && strcmp(v, "full") == 0;
}
uint64_t fingerprint(const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    uint64_t h = 0xcbf29ce484222325ull ^ n;
    if (full_weight_check()) return mix_words(h, b, n);
    h = mix_words(h, b, std::min<size_t>(n, 64));
    if (n > 64) h = mix_words(h, b + n - 64, 64);
    for (size_t o = kFingerprintStride; o + 16 <= n; o += kFingerprintStride) h = mix_words(h, b + o, 16);
    return h;
}

std::string cache_key(const void* W, uint32_t dtype, size_t rows, size_t cols) {
    char buf[96];
    snprintf(buf, sizeof(buf), "%p/%u/%zu/%zu", W, dtype, rows, cols);
    return buf;
}

int32_t cached_weight(Device& d, const void* W, uint32_t dtype, size_t rows, size_t cols, size_t bytes,
                      const void** out) {
    const std::string key = cache_key(W, dtype, rows, cols);
    const uint64_t fp = fingerprint(W, bytes);
    auto it = d.cache.find(key);
    if (it != d.cache.end() && it->second.fingerprint == fp) {
        *out = it->second.dptr;
        return NEXUS_GPU_SUCCESS;
    }
    if (it != d.cache.end()) {
        CUDA_TRY(cudaStreamSynchronize(d.stream));
        CUDA_TRY(cudaFree(it->second.dptr));
        d.cache_bytes -= it->second.bytes;
        d.cache.erase(it);
    }
    CachedWeight cw;
    CUDA_TRY(cudaMalloc(&cw.dptr, align256(bytes)));
    cw.bytes = align256(bytes);
    cw.fingerprint = fp;
    cudaError_t e = cudaMemcpy(cw.dptr, W, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(cw.dptr);
        return fail(NEXUS_GPU_ERROR_CUDA, "weight upload failed: %s", cudaGetErrorString(e));
    }
    d.cache_bytes += cw.bytes;
    d.cache.emplace(key, cw);
    *out = cw.dptr;
    return NEXUS_GPU_SUCCESS;
}

int32_t grow(void** p, size_t* cap, size_t need) {
    if (*cap >= need) return NEXUS_GPU_SUCCESS;
    if (*p) CUDA_TRY(cudaFree(*p));
    *p = nullptr;
    *cap = 0;
    const size_t sz = align256(std::max<size_t>(need, 4096));
    CUDA_TRY(cudaMalloc(p, sz));
    *cap = sz;
    return NEXUS_GPU_SUCCESS;
}

// The synchronous host-pointer GEMV behind layers 1 and 2.
int32_t host_gemv(const void* W, uint32_t dtype, const float* x, float* y, size_t rows, size_t cols) {
    if (!W) return NEXUS_GPU_SUCCESS;  // transformer_ops.hpp:158
    FormatInfo f;
    int32_t rc = check_shape(dtype, rows, cols, f);
    if (rc) return rc;
    if (rows == 0) return NEXUS_GPU_SUCCESS;
    if (!x || !y) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null x or y");
    Device* d = nullptr;
    if ((rc = get_device(&d))) return rc;
    std::lock_guard<std::mutex> lk(d->mu);
    const void* dW = nullptr;
    if ((rc = cached_weight(*d, W, dtype, rows, cols, rows * row_bytes_of(f, cols), &dW))) return rc;
    if ((rc = grow(&d->dx, &d->dx_cap, cols * 4 + xq_bytes(dtype, 1, cols) + 256))) return rc;
    if ((rc = grow(&d->dy, &d->dy_cap, rows * 4))) return rc;
    uint8_t* ws = static_cast<uint8_t*>(d->dx) + align256(cols * 4);
    CUDA_TRY(cudaMemcpyAsync(d->dx, x, cols * 4, cudaMemcpyHostToDevice, d->stream));
    if ((rc = run_gemv(*d, dW, dtype, d->dx, NEXUS_GPU_FP32, static_cast<float*>(d->dy), 1, rows, cols, ws,
                       d->stream)))
        return rc;
    CUDA_TRY(cudaMemcpyAsync(y, d->dy, rows * 4, cudaMemcpyDeviceToHost, d->stream));
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    return NEXUS_GPU_SUCCESS;
}

int32_t host_dequant(const void* blocks, uint32_t dtype, float* out, size_t num_blocks) {
    FormatInfo f;
    if (!format_info(dtype, f)) return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "unsupported dtype %u", dtype);
    if (num_blocks == 0) return NEXUS_GPU_SUCCESS;
    if (!blocks || !out) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(d->mu);
    const size_t in_bytes = num_blocks * (size_t)f.bytes, count = num_blocks * (size_t)f.elems;
    if ((rc = grow(&d->dx, &d->dx_cap, in_bytes))) return rc;
    if ((rc = grow(&d->dy, &d->dy_cap, count * 4))) return rc;
    CUDA_TRY(cudaMemcpyAsync(d->dx, blocks, in_bytes, cudaMemcpyHostToDevice, d->stream));
    if ((rc = run_dequant(d->dx, dtype, static_cast<float*>(d->dy), count, d->stream))) return rc;
    CUDA_TRY(cudaMemcpyAsync(out, d->dy, count * 4, cudaMemcpyDeviceToHost, d->stream));
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    return NEXUS_GPU_SUCCESS;
}

// Host-pointer INT4-AWQ / FP8 GEMV and dequantization (the reference's
// signatures): weights, scales and zeros are cached on the device like the
// GGUF weights (keyed by host pointer, shape and a sampled fingerprint).
constexpr uint32_t kCacheInt4 = 5, kCacheInt4Scales = 0x10005, kCacheInt4Zeros = 0x20005, kCacheFp8 = 3;

int32_t host_gemv_int4(const uint32_t* W, const float* x, const float* scales, const float* zeros, float* y,
                       size_t rows, size_t cols, size_t gs) {
    int32_t rc = check_int4(rows, cols, gs);
    if (rc) return rc;
    if (rows == 0 || cols == 0) return NEXUS_GPU_SUCCESS;
    if (!W || !x || !scales || !y) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    Device* d = nullptr;
    if ((rc = get_device(&d))) return rc;
    std::lock_guard<std::mutex> lk(d->mu);
    const size_t ng = rows * (cols / gs);
    const void *dW = nullptr, *dS = nullptr, *dZ = nullptr;
    if ((rc = cached_weight(*d, W, kCacheInt4, rows, cols, rows * cols / 2, &dW))) return rc;
    if ((rc = cached_weight(*d, scales, kCacheInt4Scales, rows, cols / gs, ng * 4, &dS))) return rc;
    if (zeros && (rc = cached_weight(*d, zeros, kCacheInt4Zeros, rows, cols / gs, ng * 4, &dZ))) return rc;
    if ((rc = grow(&d->dx, &d->dx_cap, align256(cols * 4) + int4_ws_bytes(cols) + 256))) return rc;
    if ((rc = grow(&d->dy, &d->dy_cap, rows * 4))) return rc;
    uint8_t* ws = static_cast<uint8_t*>(d->dx) + align256(cols * 4);
    CUDA_TRY(cudaMemcpyAsync(d->dx, x, cols * 4, cudaMemcpyHostToDevice, d->stream));
    if ((rc = run_gemv_int4(*d, static_cast<const uint32_t*>(dW), static_cast<const float*>(dS),
                            static_cast<const float*>(dZ), static_cast<const float*>(d->dx),
                            static_cast<float*>(d->dy), rows, cols, gs, ws, d->stream)))
        return rc;
    CUDA_TRY(cudaMemcpyAsync(y, d->dy, rows * 4, cudaMemcpyDeviceToHost, d->stream));
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    return NEXUS_GPU_SUCCESS;
}

int32_t host_gemv_fp8(const uint8_t* W, const float* x, float* y, size_t rows, size_t cols, float scale) {
    if (rows == 0 || cols == 0) return NEXUS_GPU_SUCCESS;
    if (!W || !x || !y) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(d->mu);
    const void* dW = nullptr;
    if ((rc = cached_weight(*d, W, kCacheFp8, rows, cols, rows * cols, &dW))) return rc;
    if ((rc = grow(&d->dx, &d->dx_cap, cols * 4))) return rc;
    if ((rc = grow(&d->dy, &d->dy_cap, rows * 4))) return rc;
    CUDA_TRY(cudaMemcpyAsync(d->dx, x, cols * 4, cudaMemcpyHostToDevice, d->stream));
    if ((rc = run_gemv_fp8(*d, static_cast<const uint8_t*>(dW), static_cast<const float*>(d->dx),
                           static_cast<float*>(d->dy), rows, cols, scale, d->stream)))
        return rc;
    CUDA_TRY(cudaMemcpyAsync(y, d->dy, rows * 4, cudaMemcpyDeviceToHost, d->stream));
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    return NEXUS_GPU_SUCCESS;
}

int32_t host_dequant_int4(const uint32_t* packed, const float* scales, const float* zeros, float* out, size_t count,
                          size_t gs) {
    if (gs == 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "group_size is 0");
    if (count == 0) return NEXUS_GPU_SUCCESS;
    if (!packed || !scales || !out) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(d->mu);
    const size_t words = (count + 7) / 8, ng = (count + gs - 1) / gs;
    const size_t o_s = align256(words * 4), o_z = o_s + align256(ng * 4);
    if ((rc = grow(&d->dx, &d->dx_cap, o_z + align256(ng * 4)))) return rc;
    if ((rc = grow(&d->dy, &d->dy_cap, count * 4))) return rc;
    uint8_t* base = static_cast<uint8_t*>(d->dx);
    CUDA_TRY(cudaMemcpyAsync(base, packed, words * 4, cudaMemcpyHostToDevice, d->stream));
    CUDA_TRY(cudaMemcpyAsync(base + o_s, scales, ng * 4, cudaMemcpyHostToDevice, d->stream));
    if (zeros) CUDA_TRY(cudaMemcpyAsync(base + o_z, zeros, ng * 4, cudaMemcpyHostToDevice, d->stream));
    if ((rc = run_dequant_int4(reinterpret_cast<const uint32_t*>(base), reinterpret_cast<const float*>(base + o_s),
                               zeros ? reinterpret_cast<const float*>(base + o_z) : nullptr,
                               static_cast<float*>(d->dy), count, gs, d->stream)))
        return rc;
    CUDA_TRY(cudaMemcpyAsync(out, d->dy, count * 4, cudaMemcpyDeviceToHost, d->stream));
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    return NEXUS_GPU_SUCCESS;
}

int32_t host_dequant_fp8(const uint8_t* in, float* out, size_t count, float scale) {
    if (count == 0) return NEXUS_GPU_SUCCESS;
    if (!in || !out) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null pointer");
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(d->mu);
    if ((rc = grow(&d->dx, &d->dx_cap, count))) return rc;
    if ((rc = grow(&d->dy, &d->dy_cap, count * 4))) return rc;
    CUDA_TRY(cudaMemcpyAsync(d->dx, in, count, cudaMemcpyHostToDevice, d->stream));
    if ((rc = run_dequant_fp8(static_cast<const uint8_t*>(d->dx), static_cast<float*>(d->dy), count, scale,
                              d->stream)))
        return rc;
    CUDA_TRY(cudaMemcpyAsync(out, d->dy, count * 4, cudaMemcpyDeviceToHost, d->stream));
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    return NEXUS_GPU_SUCCESS;
}

void report_void(const char* fn, int32_t rc) {
    if (rc != NEXUS_GPU_SUCCESS) fprintf(stderr, "[nexus_gpu] %s: %s (status %d)\n", fn, t_last_error.c_str(), rc);
}


// ------------------------------------------------------------ GEMV stacks
// Device block of a stack: the control area (abort flag, run epoch, CTA-exit
// count, end-of-run counts), then -- sharded stacks only -- every task's
// full-length output, then the tagged copy (a 32-bit word per row, the run's
// parity in the lowest bit) of every task that a later task depends on.
// Peers map this block through CUDA IPC.
struct StackLayout {
    size_t abort = 0, epoch = 0, fin = 0, end = 0, local_end = 0, ctrl = 0, total = 0;
    std::vector<uint64_t> out_off;  // sharded: output of task i at float offset out_off[i]
    std::vector<uint64_t> tg_off;   // task i's tagged copy at 32-bit word offset tg_off[i] (0: none)
};

struct StackHandle {
    int dev = -1;
    uint32_t dtype = 0;
    int group = 1;
    int grid = 0;
    size_t smem = 0;
    int n_tasks = 0;
    int world = 1, rank = 0;
    bool connected = true;  // sharded stacks need nexus_gpu_stack_connect first
    bool fused = false;     // some task has a norm, a SwiGLU or a residual: the kernel variant with them
    int tokens = 1;         // activation vectors per run (2..4: the multi-token kernel; 16..64: tensor cores)
    bool mma = false;       // the tcgen05 stack (tokens >= 16): mparams, tmX, d_block
    MmaStackParams mparams{};
    CUtensorMap tmXin{}, tmX{};  // tensor-core stack: x slots 0 (stack input) and 1
    uint64_t fingerprint = 0;
    StackParams params{};
    StackTask* d_tasks = nullptr;
    uint8_t* d_block = nullptr;
    StackLayout lay;
    std::vector<float*> outputs;        // this rank's output of each task
    std::vector<void*> peer_mappings;   // IPC mappings opened by connect
    // 5..15 tokens: multi-token stacks of 2..4 tokens each, run one after another
    // (part k serves tokens [part_tok0[k], part_tok0[k + 1])); no kernel of its own
    std::vector<StackHandle*> parts;
    std::vector<int> part_tok0;
    uint64_t input_cols = 0;
};

// What a rank publishes to its peers (nexus_gpu_stack_export).
struct StackBlob {
    uint32_t magic, version, world, rank, n_tasks, grid;
    uint64_t fingerprint, block_bytes;
    cudaIpcMemHandle_t handle;
};
constexpr uint32_t kStackBlobMagic = 0x4e535442u;  // "NSTB"

template <class F, int G, bool FX>
int32_t stack_kernel_attrs(const Device& d, size_t smem) {
    CUDA_TRY(cudaFuncSetAttribute(gemv_stack_kernel<F, G, FX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  d.smem_optin));
    int per_sm = 0;
    CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_stack_kernel<F, G, FX>, kGemvThreads, smem));
    if (per_sm < 1) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "stack kernel cannot be resident (smem %zu)", smem);
    return NEXUS_GPU_SUCCESS;
}

template <class F, int MT, int G>
int32_t stack_mt_kernel_attrs(const Device& d, size_t smem) {
    CUDA_TRY(cudaFuncSetAttribute(gemv_stack_mt_kernel<F, MT, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  d.smem_optin));
    int per_sm = 0;
    CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_stack_mt_kernel<F, MT, G>, kGemvThreads, smem));
    if (per_sm < 1) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "stack kernel cannot be resident (smem %zu)", smem);
    return NEXUS_GPU_SUCCESS;
}

template <class F>
int32_t stack_attrs_for(int group, bool fused, int tokens, const Device& d, size_t smem) {
    if (tokens == 2) {
        if constexpr (F::kGroup == 2)
            if (group == 2) return stack_mt_kernel_attrs<F, 2, 2>(d, smem);
        return stack_mt_kernel_attrs<F, 2, 1>(d, smem);
    }
    if (tokens == 3) return stack_mt_kernel_attrs<F, 3, 1>(d, smem);
    if (tokens == 4) return stack_mt_kernel_attrs<F, 4, 1>(d, smem);
    const bool grouped = F::kGroup > 1 && group == F::kGroup;
    if (fused) return grouped ? stack_kernel_attrs<F, F::kGroup, true>(d, smem) : stack_kernel_attrs<F, 1, true>(d, smem);
    return grouped ? stack_kernel_attrs<F, F::kGroup, false>(d, smem) : stack_kernel_attrs<F, 1, false>(d, smem);
}

template <class F>
int32_t stack_launch_for(const StackHandle& h, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(h.grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = h.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // CTAs wait on one another: all must be resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (h.tokens > 1) {
        bool paired = false;
        if constexpr (F::kGroup == 2) paired = h.group == 2;
        if (h.tokens == 2 && paired) {
            if constexpr (F::kGroup == 2) CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_mt_kernel<F, 2, F::kGroup>, h.params));
        } else if (h.tokens == 2) {
            CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_mt_kernel<F, 2, 1>, h.params));
        } else if (h.tokens == 3) {
            CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_mt_kernel<F, 3, 1>, h.params));
        } else {
            CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_mt_kernel<F, 4, 1>, h.params));
        }
        return NEXUS_GPU_SUCCESS;
    }
    const bool grouped = F::kGroup > 1 && h.group == F::kGroup;
    if (h.fused) {
        if (grouped) CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_kernel<F, F::kGroup, true>, h.params));
        else CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_kernel<F, 1, true>, h.params));
    } else {
        if (grouped) CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_kernel<F, F::kGroup, false>, h.params));
        else CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stack_kernel<F, 1, false>, h.params));
    }
    return NEXUS_GPU_SUCCESS;
}

void stack_free(StackHandle* h) {
    if (!h) return;
    for (StackHandle* p : h->parts) stack_free(p);
    int cur = -1;
    cudaGetDevice(&cur);
    if (h->dev >= 0 && cur != h->dev) cudaSetDevice(h->dev);
    for (void* m : h->peer_mappings)
        if (m) cudaIpcCloseMemHandle(m);
    if (h->d_tasks) cudaFree(h->d_tasks);
    if (h->d_block) cudaFree(h->d_block);
    if (h->dev >= 0 && cur >= 0 && cur != h->dev) cudaSetDevice(cur);
    delete h;
}

// Rows [r0, r1) of an N-row matrix that rank `rank` of `world` owns.
inline void shard_rows(uint64_t N, int world, int rank, uint64_t& r0, uint64_t& r1) {
    r0 = N * (uint64_t)rank / (uint64_t)world;
    r1 = N * (uint64_t)(rank + 1) / (uint64_t)world;
}

uint64_t stack_fingerprint(uint32_t dtype, const NexusGpuStackTaskEx* tasks, uint32_t n, uint64_t input_cols,
                           int world) {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](uint64_t v) {
        for (int i = 0; i < 8; ++i) {
            h ^= (v >> (8 * i)) & 0xffu;
            h *= 1099511628211ull;
        }
    };
    mix(dtype);
    mix(n);
    mix(input_cols);
    mix((uint64_t)world);
    for (uint32_t i = 0; i < n; ++i) {
        mix(tasks[i].rows);
        mix(tasks[i].cols);
        mix((uint64_t)(int64_t)tasks[i].x_source);
        mix((uint64_t)(int64_t)tasks[i].after);
        mix((uint64_t)(int64_t)tasks[i].x_source2);
        mix((uint64_t)(int64_t)tasks[i].residual_source);
        mix(tasks[i].norm_weight != nullptr);
        uint32_t eb;
        memcpy(&eb, &tasks[i].norm_eps, 4);
        mix(tasks[i].norm_weight ? eb : 0u);
        mix(tasks[i].W_up != nullptr);
    }
    return h;
}

int32_t mma_stack_create(uint32_t dtype, const NexusGpuStackTaskEx* tasks, uint32_t n, uint64_t input_cols,
                         int tokens, void** out);

int32_t stack_create(uint32_t dtype, const NexusGpuStackTaskEx* tasks, uint32_t n, uint64_t input_cols, int world,
                     int rank, void** out, int tokens = 1) {
    if (tokens >= kMmaMinTokens && tokens <= kMaxTokens && world == 1)
        return mma_stack_create(dtype, tasks, n, input_cols, tokens, out);
    if (!out || (!tasks && n)) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "rank %d of world %d (1..%d GPUs)", rank, world, kMaxWorld);
    const bool sharded = world > 1;
    if (tokens < 1 || tokens > kMaxStackTokens)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "%d tokens per run (1..%d on CUDA cores, %d..%d on tensor cores)",
                    tokens, kMaxStackTokens, kMmaMinTokens, kMaxTokens);
    if (tokens > 1 && sharded)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "a multi-token stack is not sharded");
    if (dtype == NEXUS_GPU_FP16)
        return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "GEMV stacks serve the integer GGUF formats");
    FormatInfo f;
    if (!format_info(dtype, f)) return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "unsupported weight dtype %u", dtype);
    if (n == 0 || n > 100000) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task count %u", n);
    if (input_cols == 0 || input_cols % 32 || input_cols > (uint64_t)INT32_MAX)
        return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "stack input length %llu is not a positive multiple of 32",
                    (unsigned long long)input_cols);
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    if ((rc = ensure_attrs(*d))) return rc;

    std::vector<StackTask> ht(n);
    std::vector<uint64_t> local_rows(n), row_off(n);
    int group = -1;
    size_t slot = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const NexusGpuStackTaskEx& u = tasks[i];
        if ((rc = check_shape(dtype, u.rows, u.cols, f))) return fail(rc, "task %u: %s", i, t_last_error.c_str());
        if (!u.W || u.rows == 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: null W or no rows", i);
        if (sharded ? u.y != nullptr : u.y == nullptr)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT,
                        sharded ? "task %u: y must be NULL in a sharded stack (outputs belong to the stack)"
                                : "task %u: null y", i);
        if (((uintptr_t)u.W & 15) != 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: W not 16-byte aligned", i);
        if (tokens > 1 && (u.x_source2 != -1 || u.residual_source != -2 || u.norm_weight || u.W_up))
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: a multi-token stack has no fused operations", i);
        const uint64_t xlen = u.x_source < 0 ? input_cols : (u.x_source < (int32_t)i ? tasks[u.x_source].rows : 0);
        if (u.x_source >= (int32_t)i || xlen != u.cols)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "task %u: x_source %d does not give a vector of %llu", i,
                        u.x_source, (unsigned long long)u.cols);
        if (u.after >= (int32_t)i || u.after < -1)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: after=%d is not an earlier task", i, u.after);
        if (!sharded && u.x_source >= 0 && ((uintptr_t)tasks[u.x_source].y & 15) != 0)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %d feeds x but its y is not 16-byte aligned",
                        u.x_source);
        if (u.x_source2 != -1 &&
            (u.x_source2 < 0 || u.x_source2 >= (int32_t)i || tasks[u.x_source2].rows != u.cols || u.x_source < 0))
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH,
                        "task %u: x_source2 %d must be an earlier task of %llu rows beside a task x_source", i,
                        u.x_source2, (unsigned long long)u.cols);
        if (!sharded && u.x_source2 >= 0 && ((uintptr_t)tasks[u.x_source2].y & 15) != 0)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %d feeds x2 but its y is not 16-byte aligned",
                        u.x_source2);
        if (u.residual_source < -2 || u.residual_source >= (int32_t)i ||
            (u.residual_source == -1 && input_cols != u.rows) ||
            (u.residual_source >= 0 && tasks[u.residual_source].rows != u.rows))
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "task %u: residual_source %d does not give %llu values", i,
                        u.residual_source, (unsigned long long)u.rows);
        if (u.norm_weight && ((uintptr_t)u.norm_weight & 15) != 0)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: norm_weight not 16-byte aligned", i);
        if (u.W_up && ((uintptr_t)u.W_up & 15) != 0)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: W_up not 16-byte aligned", i);
        uint64_t r0 = 0, r1 = u.rows;
        if (sharded) shard_rows(u.rows, world, rank, r0, r1);
        if (r1 <= r0 || u.rows > (uint64_t)INT32_MAX)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "task %u: %llu rows leave rank %d of %d no rows", i,
                        (unsigned long long)u.rows, rank, world);
        local_rows[i] = r1 - r0;
        row_off[i] = r0;
        GemvParams gp{};
        size_t sm = 0;
        const uint64_t rb = row_bytes_of(f, u.cols);
        // a gate+up pair plans with its two rows as one (twice the bytes per ring row)
        // multi-token stacks: one (two for 2 tokens) single-block work items per lane, smaller stages
        const bool ok_plan = tokens > 1
                                 ? plan_for(dtype, *d, (int)local_rows[i], (int)u.cols, rb, gp, sm, kStageTargetBytes,
                                            kMaxJ / (tokens == 2 ? 2 : 4),
                                            tokens == 2 && (dtype == NEXUS_GPU_GGUF_Q4_0 || dtype == NEXUS_GPU_GGUF_Q8_0))
                                 : plan_for(dtype, *d, (int)local_rows[i], (int)u.cols, u.W_up ? 2 * rb : rb, gp, sm,
                                            kStackStageTargetBytes);
        if (!ok_plan)
            return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "task %u (%llux%llu) is outside the fast kernel's limits", i,
                        (unsigned long long)local_rows[i], (unsigned long long)u.cols);
        if (group < 0) group = gp.group;
        if (gp.group != group)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "task %u: mixed block-grouping in one stack", i);
        StackTask& T = ht[i];
        T.W = static_cast<const uint8_t*>(u.W);
        T.row_bytes = rb;
        T.total_bytes = rb * local_rows[i];
        T.N = (int)local_rows[i];
        T.K = (int)u.cols;
        T.nwi = gp.nwi;
        T.segments = gp.segments;
        T.seg_wi = gp.seg_wi;
        T.wi_per_lane = gp.wi_per_lane;
        T.stage_rows = gp.stage_rows;
        T.stage_bytes = gp.stage_bytes;
        T.rot_step = gp.stage_rows % (kConsumerWarps / gp.segments);
        T.row_off = (int)row_off[i];
        if (u.W_up) {  // the up rows of a stage sit half a slot after the gate rows
            T.W2 = static_cast<const uint8_t*>(u.W_up);
            T.half = (int)((gp.stage_rows * rb + 32 + 15) / 16 * 16);
            T.stage_bytes = 2 * T.half;
        }
        slot = std::max(slot, (size_t)T.stage_bytes);
    }
    size_t x_smem = 0;
    for (const StackTask& T : ht)
        x_smem = std::max(x_smem, (size_t)tokens * x_stage_planes_len(T.K) * (kXQLimbBytes + kXQMetaBytes));
    x_smem = (x_smem + 127) / 128 * 128;
    if ((uint64_t)d->smem_optin < kStackSmemHeader + x_smem + 128 + 2 * slot)
        return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "stack stages do not fit shared memory");
    const uint64_t avail = (uint64_t)d->smem_optin - kStackSmemHeader - x_smem - 128;
    int ns = (int)std::min<uint64_t>(kMaxStages, avail / slot);
    auto fits = [&](int k) {
        for (const StackTask& T : ht)
            if (T.stage_rows * T.segments * (T.W2 ? 2 : 1) * tokens > kMaxSlots / k) return false;
        return true;
    };
    while (ns > 2 && !fits(ns)) --ns;
    if (ns < 2 || !fits(ns)) return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "stack stages do not fit shared memory");

    auto h = new StackHandle();
    h->dev = d->id;
    h->dtype = dtype;
    h->group = group;
    h->grid = d->sms;
    h->n_tasks = (int)n;
    h->world = world;
    h->rank = rank;
    h->connected = !sharded;
    h->tokens = tokens;
    h->fingerprint = stack_fingerprint(dtype, tasks, n, input_cols, world);
    h->smem = kStackSmemHeader + x_smem + (size_t)ns * slot;
    for (uint32_t i = 0; i < n; ++i)
        h->fused |= tasks[i].x_source2 >= 0 || tasks[i].residual_source != -2 || tasks[i].norm_weight != nullptr ||
                    tasks[i].W_up != nullptr;

    std::vector<char> waited_for(n, 0);
    for (uint32_t i = 0; i < n; ++i) {
        if (tasks[i].after >= 0) waited_for[tasks[i].after] = 1;
        if (tasks[i].x_source >= 0) waited_for[tasks[i].x_source] = 1;
        if (tasks[i].x_source2 >= 0) waited_for[tasks[i].x_source2] = 1;
        if (tasks[i].residual_source >= 0) waited_for[tasks[i].residual_source] = 1;
    }
    StackLayout& lay = h->lay;
    lay.abort = 0;
    lay.epoch = lay.abort + 128;
    lay.fin = lay.epoch + 128;
    lay.end = lay.fin + 128;
    lay.local_end = lay.end + 128;
    lay.ctrl = align256(lay.local_end + 128);
    lay.total = lay.ctrl;
    if (sharded) {
        lay.out_off.resize(n);
        for (uint32_t i = 0; i < n; ++i) {
            lay.out_off[i] = lay.total / sizeof(float);
            lay.total += align256(tasks[i].rows * sizeof(float));
        }
    }
    lay.tg_off.assign(n, 0);
    for (uint32_t i = 0; i < n; ++i) {
        if (!waited_for[i]) continue;
        lay.tg_off[i] = lay.total / sizeof(uint32_t);
        lay.total += align256(tasks[i].rows * tokens * sizeof(uint32_t));
    }

    // each task's rows for each CTA, balanced: [N*c/grid, N*(c+1)/grid) of this rank's slice
    const size_t task_bytes = align256(n * sizeof(StackTask));
    std::vector<int2> cta_rows((size_t)n * h->grid);
    for (uint32_t i = 0; i < n; ++i)
        for (int c = 0; c < h->grid; ++c)
            cta_rows[(size_t)i * h->grid + c] = make_int2((int)(local_rows[i] * (uint64_t)c / (uint64_t)h->grid),
                                                          (int)(local_rows[i] * (uint64_t)(c + 1) / (uint64_t)h->grid));
    cudaError_t e = cudaMalloc(&h->d_tasks, task_bytes + cta_rows.size() * sizeof(int2));
    if (e == cudaSuccess) e = cudaMalloc(&h->d_block, lay.total);
    if (e == cudaSuccess) e = cudaMemset(h->d_block, 0, lay.total);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        stack_free(h);
        cudaGetLastError();
        return fail(NEXUS_GPU_ERROR_OUT_OF_TIER0_MEMORY, "stack allocation failed: %s", cudaGetErrorString(e));
    }
    h->outputs.resize(n);
    for (uint32_t i = 0; i < n; ++i)
        h->outputs[i] = sharded ? reinterpret_cast<float*>(h->d_block) + lay.out_off[i] : tasks[i].y;
    for (uint32_t i = 0; i < n; ++i) {
        StackTask& T = ht[i];
        T.y = h->outputs[i];
        T.y_off = sharded ? lay.out_off[i] : 0;
        T.tg = waited_for[i] ? reinterpret_cast<uint32_t*>(h->d_block) + lay.tg_off[i] : nullptr;
        T.tg_off = lay.tg_off[i];
        T.src = tasks[i].x_source < 0 ? -1 : tasks[i].x_source;
        T.after = tasks[i].after;
        T.after_rows = tasks[i].after >= 0 ? (int)tasks[tasks[i].after].rows : 0;
        T.src2 = tasks[i].x_source2 < 0 ? -1 : tasks[i].x_source2;
        T.norm_w = tasks[i].norm_weight;
        T.norm_eps = tasks[i].norm_eps;
        T.res_input = tasks[i].residual_source == -1;
        T.res_src = tasks[i].residual_source >= 0 ? tasks[i].residual_source : -1;
        // same input (and fusions), same plan (same cols), and no new ordering
        // dependency: keep the previous task's x slices, skip the wait and the staging
        T.reuse_x = i > 0 && tasks[i].x_source == tasks[i - 1].x_source && tasks[i].cols == tasks[i - 1].cols &&
                    tasks[i].x_source2 == tasks[i - 1].x_source2 && tasks[i].norm_weight == tasks[i - 1].norm_weight &&
                    (!tasks[i].norm_weight || memcmp(&tasks[i].norm_eps, &tasks[i - 1].norm_eps, 4) == 0) &&
                    (tasks[i].after == -1 || tasks[i].after == tasks[i - 1].after) &&
                    (tasks[i].residual_source < 0 || tasks[i].residual_source == tasks[i - 1].residual_source);
    }
    e = cudaMemcpy(h->d_tasks, ht.data(), n * sizeof(StackTask), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(reinterpret_cast<uint8_t*>(h->d_tasks) + task_bytes, cta_rows.data(),
                       cta_rows.size() * sizeof(int2), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        stack_free(h);
        return fail(NEXUS_GPU_ERROR_CUDA, "stack upload failed: %s", cudaGetErrorString(e));
    }
    StackParams& P = h->params;
    P.tasks = h->d_tasks;
    P.cta_rows = reinterpret_cast<const int2*>(reinterpret_cast<uint8_t*>(h->d_tasks) + task_bytes);
    P.n_tasks = (int)n;
    P.n_stages = ns;
    P.stage_slot = (int)slot;
    P.x_smem = (int)x_smem;
    P.slot_stride = kMaxSlots / ns;
    P.x_in = nullptr;
    P.wait_ns = kWaitLimitNs;
    P.wait_polls = (uint32_t)(kWaitLimitNs / kTagPollNs);
    P.abort_flag = reinterpret_cast<unsigned*>(h->d_block + lay.abort);
    P.epoch = reinterpret_cast<unsigned long long*>(h->d_block + lay.epoch);
    P.fin = reinterpret_cast<unsigned long long*>(h->d_block + lay.fin);
    P.end_done = reinterpret_cast<unsigned long long*>(h->d_block + lay.end);
    P.local_end = reinterpret_cast<unsigned long long*>(h->d_block + lay.local_end);
    P.world = world;
    P.rank = rank;
    P.peer_end[rank] = P.end_done;
    P.peer_block[rank] = h->d_block;

    switch (dtype) {
        case NEXUS_GPU_GGUF_Q4_0: rc = stack_attrs_for<FmtQ4_0>(group, h->fused, tokens, *d, h->smem); break;
        case NEXUS_GPU_GGUF_Q8_0: rc = stack_attrs_for<FmtQ8_0>(group, h->fused, tokens, *d, h->smem); break;
        case NEXUS_GPU_GGUF_Q5_K: rc = stack_attrs_for<FmtQ5_K>(group, h->fused, tokens, *d, h->smem); break;
        default: rc = stack_attrs_for<FmtQ6_K>(group, h->fused, tokens, *d, h->smem); break;
    }
    if (rc) {
        stack_free(h);
        return rc;
    }
    *out = h;
    return NEXUS_GPU_SUCCESS;
}

// ---------------------------------------------------- tensor-core stacks
// A stack for 16..64 tokens on the tcgen05 tensor cores
// (gemm_q4_0_mma_stack_kernel): GGUF Q4_0, every task's cols a multiple of
// 256, unsharded, no fused operations.  Every task's y holds tokens x rows
// floats; the stack input tokens x input_cols.
int32_t mma_stack_create(uint32_t dtype, const NexusGpuStackTaskEx* tasks, uint32_t n, uint64_t input_cols,
                         int tokens, void** out) {
    if (!out || (!tasks && n)) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (dtype != NEXUS_GPU_GGUF_Q4_0)
        return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "tensor-core stacks (%d..%d tokens) serve GGUF Q4_0",
                    kMmaMinTokens, kMaxTokens);
    if (n == 0 || n > 100000) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task count %u", n);
    if (input_cols == 0 || input_cols % kRawK || input_cols > (uint64_t)INT32_MAX)
        return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "stack input length %llu is not a positive multiple of %d",
                    (unsigned long long)input_cols, kRawK);
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    if ((rc = ensure_attrs(*d))) return rc;
    if (d->smem_optin < kMmaStackSmemBytes)
        return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "tensor-core stack needs %d bytes of shared memory",
                    kMmaStackSmemBytes);
    TensorMapEncodeTiled encode = tensor_map_encoder();
    if (!encode) return fail(NEXUS_GPU_ERROR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const int NB = (tokens + 15) / 16 * 16, G = d->sms;
    std::vector<MmaTask> ht(n);
    std::vector<MmaGroup> hg;
    std::vector<size_t> arr_off(n);
    size_t arr_words = 0;
    int kmax = 0, last_hop = 0, pubs = 0, in_pub = -1, cur_pub = -1;
    for (uint32_t i = 0; i < n; ++i) {
        const NexusGpuStackTaskEx& u = tasks[i];
        if (!u.W || !u.y || u.rows == 0 || u.rows > (uint64_t)INT32_MAX)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: null W or y, or no rows", i);
        if (u.cols == 0 || u.cols % kRawK || u.cols > (uint64_t)INT32_MAX)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "task %u: cols %llu is not a positive multiple of %d", i,
                        (unsigned long long)u.cols, kRawK);
        if (((uintptr_t)u.W & 15) || ((uintptr_t)u.y & 15))
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: W or y not 16-byte aligned", i);
        if (u.x_source2 != -1 || u.residual_source != -2 || u.norm_weight || u.W_up)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: a multi-token stack has no fused operations", i);
        const uint64_t xlen = u.x_source < 0 ? input_cols : (u.x_source < (int32_t)i ? tasks[u.x_source].rows : 0);
        if (u.x_source >= (int32_t)i || xlen != u.cols)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "task %u: x_source %d does not give a vector of %llu", i,
                        u.x_source, (unsigned long long)u.cols);
        if (u.after >= (int32_t)i || u.after < -1)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u: after=%d is not an earlier task", i, u.after);
        // a hop (grid barriers, x conversion) where the input changes, or where an `after`
        // task has not been behind a barrier yet: it starts a new group
        const bool hop = i == 0 || u.x_source != tasks[i - 1].x_source || (u.after >= 0 && u.after >= last_hop);
        if (hop) {
            last_hop = (int)i;
            MmaGroup g;
            memset(&g, 0, sizeof(g));
            g.x = u.x_source < 0 ? nullptr : tasks[u.x_source].y;
            g.first = (int)i;
            g.n_chunks = (int)(u.cols / kRawK);
            g.K = (int)u.cols;
            g.hidx = (int)hg.size();
            // x slot 0 holds the stack input, converted at its first hop of a run; slot 1 the
            // latest earlier task's y, converted at every hop that reads one
            g.xslot = u.x_source < 0 ? 0 : 1;
            if (u.x_source >= 0 || in_pub < 0) {
                g.conv = 1;
                cur_pub = pubs++;
                if (u.x_source < 0) in_pub = cur_pub;
            }
            g.pidx = u.x_source < 0 ? in_pub : cur_pub;
            hg.push_back(g);
        }
        MmaGroup& grp = hg.back();
        MmaTask& T = ht[i];
        memset(&T, 0, sizeof(T));
        const uint64_t rb = u.cols / 32 * 18;
        const cuuint64_t dims[2] = {(cuuint64_t)rb, (cuuint64_t)u.rows};
        const cuuint64_t strides[1] = {(cuuint64_t)rb};
        const cuuint32_t box[2] = {(cuuint32_t)kRawRowBytes, (cuuint32_t)kMmaRows};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&T.tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(u.W), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return fail(NEXUS_GPU_ERROR_CUDA, "task %u: weight tensor map rejected", i);
        T.y = u.y;
        T.N = (int)u.rows;
        T.tiles = (int)((u.rows + kMmaRows - 1) / kMmaRows);
        T.tile0 = grp.tiles;
        grp.tiles += T.tiles;
        grp.count += 1;
        arr_off[i] = arr_words;
        arr_words += (size_t)T.tiles;
        kmax = std::max(kmax, (int)u.cols);
    }
    for (MmaGroup& g : hg) {  // each group one stream-K GEMM over its members' tiles
        g.total = (long long)g.tiles * g.n_chunks;
        g.G = tc_ctas(G, g.tiles, g.n_chunks);
    }
    const int n_groups = (int)hg.size();
    // device block: tasks (64-byte aligned maps), fp16 x, scales, partial sums, arrival
    // counters, grid barrier / run / exit counters and the abort flag
    size_t off = 0;
    const size_t o_tasks = off;
    off = align256(off + n * sizeof(MmaTask));
    const size_t o_groups = off;
    off = align256(off + n_groups * sizeof(MmaGroup));
    const size_t o_x = off;
    off = align256(off + 2 * (size_t)NB * kmax * sizeof(__half));
    const size_t o_scale = off;
    off = align256(off + 2 * kMaxTokens * sizeof(float));
    const size_t o_part = off;
    off = align256(off + (size_t)G * 2 * NB * kMmaRows * sizeof(float));
    const size_t o_arr = off;
    off = align256(off + arr_words * sizeof(unsigned));
    const size_t o_ctrl = off;
    off = align256(off + 5 * sizeof(unsigned long long));
    auto h = new StackHandle();
    h->dev = d->id;
    h->dtype = dtype;
    h->grid = G;
    h->n_tasks = (int)n;
    h->tokens = tokens;
    h->mma = true;
    cudaError_t e = cudaMalloc(&h->d_block, off);
    if (e == cudaSuccess) e = cudaMemset(h->d_block, 0, off);
    if (e != cudaSuccess) {
        stack_free(h);
        cudaGetLastError();
        return fail(NEXUS_GPU_ERROR_OUT_OF_TIER0_MEMORY, "stack allocation failed: %s", cudaGetErrorString(e));
    }
    uint8_t* blk = h->d_block;
    for (uint32_t i = 0; i < n; ++i) ht[i].arrivals = reinterpret_cast<unsigned*>(blk + o_arr) + arr_off[i];
    e = cudaMemcpy(blk + o_tasks, ht.data(), n * sizeof(MmaTask), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(blk + o_groups, hg.data(), n_groups * sizeof(MmaGroup), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        stack_free(h);
        return fail(NEXUS_GPU_ERROR_CUDA, "stack upload failed: %s", cudaGetErrorString(e));
    }
    for (int slot = 0; slot < 2; ++slot) {
        const cuuint64_t dims[2] = {(cuuint64_t)kmax, (cuuint64_t)NB};
        const cuuint64_t strides[1] = {(cuuint64_t)kmax * sizeof(__half)};
        const cuuint32_t box[2] = {(cuuint32_t)kUnitK, (cuuint32_t)NB};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(slot ? &h->tmX : &h->tmXin, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   blk + o_x + (size_t)slot * NB * kmax * sizeof(__half), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            stack_free(h);
            return fail(NEXUS_GPU_ERROR_CUDA, "activation tensor map rejected (%d x %d)", NB, kmax);
        }
    }
    MmaStackParams& P = h->mparams;
    P.tasks = reinterpret_cast<const MmaTask*>(blk + o_tasks);
    P.groups = reinterpret_cast<const MmaGroup*>(blk + o_groups);
    P.n_groups = n_groups;
    P.n_pubs = pubs;
    P.M = tokens;
    P.NB = NB;
    P.kmax = kmax;
    // the ring budget: x tiles for about 6 chunks' MMAs (at least 3), raw chunks in the rest
    P.b_stages = std::max(3, std::min(6, 48 * 1024 / (NB * 512)));
    P.raw_base = (P.b_stages * NB * 512 + 1023) / 1024 * 1024;
    P.raw_stages = std::min(kStackRawMax, (kStackRingBytes - P.raw_base) / kRawChunkBytes);
    P.xbuf = reinterpret_cast<__half*>(blk + o_x);
    P.xscale = reinterpret_cast<float*>(blk + o_scale);
    P.partial = reinterpret_cast<float*>(blk + o_part);
    unsigned long long* ctrl = reinterpret_cast<unsigned long long*>(blk + o_ctrl);
    P.bar_done = ctrl;
    P.bar_pub = ctrl + 1;
    P.epoch = ctrl + 2;
    P.fin = ctrl + 3;
    P.abort_flag = reinterpret_cast<unsigned*>(ctrl + 4);
    h->params.abort_flag = P.abort_flag;  // nexus_gpu_stack_wait reads it
    h->outputs.resize(n);
    for (uint32_t i = 0; i < n; ++i) h->outputs[i] = tasks[i].y;
    auto attrs = [&]() -> int32_t {
        CUDA_TRY(cudaFuncSetAttribute(gemm_q4_0_mma_stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kMmaStackSmemBytes));
        int per_sm = 0;
        CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_q4_0_mma_stack_kernel, kMmaStackThreads,
                                                               kMmaStackSmemBytes));
        if (per_sm < 1) {
            cudaFuncAttributes fa = {};
            cudaFuncGetAttributes(&fa, gemm_q4_0_mma_stack_kernel);
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT,
                        "tensor-core stack kernel cannot be resident (%d registers a thread, at most %d threads, "
                        "%d threads and %d bytes of shared memory asked)",
                        fa.numRegs, fa.maxThreadsPerBlock, kMmaStackThreads, kMmaStackSmemBytes);
        }
        return NEXUS_GPU_SUCCESS;
    };
    if ((rc = attrs())) {
        stack_free(h);
        return rc;
    }
    *out = h;
    return NEXUS_GPU_SUCCESS;
}

int32_t mma_stack_launch(StackHandle& h, const float* x_in, cudaStream_t st) {
    h.mparams.x_in = x_in;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(h.grid);
    cfg.blockDim = dim3(kMmaStackThreads);
    cfg.dynamicSmemBytes = kMmaStackSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // CTAs wait on one another at grid barriers: all resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_q4_0_mma_stack_kernel, h.tmXin, h.tmX, h.mparams));
    return NEXUS_GPU_SUCCESS;
}

int32_t stack_current_device(const StackHandle* h) {
    int cur = -1;
    CUDA_TRY(cudaGetDevice(&cur));
    if (cur != h->dev) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "stack belongs to device %d, current is %d", h->dev, cur);
    return NEXUS_GPU_SUCCESS;
}

int32_t stack_export(void* handle, void* blob, uint64_t* bytes) {
    StackHandle* h = static_cast<StackHandle*>(handle);
    if (!h || !bytes) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null handle or size");
    if (!blob) {
        *bytes = sizeof(StackBlob);
        return NEXUS_GPU_SUCCESS;
    }
    if (*bytes < sizeof(StackBlob)) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "blob buffer of %llu bytes, need %zu",
                                                (unsigned long long)*bytes, sizeof(StackBlob));
    if (h->world < 2) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "not a sharded stack");
    int32_t rc = stack_current_device(h);
    if (rc) return rc;
    StackBlob b{};
    b.magic = kStackBlobMagic;
    b.version = 1;
    b.world = (uint32_t)h->world;
    b.rank = (uint32_t)h->rank;
    b.n_tasks = (uint32_t)h->n_tasks;
    b.grid = (uint32_t)h->grid;
    b.fingerprint = h->fingerprint;
    b.block_bytes = h->lay.total;
    CUDA_TRY(cudaIpcGetMemHandle(&b.handle, h->d_block));
    std::memcpy(blob, &b, sizeof(b));
    *bytes = sizeof(StackBlob);
    return NEXUS_GPU_SUCCESS;
}

int32_t stack_connect(void* handle, const void* blobs, uint64_t bytes) {
    StackHandle* h = static_cast<StackHandle*>(handle);
    if (!h || !blobs) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null handle or blobs");
    if (h->world < 2) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "not a sharded stack");
    if (h->connected) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "stack already connected");
    if (bytes != (uint64_t)h->world * sizeof(StackBlob))
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "%llu blob bytes, need %d x %zu", (unsigned long long)bytes,
                    h->world, sizeof(StackBlob));
    int32_t rc = stack_current_device(h);
    if (rc) return rc;
    std::vector<StackBlob> b(h->world);
    std::memcpy(b.data(), blobs, bytes);
    for (int p = 0; p < h->world; ++p) {
        if (b[p].magic != kStackBlobMagic || b[p].version != 1 || b[p].world != (uint32_t)h->world ||
            b[p].rank != (uint32_t)p)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "blob %d is not rank %d's stack export", p, p);
        if (b[p].fingerprint != h->fingerprint || b[p].n_tasks != (uint32_t)h->n_tasks ||
            b[p].block_bytes != h->lay.total)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "rank %d built a different task list", p);
        if (b[p].grid != (uint32_t)h->grid)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "rank %d runs %u CTAs, this rank %d", p, b[p].grid, h->grid);
    }
    std::vector<void*> maps(h->world, nullptr);
    for (int p = 0; p < h->world; ++p) {
        if (p == h->rank) continue;
        cudaError_t e = cudaIpcOpenMemHandle(&maps[p], b[p].handle, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (void* m : maps)
                if (m) cudaIpcCloseMemHandle(m);
            cudaGetLastError();
            return fail(NEXUS_GPU_ERROR_CUDA, "opening rank %d's stack memory: %s", p, cudaGetErrorString(e));
        }
    }
    StackParams& P = h->params;
    for (int p = 0; p < h->world; ++p) {
        if (p == h->rank) continue;
        uint8_t* base = static_cast<uint8_t*>(maps[p]);
        P.peer_end[p] = reinterpret_cast<unsigned long long*>(base + h->lay.end);
        P.peer_block[p] = base;
    }
    h->peer_mappings = maps;
    h->connected = true;
    return NEXUS_GPU_SUCCESS;
}

// Ranks of one sharded stack that live in this process (one thread or one
// loop driving several GPUs, or -- for tests -- several ranks on one GPU):
// connect them by their device pointers, with peer access enabled between
// distinct devices.  Same checks as stack_connect.
int32_t stack_connect_local(void* const* stacks, uint32_t n) {
    if (!stacks || n < 2 || n > (uint32_t)kMaxWorld)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "%u stacks (2..%d ranks)", n, kMaxWorld);
    std::vector<StackHandle*> hs(n);
    for (uint32_t i = 0; i < n; ++i) {
        hs[i] = static_cast<StackHandle*>(stacks[i]);
        if (!hs[i]) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null stack %u", i);
        if (hs[i]->world != (int)n || hs[i]->rank != (int)i)
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "stack %u is rank %d of %d, not rank %u of %u", i,
                        hs[i]->rank, hs[i]->world, i, n);
        if (hs[i]->connected) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "stack %u already connected", i);
        if (hs[i]->fingerprint != hs[0]->fingerprint || hs[i]->lay.total != hs[0]->lay.total)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "rank %u built a different task list", i);
        if (hs[i]->grid != hs[0]->grid)
            return fail(NEXUS_GPU_ERROR_SHAPE_MISMATCH, "rank %u runs %d CTAs, rank 0 %d", i, hs[i]->grid, hs[0]->grid);
    }
    int cur = -1;
    CUDA_TRY(cudaGetDevice(&cur));
    for (uint32_t i = 0; i < n; ++i)
        for (uint32_t j = 0; j < n; ++j) {
            if (hs[i]->dev == hs[j]->dev) continue;
            int can = 0;
            CUDA_TRY(cudaDeviceCanAccessPeer(&can, hs[i]->dev, hs[j]->dev));
            if (!can) {
                cudaSetDevice(cur);
                return fail(NEXUS_GPU_ERROR_CUDA, "device %d cannot reach device %d", hs[i]->dev, hs[j]->dev);
            }
            CUDA_TRY(cudaSetDevice(hs[i]->dev));
            const cudaError_t e = cudaDeviceEnablePeerAccess(hs[j]->dev, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) {
                cudaSetDevice(cur);
                return fail(NEXUS_GPU_ERROR_CUDA, "peer access %d -> %d: %s", hs[i]->dev, hs[j]->dev,
                            cudaGetErrorString(e));
            }
        }
    CUDA_TRY(cudaSetDevice(cur));
    for (uint32_t i = 0; i < n; ++i) {
        StackParams& P = hs[i]->params;
        for (uint32_t p = 0; p < n; ++p) {
            P.peer_end[p] = hs[p]->params.end_done;
            P.peer_block[p] = hs[p]->d_block;
        }
        hs[i]->connected = true;
    }
    return NEXUS_GPU_SUCCESS;
}

// Wait for the stack's last run on `stream`; a wait that gave up (a peer that
// never ran, a stalled pipeline) poisons the stack and is reported here.
int32_t stack_wait(void* handle, cudaStream_t st) {
    StackHandle* h = static_cast<StackHandle*>(handle);
    if (!h) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null handle");
    int32_t rc = stack_current_device(h);
    if (rc) return rc;
    for (StackHandle* p : h->parts)
        if ((rc = stack_wait(p, st))) return rc;
    if (!h->parts.empty()) return NEXUS_GPU_SUCCESS;
    CUDA_TRY(cudaStreamSynchronize(st));
    unsigned aborted = 0;
    CUDA_TRY(cudaMemcpy(&aborted, h->params.abort_flag, sizeof(aborted), cudaMemcpyDeviceToHost));
    if (aborted) return fail(NEXUS_GPU_ERROR_TIMEOUT, "a bounded wait of the stack expired; destroy the stack");
    return NEXUS_GPU_SUCCESS;
}

int32_t stack_output(void* handle, uint32_t task, float** y) {
    StackHandle* h = static_cast<StackHandle*>(handle);
    if (!h || !y) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null handle or output pointer");
    if (task >= (uint32_t)h->n_tasks) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "task %u of %d", task, h->n_tasks);
    *y = h->outputs[task];
    return NEXUS_GPU_SUCCESS;
}

int32_t stack_run(void* handle, const float* x_in, cudaStream_t st) {
    StackHandle* h = static_cast<StackHandle*>(handle);
    if (!h || !x_in) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null handle or input");
    if (((uintptr_t)x_in & 15) != 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "stack input not 16-byte aligned");
    if (!h->connected) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "sharded stack not connected to its peers");
    int32_t rc = stack_current_device(h);
    if (rc) return rc;
    for (size_t k = 0; k < h->parts.size(); ++k)  // a split stack: its parts in token order
        if ((rc = stack_run(h->parts[k], x_in + (size_t)h->part_tok0[k] * h->input_cols, st))) return rc;
    if (!h->parts.empty()) return NEXUS_GPU_SUCCESS;
    if (h->mma) return mma_stack_launch(*h, x_in, st);
    h->params.x_in = x_in;
    switch (h->dtype) {
        case NEXUS_GPU_GGUF_Q4_0: return stack_launch_for<FmtQ4_0>(*h, st);
        case NEXUS_GPU_GGUF_Q8_0: return stack_launch_for<FmtQ8_0>(*h, st);
        case NEXUS_GPU_GGUF_Q5_K: return stack_launch_for<FmtQ5_K>(*h, st);
        default: return stack_launch_for<FmtQ6_K>(*h, st);
    }
}

// ------------------------------------------------ no-allocation entry point
// Scratch of nexus_gpu_gemv_noalloc: the quantized activations (int16 X and
// block metadata) that xquant_kernel writes and the GEMV kernel reads.  It is
// part of the loaded module, so every GPU that loads the library holds these
// kNoAllocScratchBytes until the process exits, and no call ever allocates.
// In host code the array's name is only a host-side stand-in: the device
// address comes from cudaGetSymbolAddress, once per device.
constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB
constexpr int kNoAllocMaxDevices = 64;
static_assert(sizeof(g_noalloc_scratch) == kNoAllocScratchBytes, "scratch array and its stated limit differ");

struct NoAllocDevice {
    bool ready = false;
    uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
    Device dev;                  // geometry and kernel attributes only; no stream, no memory
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc[kNoAllocMaxDevices];  // constructed at load time: calls never allocate

// First call on a device (with that device current): resolve the scratch
// array's device address and read the device geometry.
int32_t noalloc_device(Device** out_dev, uint8_t** out_scratch) {
    int id = 0, n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(NEXUS_GPU_ERROR_NO_DEVICE, "no CUDA device");
    }
    CUDA_TRY(cudaGetDevice(&id));
    if (id < 0 || id >= kNoAllocMaxDevices)
        return fail(NEXUS_GPU_ERROR_NO_DEVICE, "device %d beyond the %d devices the no-allocation path serves", id,
                    kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocDevice& e = g_noalloc[id];
    if (!e.ready) {
        void* ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (err != cudaSuccess)
            return fail(NEXUS_GPU_ERROR_CUDA, "cudaGetSymbolAddress(no-allocation scratch) failed: %s",
                        cudaGetErrorString(err));
        e.dev.id = id;
        CUDA_TRY(cudaDeviceGetAttribute(&e.dev.sms, cudaDevAttrMultiProcessorCount, id));
        CUDA_TRY(cudaDeviceGetAttribute(&e.dev.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, id));
        e.scratch = static_cast<uint8_t*>(ptr);
        // kernel attributes too, under the lock: later calls only read e.dev
        int32_t rc = ensure_attrs(e.dev);
        if (rc) return rc;
        e.ready = true;
    }
    *out_dev = &e.dev;
    *out_scratch = e.scratch;
    return NEXUS_GPU_SUCCESS;
}

}  // namespace
}  // namespace nexus_gpu

using namespace nexus_gpu;

// ================================================================ C ABI
extern "C" {

NEXUS_GPU_API void nexus_fused_gemv_q4_0(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    report_void(__func__, host_gemv(W, NEXUS_GPU_GGUF_Q4_0, x, y, rows, cols));
}
NEXUS_GPU_API void nexus_fused_gemv_q8_0(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    report_void(__func__, host_gemv(W, NEXUS_GPU_GGUF_Q8_0, x, y, rows, cols));
}
NEXUS_GPU_API void nexus_fused_gemv_fp16(const uint16_t* W, const float* x, float* y, size_t rows, size_t cols) {
    report_void(__func__, host_gemv(W, NEXUS_GPU_FP16, x, y, rows, cols));
}
NEXUS_GPU_API void nexus_fused_gemv_q5_k(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    report_void(__func__, host_gemv(W, NEXUS_GPU_GGUF_Q5_K, x, y, rows, cols));
}
NEXUS_GPU_API void nexus_fused_gemv_q6_k(const void* W, const float* x, float* y, size_t rows, size_t cols) {
    report_void(__func__, host_gemv(W, NEXUS_GPU_GGUF_Q6_K, x, y, rows, cols));
}

NEXUS_GPU_API void nexus_dequantize_gguf_q4_0(const void* blocks, float* out, size_t nb) {
    report_void(__func__, host_dequant(blocks, NEXUS_GPU_GGUF_Q4_0, out, nb));
}
NEXUS_GPU_API void nexus_dequantize_gguf_q5_k(const void* blocks, float* out, size_t nb) {
    report_void(__func__, host_dequant(blocks, NEXUS_GPU_GGUF_Q5_K, out, nb));
}
NEXUS_GPU_API void nexus_dequantize_gguf_q6_k(const void* blocks, float* out, size_t nb) {
    report_void(__func__, host_dequant(blocks, NEXUS_GPU_GGUF_Q6_K, out, nb));
}

NEXUS_GPU_API void nexus_fused_gemv_int4(const uint32_t* W_packed, const float* x, const float* scales,
                                         const float* zeros, float* y, size_t rows, size_t cols, size_t group_size) {
    report_void(__func__, host_gemv_int4(W_packed, x, scales, zeros, y, rows, cols, group_size));
}
NEXUS_GPU_API void nexus_fused_gemv_fp8(const uint8_t* W_fp8, const float* x, float* y, size_t rows, size_t cols,
                                        float scale) {
    report_void(__func__, host_gemv_fp8(W_fp8, x, y, rows, cols, scale));
}
NEXUS_GPU_API void nexus_dequantize_int4_awq(const uint32_t* packed, const float* scales, const float* zeros,
                                             float* output, size_t count, size_t group_size) {
    report_void(__func__, host_dequant_int4(packed, scales, zeros, output, count, group_size));
}
NEXUS_GPU_API void nexus_dequantize_fp8_e4m3(const uint8_t* input, float* output, size_t count, float scale) {
    report_void(__func__, host_dequant_fp8(input, output, count, scale));
}

NEXUS_GPU_API int32_t nexus_gpu_gemv_dispatch(const void* W, uint32_t dtype, const float* x, float* y, size_t rows,
                                              size_t cols) {
    t_last_error.clear();
    return host_gemv(W, dtype, x, y, rows, cols);
}

NEXUS_GPU_API void* nexus_gpu_allocate_device_memory(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        fail(NEXUS_GPU_ERROR_OUT_OF_TIER0_MEMORY, "cudaMalloc(%zu) failed", bytes);
        return nullptr;
    }
    return p;
}
NEXUS_GPU_API void nexus_gpu_free_device_memory(void* ptr) {
    if (ptr) cudaFree(ptr);
}
NEXUS_GPU_API int32_t nexus_gpu_copy_host_to_device_async(void* dst, const void* src, size_t bytes, void* stream) {
    CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
    return NEXUS_GPU_SUCCESS;
}
NEXUS_GPU_API int32_t nexus_gpu_copy_device_to_host_async(void* dst, const void* src, size_t bytes, void* stream) {
    CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
    return NEXUS_GPU_SUCCESS;
}
NEXUS_GPU_API int32_t nexus_gpu_synchronize(void* stream) {
    CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_weight_cache_invalidate(const void* host_W) {
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(d->mu);
    CUDA_TRY(cudaStreamSynchronize(d->stream));
    char prefix[32];
    snprintf(prefix, sizeof(prefix), "%p/", host_W);
    for (auto it = d->cache.begin(); it != d->cache.end();) {
        if (host_W == nullptr || it->first.rfind(prefix, 0) == 0) {
            CUDA_TRY(cudaFree(it->second.dptr));
            d->cache_bytes -= it->second.bytes;
            it = d->cache.erase(it);
        } else {
            ++it;
        }
    }
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API size_t nexus_gpu_weight_cache_bytes(void) {
    Device* d = nullptr;
    if (get_device(&d)) return 0;
    std::lock_guard<std::mutex> lk(d->mu);
    return d->cache_bytes;
}

NEXUS_GPU_API size_t nexus_gpu_weight_bytes(uint32_t dtype, size_t rows, size_t cols) {
    FormatInfo f;
    if (!format_info(dtype, f) || cols % (size_t)f.elems) return 0;
    return rows * row_bytes_of(f, cols);
}

// SM count of the current device (148, a B200's, when there is none: sizes
// then cover a B200).
int current_sms() {
    int id = 0, sms = 0;
    if (cudaGetDevice(&id) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, id) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    return sms;
}

NEXUS_GPU_API size_t nexus_gpu_gemv_workspace_size(uint32_t dtype, size_t M, size_t rows, size_t cols) {
    return gemv_ws_bytes(current_sms(), dtype, M, rows, cols, true);
}

NEXUS_GPU_API int32_t nexus_gpu_gemv_ws(const void* dW, uint32_t dtype, const void* dX, uint32_t x_dtype, float* dY,
                                        size_t M, size_t rows, size_t cols, void* workspace, size_t workspace_bytes,
                                        void* stream) {
    t_last_error.clear();
    if (M > kMaxActivationRows)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "M=%zu activation rows, at most %zu", M, kMaxActivationRows);
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    const size_t need = gemv_ws_bytes(d->sms, dtype, M, rows, cols, true);
    if (workspace_bytes < need || (need && !workspace))
        return fail(NEXUS_GPU_ERROR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    if (need && ((uintptr_t)workspace & 255))
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
    return run_gemv(*d, dW, dtype, dX, x_dtype, dY, M, rows, cols, static_cast<uint8_t*>(workspace),
                    static_cast<cudaStream_t>(stream));
}

NEXUS_GPU_API int32_t nexus_gpu_gemv(const void* dW, uint32_t dtype, const void* dX, uint32_t x_dtype, float* dY,
                                     size_t M, size_t rows, size_t cols, void* stream) {
    t_last_error.clear();
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    FormatInfo f;
    if ((rc = check_shape(dtype, rows, cols, f))) return rc;
    uint8_t* ws = nullptr;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = get_workspace(*d, st, gemv_ws_bytes(d->sms, dtype, M, rows, cols, true), &ws))) return rc;
    return run_gemv(*d, dW, dtype, dX, x_dtype, dY, M, rows, cols, ws, st);
}

NEXUS_GPU_API int32_t nexus_gpu_gemv_noalloc(const void* dW, uint32_t dtype, const void* dX, uint32_t x_dtype,
                                             float* dY, size_t M, size_t rows, size_t cols, void* stream) {
    t_last_error.clear();
    FormatInfo f;
    int32_t rc = check_shape(dtype, rows, cols, f);
    if (rc) return rc;
    // bound M first, so that the scratch size below cannot overflow
    if (M > kMaxActivationRows)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "M=%zu activation rows, at most %zu", M, kMaxActivationRows);
    const size_t need = xq_bytes(dtype, M, cols);
    if (need > kNoAllocScratchBytes)
        return fail(NEXUS_GPU_ERROR_WORKSPACE,
                    "nexus_gpu_gemv_noalloc: M=%zu x cols=%zu needs %zu bytes of scratch, above its fixed %zu-byte "
                    "array (M * cols / 32 * 80 bytes must fit); use nexus_gpu_gemv_ws for larger shapes",
                    M, cols, need, kNoAllocScratchBytes);
    Device* d = nullptr;
    uint8_t* scratch = nullptr;
    if ((rc = noalloc_device(&d, &scratch))) return rc;
    // the fixed scratch serves the CUDA-core path only (no tensor-core workspace)
    return run_gemv(*d, dW, dtype, dX, x_dtype, dY, M, rows, cols, scratch, static_cast<cudaStream_t>(stream), false);
}

// The plain stack tasks as fused-task descriptions with no fusions.
std::vector<NexusGpuStackTaskEx> plain_tasks(const NexusGpuStackTask* tasks, uint32_t n) {
    std::vector<NexusGpuStackTaskEx> v(tasks ? n : 0);
    for (size_t i = 0; i < v.size(); ++i) {
        v[i].W = tasks[i].W;
        v[i].rows = tasks[i].rows;
        v[i].cols = tasks[i].cols;
        v[i].y = tasks[i].y;
        v[i].x_source = tasks[i].x_source;
        v[i].after = tasks[i].after;
        v[i].x_source2 = -1;
        v[i].residual_source = -2;
        v[i].norm_weight = nullptr;
        v[i].norm_eps = 0.0f;
        v[i].W_up = nullptr;
    }
    return v;
}

NEXUS_GPU_API int32_t nexus_gpu_stack_create(uint32_t dtype, const NexusGpuStackTask* tasks, uint32_t n_tasks,
                                             uint64_t input_cols, void** out_stack) {
    t_last_error.clear();
    const auto ex = plain_tasks(tasks, n_tasks);
    return stack_create(dtype, tasks ? ex.data() : nullptr, n_tasks, input_cols, 1, 0, out_stack);
}

// 5..15 tokens (between the CUDA-core and the tensor-core stacks): ceil(tokens / 4)
// multi-token stacks of 2..4 tokens each over the same tasks, part k writing its
// tokens' rows of every y and reading its tokens' rows of the input; a run launches
// them one after another, so every weight is read ceil(tokens / 4) times a run.
int32_t stack_create_split(uint32_t dtype, const NexusGpuStackTaskEx* tasks, uint32_t n, uint64_t input_cols,
                           int tokens, void** out) {
    if (!out || !tasks || n == 0) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null argument or no tasks");
    *out = nullptr;
    const int k = (tokens + kMaxStackTokens - 1) / kMaxStackTokens;
    auto h = new StackHandle();
    h->dtype = dtype;
    h->n_tasks = (int)n;
    h->tokens = tokens;
    h->input_cols = input_cols;
    for (uint32_t i = 0; i < n; ++i) h->outputs.push_back(static_cast<float*>(tasks[i].y));
    std::vector<NexusGpuStackTaskEx> part(tasks, tasks + n);
    int tok0 = 0;
    for (int j = 0; j < k; ++j) {
        const int m = tokens / k + (j < tokens % k ? 1 : 0);  // 2..4: tokens >= 5 and k = ceil(tokens / 4)
        for (uint32_t i = 0; i < n; ++i)
            part[i].y = tasks[i].y ? static_cast<float*>(tasks[i].y) + (size_t)tok0 * tasks[i].rows : nullptr;
        void* p = nullptr;
        const int32_t rc = stack_create(dtype, part.data(), n, input_cols, 1, 0, &p, m);
        if (rc) {
            stack_free(h);
            return rc;
        }
        h->parts.push_back(static_cast<StackHandle*>(p));
        h->part_tok0.push_back(tok0);
        tok0 += m;
    }
    h->dev = h->parts[0]->dev;
    *out = h;
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_stack_create_tokens(uint32_t dtype, const NexusGpuStackTask* tasks, uint32_t n_tasks,
                                                    uint64_t input_cols, uint32_t tokens, void** out_stack) {
    t_last_error.clear();
    const auto ex = plain_tasks(tasks, n_tasks);
    if (tokens > (uint32_t)kMaxStackTokens && tokens < (uint32_t)kMmaMinTokens)
        return stack_create_split(dtype, tasks ? ex.data() : nullptr, n_tasks, input_cols, (int)tokens, out_stack);
    return stack_create(dtype, tasks ? ex.data() : nullptr, n_tasks, input_cols, 1, 0, out_stack,
                        tokens > (uint32_t)kMaxTokens ? kMaxTokens + 1 : (int)tokens);
}

NEXUS_GPU_API int32_t nexus_gpu_stack_create_ex(uint32_t dtype, const NexusGpuStackTaskEx* tasks, uint32_t n_tasks,
                                                uint64_t input_cols, uint32_t world, uint32_t rank, void** out_stack) {
    t_last_error.clear();
    if (world < 1 || world > (uint32_t)kMaxWorld || rank >= world)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "rank %u of world %u (1..%d GPUs)", rank, world, kMaxWorld);
    return stack_create(dtype, tasks, n_tasks, input_cols, (int)world, (int)rank, out_stack);
}

NEXUS_GPU_API int32_t nexus_gpu_stack_create_sharded(uint32_t dtype, const NexusGpuStackTask* tasks, uint32_t n_tasks,
                                                     uint64_t input_cols, uint32_t world, uint32_t rank,
                                                     void** out_stack) {
    t_last_error.clear();
    if (world < 2) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "a sharded stack needs 2..%d ranks", kMaxWorld);
    if (world > (uint32_t)kMaxWorld || rank >= world)
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "rank %u of world %u (2..%d GPUs)", rank, world, kMaxWorld);
    const auto ex = plain_tasks(tasks, n_tasks);
    return stack_create(dtype, tasks ? ex.data() : nullptr, n_tasks, input_cols, (int)world, (int)rank, out_stack);
}

NEXUS_GPU_API int32_t nexus_gpu_stack_export(void* stack, void* blob, uint64_t* blob_bytes) {
    t_last_error.clear();
    return stack_export(stack, blob, blob_bytes);
}

NEXUS_GPU_API int32_t nexus_gpu_stack_connect(void* stack, const void* blobs, uint64_t blobs_bytes) {
    t_last_error.clear();
    return stack_connect(stack, blobs, blobs_bytes);
}

NEXUS_GPU_API int32_t nexus_gpu_stack_output(void* stack, uint32_t task, float** y) {
    t_last_error.clear();
    return stack_output(stack, task, y);
}

NEXUS_GPU_API int32_t nexus_gpu_stack_run(void* stack, const float* dX, void* stream) {
    t_last_error.clear();
    return stack_run(stack, dX, static_cast<cudaStream_t>(stream));
}

NEXUS_GPU_API int32_t nexus_gpu_stack_connect_local(void* const* stacks, uint32_t n_stacks) {
    t_last_error.clear();
    return stack_connect_local(stacks, n_stacks);
}

NEXUS_GPU_API int32_t nexus_gpu_stack_set_wait_limit(void* stack, uint64_t limit_ns) {
    t_last_error.clear();
    StackHandle* h = static_cast<StackHandle*>(stack);
    if (!h) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null stack");
    for (StackHandle* p : h->parts) nexus_gpu_stack_set_wait_limit(p, limit_ns);
    h->params.wait_ns = limit_ns ? limit_ns : kWaitLimitNs;
    h->params.wait_polls = (uint32_t)std::min<uint64_t>(h->params.wait_ns / kTagPollNs + 1, UINT32_MAX);
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_stack_wait(void* stack, void* stream) {
    t_last_error.clear();
    return stack_wait(stack, static_cast<cudaStream_t>(stream));
}

NEXUS_GPU_API int32_t nexus_gpu_stack_destroy(void* stack) {
    stack_free(static_cast<StackHandle*>(stack));
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_dequantize(const void* dW, uint32_t dtype, float* dOut, size_t count, void* stream) {
    t_last_error.clear();
    return run_dequant(dW, dtype, dOut, count, static_cast<cudaStream_t>(stream));
}

NEXUS_GPU_API size_t nexus_gpu_gemv_int4_workspace_size(size_t cols) { return int4_ws_bytes(cols); }

NEXUS_GPU_API int32_t nexus_gpu_gemv_int4(const void* dW, const float* dScales, const float* dZeros, const float* dX,
                                          float* dY, size_t rows, size_t cols, size_t group_size, void* workspace,
                                          size_t workspace_bytes, void* stream) {
    t_last_error.clear();
    int32_t rc = check_int4(rows, cols, group_size);  // before touching a device
    if (rc) return rc;
    Device* d = nullptr;
    if ((rc = get_device(&d))) return rc;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const size_t need = int4_ws_bytes(cols);
    if (!ws) {
        if ((rc = get_workspace(*d, st, need, &ws))) return rc;
    } else if (workspace_bytes < need) {
        return fail(NEXUS_GPU_ERROR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes, need);
    }
    return run_gemv_int4(*d, static_cast<const uint32_t*>(dW), dScales, dZeros, dX, dY, rows, cols, group_size, ws,
                         st);
}

NEXUS_GPU_API int32_t nexus_gpu_gemv_fp8(const void* dW, const float* dX, float* dY, size_t rows, size_t cols,
                                         float scale, void* stream) {
    t_last_error.clear();
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    return run_gemv_fp8(*d, static_cast<const uint8_t*>(dW), dX, dY, rows, cols, scale,
                        static_cast<cudaStream_t>(stream));
}

NEXUS_GPU_API int32_t nexus_gpu_dequantize_int4_awq(const void* dPacked, const float* dScales, const float* dZeros,
                                                    float* dOut, size_t count, size_t group_size, void* stream) {
    t_last_error.clear();
    return run_dequant_int4(static_cast<const uint32_t*>(dPacked), dScales, dZeros, dOut, count, group_size,
                            static_cast<cudaStream_t>(stream));
}

NEXUS_GPU_API int32_t nexus_gpu_dequantize_fp8_e4m3(const void* dIn, float* dOut, size_t count, float scale,
                                                    void* stream) {
    t_last_error.clear();
    return run_dequant_fp8(static_cast<const uint8_t*>(dIn), dOut, count, scale, static_cast<cudaStream_t>(stream));
}

NEXUS_GPU_API const char* nexus_gpu_last_error(void) { return t_last_error.c_str(); }

NEXUS_GPU_API int32_t nexus_gpu_device_status(uint32_t* out_bits) {
    if (!out_bits) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null out_bits");
    CUDA_TRY(cudaDeviceSynchronize());
    unsigned v = 0, zero = 0;
    CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)));
    CUDA_TRY(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)));
    *out_bits = v;
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_device_info(char* name, size_t name_len, int* sm_count, int* cc_major,
                                            int* cc_minor) {
    int id = 0;
    CUDA_TRY(cudaGetDevice(&id));
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, id));
    if (name && name_len) {
        strncpy(name, prop.name, name_len - 1);
        name[name_len - 1] = '\0';
    }
    if (sm_count) *sm_count = prop.multiProcessorCount;
    if (cc_major) *cc_major = prop.major;
    if (cc_minor) *cc_minor = prop.minor;
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API const char* nexus_gpu_version(void) { return "nexus_gpu 0.1.0 (sm_100a)"; }

// ------------------------------------------------ GGUF file -> device upload

NEXUS_GPU_API int32_t nexus_gpu_gguf_open(const char* path, void** out_file) {
    if (!path || !out_file) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null path or out_file");
    *out_file = nullptr;
    auto* f = new (std::nothrow) gguf::File();
    if (!f) return fail(NEXUS_GPU_ERROR_OUT_OF_HOST_MEMORY, "out of host memory");
    std::string err;
    bool ok = false;
    try {
        ok = gguf::parse(path, *f, err);
    } catch (const std::bad_alloc&) {
        err = "out of host memory while parsing";
    }
    if (!ok) {
        gguf::close_file(*f);
        delete f;
        return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "%s: %s", path, err.c_str());
    }
    *out_file = f;
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_gguf_close(void* file) {
    if (!file) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null file");
    auto* f = static_cast<gguf::File*>(file);
    int cur = -1;
    if (!f->ring.empty()) {  // the staging buffers belong to the upload's device
        cudaGetDevice(&cur);
        cudaSetDevice(f->device);
    }
    gguf::close_file(*f);
    if (cur >= 0) cudaSetDevice(cur);  // leave the caller's current device as it was
    delete f;
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_gguf_model(void* file, NexusGpuGgufModel* out) {
    if (!file || !out) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null file or out");
    const gguf::File& f = *static_cast<gguf::File*>(file);
    const gguf::Model& m = f.model;
    memset(out, 0, sizeof(*out));
    snprintf(out->architecture, sizeof(out->architecture), "%s", m.architecture.c_str());
    out->version = f.version;
    out->alignment = (uint32_t)f.alignment;  // at most 2^31: checked by the parser
    out->tensor_count = f.tensors.size();
    out->skipped = f.skipped;
    out->data_offset = f.data_offset;
    out->vocab_size = m.vocab;
    out->hidden_size = m.hidden;
    out->intermediate_size = m.ffn;
    out->num_hidden_layers = m.layers;
    out->num_attention_heads = m.heads;
    out->num_key_value_heads = m.kv_heads;
    out->max_position_embeddings = m.ctx;
    out->rms_norm_eps = m.eps;
    out->rope_theta = m.rope;
    out->is_moe = m.moe;
    out->num_experts = m.experts;
    out->num_experts_per_tok = m.experts_per_tok;
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_gguf_tensor(void* file, uint64_t index, NexusGpuGgufTensor* out) {
    if (!file || !out) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null file or out");
    const gguf::File& f = *static_cast<gguf::File*>(file);
    if (index >= f.tensors.size())
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "tensor index %llu of %zu", (unsigned long long)index,
                    f.tensors.size());
    const gguf::Tensor& t = f.tensors[index];
    memset(out, 0, sizeof(*out));
    snprintf(out->name, sizeof(out->name), "%s", t.name.c_str());
    out->ggml_type = t.ggml_type;
    out->dtype = t.dtype;
    out->served = gguf::served(t.dtype);
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; ++d) out->dims[d] = d < (int)t.n_dims ? t.dims[d] : 1;
    out->cols = t.dims[0];
    out->rows = t.dims[1] * t.dims[2] * t.dims[3];
    out->file_offset = t.file_offset;
    out->bytes = t.bytes;
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API int32_t nexus_gpu_gguf_find(void* file, const char* name, uint64_t* index) {
    if (!file || !name || !index) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null argument");
    if (!gguf::find(*static_cast<gguf::File*>(file), name, *index))
        return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "no tensor named %s", name);
    return NEXUS_GPU_SUCCESS;
}

NEXUS_GPU_API uint64_t nexus_gpu_gguf_upload_size(void* file, const uint64_t* indices, uint64_t n) {
    if (!file || (n && !indices)) return 0;
    const gguf::File& f = *static_cast<gguf::File*>(file);
    for (uint64_t i = 0; i < n; ++i)
        if (indices[i] >= f.tensors.size()) return 0;
    return gguf::image_layout(f, indices, n, nullptr);
}

NEXUS_GPU_API int32_t nexus_gpu_gguf_upload(void* file, const uint64_t* indices, uint64_t n, void* d_dst,
                                            uint64_t dst_bytes, uint64_t* offsets, void* stream) {
    if (!file || (n && (!indices || !offsets))) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null argument");
    gguf::File& f = *static_cast<gguf::File*>(file);
    for (uint64_t i = 0; i < n; ++i) {
        if (indices[i] >= f.tensors.size())
            return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "tensor index %llu of %zu", (unsigned long long)indices[i],
                        f.tensors.size());
        const gguf::Tensor& t = f.tensors[indices[i]];
        if (t.dtype < 0 || t.bytes == 0)
            return fail(NEXUS_GPU_ERROR_FORMAT_UNSUPPORTED, "tensor %s: ggml type %u has no NexusLLM data type",
                        t.name.c_str(), t.ggml_type);
    }
    const uint64_t total = gguf::image_layout(f, indices, n, offsets);
    if (total == 0) return NEXUS_GPU_SUCCESS;
    if (!d_dst) return fail(NEXUS_GPU_ERROR_INVALID_ARGUMENT, "null device buffer");
    if (dst_bytes < total)
        return fail(NEXUS_GPU_ERROR_WORKSPACE, "device buffer of %llu bytes, the image needs %llu",
                    (unsigned long long)dst_bytes, (unsigned long long)total);
    Device* d = nullptr;
    int32_t rc = get_device(&d);
    if (rc) return rc;
    if (!f.ring.empty() && f.device != d->id) {  // staging of another device: remake it here
        CUDA_TRY(cudaSetDevice(f.device));
        for (gguf::Staging& s : f.ring) {
            cudaEventSynchronize(s.done);
            cudaEventDestroy(s.done);
            cudaFreeHost(s.host);
        }
        f.ring.clear();
        CUDA_TRY(cudaSetDevice(d->id));
    }
    if (f.ring.empty()) {  // pinned staging ring, kept for later uploads; all or nothing
        std::vector<gguf::Staging> ring(gguf::kStages);
        cudaError_t e = cudaSuccess;
        for (gguf::Staging& s : ring) {
            if (e == cudaSuccess) e = cudaHostAlloc(&s.host, gguf::kStageBytes, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming);
        }
        if (e != cudaSuccess) {
            for (gguf::Staging& s : ring) {
                if (s.done) cudaEventDestroy(s.done);
                if (s.host) cudaFreeHost(s.host);
            }
            cudaGetLastError();
            return fail(NEXUS_GPU_ERROR_OUT_OF_HOST_MEMORY, "pinned staging buffers: %s", cudaGetErrorString(e));
        }
        f.device = d->id;
        f.ring = std::move(ring);
    }
    std::vector<gguf::Segment> seg(n);
    for (uint64_t i = 0; i < n; ++i) {
        const gguf::Tensor& t = f.tensors[indices[i]];
        seg[i] = {offsets[i], t.bytes, f.base + t.file_offset};
    }
    std::sort(seg.begin(), seg.end(), [](const gguf::Segment& a, const gguf::Segment& b) {
        return a.image_off < b.image_off;
    });
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int threads = (int)std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    auto drain = [&]() {  // leave no copy in flight from the staging buffers
        for (gguf::Staging& s : f.ring)
            if (s.busy) {
                cudaEventSynchronize(s.done);
                s.busy = false;
            }
    };
    int k = 0;
    for (uint64_t c0 = 0; c0 < total; c0 += gguf::kStageBytes, ++k) {
        gguf::Staging& s = f.ring[k % gguf::kStages];
        if (s.busy) {
            const cudaError_t e = cudaEventSynchronize(s.done);
            s.busy = false;
            if (e != cudaSuccess) {
                drain();
                return fail(NEXUS_GPU_ERROR_CUDA, "staging copy failed: %s", cudaGetErrorString(e));
            }
        }
        const uint64_t c1 = std::min<uint64_t>(total, c0 + gguf::kStageBytes);
        uint8_t* host = static_cast<uint8_t*>(s.host);
        // host threads copy slices of the piece out of the mapping
        const uint64_t slice = ((c1 - c0 + threads - 1) / threads + 4095) / 4096 * 4096;
        std::vector<std::thread> pool;
        try {
            for (uint64_t a = c0 + slice; a < c1; a += slice)
                pool.emplace_back(gguf::fill_range, std::cref(seg), a, std::min(c1, a + slice), host + (a - c0));
        } catch (const std::exception&) {  // no more threads: this one copies the rest
            const uint64_t a = c0 + slice * (pool.size() + 1);
            if (a < c1) gguf::fill_range(seg, a, c1, host + (a - c0));
        }
        gguf::fill_range(seg, c0, std::min(c1, c0 + slice), host);
        for (std::thread& th : pool) th.join();
        cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(d_dst) + c0, host, c1 - c0, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaEventRecord(s.done, st);
        if (e != cudaSuccess) {
            drain();
            cudaStreamSynchronize(st);
            return fail(NEXUS_GPU_ERROR_CUDA, "upload copy failed: %s", cudaGetErrorString(e));
        }
        s.busy = true;
    }
    drain();
    return NEXUS_GPU_SUCCESS;
}

}  // extern "C"
