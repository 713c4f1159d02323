// stack_kernels.cuh -- persistent multi-GEMV kernel (a decode step's GEMVs in
// one cooperative launch) for sm_100a.
//
// A decode step runs its GEMVs back to back (src/forward_pass.cpp:504-585:
// q, k, v, o, gate, up, down per layer, then the LM head).  Launched one by
// one, each GEMV pays a fixed pipeline fill and launch latency that is larger
// than the HBM time of the small matrices.  Here one launch runs a list of
// GEMV tasks:
//  * The producer warp of every CTA streams the CTA's rows of task after task
//    through the same shared-memory ring, without ever waiting for data:
//    weights do not depend on activations, so HBM keeps streaming while the
//    consumers wait for a task's input.
//  * Each task's consumer work is the single-GEMV kernel's (same plan, same
//    per-row arithmetic, so results are bit-identical to nexus_gpu_gemv).
//  * A task's x is either the stack input or the y of an earlier task.  A task
//    whose y feeds a later task splits its rows over the CTAs in whole 32-row
//    blocks, so each 32-element block of y is computed by one CTA: when a CTA's
//    warps have finished the task, the last of them quantizes the CTA's own
//    blocks of y into the 16-bit fixed-point form consumers load
//    (quantize_x_block) and only then bumps the task's global completion
//    counter.  One counter per task therefore means "y written and quantized";
//    a task starts when its source's counter and, optionally, another task's
//    counter (the ordering a real decode has between layers) reach the CTA
//    count.  The consumer warps of a CTA step through the tasks together:
//    one thread polls the grid counters, and the task's quantized x is staged
//    once per CTA in shared memory.  The stack input is quantized the same way
//    at kernel start.
//  * All CTAs must be resident at once (they wait on one another): the host
//    launches the kernel cooperatively with one CTA per SM.  Every wait is
//    bounded; an expired wait raises a global abort flag that ends every CTA's
//    work and sets the device status word.
#pragma once

#include "gemv_kernels.cuh"

namespace nexus_gpu {

struct StackTask {
    const uint8_t* W;
    uint64_t row_bytes, total_bytes;
    int N, K;
    int nwi, segments, seg_wi, wi_per_lane, stage_rows, stage_bytes;
    float* y;
    const uint8_t* x_limbs;  // quantized x of this task's source
    const int4* x_meta;
    int src;                 // counter index of the source: a task index, or n_tasks (the stack input)
    int after;               // -1, or a task that must complete before this one starts
    uint8_t* q_limbs;        // non-null when y is some later task's x: quantize y here, and
    int4* q_meta;            // split rows over CTAs in whole 32-row blocks
    int signal;              // some later task waits for this one: count CTAs when done
    int reuse_x;             // same input and plan as the previous task: keep its x, skip the wait
};

struct StackParams {
    const StackTask* tasks;
    int n_tasks;
    int n_stages;
    int stage_slot;          // bytes per ring slot (>= every task's stage_bytes)
    int x_smem;              // bytes of the shared x staging buffer (>= every task's K/32 * 80)
    int slot_stride;         // partial-sum floats per ring slot (>= R * S of every task)
    const float* x_in;       // stack input, fp32 [in_K]
    int in_K;
    uint8_t* in_limbs;
    int4* in_meta;
    unsigned* done;          // [(n_tasks + 1) * kCounterStride]: CTAs that finished (and quantized)
                             // each task; slot n_tasks counts the quantized stack input
    unsigned* abort_flag;
};

constexpr int kCounterStride = 32;  // one 128-byte line per counter

// Rows [rb, re) of an N-row task for CTA c of n_cta: balanced, or in whole
// 32-row blocks for tasks whose y is quantized by the CTAs that computed it.
__device__ __forceinline__ void cta_rows(int N, bool blocks32, int c, int n_cta, int& rb, int& re) {
    if (blocks32) {
        const int nb = N / 32;
        rb = 32 * (int)((int64_t)nb * c / n_cta);
        re = 32 * (int)((int64_t)nb * (c + 1) / n_cta);
    } else {
        rb = (int)((int64_t)N * c / n_cta);
        re = (int)((int64_t)N * (c + 1) / n_cta);
    }
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait (one thread) until *ctr >= target.  Bounded: gives up when another CTA
// raised the abort flag or after kWaitLimitNs, raising it itself.
__device__ __noinline__ bool wait_count_bounded(const unsigned* ctr, unsigned target, unsigned* abort_flag) {
    if (ld_acquire_u32(ctr) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t k = 1;; ++k) {
        __nanosleep(64);
        if (ld_acquire_u32(ctr) >= target) return true;
        if ((k & 15u) == 0) {
            if (*reinterpret_cast<volatile unsigned*>(abort_flag)) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&g_device_status, kStatusWaitTimeout);
                atomicExch(abort_flag, 1u);
                return false;
            }
        }
    }
}

constexpr int kStackBarBytes = 16 * kMaxStages + 16;  // mbarriers + a broadcast flag
constexpr int kStackSmemHeader = ((kStackBarBytes + 127) / 128) * 128 + kSmemHeader - kBarBytes;

// Named barrier of the consumer warps (the producer warp never joins it).
__device__ __forceinline__ void consumer_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}
// The same barrier, returning whether any consumer thread passed `v` true.
__device__ __forceinline__ bool consumer_bar_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kConsumers)
        : "memory");
    return r != 0;
}

// x slice of work item gj from the shared staging buffer (limbs at xl, meta at xm).
__device__ __forceinline__ void load_xint_smem(uint32_t xl, uint32_t xm, int gj, XInt& X) {
    const uint32_t a = xl + (uint32_t)gj * kXQLimbBytes;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const uint4 v = lds128(a + 16 * q);
        X.h[4 * q + 0] = v.x; X.h[4 * q + 1] = v.y; X.h[4 * q + 2] = v.z; X.h[4 * q + 3] = v.w;
        const uint4 u = lds128(a + 32 + 16 * q);
        X.l[4 * q + 0] = u.x; X.l[4 * q + 1] = u.y; X.l[4 * q + 2] = u.z; X.l[4 * q + 3] = u.w;
    }
    const uint4 m = lds128(xm + (uint32_t)gj * kXQMetaBytes);
    X.s = __uint_as_float(m.x);
    X.sa = (int)m.y;
    X.sb = (int)m.z;
    X.sx = (int)m.w;
}

template <class F, int G>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_stack_kernel(const StackParams P) {
    using XT = typename std::conditional<F::kIntX, XInt, XF16>::type;
    static_assert(F::kIntX, "the stack kernel serves the integer formats");
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full_bar = sbase;
    const uint32_t empty_bar = sbase + 8 * kMaxStages;
    volatile int* s_flag = reinterpret_cast<volatile int*>(smem + 16 * kMaxStages);  // warp-0 verdicts
    constexpr int kHdr = ((kStackBarBytes + 127) / 128) * 128;
    float* slots = reinterpret_cast<float*>(smem + kHdr);
    int* counters = reinterpret_cast<int*>(smem + kHdr + kMaxSlots * 4);  // [kMaxStages][kMaxStageRows]
    const uint32_t stage0 = sbase + kStackSmemHeader + (uint32_t)P.x_smem;  // after the x staging buffer

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_cta = gridDim.x, c = blockIdx.x;
    const int NS = P.n_stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, kConsumerWarps);
        }
        s_flag[0] = 1;
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < kMaxStages * kMaxStageRows; i += blockDim.x) counters[i] = 0;
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------- producer
        if (lane != 0) return;
        int it = 0, s = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = 0; t < P.n_tasks && ok; ++t) {
            const StackTask& T = P.tasks[t];
            const uint64_t rb = __ldg(&T.row_bytes), total = __ldg(&T.total_bytes);
            const uint8_t* W = reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.W)));
            const int N = __ldg(&T.N), R = __ldg(&T.stage_rows);
            int row_begin, row_end;
            cta_rows(N, __ldg(reinterpret_cast<const unsigned long long*>(&T.q_limbs)) != 0ull, c, n_cta, row_begin,
                     row_end);
            const uint64_t floor16 = total & ~(uint64_t)15;
            const uint64_t span = (uint64_t)R * rb, cta_end = (uint64_t)row_end * rb;
            for (uint64_t start = (uint64_t)row_begin * rb; start < cta_end; ++it) {
                if (it >= NS && !mbar_wait_bounded(empty_bar + 8 * s, phase)) {
                    ok = false;
                    break;
                }
                const uint64_t end = min(start + span, cta_end);
                const uint64_t a = start & ~(uint64_t)15;
                const uint64_t bend = min((end + 15) & ~(uint64_t)15, floor16);
                const uint32_t dst = stage0 + (uint32_t)(s * P.stage_slot);
                if (bend < end) {
                    for (uint64_t pos = (bend > a ? bend : a); pos < end; pos += 2)
                        sts16(dst + (uint32_t)(pos - a), *reinterpret_cast<const uint16_t*>(W + pos));
                    fence_proxy_async_smem();
                }
                const uint32_t n = bend > a ? (uint32_t)(bend - a) : 0u;
                mbar_arrive_expect_tx(full_bar + 8 * s, n);
                if (n) bulk_g2s(dst, W + a, n, full_bar + 8 * s);
                start = end;
                if (++s == NS) {
                    s = 0;
                    if (it >= NS) phase ^= 1;
                }
            }
        }
        if (!ok) {  // leave no copy in flight
            for (int k = 0; k < NS && k < it; ++k) {
                const int j = it - 1 - k;
                mbar_wait_bounded(full_bar + 8 * (j % NS), (j / NS) & 1);
            }
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    // Consumer warps step through the tasks together: at each task start the
    // CTA loads the task's quantized x once into shared memory (every warp
    // reading it from L2 on its own multiplied the L2 traffic by the warp count
    // and stalled behind the weight stream), then each warp copies its slices
    // into registers.  Warp 0 polls the grid counters for the CTA.
    const int tid = threadIdx.x;  // 0 .. kConsumers-1
    const uint32_t xs = sbase + kStackSmemHeader;  // x staging: limbs [nxb][64] then meta [nxb][16]
    bool alive = true;
    // this CTA's 32-element blocks of the stack input
    {
        int b0, b1;
        cta_rows(P.in_K, true, c, n_cta, b0, b1);
        for (int b = b0 / 32 + warp; b < b1 / 32; b += kConsumerWarps)
            quantize_x_block(__ldcg(P.x_in + 32 * b + lane), lane, P.in_limbs + (size_t)b * kXQLimbBytes,
                             P.in_meta + b);
        __threadfence();
    }
    consumer_bar();
    if (tid == 0) atomicAdd(&P.done[P.n_tasks * kCounterStride], 1u);

    int s = 0;
    uint32_t phase = 0;
    XT X[kMaxJ];
    for (int t = 0; t < P.n_tasks; ++t) {
        const StackTask& T = P.tasks[t];
        const int N = __ldg(&T.N), K = __ldg(&T.K), R = __ldg(&T.stage_rows), S = __ldg(&T.segments);
        const int NW = __ldg(&T.nwi), SW = __ldg(&T.seg_wi), J = __ldg(&T.wi_per_lane);
        const uint64_t rbytes = __ldg(&T.row_bytes);
        float* y = reinterpret_cast<float*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.y)));
        uint8_t* ql = reinterpret_cast<uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.q_limbs)));
        const bool reuse = __ldg(&T.reuse_x) != 0;
        const int sg = warp % S, grp = warp / S, n_grp = kConsumerWarps / S;
        int wi[kMaxJ];
        bool has[kMaxJ];
        lane_items<G>(lane, sg, SW, J, NW, wi, has);
        if (!reuse) {
        // the task's input must be written and quantized, and its ordering dependency done
        int ok = 1;
        if (tid == 0) {
            const int after = __ldg(&T.after);
            ok = wait_count_bounded(&P.done[__ldg(&T.src) * kCounterStride], (unsigned)n_cta, P.abort_flag);
            if (ok && after >= 0) ok = wait_count_bounded(&P.done[after * kCounterStride], (unsigned)n_cta, P.abort_flag);
            s_flag[0] = ok;
        }
        consumer_bar();  // also: every warp is done with the previous task's x staging
        if (!s_flag[0]) break;
        __threadfence();
        {   // stage x: limbs and meta, 16 bytes per thread per step
            const int nxb = K / 32;
            const int4* gl = reinterpret_cast<const int4*>(
                __ldg(reinterpret_cast<const unsigned long long*>(&T.x_limbs)));
            const int4* gm = reinterpret_cast<const int4*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.x_meta)));
            for (int i = tid; i < nxb * (kXQLimbBytes / 16); i += kConsumers) {
                const int4 v = __ldcg(gl + i);
                asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(xs + 16 * i), "r"(v.x), "r"(v.y),
                             "r"(v.z), "r"(v.w)
                             : "memory");
            }
            const uint32_t xm = xs + (uint32_t)nxb * kXQLimbBytes;
            for (int i = tid; i < nxb; i += kConsumers) {
                const int4 v = __ldcg(gm + i);
                asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(xm + 16 * i), "r"(v.x), "r"(v.y),
                             "r"(v.z), "r"(v.w)
                             : "memory");
            }
        }
        consumer_bar();
        {
            const uint32_t xm = xs + (uint32_t)(K / 32) * kXQLimbBytes;
#pragma unroll
            for (int j = 0; j < kMaxJ; ++j)
                if (has[j]) load_xint_smem(xs, xm, wi[j], X[j]);
        }
        }  // !reuse

        int row_begin, row_end;
        cta_rows(N, ql != nullptr, c, n_cta, row_begin, row_end);
        const int n_st = (row_end - row_begin + R - 1) / R;
        int rot = 0;
        for (int i = 0; i < n_st; ++i) {
            const int r0 = row_begin + i * R;
            const int nr = min(R, row_end - r0);
            if (alive && !mbar_wait_bounded(full_bar + 8 * s, phase)) {
                atomicExch(P.abort_flag, 1u);
                alive = false;  // no more waits; the loop ends at the next reducing barrier
            }
            if (alive) {
                const uint32_t base =
                    stage0 + (uint32_t)(s * P.stage_slot) + (uint32_t)(((uint64_t)r0 * rbytes) & 15);
                int rl = grp - rot;
                if (rl < 0) rl += n_grp;
                for (; rl < nr; rl += n_grp) {
                    const uint32_t row = base + (uint32_t)(rl * rbytes);
                    float acc = row_partial<F, G>(row, wi, has, X);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                    if (S == 1) {
                        if (lane == 0) y[r0 + rl] = acc;
                    } else if (lane == 0) {
                        float* sl = slots + s * P.slot_stride + rl * S;
                        sl[sg] = acc;
                        __threadfence_block();
                        const int prev = atomicAdd(&counters[s * kMaxStageRows + rl], 1);
                        if (prev == S - 1) {  // last segment of this row: sum in segment order
                            __threadfence_block();
                            float v = 0.f;
                            for (int k = 0; k < S; ++k) v += *(volatile float*)(sl + k);
                            y[r0 + rl] = v;
                            counters[s * kMaxStageRows + rl] = 0;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar + 8 * s);
            if (++s == P.n_stages) {
                s = 0;
                phase ^= 1;
            }
            rot += R % n_grp;
            if (rot >= n_grp) rot -= n_grp;
        }
        // this CTA's rows of task t are written; when a later task waits for
        // it, warp 0 quantizes the CTA's blocks of y (when y feeds a later
        // task) and counts the CTA
        if (!__ldg(&T.signal)) continue;  // a failed wait ends the loop at the next reducing barrier
        __threadfence();
        if (consumer_bar_any(!alive)) break;  // every consumer leaves together after a failed wait
        if (warp == 0) {
            if (ql != nullptr) {
                int4* qm = reinterpret_cast<int4*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.q_meta)));
                for (int b = row_begin / 32; b < row_end / 32; ++b)
                    quantize_x_block(__ldcg(y + 32 * b + lane), lane, ql + (size_t)b * kXQLimbBytes, qm + b);
                __threadfence();
                __syncwarp();
            }
            if (lane == 0) atomicAdd(&P.done[t * kCounterStride], 1u);
        }
    }
}

}  // namespace nexus_gpu
