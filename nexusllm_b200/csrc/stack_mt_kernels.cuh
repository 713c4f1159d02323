// stack_mt_kernels.cuh -- the GEMV stack for MT = 2..4 tokens per step
// (batched decode below the tensor-core range) for sm_100a.
//
// A decode step over M requests runs every GEMV of the step for M
// activation vectors (src/forward_pass.cpp:633-667 serves them one request
// at a time, reading every weight M times).  This kernel runs the stack's task
// list once for MT tokens, so every weight is read from HBM once per step:
//  * The producer, the ring, the row split over CTAs, the parity-tagged rows
//    that carry dependencies and the bounded waits are the plain stack's
//    (stack_kernels.cuh).  A task's output holds MT rows of values, token t at
//    y[t * N + r], and so does its tagged copy; the stack input holds MT
//    vectors, token t at x[t * K].
//  * A group head stages all MT tokens' x into shared memory, quantized to
//    the library's 16-bit fixed point (quantize_x_pair, the same rule as
//    every other path), token t in its own plane set.
//  * A lane holds, for its work items (one 32-weight item per lane when MT >
//    2, two when MT == 2 -- a block pair for Q4_0 and Q8_0), the x slices of
//    every token in registers.  It
//    decodes a weight item once and takes its exact int32 dp2a dot product
//    with each token's slice (Q4_0, Q8_0; the K-quant formats re-read the
//    item per token), scaled once per item and token as the reference scales
//    once per block.
//  * A row's MT partial sums are reduced across the warp with a transposed
//    butterfly (for MT = 4: 2 + 1 + 3 shuffles instead of 4 x 5): afterwards
//    the 8 (MT > 2) or 16 (MT == 2) lanes of a token hold that token's sum,
//    and one of them stores it.  K-split rows meet in shared slots as in the
//    plain stack, per (row, token).
// Unsharded only (world 1).
#pragma once

#include "stack_kernels.cuh"

namespace nexus_gpu {

constexpr int kMaxStackTokens = 4;

// Work items per lane for MT tokens: the x slices of MT tokens per item fill
// the registers the single-token kernel gives four items.
template <int MT>
struct MtPlan {
    static constexpr int kJ = MT == 2 ? 2 : 1;
};

// Item j of a row (shared address b of its block or super-block) against MT
// tokens' slices X[0..MT), added to acc[t].
template <class F, int MT>
__device__ __forceinline__ void dot_item_mt(uint32_t b, int wi, const XInt (&X)[MT], float (&acc)[MT]) {
    if constexpr (F::kBlockBytes == 18) {  // Q4_0: decode once
        uint32_t q[4];
        lds_words_2a<4>(b + 2, q);
        const float d = nexus_fp16(lds16(b));
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] += q4_0_block(d, q, X[t]);
    } else if constexpr (F::kBlockBytes == 34) {  // Q8_0: decode once
        uint32_t q[8];
        lds_words_2a<8>(b + 2, q);
        const float d = nexus_fp16(lds16(b));
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] += q8_0_block(d, q, X[t]);
    } else {
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] += dot_wi<F>(b - wi_offset<F>(wi), wi, X[t]);
    }
}

// Two consecutive Q4_0 / Q8_0 blocks (a lane's pair of items when MT == 2) at
// a 4-byte-aligned shared address against MT tokens' slices of each: one
// realignment for both blocks, and lanes 9 (Q4_0) or 17 (Q8_0) words apart,
// so their shared loads do not conflict.
template <class F, int MT>
__device__ __forceinline__ void dot_pair_mt(uint32_t p, const XInt (&X0)[MT], const XInt (&X1)[MT],
                                            float (&acc)[MT]) {
    if constexpr (F::kBlockBytes == 18) {
        uint32_t w[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = lds32(p + 4 * k);
        uint32_t q0[4], q1[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            q0[k] = __byte_perm(w[k], w[k + 1], 0x5432);  // bytes 2..17
            q1[k] = w[5 + k];                             // bytes 20..35
        }
        const float d0 = nexus_fp16(w[0] & 0xffffu), d1 = nexus_fp16_hi(w[4]);
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] += q4_0_block(d0, q0, X0[t]) + q4_0_block(d1, q1, X1[t]);
    } else {
        static_assert(F::kBlockBytes == 34, "block pairs serve Q4_0 and Q8_0");
        uint32_t w[17];
#pragma unroll
        for (int k = 0; k < 17; ++k) w[k] = lds32(p + 4 * k);
        uint32_t q0[8], q1[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            q0[k] = __byte_perm(w[k], w[k + 1], 0x5432);  // bytes 2..33
            q1[k] = w[9 + k];                             // bytes 36..67
        }
        const float d0 = nexus_fp16(w[0] & 0xffffu), d1 = nexus_fp16_hi(w[8]);
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] += q8_0_block(d0, q0, X0[t]) + q8_0_block(d1, q1, X1[t]);
    }
}

// The token whose full sum lane `lane` holds after reduce_tokens, and whether
// the lane is the one that stores it.
template <int MT>
__device__ __forceinline__ int token_of(int lane) {
    return MT == 2 ? (lane >> 4) & 1 : (lane >> 3) & 3;
}
template <int MT>
__device__ __forceinline__ bool token_lead(int lane) {
    return MT == 2 ? (lane & 15) == 0 : ((lane & 7) == 0 && token_of<MT>(lane) < MT);
}

// Sum each a[t] over the warp.  Transposed butterfly: the first exchange
// (lanes 16 apart) trades half of the values, the second (8 apart, MT > 2)
// half of the rest, then every lane adds its partners' single value.  Every
// lane of a token ends with the same sum, in a fixed order.
template <int MT>
__device__ __forceinline__ float reduce_tokens(const float (&a)[MT], int lane) {
    static_assert(MT >= 2 && MT <= 4, "2 to 4 tokens");
    float v;
    if constexpr (MT == 2) {
        const bool h = (lane & 16) != 0;
        v = (h ? a[1] : a[0]) + __shfl_xor_sync(0xffffffffu, h ? a[0] : a[1], 16);
    } else {
        const float a3 = MT == 4 ? a[MT - 1] : 0.0f;
        const bool h = (lane & 16) != 0;
        float k0 = (h ? a[2] : a[0]) + __shfl_xor_sync(0xffffffffu, h ? a[0] : a[2], 16);
        float k1 = (h ? a3 : a[1]) + __shfl_xor_sync(0xffffffffu, h ? a[1] : a3, 16);
        const bool g = (lane & 8) != 0;
        v = (g ? k1 : k0) + __shfl_xor_sync(0xffffffffu, g ? k0 : k1, 8);
    }
#pragma unroll
    for (int o = MT == 2 ? 8 : 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Row r of token t of a task: its output and, when a later task depends on
// it, its tagged copy (both hold MT rows of N values).
__device__ __forceinline__ void put_row_mt(float* y, uint32_t* tg, int N, uint32_t par, int t, int r, float v) {
    y[(size_t)t * N + r] = v;
    if (tg) st_tagged(tg + (size_t)t * N + r, v, par, false);
}

// G = 2: a lane's two items are a block pair (MT == 2, Q4_0 / Q8_0).
template <class F, int MT, int G>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_stack_mt_kernel(const StackParams P) {
    static_assert(F::kIntX, "the stack kernel serves the integer formats");
    constexpr int JM = MtPlan<MT>::kJ;
    static_assert(G == 1 || (G == 2 && JM == 2 && F::kGroup == 2), "block pairs: two tokens, Q4_0 or Q8_0");
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full_bar = sbase;
    const uint32_t empty_bar = sbase + 8 * kMaxStages;
    constexpr int kHdr = ((kStackBarBytes + 127) / 128) * 128;
    float* slots = reinterpret_cast<float*>(smem + kHdr);
    const uint32_t stage0 = sbase + kStackSmemHeader + (uint32_t)P.x_smem;  // after the x staging buffer

    // x groups staged by the consumers (read by the producer, stack_producer)
    volatile int* s_staged = reinterpret_cast<volatile int*>(smem + 16 * kMaxStages + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_cta = gridDim.x, c = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < P.n_stages; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, kConsumerWarps);
        }
        s_staged[0] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0) stack_producer<false>(P, full_bar, empty_bar, stage0, c, n_cta, s_staged);
        return;
    }

    // ----------------------------------------------------------- consumers
    const int tid = threadIdx.x;
    const uint32_t xs = sbase + kStackSmemHeader;  // x staging: MT plane sets (xsw layout)
    const uint32_t par = (uint32_t)(*reinterpret_cast<volatile unsigned long long*>(P.epoch) + 1) & 1u;
    bool alive = true;
    int s = 0;
    uint32_t phase = 0;
    for (int t = 0; t < P.n_tasks;) {
        // ---- group head: wait, stage every token's x, load the slices
        const StackTask& H = P.tasks[t];
        const int K = __ldg(&H.K), S = __ldg(&H.segments);
        const int NW = __ldg(&H.nwi), SW = __ldg(&H.seg_wi), J = __ldg(&H.wi_per_lane);
        bool ok = *reinterpret_cast<volatile unsigned*>(P.abort_flag) == 0;
        const int src = __ldg(&H.src), after = __ldg(&H.after);
        consumer_bar();  // every warp is done with the previous group's x staging
        const int nxb = K / 32, nxbp = x_stage_planes_len(K), hf = lane & 1;
        const uint32_t tok_bytes = 80u * (uint32_t)nxbp;  // one token's plane set
        {
            const uint32_t* xt = src >= 0 ? ld_task_ptr(&P.tasks[src].tg) : nullptr;
            const float4* xv = reinterpret_cast<const float4*>(P.x_in);
            for (int base = 0; base < MT * nxb; base += kConsumers / 2) {
                const int idx = base + (tid >> 1);
                const int tk = idx / nxb, b = idx - tk * nxb;
                float e[16];
                if (idx >= MT * nxb) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) e[k] = 0.0f;
                } else if (xt != nullptr) {
                    ok = wait_tagged16(xt + (size_t)tk * K + 32 * b + 16 * hf, par, false, e, P.abort_flag,
                                       P.wait_polls) && ok;
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 v = __ldcg(xv + (size_t)tk * (K / 4) + 8 * b + 4 * hf + q);
                        e[4 * q + 0] = v.x;
                        e[4 * q + 1] = v.y;
                        e[4 * q + 2] = v.z;
                        e[4 * q + 3] = v.w;
                    }
                }
                quantize_x_pair(e, hf, idx < MT * nxb, xs + (uint32_t)min(tk, MT - 1) * tok_bytes, nxbp, b);
            }
        }
        // the `after` rows after the staging, which never depends on them (as the
        // single-token kernel does): the staging's L2 reads overlap the wait
        if (ok && after >= 0)
            ok = wait_rows_tagged(ld_task_ptr(&P.tasks[after].tg), MT * __ldg(&H.after_rows), par, false, tid,
                                  P.abort_flag, P.wait_polls);
        if (consumer_bar_any(!ok)) break;  // every consumer leaves together after a failed wait
        if (tid == 0) s_staged[0] = s_staged[0] + 1;  // this group's x is staged: the producer may run ahead
        const int sg = warp % S, grp = warp / S, n_grp = kConsumerWarps / S;
        int wi4[kMaxJ];
        bool has4[kMaxJ];
        lane_items<G>(lane, sg, SW, J, NW, wi4, has4);
        int wi[JM];
        bool has[JM];
        XInt X[JM][MT];
#pragma unroll
        for (int j = 0; j < JM; ++j) {
            wi[j] = wi4[j];
            has[j] = has4[j];
            if (has[j]) {
#pragma unroll
                for (int k = 0; k < MT; ++k) load_xint_smem(xs + (uint32_t)k * tok_bytes, nxbp, wi[j], X[j][k]);
            }
        }

        // ---- the group's tasks
        for (;;) {
            const StackTask& T = P.tasks[t];
            const int R = __ldg(&T.stage_rows), rot_step = __ldg(&T.rot_step), N = __ldg(&T.N);
            const uint32_t rbytes = (uint32_t)__ldg(&T.row_bytes);
            const int2 rr = __ldg(P.cta_rows + (size_t)t * n_cta + c);
            float* const y = reinterpret_cast<float*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.y)));
            uint32_t* const tg = ld_task_ptr(&T.tg);
            int rot = 0;
            for (int r0 = rr.x; r0 < rr.y; r0 += R) {
                const int nr = min(R, rr.y - r0);
                if (alive && !mbar_wait_bounded(full_bar + 8 * s, phase)) {
                    atomicExch(P.abort_flag, 1u);
                    alive = false;
                }
                if (alive) {
                    const uint32_t base = stage0 + (uint32_t)(s * P.stage_slot) + (((uint32_t)r0 * rbytes) & 15u);
                    int rl = grp - rot;
                    if (rl < 0) rl += n_grp;
                    if (grp >= n_grp) rl = nr;
                    for (; rl < nr; rl += n_grp) {
                        const uint32_t row = base + (uint32_t)(rl * rbytes);
                        float acc[MT];
#pragma unroll
                        for (int k = 0; k < MT; ++k) acc[k] = 0.0f;
                        if constexpr (G == 2) {
                            if (has[0]) dot_pair_mt<F, MT>(row + wi_offset<F>(wi[0]), X[0], X[1], acc);
                        } else {
#pragma unroll
                            for (int j = 0; j < JM; ++j)
                                if (has[j]) dot_item_mt<F, MT>(row + wi_offset<F>(wi[j]), wi[j], X[j], acc);
                        }
                        const float v = reduce_tokens<MT>(acc, lane);
                        if (token_lead<MT>(lane)) {
                            const int tk = token_of<MT>(lane);
                            if (S == 1) put_row_mt(y, tg, N, par, tk, r0 + rl, v);
                            else slots[s * P.slot_stride + (rl * MT + tk) * S + sg] = v;
                        }
                    }
                }
                if (S > 1 && grp < n_grp) {
                    // the S warps of the row group meet once per stage (named barrier
                    // 2 + grp); the segment-0 warp's lanes then finish the group's
                    // (row, token) pairs, summing the partials in segment order
                    asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "r"(32 * S) : "memory");
                    if (alive && sg == 0) {
                        int first = grp - rot;
                        if (first < 0) first += n_grp;
                        for (int idx = lane;; idx += 32) {
                            const int rl = first + n_grp * (idx / MT), tk = idx % MT;
                            if (rl >= nr) break;
                            const float* sl = slots + s * P.slot_stride + (rl * MT + tk) * S;
                            float v = 0.f;
                            for (int k = 0; k < S; ++k) v += sl[k];
                            put_row_mt(y, tg, N, par, tk, r0 + rl, v);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_bar + 8 * s);
                if (++s == P.n_stages) {
                    s = 0;
                    phase ^= 1;
                }
                rot += rot_step;
                if (rot >= n_grp) rot -= n_grp;
            }
            if (++t >= P.n_tasks || !__ldg(&P.tasks[t].reuse_x)) break;
        }
    }
    // the last CTA to leave advances the epoch for the next run
    const unsigned long long run = *reinterpret_cast<volatile unsigned long long*>(P.epoch);
    consumer_bar();
    if (tid == 0) {
        __threadfence();
        const unsigned long long left = atomicAdd(P.fin, 1ull) + 1;
        if (left == (run + 1) * (unsigned long long)n_cta) atomicExch(P.epoch, run + 1);
    }
}

}  // namespace nexus_gpu
