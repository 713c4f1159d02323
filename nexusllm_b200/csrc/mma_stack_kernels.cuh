// mma_stack_kernels.cuh -- batched decode (16..64 tokens) of a whole GEMV
// stack on the tcgen05 tensor cores in ONE persistent launch, GGUF Q4_0.
//
// A decode step over M requests runs the step's GEMVs with M activation rows
// each (src/forward_pass.cpp:504-585 per request; the reference serves
// requests one after another, :633-667).  Launched one GEMM at a time, each
// pays a launch, an x-preparation kernel, a TMEM allocation and a pipeline
// fill and drain that cost more than its HBM time.  Here one cooperative
// launch (one CTA per SM) runs the task list:
//  * Each task is the single-GEMM kernel's work (gemm_q4_0_mma_kernel):
//    128-row tiles x 256-weight chunks split stream-K over the task's CTAs,
//    raw Q4_0 chunks and x tiles by TMA, the nibble decode into tensor memory
//    by sixteen warps, tcgen05.mma from tensor memory and shared memory, and
//    the fix-up of shared tiles by their last CTA.  The rings, barriers and
//    accumulator carry on from task to task; only the operands change.
//  * A "hop" is a task whose input differs from the previous task's (q, k, v
//    share one input, gate and up another): there every CTA waits at a grid
//    barrier for the previous tasks' outputs (and, with them, for every read
//    of the shared x buffer), CTA b < NB converts token b of the new input
//    into the fp16 B operand (x * 2^-e per token, K permuted to the decode's
//    order, as mma_xprep_kernel does), and a second grid barrier publishes
//    it.  Tasks that share an input run back to back with no barrier.
//  * Two copy warps: one streams the raw weight chunks through the barriers
//    (weights depend on nothing; a ring slot frees as soon as its chunk is
//    decoded), the other the x tiles, which wait for the second barrier and
//    then run as far ahead as their ring allows.  Each walks its tasks with
//    incremental tile and chunk counters, so a copy costs a few instructions
//    on a scheduler it shares with the decoding warps.
//  * The per-tile arrival counters of the fix-up only grow: a tile shared by
//    n CTAs is complete at the arrival whose previous count is n - 1 modulo n,
//    so no run resets them.  The grid barrier counter and the run counter
//    grow the same way.
// Every wait is bounded; an expired wait raises the stack's abort flag and
// the device status word, every CTA stops at its next wait, the producer
// drains its copies and the tensor memory is freed.  No cluster multicast.
#pragma once

#include "mma_kernels.cuh"

namespace nexus_gpu {

constexpr int kMmaMinTokens = 16;  // below this the CUDA-core stacks serve (north star: tensor cores for M >= 16)

// One GEMM of the stack.  The tensor map comes first so that an array of
// tasks keeps every map 64-byte aligned (sizeof is a multiple of 64).
struct __align__(64) MmaTask {
    CUtensorMap tmW;        // raw Q4_0 rows: {row bytes, N}, box {144, 128}
    float* y;               // output [M][N] fp32
    unsigned* arrivals;     // [tiles] fix-up arrival counters (only grow)
    int N, tiles;           // rows; 128-row tiles
    int tile0;              // the task's first tile in its group's tile sequence
};
static_assert(sizeof(MmaTask) % 64 == 0, "tensor maps in an MmaTask array must stay 64-byte aligned");

// A hop group: the tasks from one hop to the next, which share one input and
// run as ONE GEMM over their concatenated tiles (q, k and v; gate and up), so
// the stream-K split balances the whole group over the CTAs.
struct MmaGroup {
    const float* x;         // input [M][K] fp32: an earlier task's y, or null: the stack input
    long long total;        // tiles * n_chunks
    int first, count;       // member tasks [first, first + count), their tiles in this order
    int tiles, n_chunks, K;
    int G;                  // CTAs that share the group's chunks (stream-K), <= gridDim.x
    int hidx;               // hop index: the "done" grid barrier before the group when > 0
    int conv;               // 1: convert the input into its x slot, then the "published" barrier
    int pidx;               // index of the "published" barrier that covers the group's x
    int xslot;              // x slot: 0 the stack input (converted once a run), 1 an earlier task's y
};

struct MmaStackParams {
    const MmaTask* tasks;
    const MmaGroup* groups;
    int n_groups, n_pubs;    // groups (= hops: "done" barriers + 1); "published" barriers a run
    int M, NB;               // tokens; tokens rounded up to 16 (the UMMA N)
    int kmax;                // row stride of the fp16 x slots
    int b_stages;            // x-tile ring depth in chunks
    int raw_stages;          // raw-chunk ring depth (the rest of the ring budget after the x tiles)
    int raw_base;            // byte offset of the raw-chunk ring (after the x tiles, 1024-aligned)
    __half* xbuf;            // [2][NB][kmax] x slots in fp16 (B operand): the stack input, the current y input
    float* xscale;           // [2][kMaxTokens] 2^e per token of each slot
    float* partial;          // [gridDim.x][2][NB][128] partial sums of a CTA's first and last shared tile
    unsigned long long* bar_done;  // arrivals "done with the tasks before hop h" (hops 1..), all runs
    unsigned long long* bar_pub;   // arrivals "conversion p published", all runs
    unsigned long long* epoch;     // runs completed
    unsigned long long* fin;       // CTAs that left, all runs
    unsigned* abort_flag;          // sticky: an expired wait poisons the stack
    const float* x_in;             // the stack input [M][K] fp32 of this run (tasks with x == null)
};

// Grid barrier arrival (one thread per CTA, after its CTA-local barrier):
// release its CTA's writes at GPU scope.
__device__ __forceinline__ void grid_arrive(unsigned long long* ctr) {
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
}
// Wait until `ctr` reached `target` (acquire).  Bounded: false when the abort
// flag is up or after the wait limit (which raises it and the status bit).
__device__ __forceinline__ bool grid_wait(const unsigned long long* ctr, unsigned long long target,
                                          unsigned* abort_flag) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t k = 1;; ++k) {
        __nanosleep(64);
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(ctr) : "memory");
        if (v >= target) return true;
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
// Fetch-and-add with release and acquire semantics at GPU scope.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
// The 16 dequantizing warps' barrier (named barrier 1, 512 threads).
__device__ __forceinline__ void dequant_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kDequantThreads) : "memory"); }

// Two kinds of grid barrier, each on its own counter: hop h >= 1 has a "done"
// barrier (bar_done reaches (run*(H-1) + h) * G, H hops a run), and every
// conversion p a "published" barrier after it (bar_pub reaches (run*C + p + 1)
// * G, C conversions a run; a hop whose input is the stack input converts only
// the first time).  With one counter per kind a CTA's next arrival on a counter
// always follows its own wait for that counter's current target, so early
// arrivals of a CTA that has no work between two hops cannot complete a
// barrier for a CTA that has not arrived.
__device__ __forceinline__ unsigned long long done_target(unsigned long long run, int n_hops, int h, int G) {
    return (run * (unsigned long long)(n_hops - 1) + (unsigned long long)h) * (unsigned long long)G;
}
__device__ __forceinline__ unsigned long long pub_target(unsigned long long run, int n_pubs, int p, int G) {
    return (run * (unsigned long long)n_pubs + (unsigned long long)p + 1ull) * (unsigned long long)G;
}

// This CTA's chunks of a group: the linear range [lo, hi) of tiles x chunks
// (none when b is past the group's G CTAs).
struct MmaTaskRange {
    long long lo = 0, hi = 0;
    int nc = 1, t0 = 0, t1 = -1;
    bool any = false;
};
__device__ __forceinline__ MmaTaskRange mma_group_range(const MmaGroup& g, int b) {
    MmaTaskRange r;
    const int G = __ldg(&g.G);
    r.nc = __ldg(&g.n_chunks);
    if (b >= G) return r;
    const long long total = __ldg(&g.total);
    r.lo = sk_lo(total, G, b);
    r.hi = sk_lo(total, G, b + 1);
    r.any = r.hi > r.lo;
    if (r.any) {
        r.t0 = (int)(r.lo / r.nc);
        r.t1 = (int)((r.hi - 1) / r.nc);
    }
    return r;
}

// The member task of a group tile (members' tiles are consecutive).
__device__ __forceinline__ int mma_member(const MmaStackParams& P, const MmaGroup& g, int tile) {
    int m = __ldg(&g.first);
    const int end = m + __ldg(&g.count);
    while (m + 1 < end && __ldg(&P.tasks[m + 1].tile0) <= tile) ++m;
    return m;
}

// Token b of a hop's input (fp32 [M][K]; rows b >= M are zero) -> row b of
// x slot `slot` (the fp16 B operand): x * 2^-e with amax * 2^-e in [2^13,
// 2^14), K permuted inside every 32-weight block as q4_unit_decode orders the
// weights, and the slot's xscale[b] = 2^e (mma_xprep_kernel's rule).  Run by the 512 dequantizing
// threads of CTA b; s_red holds their 16 warps' maxima.
__device__ __forceinline__ void mma_convert_token(const MmaStackParams& P, const float* x, int K, int b, int slot,
                                                  int tid, volatile uint32_t* s_red) {
    const bool real = b < P.M;
    const float* row = x + (size_t)b * K;
    uint32_t m = 0;
    if (real)
        for (int e = 4 * tid; e < K; e += 4 * kDequantThreads) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(row + e));
            m = max(m, max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                           max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu)));
        }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((tid & 31) == 0) s_red[tid >> 5] = m;
    dequant_bar();
    uint32_t amax = 0;
#pragma unroll
    for (int w = 0; w < kDequantWarps; ++w) amax = max(amax, s_red[w]);
    int ex = 0;
    if (amax != 0 && amax < 0x7f800000u) ex = max((int)((amax >> 23) & 0xff) - 127 - 13, -110);
    const float down = ldexpf(1.0f, -ex);
    __half* out = P.xbuf + ((size_t)slot * P.NB + b) * P.kmax;
    for (int e = 4 * tid; e < K; e += 4 * kDequantThreads) {
        float v4[4] = {0.f, 0.f, 0.f, 0.f};
        if (real) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(row + e));
            v4[0] = v.x;
            v4[1] = v.y;
            v4[2] = v.z;
            v4[3] = v.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int s = e + k, blk = s >> 5;
            out[32 * blk + q4_perm_dst(s & 31, blk & 1)] = __float2half_rn(v4[k] * down);
        }
    }
    if (tid == 0) P.xscale[slot * kMaxTokens + b] = real ? ldexpf(1.0f, ex) : 0.0f;
}

// Warps of the stack kernel: the single GEMM's eighteen (raw-chunk copies,
// MMA, sixteen dequantizing warps), eight epilogue warps (warps 18..25,
// tensor-memory lane quarters 2, 3, 0, 1 twice; the two halves take alternate
// groups of 16 tokens) and the x-tile copy warp (26).  The epilogue warps read a finished accumulator, store y or the
// partial sums and run the fix-up, while the other warps go on with the next
// tile segment in the second accumulator.
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kEpiWarp0 = kMmaThreads / 32;
constexpr int kXWarp = kEpiWarp0 + kEpiWarps;  // the x-tile copies
constexpr int kMmaStackThreads = kMmaThreads + kEpiThreads + 32;
// Tensor memory: accumulator 0 in columns [0, 64), the A stages, accumulator
// 1 in the last 64 columns.
constexpr int kAcc1Col = kAccCols + kAStageCols * kAStages;
static_assert(kAcc1Col + kAccCols <= kTmemCols, "two accumulators and the A stages exceed tensor memory");
// Shared memory: one ring budget, split by the host between the x tiles (a
// few chunks: they come from L2) and the raw weight chunks (as many as fit:
// they come from HBM, about 3 us after their copies are issued under load,
// so the raw ring's depth sets the streaming rate); then the barriers, the
// TMEM address and flags, the hop decision, 16 warp maxima and the second
// accumulator's two barriers, and the 1024-byte alignment slack.
constexpr int kStackRingBytes = 224 * 1024;
constexpr int kStackRawMax = 12;
constexpr int kStackBarCount = 2 * kStackRawMax + 2 * kAStages + 2 * kMaxBStages + 5;
constexpr int kStackSmemBar = kStackRingBytes;
constexpr int kMmaStackSmemBytes = kStackSmemBar + 8 * kStackBarCount + 16 + 128 + 1024;

// The hop barrier of the dequantizing and the epilogue warps (named barrier 2).
__device__ __forceinline__ void hop_bar() {
    asm volatile("bar.sync 2, %0;" ::"n"(kDequantThreads + kEpiThreads) : "memory");
}

// 16 consecutive accumulator columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Every task segment (one tile's chunks of a task, for this CTA) takes the
// accumulator k % 2, k the CTA's segment count so far: the MMA warp waits for
// the epilogue's release of its use k - 2, the epilogue warps for its commit.
// Neither the dequantizing nor the epilogue warps ever leave the task walk
// early: both meet at the hop barrier of every hop, also after a failed wait
// (they then skip all work), so the named barrier always completes.
__global__ void __launch_bounds__(kMmaStackThreads, 1)
    gemm_q4_0_mma_stack_kernel(const __grid_constant__ CUtensorMap tmXin, const __grid_constant__ CUtensorMap tmX,
                               const MmaStackParams P) {
    extern __shared__ uint8_t mma_smem_raw[];
    const uint32_t sraw = smem_u32(mma_smem_raw);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;  // 1024-byte aligned: swizzle atoms
    uint8_t* smem = mma_smem_raw + (sbase - sraw);
    const uint32_t bar0 = sbase + kStackSmemBar;
    const uint32_t raw_full = bar0, raw_empty = raw_full + 8 * kStackRawMax;
    const uint32_t a_full = raw_empty + 8 * kStackRawMax, a_empty = a_full + 8 * kAStages;
    const uint32_t b_full = a_empty + 8 * kAStages, b_empty = b_full + 8 * kMaxBStages;
    const uint32_t acc_full0 = b_empty + 8 * kMaxBStages, acc_empty0 = acc_full0 + 8, drain = acc_empty0 + 8;
    const uint32_t part_done = drain + 8, decided = part_done + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kStackSmemBar + 8 * kStackBarCount);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
    volatile int* s_go = reinterpret_cast<volatile int*>(tmem_slot + 3);
    volatile uint32_t* s_red = tmem_slot + 4;  // [16]
    const uint32_t acc_full1 = smem_u32(tmem_slot + 20), acc_empty1 = acc_full1 + 8;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x, NB = P.NB;
    const uint32_t nbs = (uint32_t)P.b_stages, b_unit = (uint32_t)NB * 128u, b_stage = 4u * b_unit;
    const uint32_t nrs = (uint32_t)P.raw_stages, raw_ring = sbase + (uint32_t)P.raw_base;
    // this run's number (runs are stream-ordered; the epoch advances after every CTA left)
    const unsigned long long run = *reinterpret_cast<volatile unsigned long long*>(P.epoch);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStackRawMax; ++s) {
            mbar_init(raw_full + 8 * s, 1);
            mbar_init(raw_empty + 8 * s, kDequantWarps);
        }
        for (int s = 0; s < kAStages; ++s) {
            mbar_init(a_full + 8 * s, kDequantWarps);
            mbar_init(a_empty + 8 * s, 1);
        }
        for (int s = 0; s < kMaxBStages; ++s) {
            mbar_init(b_full + 8 * s, 1);
            mbar_init(b_empty + 8 * s, 1);
        }
        mbar_init(acc_full0, 1);
        mbar_init(acc_full1, 1);
        mbar_init(acc_empty0, kEpiWarps);
        mbar_init(acc_empty1, kEpiWarps);
        mbar_init(drain, 1);
        mbar_init(part_done, kEpiWarps);
        mbar_init(decided, 1);
        *abort = *reinterpret_cast<volatile unsigned*>(P.abort_flag) ? 1 : 0;  // a poisoned stack does nothing
        *last_flag = 0;
        *s_go = 1;
        fence_mbar_init();
    }
    const uint32_t tcols = kTmemCols;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = __shfl_sync(0xffffffffu, *reinterpret_cast<volatile uint32_t*>(tmem_slot), 0);

    if (warp == 0) {
        // ---------------- raw weight chunks: weights depend on nothing, so they stream through
        // the hops; a ring slot is free once the dequantizing warps have decoded its chunk
        const bool leader = elect_one();
        RingPos rp;
        uint32_t issued = 0;
        bool ok = *abort == 0;
        for (int g = 0; g < P.n_groups && ok; ++g) {
            const MmaGroup& Gr = P.groups[g];
            const MmaTaskRange tr = mma_group_range(Gr, b);
            if (!tr.any) continue;
            int m = mma_member(P, Gr, tr.t0);
            int local = tr.t0 - __ldg(&P.tasks[m].tile0), mt = __ldg(&P.tasks[m].tiles);
            int c = (int)(tr.lo - (long long)tr.t0 * tr.nc);
            for (long long L = tr.lo; L < tr.hi; ++L) {
                if (issued >= nrs && !warp_wait(raw_empty + 8 * rp.stage, rp.phase ^ 1u, abort)) {
                    ok = false;
                    break;
                }
                if (leader) {
                    mbar_arrive_expect_tx(raw_full + 8 * rp.stage, kRawChunkBytes);
                    tma_load_2d(raw_ring + rp.stage * kRawChunkBytes, &P.tasks[m].tmW, c * kRawRowBytes,
                                local * kMmaRows, raw_full + 8 * rp.stage);
                }
                __syncwarp();
                ++issued;
                rp.next(nrs);
                if (++c == tr.nc) {  // next tile, of the next member at the end of this one's
                    c = 0;
                    if (++local == mt && L + 1 < tr.hi) {
                        ++m;
                        local = 0;
                        mt = __ldg(&P.tasks[m].tiles);
                    }
                }
            }
        }
        if (leader && *abort)  // leave no copy in flight
            for (uint32_t k = 0; k < issued && k < nrs; ++k) {
                const uint32_t j = issued - 1 - k;
                mbar_wait_bounded(raw_full + 8 * (j % nrs), (j / nrs) & 1);
            }
        __syncwarp();
    } else if (warp == kXWarp) {
        // ---------------- x tiles: a hop's after its input is converted and published (bar_pub),
        // made visible to the tensor-copy proxy; then as far ahead as the x ring allows
        const bool leader = elect_one();
        RingPos bp;
        uint32_t issued = 0;
        int waited = -1;  // the last conversion this warp saw published
        bool ok = *abort == 0;
        for (int g = 0; g < P.n_groups && ok; ++g) {
            const MmaGroup& Gr = P.groups[g];
            const MmaTaskRange tr = mma_group_range(Gr, b);
            if (!tr.any) continue;
            const int pidx = __ldg(&Gr.pidx);
            const CUtensorMap* map = __ldg(&Gr.xslot) ? &tmX : &tmXin;
            if (pidx > waited) {
                bool go = true;
                if (leader) {
                    go = grid_wait(P.bar_pub, pub_target(run, P.n_pubs, pidx, gridDim.x), P.abort_flag);
                    if (go) fence_proxy_async_global();
                    else *abort = 1;
                }
                if (!__all_sync(0xffffffffu, leader ? go : true)) {
                    ok = false;
                    break;
                }
                waited = pidx;
            }
            int c = (int)(tr.lo - (long long)tr.t0 * tr.nc);
            for (long long L = tr.lo; L < tr.hi; ++L) {
                if (issued >= nbs && !warp_wait(b_empty + 8 * bp.stage, bp.phase ^ 1u, abort)) {
                    ok = false;
                    break;
                }
                if (leader) {
                    const uint32_t dst = sbase + bp.stage * b_stage, bar = b_full + 8 * bp.stage;
                    mbar_arrive_expect_tx(bar, b_stage);
#pragma unroll
                    for (int u = 0; u < kUnitsPerChunk; ++u)
                        tma_load_2d(dst + u * b_unit, map, c * kRawK + u * kUnitK, 0, bar);
                }
                __syncwarp();
                ++issued;
                bp.next(nbs);
                if (++c == tr.nc) c = 0;
            }
        }
        if (leader && *abort)
            for (uint32_t k = 0; k < issued && k < nbs; ++k) {
                const uint32_t j = issued - 1 - k;
                mbar_wait_bounded(b_full + 8 * (j % nbs), (j / nbs) & 1);
            }
        __syncwarp();
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA
        const uint32_t idesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(kMmaRows >> 4) << 24);
        const uint32_t b_unit16 = b_unit >> 4;
        const bool leader = elect_one();
        RingPos ap, bp;
        bool ok = *abort == 0;
        int k = 0;  // segments (accumulator uses) so far
        for (int g = 0; g < P.n_groups && ok; ++g) {
            const MmaTaskRange tr = mma_group_range(P.groups[g], b);
            if (!tr.any) continue;
            MmaRange R;
            R.lo = tr.lo;
            R.hi = tr.hi;
            R.t0 = tr.t0;
            R.t1 = tr.t1;
            for (int tile = R.t0; tile <= R.t1 && ok; ++tile, ++k) {
                const MmaSeg S = R.seg(tile, tr.nc);
                // accumulator k % 2: its use k - 2 read out by the epilogue warps
                if (k >= 2 && !warp_wait((k & 1) ? acc_empty1 : acc_empty0, ((k >> 1) - 1) & 1, abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_d + ((k & 1) ? (uint32_t)kAcc1Col : 0u);
                for (int c = S.c0; c < S.c1; ++c, ap.next(kAStages), bp.next(nbs)) {
                    if (!warp_wait(a_full + 8 * ap.stage, ap.phase, abort) ||
                        !warp_wait(b_full + 8 * bp.stage, bp.phase, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = tmem_d + kAccCols + kAStageCols * ap.stage;
                    const uint64_t b0 = umma_desc_sw128(sbase + bp.stage * b_stage);
                    if (leader) {
#pragma unroll
                        for (int u = 0; u < kUnitsPerChunk; ++u) {
                            const uint64_t bu = b0 + (uint64_t)(u * b_unit16);
                            umma_f16_tmem_a(d, a0 + 32 * u, bu, idesc, (c > S.c0 || u > 0) ? 1u : 0u);
                            umma_f16_tmem_a(d, a0 + 32 * u + 8, bu + 2, idesc, 1u);
                            umma_f16_tmem_a(d, a0 + 32 * u + 16, bu + 4, idesc, 1u);
                            umma_f16_tmem_a(d, a0 + 32 * u + 24, bu + 6, idesc, 1u);
                        }
                        umma_commit(a_empty + 8 * ap.stage);
                        umma_commit(b_empty + 8 * bp.stage);
                    }
                    __syncwarp();
                }
                if (ok && leader) umma_commit((k & 1) ? acc_full1 : acc_full0);
                __syncwarp();
            }
        }
        if (leader) {
            umma_commit(drain);
            mbar_wait_bounded(drain, 0);
        }
        __syncwarp();
    } else if (warp < kEpiWarp0) {
        // ------------------------------- hops (barriers, x conversion) and the dequantization
        const int dw = warp - 2, grp = dw >> 2, quarter = warp & 3;
        const int r = quarter * 32 + lane;  // tensor-memory lane = weight row of the tile
        const uint32_t lane_base = tmem_d + ((uint32_t)(quarter * 32) << 16);
        const bool leader = dw == 0 && lane == 0;
        const int tid = (int)threadIdx.x - 64;
        RingPos rp, ap;
        uint32_t chunks = 0;
        bool ok = *abort == 0;
        for (int g = 0; g < P.n_groups; ++g) {
            const MmaGroup& Gr = P.groups[g];
            {
                // the group's hop: every CTA finished the groups before it (which also ends
                // every read of the y-input x slot and its scales); for a new input CTA b < NB
                // converts token b, and the result is published at GPU scope for the other
                // CTAs' tensor copies
                const int hh = __ldg(&Gr.hidx);
                if (!ok) *abort = 1;
                hop_bar();  // with the epilogue warps, through every output before the hop
                if (leader) {
                    bool go = *abort == 0;
                    if (go && hh > 0) {
                        grid_arrive(P.bar_done);
                        go = grid_wait(P.bar_done, done_target(run, P.n_groups, hh, gridDim.x), P.abort_flag);
                    }
                    *s_go = (go && *abort == 0) ? 1 : 0;
                }
                dequant_bar();
                if (!*s_go) {  // one verdict for every dequantizing warp: no more work
                    *abort = 1;
                    ok = false;
                }
                if (ok && __ldg(&Gr.conv)) {
                    if (b < NB) {
                        const float* x =
                            reinterpret_cast<const float*>(__ldg(reinterpret_cast<const unsigned long long*>(&Gr.x)));
                        mma_convert_token(P, x != nullptr ? x : P.x_in, __ldg(&Gr.K), b, __ldg(&Gr.xslot), tid, s_red);
                    }
                    fence_proxy_async_global();
                    dequant_bar();
                    if (leader) grid_arrive(P.bar_pub);
                }
            }
            // a group's chunks are decoded only after its hop, so none of its MMAs -- and none of
            // its partial sums, which reuse the previous group's slots -- comes before every
            // CTA is through the "done" barrier, even where the x tiles need no publication
            const MmaTaskRange tr = mma_group_range(Gr, b);
            if (!tr.any || !ok) continue;  // after a failed wait: no work, but the hops' structure
            // this CTA's chunks of the task, in order (tile boundaries matter only to the MMA
            // and epilogue warps)
            for (long long L = tr.lo; L < tr.hi; ++L, ++chunks, rp.next(nrs), ap.next(kAStages)) {
                if (!warp_wait(raw_full + 8 * rp.stage, rp.phase, abort) ||
                    (chunks >= kAStages && !warp_wait(a_empty + 8 * ap.stage, ap.phase ^ 1u, abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t raw_row = raw_ring + rp.stage * kRawChunkBytes + (uint32_t)r * kRawRowBytes;
                const uint32_t ta = lane_base + kAccCols + kAStageCols * ap.stage;
                switch (grp) {
                    case 0: q4_unit_tmem_lean<0>(raw_row, ta); break;
                    case 1: q4_unit_tmem_lean<1>(raw_row, ta); break;
                    case 2: q4_unit_tmem_lean<2>(raw_row, ta); break;
                    default: q4_unit_tmem_lean<3>(raw_row, ta); break;
                }
                __syncwarp();  // the warp's shared loads of the raw chunk are consumed
                if (lane == 0) mbar_arrive(raw_empty + 8 * rp.stage);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full + 8 * ap.stage);
            }
        }
        if (!ok) *abort = 1;
    } else {
        // ----------------------------- epilogue: accumulator read-out, y, partial sums, fix-up
        const int quarter = warp & 3, half = (warp - kEpiWarp0) >> 2;
        const int r = quarter * 32 + lane;  // tensor-memory lane = weight row of the tile
        const uint32_t lane_base = tmem_d + ((uint32_t)(quarter * 32) << 16);
        const bool leader = warp == kEpiWarp0 && lane == 0;
        const int etid = (int)threadIdx.x - kMmaThreads;
        uint32_t n_part = 0;
        int k = 0;  // segments so far, as the MMA warp counts them
        bool ok = *abort == 0;
        for (int g = 0; g < P.n_groups; ++g) {
            const MmaGroup& Gr = P.groups[g];
            if (!ok) *abort = 1;
            hop_bar();  // every output before the hop is stored (and every xscale read done)
            const MmaTaskRange tr = mma_group_range(Gr, b);
            if (!tr.any) continue;
            MmaRange R;
            R.lo = tr.lo;
            R.hi = tr.hi;
            R.t0 = tr.t0;
            R.t1 = tr.t1;
            const int nc = tr.nc, G = __ldg(&Gr.G);
            const float* const xscale = P.xscale + __ldg(&Gr.xslot) * kMaxTokens;
            const long long total = __ldg(&Gr.total);
            for (int tile = R.t0; tile <= R.t1; ++tile, ++k) {
                if (!ok) continue;  // no work after a failed wait, but the walk goes on to every hop
                const MmaSeg S = R.seg(tile, nc);
                const MmaTask& T = P.tasks[mma_member(P, Gr, tile)];
                const int N = __ldg(&T.N), lt = tile - __ldg(&T.tile0);  // the member's rows, its tile
                float* const y = reinterpret_cast<float*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.y)));
                unsigned* const arrivals =
                    reinterpret_cast<unsigned*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.arrivals)));
                if (!warp_wait((k & 1) ? acc_full1 : acc_full0, (k >> 1) & 1, abort)) {
                    ok = false;
                    continue;
                }
                tc_fence_after();
                const uint32_t acc = lane_base + ((k & 1) ? (uint32_t)kAcc1Col : 0u);
                const int row = lt * kMmaRows + r;
                const bool whole = S.c0 == 0 && S.c1 == nc;
                // a tile shared with other CTAs: this CTA's partial sums go to its slot for its
                // first or its last tile of the group (groups are apart by a grid barrier)
                const int slot = 2 * b + (tile == R.t0 ? 0 : 1);
                float* const mine = P.partial + (size_t)slot * NB * kMmaRows;
                for (int j0 = 16 * half; j0 < NB; j0 += 32) {
                    float v[16];
                    tmem_ld16(acc + (uint32_t)j0, v);
                    tmem_wait_ld();
                    if (whole) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int tok = j0 + j;
                            if (tok < P.M && row < N) y[(size_t)tok * N + row] = v[j] * __ldcg(xscale + tok);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) mine[(size_t)(j0 + j) * kMmaRows + r] = v[j];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive((k & 1) ? acc_empty1 : acc_empty0);
                if (whole) continue;
                // the warps' partial stores reach the leader through part_done (CTA scope);
                // its GPU-scope release then orders all of them before its arrival
                __syncwarp();
                if (lane == 0) mbar_arrive(part_done);
                const int bf = sk_owner(total, G, (long long)tile * nc);
                const int bl = sk_owner(total, G, (long long)(tile + 1) * nc - 1);
                if (leader) {
                    bool last = false;
                    if (mma_wait(part_done, n_part & 1, abort)) {
                        // the counter only grows: each run adds one arrival per sharing CTA
                        const unsigned n = (unsigned)(bl - bf + 1);
                        // release this CTA's partial sums and, for the last CTA, acquire the others'
                        last = atom_add_acq_rel_gpu(arrivals + lt, 1u) % n == n - 1;
                    }
                    *last_flag = last ? 1 : 0;
                    mbar_arrive(decided);
                }
                if (!warp_wait(decided, n_part & 1, abort)) {
                    ok = false;
                    continue;
                }
                ++n_part;
                if (*last_flag && !*abort) {
                    // the last CTA to finish the tile adds every partial in CTA order (the
                    // leader's fence after its arrival acquired them; decided passes it on)
                    // two float4s a thread per pass (n4 is a multiple of 2 * 256), partials
                    // loaded two CTAs at a time: four loads in flight; sums in CTA order
                    const int n4 = NB * (kMmaRows / 4);
                    constexpr int kFixBatch = 2;
                    // CTA bb's slot: every CTA after the first one starts inside this tile (slot
                    // 0); the first one's slot is 1 when it started in an earlier tile
                    const int slot_f = 2 * bf + (sk_lo(total, G, bf) < (long long)tile * nc ? 1 : 0);
                    for (int f0 = etid; f0 < n4; f0 += 2 * kEpiThreads) {
                        const int f1 = f0 + kEpiThreads;
                        float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
                        for (int b0 = bf; b0 <= bl; b0 += kFixBatch) {
                            float4 p0[kFixBatch], p1[kFixBatch];
#pragma unroll
                            for (int i = 0; i < kFixBatch; ++i) {
                                const int bb = b0 + i;
                                if (bb <= bl) {
                                    const int sl = bb == bf ? slot_f : 2 * bb;
                                    const float4* src = reinterpret_cast<const float4*>(P.partial + (size_t)sl * NB * kMmaRows);
                                    p0[i] = __ldcg(src + f0);
                                    p1[i] = __ldcg(src + f1);
                                }
                            }
#pragma unroll
                            for (int i = 0; i < kFixBatch; ++i)
                                if (b0 + i <= bl) {
                                    s0.x += p0[i].x;
                                    s0.y += p0[i].y;
                                    s0.z += p0[i].z;
                                    s0.w += p0[i].w;
                                    s1.x += p1[i].x;
                                    s1.y += p1[i].y;
                                    s1.z += p1[i].z;
                                    s1.w += p1[i].w;
                                }
                        }
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int f = q ? f1 : f0, tok = f / (kMmaRows / 4);
                            if (tok >= P.M) continue;
                            const float4 a = q ? s1 : s0;
                            const float sc = __ldcg(xscale + tok), a4[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int rr = lt * kMmaRows + 4 * (f % (kMmaRows / 4)) + e;
                                if (rr < N) y[(size_t)tok * N + rr] = a4[e] * sc;
                            }
                        }
                    }
                }
            }
        }
        if (!ok) *abort = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(tcols) : "memory");
    }
    // a failed wait poisons the stack; the last CTA of the run to leave advances the epoch
    if (threadIdx.x == 0) {
        if (*abort) atomicExch(P.abort_flag, 1u);
        __threadfence();
        const unsigned long long left = atomicAdd(P.fin, 1ull) + 1;
        if (left == (run + 1) * (unsigned long long)gridDim.x) atomicExch(P.epoch, run + 1);
    }
}

}  // namespace nexus_gpu
