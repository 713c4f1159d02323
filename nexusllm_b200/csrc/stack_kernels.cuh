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
//    Rows are balanced over the CTAs.
//  * A task's x is either the stack input or the y of an earlier task.  A task
//    that a later task reads or waits for also stores each output row as a
//    tagged 32-bit word (the float with its lowest mantissa bit replaced by the
//    run's parity) with a single-copy-atomic relaxed store -- into every
//    rank's copy when sharded.  A reader that sees this run's parity in a word
//    has this run's value in it: the dependent CTA's staging loads are the
//    wait, and no fence, counter or flag sits between a row's store and its
//    use (at N > 1 this removes the system-scope fences from every data
//    dependency).  An `after` dependency waits for every row of its task the
//    same way.
//  * The consumer warps of a CTA step through the tasks together, one x group
//    (a task and the following tasks with the same input and plan) at a time:
//    the CTA reads the group's x once, quantizes it into shared memory itself
//    (quantize_x_pair, the same bits as xquant_kernel), and each warp copies
//    its slices into registers for every task of the group.
//  * Sharded over GPUs, a rank computes its row slice of every task and
//    stores each output row into every peer as well (plain stores).  The
//    run ends when every rank's rows of every task have landed everywhere:
//    each rank's last CTA to finish posts the rank's end to every rank after
//    a system-scope release, and one thread per rank waits for all ranks.
//  * The fused variant (template flag FX, nexus_gpu_stack_create_ex) adds the
//    decode layer's operations around the GEMVs: the group's x staging
//    applies a SwiGLU of two sources and the RMSNorm weights and sums x^2;
//    rows are scaled by 1/rms, a gate+up pair computes both rows from one
//    ring slot and stores silu(gate) * up, and a residual vector is added at
//    the store (a group head task's residual rows of the CTA are read into
//    shared memory with the staging).  Stacks without these run the plain
//    variant.
//  * All CTAs must be resident at once (they wait on one another): the host
//    launches the kernel cooperatively with one CTA per SM.  Every wait is
//    bounded; an expired wait raises a global abort flag that ends every CTA's
//    work and sets the device status word.
#pragma once

#include "gemv_kernels.cuh"

namespace nexus_gpu {

constexpr int kMaxWorld = 8;

struct StackTask {
    const uint8_t* W;
    uint64_t row_bytes, total_bytes;
    int N, K;
    int nwi, segments, seg_wi, wi_per_lane, stage_rows, stage_bytes;
    int rot_step;                        // stage_rows % (row groups): how the row-to-group deal advances per stage
    float* y;                            // this rank's full-length output (slice written at row_off)
    uint64_t y_off;                      // sharded: y's float offset in every rank's block
    uint32_t* tg;                        // a later task depends on this one: its tagged copy (full
                                         // length, this rank's), or null
    uint64_t tg_off;                     // the tagged copy's word offset in every rank's block
    int src;                             // x is task src's output (tagged copy), or -1: the stack input
    int after;                           // -1, or a task whose every row must be stored before this one starts
    int after_rows;                      // rows of task `after`
    int row_off;                         // first global row of this rank's slice (0 unless sharded)
    int reuse_x;                         // same input and plan as the previous task: keep its x
    // fusions around the GEMV (TransformerOps, include/transformer_ops.hpp:23-44,86-95;
    // the decode layer in src/forward_pass.cpp:504-562)
    int src2;                            // SwiGLU: x = silu(x) * (task src2's output), or -1
    const float* norm_w;                 // RMSNorm of x with these fp32 weights, or null
    float norm_eps;
    int res_input;                       // the residual is the stack input
    int res_src;                         // the residual is task res_src's output (tagged copy), or -1
    const uint8_t* W2;                   // gate+up pair: the up matrix (rows as W's), or null
    int half;                            // pair: byte offset of W2's rows in a ring slot
};

struct StackParams {
    const StackTask* tasks;
    const int2* cta_rows;                // [n_tasks][n_cta]: rows [x, y) of each task for each CTA (balanced)
    int n_tasks;
    int n_stages;
    int stage_slot;                      // bytes per ring slot (>= every task's stage_bytes)
    int x_smem;                          // bytes of the shared x staging buffer
    int slot_stride;                     // partial-sum floats per ring slot (>= R * S of every task)
    const float* x_in;                   // stack input, fp32, 16-byte aligned
    uint64_t wait_ns;                    // limit of every wait on other CTAs or ranks
    uint32_t wait_polls;                 // the same limit for tag polls (wait_ns / kTagPollNs)
    unsigned* abort_flag;                // sticky: an expired wait poisons the stack
    unsigned long long* epoch;           // runs completed on this rank
    unsigned long long* fin;             // CTAs of this rank that left, summed over all runs
    unsigned long long* end_done;        // sharded: ranks whose rows all landed here, all runs
    int world, rank;                     // row sharding over `world` GPUs (1, rank 0: unsharded)
    unsigned long long* local_end;       // sharded: CTAs of this rank that stored every row, all runs
    unsigned long long* peer_end[kMaxWorld];  // every rank's end_done (own included)
    uint8_t* peer_block[kMaxWorld];           // every rank's stack block (own included)
};

// Counters and tags are never reset: run e of a stack (e = 0, 1, ...) tags
// its rows e + 1, and a sharded run ends when end_done reaches (e + 1) * world.


__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p, bool sys) {
    unsigned long long v;
    if (sys) asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    else asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Acquire side of a relaxed poll that succeeded (relaxed read + fence = acquire).
__device__ __forceinline__ void fence_acquire(bool sys) {
    if (sys) asm volatile("fence.acq_rel.sys;" ::: "memory");
    else asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
// Add 1 to a counter, on this GPU or (sys) on a peer, after the caller's fence.
__device__ __forceinline__ void red_add_u64(unsigned long long* p, bool sys) {
    if (sys) asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(p) : "memory");
    else asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(p) : "memory");
}
// Wait (one thread) until *ctr >= target, then acquire.  Bounded: gives up
// when another CTA raised the abort flag or after limit_ns, raising it itself.
__device__ __noinline__ bool wait_count_bounded(const unsigned long long* ctr, unsigned long long target,
                                                unsigned* abort_flag, bool sys, uint64_t limit_ns) {
    if (ld_relaxed_u64(ctr, sys) >= target) {
        fence_acquire(sys);
        return true;
    }
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t k = 1;; ++k) {
        __nanosleep(32);
        if (ld_relaxed_u64(ctr, sys) >= target) {
            fence_acquire(sys);
            return true;
        }
        if ((k & 15u) == 0) {
            if (*reinterpret_cast<volatile unsigned*>(abort_flag)) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicOr(&g_device_status, kStatusWaitTimeout);
                atomicExch(abort_flag, 1u);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------- tagged rows
// A task that a later task depends on also stores each output row into its
// tagged copy: the float with its lowest mantissa bit replaced by the run's
// parity, (run + 1) & 1.  Every run rewrites every row, so a word holds either
// this run's or the previous run's row, and its parity bit tells which; each
// 32-bit word is single-copy atomic, so a reader that sees this run's parity
// has this run's value.  Readers clear the bit before use, so what a task
// consumes does not depend on the run (a relative change of at most 2^-23,
// far below the 16-bit fixed-point x that follows).  The buffers start at 0
// (parity 0), and run 0 writes parity 1.
__device__ __forceinline__ void st_tagged(uint32_t* p, float v, uint32_t par, bool sys) {
    const uint32_t w = (__float_as_uint(v) & ~1u) | par;
    if (sys) asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
    else asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
}
__device__ __forceinline__ uint4 ld_tagged4(const uint32_t* p, bool sys) {
    uint4 v;
    if (sys)
        asm volatile("ld.relaxed.sys.global.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_tagged1(const uint32_t* p, bool sys) {
    uint32_t v;
    if (sys) asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    else asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float untag(uint32_t w) { return __uint_as_float(w & ~1u); }
// 16 consecutive tagged words at p (16-byte aligned) into e; true when every
// word carries this run's parity.
__device__ __forceinline__ bool ld_tagged16(const uint32_t* p, uint32_t par, bool sys, float (&e)[16]) {
    uint32_t bad = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint4 v = ld_tagged4(p + 4 * q, sys);
        e[4 * q + 0] = untag(v.x);
        e[4 * q + 1] = untag(v.y);
        e[4 * q + 2] = untag(v.z);
        e[4 * q + 3] = untag(v.w);
        bad |= (v.x ^ par) | (v.y ^ par) | (v.z ^ par) | (v.w ^ par);
    }
    return (bad & 1u) == 0;
}
// The wait's expiry.
__device__ __forceinline__ void tag_wait_expired(unsigned* abort_flag) {
    atomicOr(&g_device_status, kStatusWaitTimeout);
    atomicExch(abort_flag, 1u);
}
// Read 16 words until every one carries this run's parity.  Bounded by an
// iteration count (P.wait_polls: the stack's wait limit over kTagPollNs, less
// than any poll takes -- an L2 round trip plus the short sleep -- so the loop
// holds one counter, not a clock, and gives up no earlier than the limit):
// false when another CTA raised the abort flag or the polls ran out (raising
// it and the status bit).  The sleep between polls is short: a poll is
// already an L2 round trip, and a longer sleep only delays seeing the rows
// (16 ns in place of 100 ns: 1.322 -> 1.280 ms on the 8B step whose layers
// depend on each other through their data).
constexpr uint32_t kTagPollNs = 100;
constexpr uint32_t kTagPollSleepNs = 16;
__device__ __forceinline__ bool wait_tagged16(const uint32_t* p, uint32_t par, bool sys, float (&e)[16],
                                              unsigned* abort_flag, uint32_t polls) {
    for (uint32_t k = 0; !ld_tagged16(p, par, sys, e); ++k) {
        __nanosleep(kTagPollSleepNs);
        if ((k & 7u) == 7u && *reinterpret_cast<volatile unsigned*>(abort_flag)) return false;
        if (k >= polls) {
            tag_wait_expired(abort_flag);
            return false;
        }
    }
    return true;
}
// Every row [0, n) of a tagged copy carries this run's parity; this thread
// checks rows 4*tid .. 4*tid+3, then every 4*kConsumers on (buffer 16-byte
// aligned; a partial last group of rows is read word by word).
__device__ __forceinline__ bool tagged_group_current(const uint32_t* p, int m, uint32_t par, bool sys) {
    if (m == 4) {
        const uint4 v = ld_tagged4(p, sys);
        return (((v.x ^ par) | (v.y ^ par) | (v.z ^ par) | (v.w ^ par)) & 1u) == 0;
    }
    uint32_t bad = 0;
    for (int k = 0; k < m; ++k) bad |= ld_tagged1(p + k, sys) ^ par;
    return (bad & 1u) == 0;
}
__device__ __forceinline__ bool wait_rows_tagged(const uint32_t* tg, int n, uint32_t par, bool sys, int tid,
                                                 unsigned* abort_flag, uint32_t polls) {
    for (int i = 4 * tid; i < n; i += 4 * kConsumers) {
        const int m = min(4, n - i);
        for (uint32_t k = 0; !tagged_group_current(tg + i, m, par, sys); ++k) {
            __nanosleep(kTagPollSleepNs);
            if ((k & 7u) == 7u && *reinterpret_cast<volatile unsigned*>(abort_flag)) return false;
            if (k >= polls) {
                tag_wait_expired(abort_flag);
                return false;
            }
        }
    }
    return true;
}

// mbarriers, a broadcast flag, the end-of-run post count, the RMSNorm partial
// sums, the per-warp epilogue descriptors, the per-warp output offsets and the
// group head task's residual rows of this CTA (fused variant)
constexpr int kResStageMax = 128;
static_assert(kResStageMax <= kConsumers, "a group head stages at most one residual row a thread");
constexpr int kStackBarBytes = 16 * kMaxStages + 32 + 4 * 16 + 16 * 16 + 16 * 16 + 4 * kResStageMax;
constexpr int kStackSmemHeader = ((kStackBarBytes + 127) / 128) * 128 + kSmemHeader - kBarBytes;

__device__ __forceinline__ uint32_t atom_add_acq_rel_shared(uint32_t addr, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ unsigned long long atom_add_acq_rel_gpu(unsigned long long* p) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], 1;" : "=l"(old) : "l"(p) : "memory");
    return old;
}
__device__ __forceinline__ void red_release_gpu(unsigned long long* p) {
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p) : "memory");
}

// Sharded end of run: count this CTA as done (called by its last consumer
// warp, after it acquired the other warps' posts, so their stores -- to this
// GPU and to peers -- are ordered before).  CTAs count at GPU scope on this
// rank's counter; the CTA that completes the rank's count makes ONE
// system-scope release and adds 1 on every rank's end counter.
__device__ __forceinline__ void release_end(const StackParams& P, unsigned long long run, int n_cta) {
    if (atom_add_acq_rel_gpu(P.local_end) + 1 != (run + 1) * (unsigned long long)n_cta) return;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll 1
    for (int p = 0; p < P.world; ++p) red_add_u64(P.peer_end[p], true);
}

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

// Shared staging layout of a task's quantized x.  The 64 bytes of block b's
// int16 X are four 16-byte chunks (elements 8q .. 8q+7 in chunk q); chunk q of
// every block sits in plane q, planes of nxbp = K/32 rounded up to 8 chunks:
// chunk (q, b) at 16 * (q * nxbp + xsw(b)), then the metadata plane, block b at
// 16 * (4 * nxbp + xsw(b)).  Lanes read blocks G apart (G = 1, 2, 4); the swizzle
// xsw(b) = b ^ ((b >> 3) & 7) maps any 8 such lanes to 8 distinct 16-byte bank
// groups, so the 128-bit loads of a quarter warp never conflict.
__device__ __forceinline__ uint32_t xsw(int b) { return (uint32_t)(b ^ ((b >> 3) & 7)); }
__host__ __device__ constexpr int x_stage_planes_len(int K) { return (K / 32 + 7) / 8 * 8; }

// quantize_x_block with two lanes per block: lane half hf (0 or 1) of the
// pair holds elements 16*hf .. 16*hf+15 in e.  Same element rule and sums as
// quantize_x_block, so X and the metadata are the same bits.  Stores
// block b into the staging layout at xs when `store`; every lane must call it.
__device__ __forceinline__ void quantize_x_pair(const float (&e)[16], int hf, bool store, uint32_t xs, int nxbp,
                                                int b) {
    uint32_t mbits = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) mbits = max(mbits, __float_as_uint(e[k]) & 0x7fffffffu);
    mbits = max(mbits, __shfl_xor_sync(0xffffffffu, mbits, 1));
    const float amax = __uint_as_float(mbits);
    const bool nz = mbits < 0x7f800000u && mbits != 0;
    const bool fast = amax >= kXQTiny;
    const float s = mbits >= 0x7f800000u ? amax : (nz ? __fdiv_rn(amax, kXQMax) : 0.0f);
    const float inv = nz && fast ? xq_inv(amax) : 0.0f;
    uint32_t v[8];  // int16 pairs of elements 16hf .. 16hf+15
    int sum = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const int x0 = !nz ? 0 : (fast ? xq_elem_fast(e[2 * w], inv) : xq_elem_tiny(e[2 * w], amax));
        const int x1 = !nz ? 0 : (fast ? xq_elem_fast(e[2 * w + 1], inv) : xq_elem_tiny(e[2 * w + 1], amax));
        v[w] = ((uint32_t)x0 & 0xffffu) | ((uint32_t)x1 << 16);
        sum += x0 + x1;
    }
    const int other = __shfl_xor_sync(0xffffffffu, sum, 1);
    if (store) {
        const uint32_t col = 16 * xsw(b), plane = 16u * (uint32_t)nxbp;
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(xs + (uint32_t)(2 * hf) * plane + col), "r"(v[0]),
                     "r"(v[1]), "r"(v[2]), "r"(v[3])
                     : "memory");
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(xs + (uint32_t)(2 * hf + 1) * plane + col),
                     "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                     : "memory");
        if (hf == 0)
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(xs + 4 * plane + col), "r"(__float_as_uint(s)),
                         "r"(sum), "r"(other), "r"(sum + other)
                         : "memory");
    }
}

// x slice of work item gj (block gj) from the staging layout at xs.
__device__ __forceinline__ void load_xint_smem(uint32_t xs, int nxbp, int gj, XInt& X) {
    const uint32_t col = 16 * xsw(gj), plane = 16u * (uint32_t)nxbp;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint4 v = lds128(xs + (uint32_t)q * plane + col);
        X.v[4 * q + 0] = v.x; X.v[4 * q + 1] = v.y; X.v[4 * q + 2] = v.z; X.v[4 * q + 3] = v.w;
    }
    const uint4 m = lds128(xs + 4 * plane + col);
    X.s = __uint_as_float(m.x);
    X.sa = (int)m.y;
    X.sb = (int)m.z;
    X.sx = (int)m.w;
}

// Task fields read at the point of use (lane 0, once per output row): volatile
// loads keep the compiler from holding them in registers across the hot loop.
__device__ __forceinline__ uint64_t ld_task_u64(const void* p) {
    uint64_t v;
    asm volatile("ld.global.nc.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ int ld_task_i32(const int* p) {
    int v;
    asm volatile("ld.global.nc.s32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t* ld_task_ptr(uint32_t* const* p) {
    return reinterpret_cast<uint32_t*>(ld_task_u64(p));
}

// The fused variant's per-warp epilogue descriptor in shared memory, one
// 16-byte word per consumer warp: x,y = the residual pointer already offset to
// this rank's first row (0 when the task has none), z = the RMSNorm scale of
// the group's input (1 without one), w = 1 for a gate+up pair.  Lane 0 writes
// it once per task (z once per group) and reads it at each row, so the row
// loop holds none of it in registers and makes no dependent loads of the task.
__device__ __forceinline__ float4 ld_ep(const volatile float4* p) {
    float4 v;
    asm volatile("ld.volatile.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(smem_u32(const_cast<const float4*>(p))));
    return v;
}

// The descriptor's residual address: the stack input's floats, or -- bit 0
// set -- a task's tagged copy (both already offset to this rank's first row),
// or kResInSmem: the CTA's rows staged in shared memory at the group head.
__device__ __forceinline__ uint64_t ep_residual(const float4 e) {
    return ((uint64_t)__float_as_uint(e.y) << 32) | __float_as_uint(e.x);
}

// Row r's residual, loaded when the row starts so that the L2 latency
// overlaps its dot product.  A task's residual word is read until it carries
// this run's parity (a residual's task finished before this task's own input
// in a decode layer, so the first read almost always does); bounded like every
// wait, the expiry raising the abort flag and the status bit.
__device__ __forceinline__ uint32_t residual_wait(const uint32_t* p, uint32_t par, bool sys, unsigned* abort_flag,
                                                  uint32_t polls) {
    uint32_t w = ld_tagged1(p, sys);
    for (uint32_t k = 0; ((w ^ par) & 1u) != 0; ++k) {
        __nanosleep(kTagPollSleepNs);
        w = ld_tagged1(p, sys);
        if ((k & 7u) == 7u && *reinterpret_cast<volatile unsigned*>(abort_flag)) break;
        if (k >= polls) {
            tag_wait_expired(abort_flag);
            break;
        }
    }
    return w;
}
constexpr uint32_t kResInSmem = 2;
// The residual of row r under the descriptor e: the CTA's rows staged in shared
// memory (e.x = kResInSmem, e.y = the first staged row), a task's tagged copy
// (bit 0 set) or the stack input's floats.
__device__ __forceinline__ float residual_of(const float4 e, int r, bool sys, uint32_t par, const StackParams& P,
                                             const volatile float* s_res) {
    if (__float_as_uint(e.x) == kResInSmem) return s_res[r - __float_as_int(e.y)];
    const uint64_t a = ep_residual(e);
    if (a & 1u) {
        const uint32_t* p = reinterpret_cast<const uint32_t*>(a - 1) + r;
        uint32_t w = ld_tagged1(p, sys);
        if (((w ^ par) & 1u) != 0) w = residual_wait(p, par, sys, P.abort_flag, P.wait_polls);
        return untag(w);
    }
    return __ldcg(reinterpret_cast<const float*>(a) + r);
}

// Write row r (of this rank's slice) of task T: this rank's output and --
// sharded -- every peer's copy (plain stores over NVLink).  v is the row's
// dot product; in the fused variant (FX) the epilogue of the descriptor ep
// is applied: y = v * scale + res, or silu(v * scale) * (u * scale) + res for
// a gate+up pair (u: the up row's dot product, res: residual_of, read here
// after the dot product so that nothing of it is live during the row).
// yl: this rank's output at its first row; yo: the float offset of that row
// in every rank's stack block (sharded stacks); to: the word offset of that
// row of the task's tagged copy in every rank's block (0 when no task depends
// on this one).
template <bool FX>
__device__ __forceinline__ void put_row(const StackParams& P, float* yl, uint64_t yo, uint64_t to, uint32_t par,
                                        int r, float v, const volatile float4* ep, const volatile float* s_res,
                                        float u) {
    if constexpr (FX) {
        const float4 e = ld_ep(ep);
        if (e.z != 1.0f) v = __fmul_rn(v, e.z);
        if (__float_as_int(e.w)) {  // gate+up pair: silu(gate) * up (transformer_ops.hpp:86-95)
            if (e.z != 1.0f) u = __fmul_rn(u, e.z);
            v = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
        }
        if (ep_residual(e)) v = __fadd_rn(v, residual_of(e, r, P.world > 1, par, P, s_res));
    }
    yl[r] = v;
    const bool sys = P.world > 1;
    if (to) st_tagged(reinterpret_cast<uint32_t*>(P.peer_block[P.rank]) + to + (uint64_t)r, v, par, sys);
    if (sys) {
#pragma unroll 1
        for (int p = 0; p < P.world; ++p) {
            if (p == P.rank) continue;
            reinterpret_cast<float*>(P.peer_block[p])[yo + (uint64_t)r] = v;
            if (to) st_tagged(reinterpret_cast<uint32_t*>(P.peer_block[p]) + to + (uint64_t)r, v, par, true);
        }
    }
}

// Stage a group's input x into shared memory: read it -- the stack input's
// floats (xv), or a task's tagged copy (xt), each thread waiting for this
// run's tags on its own words -- apply the fused SwiGLU (xt2) and RMSNorm
// weights (nw), quantize two lanes per 32-element block.  Returns this
// thread's sum of squares of x (for the RMSNorm scale); `ok` turns false when
// a wait gave up (every lane still runs the quantizer's shuffles).
template <bool FX>
__device__ __forceinline__ float stage_x(const float4* xv, const uint32_t* xt,
                                         const uint32_t* xt2, const float4* nw, int K, uint32_t xs, int tid,
                                         int lane, uint32_t par, const StackParams& P, bool& ok) {
    const int nxb = K / 32, nxbp = x_stage_planes_len(K), hf = lane & 1;
    const bool sys = P.world > 1;
    float ss = 0.0f;  // in a fixed order
    for (int base = 0; base < nxb; base += kConsumers / 2) {
        const int b = base + (tid >> 1);
        float e[16];
        // fused variant: the RMSNorm weights are loaded before the wait for x, so that
        // their L2 latency overlaps it instead of following it
        float4 wv[4];
        if (FX && nw != nullptr && b < nxb) {
#pragma unroll
            for (int q = 0; q < 4; ++q) wv[q] = __ldg(nw + 8 * b + 4 * hf + q);
        }
        if (b >= nxb) {
#pragma unroll
            for (int k = 0; k < 16; ++k) e[k] = 0.0f;
        } else if (FX && xt2 != nullptr && xt != nullptr) {
            // SwiGLU input: both tagged vectors read at once, then waited for if either is stale
            float u[16];
            const bool fresh = ld_tagged16(xt + 32 * b + 16 * hf, par, sys, e);
            const bool fresh2 = ld_tagged16(xt2 + 32 * b + 16 * hf, par, sys, u);
            if (!fresh) ok = wait_tagged16(xt + 32 * b + 16 * hf, par, sys, e, P.abort_flag, P.wait_polls) && ok;
            if (!fresh2) ok = wait_tagged16(xt2 + 32 * b + 16 * hf, par, sys, u, P.abort_flag, P.wait_polls) && ok;
            // silu(gate) * up (transformer_ops.hpp:86-95).  Every CTA computes the whole
            // vector, so with the __expf / __fdividef intrinsics (relative error ~1e-6, far
            // below the 16-bit fixed-point quantization that follows)
#pragma unroll
            for (int k = 0; k < 16; ++k) e[k] = __fmul_rn(__fdividef(e[k], __fadd_rn(1.0f, __expf(-e[k]))), u[k]);
        } else if (xt != nullptr) {
            ok = wait_tagged16(xt + 32 * b + 16 * hf, par, sys, e, P.abort_flag, P.wait_polls) && ok;
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = __ldcg(xv + 8 * b + 4 * hf + q);
                e[4 * q + 0] = v.x;
                e[4 * q + 1] = v.y;
                e[4 * q + 2] = v.z;
                e[4 * q + 3] = v.w;
            }
        }
        if constexpr (FX) {
            if (nw != nullptr && b < nxb) {  // RMSNorm: sum x^2 here, quantize x * w; 1/rms scales the rows
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 w = wv[q];
                    const float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        ss = fmaf(e[4 * q + k], e[4 * q + k], ss);
                        e[4 * q + k] = __fmul_rn(e[4 * q + k], ww[k]);
                    }
                }
            }
        }
        quantize_x_pair(e, hf, b < nxb, xs, nxbp, b);
    }
    return ss;
}

// The producer (lane 0 of the last warp): streams this CTA's rows of task
// after task through the ring of NS stage slots, never waiting for
// activations; a gate+up pair (FX) copies the same rows of both matrices into
// one slot.  It leaves only after its last copies landed, on every path.
// staged: null, or a shared counter of the x groups the consumers have
// staged.  With it, the producer issues at most kAheadOfStaging stages of an
// x group before the consumers staged that group's x: the stages it would
// otherwise issue as the previous group's last slots free would cross the
// memory system together with the staging's reads of the group's input and
// delay them.
constexpr int kAheadOfStaging = 1;
template <bool FX>
__device__ __forceinline__ void stack_producer(const StackParams& P, uint32_t full_bar, uint32_t empty_bar,
                                               uint32_t stage0, int c, int n_cta,
                                               const volatile int* staged = nullptr) {
    const int NS = P.n_stages;
    int it = 0, s = 0;
    int grp = -1, in_grp = 0;  // the x group of task t, and its stages issued so far
    uint32_t phase = 0;
    bool ok = true;
    auto give_up = [&]() {
        atomicOr(&g_device_status, kStatusWaitTimeout);
        atomicExch(P.abort_flag, 1u);
        ok = false;
    };
    for (int t = 0; t < P.n_tasks && ok; ++t) {
        const StackTask& T = P.tasks[t];
        const uint64_t rb = __ldg(&T.row_bytes), total = __ldg(&T.total_bytes);
        const uint8_t* W = reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.W)));
        const uint8_t* W2 =
            FX ? reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.W2))) : nullptr;
        const int R = __ldg(&T.stage_rows);
        const int2 rr = __ldg(P.cta_rows + (size_t)t * n_cta + c);
        const int row_begin = rr.x, row_end = rr.y;
        const uint64_t floor16 = total & ~(uint64_t)15;
        const uint64_t span = (uint64_t)R * rb, cta_end = (uint64_t)row_end * rb;
        if (!__ldg(&T.reuse_x)) {
            ++grp;
            in_grp = 0;
        }
        for (uint64_t start = (uint64_t)row_begin * rb; start < cta_end; ++it, ++in_grp) {
            if (staged != nullptr && in_grp >= kAheadOfStaging && *staged <= grp) {
                // wait (bounded) until the consumers staged this group's x
                const uint64_t t0 = globaltimer_ns();
                for (uint32_t k = 1; *staged <= grp; ++k) {
                    __nanosleep(64);
                    if ((k & 15u) == 0) {
                        if (*reinterpret_cast<volatile unsigned*>(P.abort_flag)) {
                            ok = false;
                            break;
                        }
                        if (globaltimer_ns() - t0 > kWaitLimitNs) {
                            give_up();
                            break;
                        }
                    }
                }
                if (!ok) break;
            }
            if (it >= NS && !mbar_try_wait(empty_bar + 8 * s, phase)) {
                // ring full: wait (sleeping in try_wait) for the slot to drain
                const uint64_t t0 = globaltimer_ns();
                for (uint32_t k = 1; !mbar_try_wait(empty_bar + 8 * s, phase); ++k) {
                    if ((k & 15u) == 0) {
                        if (*reinterpret_cast<volatile unsigned*>(P.abort_flag)) {
                            ok = false;
                            break;
                        }
                        if (globaltimer_ns() - t0 > kWaitLimitNs) {
                            give_up();
                            break;
                        }
                    }
                }
                if (!ok) break;
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
            if (FX && W2 != nullptr) {  // gate+up pair: the same rows of the up matrix, half a slot on
                const uint32_t dst2 = dst + (uint32_t)__ldg(&T.half);
                if (bend < end) {
                    for (uint64_t pos = (bend > a ? bend : a); pos < end; pos += 2)
                        sts16(dst2 + (uint32_t)(pos - a), *reinterpret_cast<const uint16_t*>(W2 + pos));
                    fence_proxy_async_smem();
                }
                mbar_arrive_expect_tx(full_bar + 8 * s, 2 * n);
                if (n) {
                    bulk_g2s(dst, W + a, n, full_bar + 8 * s);
                    bulk_g2s(dst2, W2 + a, n, full_bar + 8 * s);
                }
            } else {
                mbar_arrive_expect_tx(full_bar + 8 * s, n);
                if (n) bulk_g2s(dst, W + a, n, full_bar + 8 * s);
            }
            start = end;
            if (++s == NS) {
                s = 0;
                if (it >= NS) phase ^= 1;
            }
        }
    }
    // leave no copy in flight: the last stages issued complete on their own
    // (consumers that stopped after a failed wait no longer wait for them)
    for (int k = 0; k < NS && k < it; ++k) {
        const int j = it - 1 - k;
        mbar_wait_bounded(full_bar + 8 * (j % NS), (j / NS) & 1);
    }
}

// FX: the variant with the fused RMSNorm / SwiGLU / residual; stacks without
// them run the variant that has none of their code.
template <class F, int G, bool FX>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_stack_kernel(const StackParams P) {
    using XT = typename std::conditional<F::kIntX, XInt, XF16>::type;
    static_assert(F::kIntX, "the stack kernel serves the integer formats");
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full_bar = sbase;
    const uint32_t empty_bar = sbase + 8 * kMaxStages;
    volatile int* s_flag = reinterpret_cast<volatile int*>(smem + 16 * kMaxStages);
    const uint32_t tend = sbase + 16 * kMaxStages + 16;  // consumer warps done with every task
    float* s_norm = reinterpret_cast<float*>(smem + 16 * kMaxStages + 32);  // [16] RMSNorm partials
    volatile float4* s_ep = reinterpret_cast<volatile float4*>(s_norm + 16);  // [16] epilogue descriptors
    volatile ulonglong2* s_od = reinterpret_cast<volatile ulonglong2*>(s_norm + 16 + 4 * 16);  // [16] output offsets
    volatile float* s_res = reinterpret_cast<volatile float*>(s_od + 16);  // [kResStageMax] head task's residual rows
    constexpr int kHdr = ((kStackBarBytes + 127) / 128) * 128;
    float* slots = reinterpret_cast<float*>(smem + kHdr);
    const uint32_t stage0 = sbase + kStackSmemHeader + (uint32_t)P.x_smem;  // after the x staging buffer

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_cta = gridDim.x, c = blockIdx.x;
    const int NS = P.n_stages;
    const bool sys = P.world > 1;  // outputs shared with peer GPUs

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, kConsumerWarps);
        }
        s_flag[0] = 1;
        s_flag[1] = 0;  // x groups staged by the consumers (read by the producer)
        for (int k = 0; k < 4; ++k) reinterpret_cast<volatile uint32_t*>(smem + 16 * kMaxStages + 16)[k] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------- producer
        // (the fused variant's producer runs ahead freely: its group heads wait on their
        // norms and residuals too, and the gate measured slower there)
        if (lane == 0) stack_producer<FX>(P, full_bar, empty_bar, stage0, c, n_cta, FX ? nullptr : s_flag + 1);
        return;
    }

    // ----------------------------------------------------------- consumers
    // Consumer warps step through the tasks together, one x group at a time:
    // the CTA reads the group's x once, quantizes it into shared memory, and each warp
    // copies its slices into registers, which then serve every task of the
    // group.  Staging from L2 once per CTA (not once per warp) keeps x off the
    // L2 path the weight stream saturates; the x registers live only inside a
    // group, so the staging loads can all be in flight at once.
    const int tid = threadIdx.x;  // 0 .. kConsumers-1
    const uint32_t xs = sbase + kStackSmemHeader;  // x staging (xsw layout)
    // this run's number: its rows carry tag run + 1
    const uint32_t par = (uint32_t)(*reinterpret_cast<volatile unsigned long long*>(P.epoch) + 1) & 1u;
    bool alive = true, stop = false;
    int s = 0;
    uint32_t phase = 0;
    for (int t = 0; t < P.n_tasks && !stop;) {
        // ---- group head: wait for the input, stage it, load the x slices
        const StackTask& H = P.tasks[t];
        const int K = __ldg(&H.K), S = __ldg(&H.segments);
        const int NW = __ldg(&H.nwi), SW = __ldg(&H.seg_wi), J = __ldg(&H.wi_per_lane);
        bool ok = *reinterpret_cast<volatile unsigned*>(P.abort_flag) == 0;  // poisoned by an earlier run
        const int src = __ldg(&H.src), after = __ldg(&H.after);
        consumer_bar();  // every warp is done with the previous group's x staging
        const float4* nw =
            FX ? reinterpret_cast<const float4*>(__ldg(reinterpret_cast<const unsigned long long*>(&H.norm_w))) : nullptr;
        // fused variant: the head task's residual rows of this CTA (at most one a thread),
        // loaded before the staging so that their L2 latency overlaps it; checked and
        // written to shared memory after it
        int res_rows = 0;  // > 0: the head task's residual rows of this CTA are staged
        bool res_in = false;
        uint32_t res_w = 0;
        if constexpr (FX) {
            const int rs = __ldg(&H.res_src);
            res_in = __ldg(&H.res_input) != 0;
            const int2 hr = __ldg(P.cta_rows + (size_t)t * n_cta + c);
            if ((res_in || rs >= 0) && hr.y - hr.x <= kResStageMax) {
                res_rows = hr.y - hr.x;
                const int first = __ldg(&H.row_off) + hr.x;
                if (tid < res_rows)
                    res_w = res_in ? __float_as_uint(__ldcg(P.x_in + first + tid))
                                   : ld_tagged1(ld_task_ptr(&P.tasks[rs].tg) + first + tid, sys);
            }
        }
        {   // read x (L2; a task's output waits for this run's tags), apply the fusions,
            // quantize, two lanes per 32-element block
            const float4* xv = reinterpret_cast<const float4*>(P.x_in);
            const uint32_t* xt = src >= 0 ? ld_task_ptr(&P.tasks[src].tg) : nullptr;
            const int src2 = FX ? __ldg(&H.src2) : -1;
            const uint32_t* xt2 = src2 >= 0 ? ld_task_ptr(&P.tasks[src2].tg) : nullptr;
            float ss;  // RMSNorm: sum of squares of this thread's elements
            if (FX && (xt2 != nullptr || nw != nullptr)) ss = stage_x<FX>(xv, xt, xt2, nw, K, xs, tid, lane, par, P, ok);
            else ss = stage_x<false>(xv, xt, nullptr, nullptr, K, xs, tid, lane, par, P, ok);
            if (nw != nullptr) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                if (lane == 0) s_norm[warp] = ss;
            }
        }
        // ordering dependency: every row of `after` stored in this run, checked after the
        // staging (which never depends on it: the stack input is fixed for the run and a
        // task's output carries its own tags), so the staging's L2 reads overlap the wait
        // for the other CTAs' last rows; each thread checks its share of the rows (a
        // residual's rows are checked as they are read, residual_of)
        if (ok && after >= 0)
            ok = wait_rows_tagged(ld_task_ptr(&P.tasks[after].tg), __ldg(&H.after_rows), par, sys, tid, P.abort_flag,
                                  P.wait_polls);
        // fused variant: the head task's residual rows of this CTA into shared memory (the
        // residual's task finished before this group's input in a decode layer, so its word
        // loaded above almost always carries this run's parity), so the row stores read no
        // global memory
        if constexpr (FX) {
            if (tid < res_rows) {
                if (res_in) {
                    s_res[tid] = __uint_as_float(res_w);
                } else {
                    if (((res_w ^ par) & 1u) != 0) {  // not yet stored: wait for it (rare)
                        const int2 hr = __ldg(P.cta_rows + (size_t)t * n_cta + c);
                        res_w = residual_wait(ld_task_ptr(&P.tasks[__ldg(&H.res_src)].tg) + __ldg(&H.row_off) + hr.x + tid,
                                              par, sys, P.abort_flag, P.wait_polls);
                    }
                    s_res[tid] = untag(res_w);
                }
            }
        }
        if (consumer_bar_any(!ok)) {  // every consumer leaves together after a failed wait
            stop = true;
            break;
        }
        if (tid == 0) s_flag[1] = s_flag[1] + 1;  // this group's x is staged: the producer may run ahead
        // RMSNorm scale of this group's input: 1 / sqrt(sum x^2 / K + eps)
        // (transformer_ops.hpp:23-30), the warps' sums added in warp order
        float gscale = 1.0f;
        if (nw != nullptr) {
            float tot = 0.0f;
#pragma unroll 1
            for (int w = 0; w < kConsumerWarps; ++w) tot = __fadd_rn(tot, s_norm[w]);
            gscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), __ldg(&H.norm_eps))));
        }
        if (FX && lane == 0) s_ep[warp].z = gscale;  // read back by this lane at its row stores
        // this lane's work items (after the staging, so they hold no registers through it)
        const int sg = warp % S, grp = warp / S, n_grp = kConsumerWarps / S;
        int wi[kMaxJ];
        bool has[kMaxJ];
        lane_items<G>(lane, sg, SW, J, NW, wi, has);
        XT X[kMaxJ];
        {
            const int nxbp = x_stage_planes_len(K);
#pragma unroll
            for (int j = 0; j < kMaxJ; ++j)
                if (has[j]) load_xint_smem(xs, nxbp, wi[j], X[j]);
        }

        // ---- the group's tasks
        bool res_head = res_rows > 0;  // the next task is the head: its residual rows are staged
        for (;;) {
            const StackTask& T = P.tasks[t];
            // task constants, held in registers for the task's rows
            const int R = __ldg(&T.stage_rows), rot_step = __ldg(&T.rot_step);
            const uint32_t rbytes = (uint32_t)__ldg(&T.row_bytes);
            const uint32_t half = FX ? (uint32_t)__ldg(&T.half) : 0u;  // a gate+up pair when non-zero
            const int2 rr = __ldg(P.cta_rows + (size_t)t * n_cta + c);
            const int row_off = __ldg(&T.row_off);
            float* const yl = reinterpret_cast<float*>(__ldg(reinterpret_cast<const unsigned long long*>(&T.y))) + row_off;
            const uint64_t yo = __ldg(reinterpret_cast<const unsigned long long*>(&T.y_off)) + (uint64_t)row_off;
            const uint64_t tg_off = __ldg(reinterpret_cast<const unsigned long long*>(&T.tg_off));
            const uint64_t to = tg_off ? tg_off + (uint64_t)row_off : 0ull;
            if (FX && lane == 0) {  // this task's residual and pair flag into the warp's descriptor
                const int rs = ld_task_i32(&T.res_src);
                uint64_t rp = 0;
                if (ld_task_i32(&T.res_input)) rp = (uint64_t)(P.x_in + ld_task_i32(&T.row_off));
                else if (rs >= 0) rp = (uint64_t)(ld_task_ptr(&P.tasks[rs].tg) + ld_task_i32(&T.row_off)) | 1u;
                if (rp && res_head) {  // staged at the group head: e.y = the CTA's first row
                    s_ep[warp].x = __uint_as_float(kResInSmem);
                    s_ep[warp].y = __int_as_float(rr.x);
                } else {
                    s_ep[warp].x = __uint_as_float((uint32_t)rp);
                    s_ep[warp].y = __uint_as_float((uint32_t)(rp >> 32));
                }
                s_ep[warp].w = __int_as_float(half != 0u);
            }
            res_head = false;
            int rot = 0;  // (stage index * R) % n_grp: the group that takes a stage's first row
            for (int r0 = rr.x; r0 < rr.y; r0 += R) {
                const int nr = min(R, rr.y - r0);
                if (alive && !mbar_wait_bounded(full_bar + 8 * s, phase)) {
                    atomicExch(P.abort_flag, 1u);
                    alive = false;  // no more waits; the loop ends at the next group head
                }
                if (alive) {
                    // the stage's copy starts at the 16-byte boundary at or below row r0
                    const uint32_t base = stage0 + (uint32_t)(s * P.stage_slot) + (((uint32_t)r0 * rbytes) & 15u);
                    int rl = grp - rot;
                    if (rl < 0) rl += n_grp;
                    if (grp >= n_grp) rl = nr;  // the 15 - S*n_grp warps past the last row group idle
                    if (!FX || half == 0) {
                        // two rows of the stage at once: two independent dot products on the
                        // same x slices, and one reduction for both -- lanes 0-15 finish the
                        // first row, lanes 16-31 the second (each half's sum the same tree as
                        // the one-row reduction's, up to the order of commutative adds)
                        for (; rl + n_grp < nr; rl += 2 * n_grp) {
                            const uint32_t row = base + (uint32_t)(rl * rbytes);
                            const float a = row_partial<F, G>(row, wi, has, X);
                            const float b = row_partial<F, G>(row + (uint32_t)(n_grp * rbytes), wi, has, X);
                            float v = (lane < 16 ? a : b) + __shfl_xor_sync(0xffffffffu, lane < 16 ? b : a, 16);
#pragma unroll
                            for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                            const int rme = rl + (lane < 16 ? 0 : n_grp);
                            if ((lane & 15) == 0) {
                                if (S == 1)
                                    put_row<FX>(P, yl, yo, to, par, r0 + rme, v, s_ep + warp, s_res, 0.0f);
                                else slots[s * P.slot_stride + rme * S + sg] = v;
                            }
                        }
                    }
                    for (; rl < nr; rl += n_grp) {
                        const uint32_t row = base + (uint32_t)(rl * rbytes);
                        float acc = row_partial<F, G>(row, wi, has, X);
                        float up = 0.0f;  // a pair's up row: the same row of W2, half a slot on
                        if (FX && half) {
                            // both dot products, then one reduction for both as the two-row path
                            // does (lanes 0-15 the gate row's sum, 16-31 the up row's: the same
                            // trees as two one-row reductions)
                            const float u = row_partial<F, G>(row + half, wi, has, X);
                            float v = (lane < 16 ? acc : u) + __shfl_xor_sync(0xffffffffu, lane < 16 ? u : acc, 16);
#pragma unroll
                            for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                            acc = v;
                            up = __shfl_sync(0xffffffffu, v, 16);
                        } else {
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                        }
                        if (S == 1) {
                            if (lane == 0) put_row<FX>(P, yl, yo, to, par, r0 + rl, acc, s_ep + warp, s_res, up);
                        } else if (lane == 0) {  // this segment's partial (summed below)
                            float* sl = slots + s * P.slot_stride + rl * S * (half ? 2 : 1);
                            sl[sg] = acc;
                            if (FX && half) sl[S + sg] = up;
                        }
                    }
                }
                if (S > 1 && grp < n_grp) {
                    // The S warps of the row group meet once per stage (named barrier 2 + grp,
                    // which orders their partials in shared memory); then the lanes of the
                    // segment-0 warp finish the group's rows of the stage, one row per lane,
                    // summing the partials in segment order.  Every warp of the group reaches
                    // this barrier once per stage on every path, so a failed wait cannot
                    // leave another warp waiting here.
                    asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "r"(32 * S) : "memory");
                    if (alive && sg == 0) {
                        int first = grp - rot;
                        if (first < 0) first += n_grp;
                        for (int rl = first + n_grp * lane; rl < nr; rl += 32 * n_grp) {
                            const float* sl = slots + s * P.slot_stride + rl * S * (half ? 2 : 1);
                            float v = 0.f, u = 0.f;
                            for (int k = 0; k < S; ++k) v += sl[k];
                            if (FX && half)
                                for (int k = 0; k < S; ++k) u += sl[S + k];
                            put_row<FX>(P, yl, yo, to, par, r0 + rl, v, s_ep + warp, s_res, u);
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
    // A sharded run ends only when every rank's rows of every task have landed
    // here: each warp posts that it is done, the CTA's last warp counts the CTA
    // (release_end: the rank's last CTA tells every rank), and one thread of
    // CTA 0 waits for all ranks (the kernel, and so the stream, completes after it).
    // this run's number (the epoch advances only after every CTA of the rank left)
    const unsigned long long run = *reinterpret_cast<volatile unsigned long long*>(P.epoch);
    if (sys) {
        __syncwarp();
        if (lane == 0 && atom_add_acq_rel_shared(tend, 1u) + 1 == (uint32_t)kConsumerWarps &&
            *reinterpret_cast<volatile unsigned*>(P.abort_flag) == 0)
            release_end(P, run, n_cta);
        if (c == 0 && tid == 0 && !stop)
            wait_count_bounded(P.end_done, (run + 1) * (unsigned long long)P.world, P.abort_flag, true, P.wait_ns);
    }
    // the last CTA of this rank to leave advances the epoch for the next run
    consumer_bar();
    if (tid == 0) {
        __threadfence();
        const unsigned long long left = atomicAdd(P.fin, 1ull) + 1;
        if (left == (run + 1) * (unsigned long long)n_cta) atomicExch(P.epoch, run + 1);
    }
}

}  // namespace nexus_gpu
