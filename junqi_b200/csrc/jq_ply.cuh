// jq_ply.cuh -- one ply of one env by one warp (the rules kernel's unit of
// work), and the rules kernel itself.
#pragma once
#include "jq_rules.cuh"
#include "jq_trace.cuh"

namespace jq {

constexpr int RULE_WARPS = 8;
constexpr int RULE_THREADS = RULE_WARPS * 32;

enum : int { DO_STEP = 1, DO_RESET = 2, DO_LEGAL = 4, RESET_ALL = 8, DO_BELIEF_INIT = 16 };

struct RuleSmem {
    TopoCore topo;
    WEnv w[RULE_WARPS];
    int applied;  // plies applied by this CTA (statistics)
};

// four CTAs per SM (one wave at 4,096 envs): 228 KB of shared memory, 1 KB reserved per CTA
static_assert(sizeof(RuleSmem) + 1024 <= 228 * 1024 / 4, "rules kernel shared memory exceeds four CTAs per SM");

struct RuleArgs {
    jq_batch b;
    const int32_t *acts;
    int mode;
    jq_step_out out;
    uint64_t seed, ply;
    const int8_t *pool;
    int pool_size;
    int32_t *counts, *ids;
    int cap;
    uint8_t *mask;
    int64_t *stats;
    const int8_t *seats;
    const int32_t *rows;  // explicit pool rows for DO_RESET (NULL: hashed index)
    int flags;
};

__device__ __forceinline__ int pool_index(uint64_t seed, uint64_t ply, int e, int P) {
    return (int)(hash3(seed, ply, (uint64_t)e) % (uint64_t)P);
}

// The rules kernel's board tables into shared memory, 16 bytes per thread
// and step.
static_assert(sizeof(TopoCore) % 16 == 0, "TopoCore copies in 16-byte words");
__device__ __forceinline__ void stage_topo(TopoCore &dst_t, int tid, int nthreads) {
    const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const TopoCore *>(&g_topo));
    uint4 *dst = reinterpret_cast<uint4 *>(&dst_t);
    for (int k = tid; k < (int)(sizeof(TopoCore) / 16); k += nthreads) dst[k] = src[k];
}

// The parts of a ply `a.flags` selects, for env e, by one warp.  Returns (on
// every lane) whether a step was applied.
__device__ bool warp_ply_env(const RuleArgs &a, const TopoCore &T, WEnv &w, int e, int lane) {
    const jq_batch &b = a.b;
    bool applied = false;
    const bool traced = threadIdx.x == 0 && e < RULE_WARPS * (int)gridDim.x;  // warp 0's first env
    warp_load(b, T, w, e, lane, (a.flags & DO_STEP) != 0);
    if (traced) JQ_TRACE_AT(1, TR_LOADED);
    if (a.flags & DO_BELIEF_INIT) {
        warp_belief_init(b, T, w, e, lane, a.mode);
        b.hist_src[(size_t)e * HIST + lane] = -1;
        b.hist_dst[(size_t)e * HIST + lane] = -1;
        if (lane == 0) b.hist_count[e] = 0;
        __syncwarp();
    }
    if (a.flags & DO_STEP) applied = warp_step(b, T, w, e, lane, a.acts[e], a.mode, a.out, a.stats, traced);
    if (traced) JQ_TRACE_AT(1, TR_STEPPED);
    if ((a.flags & DO_RESET) && a.pool && a.pool_size > 0) {
        int row = -1;
        if (a.rows) {
            const int r = a.rows[e];
            row = (r >= 0 && r < a.pool_size) ? r : -1;
        } else if ((a.flags & RESET_ALL) || b.terminated[e]) {
            row = pool_index(a.seed, a.ply, e, a.pool_size);
        }
        if (row >= 0) warp_reset(b, T, w, e, lane, a.pool + (size_t)row * NP, a.mode);
    }
    __syncwarp();
    if (traced) JQ_TRACE_AT(1, TR_RESET);
    if (a.flags & DO_LEGAL) {
        int seat = a.seats ? a.seats[e] : b.turn[e];
        const bool skip = seat < 0 || seat > 3 || b.terminated[e] || w.sdead[seat & 3];
        seat &= 3;
        const int cnt = warp_legal(T, w, lane, seat, skip, a.ids ? a.ids + (size_t)e * a.cap : nullptr, a.cap,
                                   a.mask ? a.mask + (size_t)e * MASK_BYTES : nullptr, traced);
        if (lane == 0 && a.counts) a.counts[e] = cnt;
    }
    __syncwarp();
    if (traced) JQ_TRACE_AT(1, TR_MASKED);
    return applied;
}

__global__ void __launch_bounds__(RULE_THREADS, 4) rules_kernel(RuleArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    RuleSmem &S = *reinterpret_cast<RuleSmem *>(smem_raw);
    if (threadIdx.x == 0) JQ_TRACE_AT(1, TR_ENTRY);
    // launched as a programmatic dependent: the next kernel may start its
    // own table loads now; state is touched only after the previous kernel
    // in the stream has completed
    asm volatile("griddepcontrol.launch_dependents;");
    stage_topo(S.topo, threadIdx.x, RULE_THREADS);
    if (threadIdx.x == 0) S.applied = 0;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) JQ_TRACE_AT(1, TR_WAITED);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    WEnv &w = S.w[warp];
    for (int e = blockIdx.x * RULE_WARPS + warp; e < a.b.n; e += gridDim.x * RULE_WARPS) {
        const bool applied = warp_ply_env(a, S.topo, w, e, lane);
        if (applied && lane == 0 && a.stats) atomicAdd_block(&S.applied, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) JQ_TRACE_AT(1, TR_EXIT);
    if (threadIdx.x == 0 && a.stats && S.applied) atomicAdd((unsigned long long *)&a.stats[5], (unsigned long long)S.applied);
}

}  // namespace jq
