// jq_lib.cu -- kernels and the extern "C" entry points of libjq.so.
//
// Launch shapes: rules kernels run one warp per env with eight envs per CTA
// and a grid sized to fill the device (grid-stride over envs), the board
// tables staged once per CTA in shared memory; the observation kernel runs a
// persistent grid of (SMs x resident CTAs) CTAs, one (env, observer) unit at a
// time.  No entry point synchronises the device; every launch goes to the
// caller's stream.
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "jq_cellbel.cuh"
#include "jq_hist.cuh"
#include "jq_obs.cuh"
#include "jq_ply.cuh"
#include "jq_rules.cuh"
#include "jq_slots.cuh"
#include "jq_topo_build.h"

namespace jq {

// Zobrist hash of every env rebuilt from scratch (state.py:1761-1815), one
// warp per env.
__global__ void rehash_kernel(jq_batch b, int mode) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (e >= b.n) return;
    int64_t h = 0;
    for (int p = lane; p < NP; p += 32) {
        const size_t q = PI(e, p);
        const int t = b.piece_type[q], x = b.pos_x[q], y = b.pos_y[q];
        if (b.alive[q] && t >= 0 && x >= 0 && x < 17 && y >= 0 && y < 17) h ^= zpiece(p, t, y * 17 + x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) h ^= __shfl_xor_sync(FULL, h, o);
    if (lane == 0) {
        const int w = b.winner[e];
        h ^= c_zturn[b.turn[e] & 3] ^ g_zmc[b.move_counter[e] & 0xFFF] ^ g_zmslc[b.mslc[e] & 0x1FF];
        h ^= c_zwin[(w == 0 || w == 1) ? w + 1 : 0] ^ c_zshow[mode & 3];
        if (b.terminated[e]) h ^= c_zterm;
        if (b.draw[e]) h ^= c_zdraw;
        for (int s = 0; s < 4; ++s) {
            if (b.seat_dead[(size_t)e * 4 + s]) h ^= c_zsdead[s];
            if (b.seat_flag[(size_t)e * 4 + s]) h ^= c_zsflag[s];
        }
        b.zobrist[e] = h;
    }
}

// Entry of the small kernels launched with programmatic dependent launch
// (launch_pdl): let the next kernel in the stream be scheduled early, then
// wait until the previous one has completed and its writes are visible,
// before the first access to caller memory.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// compact canonical action -> world flat action (game_state.cu:2639-2685 semantics)
__global__ void rotate_actions_kernel(int n, const int32_t *can, const int8_t *seats, const int8_t *turn,
                                      int32_t *world) {
    pdl_enter();
    int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    int a = can[e];
    int seat = (seats ? seats[e] : turn[e]) & 3;
    if (a < 0 || a >= NB * NB) { world[e] = -1; return; }
    int cs = a / NB, cd = a % NB;
    // canonical -> world: invert the per-seat rotation by search over the 129 cells
    int ws = -1, wd = -1;
    for (int c = 0; c < NB; ++c) {
        int r = g_topo.rot[seat][c];
        if (r == cs) ws = c;
        if (r == cd) wd = c;
    }
    world[e] = (ws < 0 || wd < 0) ? -1 : g_topo.c2f[ws] * NC + g_topo.c2f[wd];
}

// ---------------------------------------------------------------------------
// CSR: block sums, per-block exclusive scan, then value compaction with one
// warp per env (every env's copy in flight at once)
// ---------------------------------------------------------------------------
constexpr int CSR_BLOCK = 1024;   // envs per block sum
constexpr int CSR_COPY_WARPS = 8; // envs per block of csr_values_kernel

__global__ void csr_partial_kernel(int n, const int32_t *counts, int cap, int32_t *partial) {
    __shared__ int32_t red[32];
    pdl_enter();
    int e = blockIdx.x * CSR_BLOCK + threadIdx.x;
    int v = e < n ? min(counts[e], cap) : 0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        int s = red[threadIdx.x];
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
        if (threadIdx.x == 0) partial[blockIdx.x] = s;
    }
}

__global__ void csr_offsets_kernel(int n, const int32_t *counts, int cap, const int32_t *partial,
                                   int32_t *offsets) {
    __shared__ int32_t wsum[32];
    __shared__ int32_t base_s;
    pdl_enter();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (wid == 0) {  // sum of the block sums before this block
        int s = 0;
        for (int k = lane; k < (int)blockIdx.x; k += 32) s += partial[k];
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
        if (lane == 0) base_s = s;
    }
    int e = blockIdx.x * CSR_BLOCK + threadIdx.x;
    int v = e < n ? min(counts[e], cap) : 0, inc = v;
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) wsum[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        int s = wsum[lane], si = s;
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(FULL, si, o);
            if (lane >= o) si += t;
        }
        wsum[lane] = si - s;
    }
    __syncthreads();
    int excl = base_s + wsum[wid] + inc - v;
    if (e < n) offsets[e] = excl;
    if (e == n - 1) offsets[n] = excl + v;
}

__global__ void csr_values_kernel(int n, const int32_t *counts, const int32_t *ids, int cap,
                                  const int32_t *offsets, int32_t *values) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * CSR_COPY_WARPS + (threadIdx.x >> 5);
    if (e >= n) return;
    const int c = min(counts[e], cap), o = offsets[e];
    for (int j = lane; j < c; j += 32) values[o + j] = ids[(size_t)e * cap + j];
}

// ---------------------------------------------------------------------------
// Samplers (stand-in policies for benchmarks)
// ---------------------------------------------------------------------------
__global__ void sample_uniform_kernel(int n, const int32_t *counts, const int32_t *ids, int cap, uint64_t seed,
                                      uint64_t ply, int32_t *acts) {
    pdl_enter();
    int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    int c = min(counts[e], cap);
    acts[e] = c > 0 ? ids[(size_t)e * cap + (int)(hash3(seed, ply, (uint64_t)e) % (uint64_t)c)] : -1;
}

__device__ __forceinline__ float u01(uint64_t h) {  // (0, 1)
    return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

// Gumbel-max over the legal set: argmax_a logit(a) + G(a), logit ~ N(0,1)
// (Box-Muller) and G ~ Gumbel(0,1), both keyed on (seed, ply, env, action).
__global__ void sample_softmax_kernel(int n, const int8_t *turn, const int32_t *counts, const int32_t *ids, int cap,
                                      uint64_t seed, uint64_t ply, int32_t *can_out, int32_t *world_out) {
    pdl_enter();
    int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    int c = min(counts[e], cap), seat = turn[e] & 3;
    float best = -3.0e38f;
    int best_w = -1, best_c = -1;
    for (int j = 0; j < c; ++j) {
        int id = ids[(size_t)e * cap + j];
        int sc = g_topo.f2c[id / NC], dc = g_topo.f2c[id % NC];
        if (sc < 0 || dc < 0) continue;
        int can = g_topo.rot[seat][sc] * NB + g_topo.rot[seat][dc];
        uint64_t h = hash3(seed ^ 0xA5A5A5A5ull, ply, ((uint64_t)e << 16) ^ (uint64_t)can);
        float r1 = u01(h), r2 = u01(mix64(h)), r3 = u01(mix64(h ^ 0x5bd1e995ull));
        float logit = sqrtf(-2.f * logf(r1)) * cosf(6.2831853f * r2);
        float score = logit - logf(-logf(r3));
        if (score > best) { best = score; best_w = id; best_c = can; }
    }
    if (can_out) can_out[e] = best_c;
    if (world_out) world_out[e] = best_w;
}

// ---------------------------------------------------------------------------
// Host-side state
// ---------------------------------------------------------------------------
constexpr int OBS_TICKETS = 256;  // observation launches that may be in flight on one GPU at once
struct DeviceState {
    bool topo = false, zob = false, obs = false;
    const int8_t *pool = nullptr;
    int pool_size = 0;
    int sms = 0, rule_blocks_per_sm = 0, obs_blocks_per_sm = 0;
    int *obs_ticket = nullptr;             // OBS_TICKETS x {next unit, finished CTAs}, zero between launches
    std::atomic<unsigned> obs_calls{0};
};
constexpr int MAX_DEV = 64;
static DeviceState g_dev[MAX_DEV];
static std::mutex g_mu;
static thread_local char g_err[512] = "";

static int fail(int code, const char *msg) {
    std::snprintf(g_err, sizeof g_err, "%s", msg);
    return code;
}
static int cuda_fail(cudaError_t err, const char *where) {
    std::snprintf(g_err, sizeof g_err, "%s: %s", where, cudaGetErrorString(err));
    return JQ_ERR_CUDA;
}
#define CU(call)                                                    \
    do {                                                            \
        cudaError_t _e = (call);                                    \
        if (_e != cudaSuccess) return cuda_fail(_e, #call);         \
    } while (0)

static int current_dev(DeviceState *&st) {
    int d = 0;
    CU(cudaGetDevice(&d));
    if (d < 0 || d >= MAX_DEV) return fail(JQ_ERR_ARG, "device index out of range");
    st = &g_dev[d];
    return JQ_OK;
}

static int check_batch(const jq_batch *b) {
    if (!b || b->n <= 0) return fail(JQ_ERR_ARG, "batch is null or empty");
    const void *ptrs[] = {b->alive, b->piece_type, b->piece_seat, b->pos_x, b->pos_y, b->zero_x, b->zero_y,
                          b->move_count, b->active_eat, b->passive_surv, b->death_reason, b->death_step,
                          b->death_loc, b->cell_pid, b->seat_dead, b->seat_flag, b->turn, b->zobrist,
                          b->move_counter, b->mslc, b->terminated, b->winner, b->draw, b->cm_direct_lo,
                          b->cm_direct_hi, b->cm_direct_type, b->cm_last_direct_step, b->cm_direct_other,
                          b->cm_chain_lo, b->cm_chain_hi, b->cm_chain_type, b->cm_last_chain_step,
                          b->cm_eaten_lo, b->cm_eaten_hi, b->cm_rank_floor, b->cm_rank_floor_step,
                          b->cm_is_gongb, b->cm_not_gongb, b->cm_atk_gongb, b->hist_src, b->hist_dst,
                          b->hist_count, b->bel_code, b->remaining, b->rem_tracked};
    for (const void *p : ptrs)
        if (!p) return fail(JQ_ERR_ARG, "a batch field pointer is null");
    const void *wide[] = {b->move_count, b->active_eat, b->passive_surv, b->death_step, b->death_loc, b->cell_pid,
                          b->zobrist, b->move_counter, b->mslc, b->cm_direct_lo, b->cm_direct_hi,
                          b->cm_direct_type, b->cm_last_direct_step, b->cm_direct_other, b->cm_chain_lo,
                          b->cm_chain_hi, b->cm_chain_type, b->cm_last_chain_step, b->cm_eaten_lo, b->cm_eaten_hi,
                          b->cm_rank_floor_step, b->hist_src, b->hist_dst, b->hist_count, b->remaining};
    for (const void *p : wide)
        if ((uintptr_t)p & 1) return fail(JQ_ERR_ARG, "a multi-byte batch field is misaligned");
    if (((uintptr_t)b->zobrist | (uintptr_t)b->cm_direct_lo | (uintptr_t)b->cm_direct_hi | (uintptr_t)b->cm_chain_lo |
         (uintptr_t)b->cm_chain_hi | (uintptr_t)b->cm_eaten_lo | (uintptr_t)b->cm_eaten_hi) & 7)
        return fail(JQ_ERR_ARG, "64-bit batch fields must be 8-byte aligned");
    if (((uintptr_t)b->move_counter | (uintptr_t)b->mslc | (uintptr_t)b->hist_count) & 3)
        return fail(JQ_ERR_ARG, "32-bit batch fields must be 4-byte aligned");
    if ((uintptr_t)b->bel_code & 15) return fail(JQ_ERR_ARG, "bel_code must be 16-byte aligned");
    if (b->rules != JQ_RULES_BATCHED && b->rules != JQ_RULES_GAMESTATE) return fail(JQ_ERR_ARG, "unknown rules value");
    return JQ_OK;
}

static size_t rule_smem() { return sizeof(RuleSmem); }
static size_t obs_smem() { return sizeof(ObsSmem); }

// Programmatic dependent launch: the kernel may be scheduled while the
// previous kernel in the stream drains (the rules kernel's slowest envs, the
// observation kernel's last units), load its board tables into shared
// memory, then wait (griddepcontrol.wait) for that kernel to complete
// before touching any state.  Kernels launched this way call
// griddepcontrol.wait before their first access to caller memory.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

static int launch_rules(RuleArgs &a, cudaStream_t s) {
    DeviceState *st;
    int rc = current_dev(st);
    if (rc) return rc;
    if (!st->topo) return fail(JQ_ERR_NOT_READY, "jq_init was not called on this device");
    int blocks = (a.b.n + RULE_WARPS - 1) / RULE_WARPS;
    int cap_blocks = st->sms * (st->rule_blocks_per_sm > 0 ? st->rule_blocks_per_sm : 1) * 4;
    if (blocks > cap_blocks) blocks = cap_blocks;
    CU(launch_pdl(rules_kernel, (unsigned)blocks, RULE_THREADS, rule_smem(), s, a));
    return JQ_OK;
}

// The three CSR kernels; scratch holds ceil(n / CSR_BLOCK) block sums, all
// written by csr_partial_kernel before csr_offsets_kernel reads them.
static int launch_csr(int32_t n, const int32_t *counts, const int32_t *ids, int32_t cap, int32_t *scratch,
                      int32_t *offsets, int32_t *values, cudaStream_t s) {
    const unsigned blocks = (unsigned)((n + CSR_BLOCK - 1) / CSR_BLOCK);
    CU(launch_pdl(csr_partial_kernel, blocks, CSR_BLOCK, 0, s, (int)n, counts, (int)cap, scratch));
    CU(launch_pdl(csr_offsets_kernel, blocks, CSR_BLOCK, 0, s, (int)n, counts, (int)cap,
                  (const int32_t *)scratch, offsets));
    CU(launch_pdl(csr_values_kernel, (unsigned)((n + CSR_COPY_WARPS - 1) / CSR_COPY_WARPS), 32 * CSR_COPY_WARPS, 0,
                  s, (int)n, counts, ids, (int)cap, (const int32_t *)offsets, values));
    return JQ_OK;
}

}  // namespace jq

using namespace jq;

extern "C" {

int jq_abi_version(void) { return JQ_ABI_VERSION; }

int jq_topology_dump(int32_t *on_board, int32_t *rail, int32_t *curve, int32_t *rail_adj, int32_t *srays,
                     int32_t *crays, int32_t *compact_to_flat, int32_t *flags) {
    static Topo T;
    build_topo(T);
    auto flat = [&](int c) { return c == NONE8 ? -1 : (int)T.c2f[c]; };
    for (int f = 0; f < NC; ++f) {
        int c = T.f2c[f];
        on_board[f] = c >= 0;
        rail[f] = c >= 0 && (T.flags[c] & F_RAIL) ? 1 : 0;
        curve[f] = c >= 0 ? T.curve[c] : 0;
        flags[f] = c >= 0 ? T.flags[c] : 0;
        int n = 0;
        for (int k = 0; k < 4; ++k) rail_adj[f * 4 + k] = -1;
        if (c >= 0)
            for (int v = 0; v < NB; ++v)
                if ((T.railnb[c][v >> 5] >> (v & 31)) & 1u) rail_adj[f * 4 + n++] = T.c2f[v];
        for (int k = 0; k < 4; ++k)
            for (int l = 0; l < 12; ++l) srays[(f * 4 + k) * 12 + l] = c >= 0 ? flat(T.sray[c][k][l]) : -1;
        for (int k = 0; k < 2; ++k)
            for (int l = 0; l < 11; ++l) crays[(f * 2 + k) * 11 + l] = c >= 0 ? flat(T.cray[c][k][l]) : -1;
    }
    for (int c = 0; c < NB; ++c) compact_to_flat[c] = T.c2f[c];
    return JQ_OK;
}
const char *jq_last_error(void) { return g_err; }

int jq_init(int device) {
    if (device < 0 || device >= MAX_DEV) return fail(JQ_ERR_ARG, "device index out of range");
    CU(cudaSetDevice(device));
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState &st = g_dev[device];
    if (st.topo) return JQ_OK;
    static Topo host_topo;
    static SlotTopo host_slot;
    static bool built = false;
    if (!built) {
        build_topo(host_topo);
        if (!build_ray_masks(host_topo, host_topo.ray)) return fail(JQ_ERR_ARG, "straight rail rays out of order");
        build_slot_topo(host_topo, host_slot);
        built = true;
    }
    CU(cudaMemcpyToSymbol(g_topo, &host_topo, sizeof(Topo)));
    CU(cudaMemcpyToSymbol(g_slot, &host_slot, sizeof(SlotTopo)));
    {
        static uint32_t statw[4][OBS_VEC][STAT_WORDS];
        build_static_words(host_topo, statw);
        CU(cudaMemcpyToSymbol(g_statw, statw, sizeof(statw)));
    }
    CU(cudaFuncSetAttribute(rules_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rule_smem()));
    CU(cudaFuncSetAttribute(obs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)obs_smem()));
    CU(cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, device));
    CU(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&st.rule_blocks_per_sm, rules_kernel, RULE_THREADS, rule_smem()));
    CU(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&st.obs_blocks_per_sm, obs_kernel, OBS_THREADS, obs_smem()));
    if (st.obs_blocks_per_sm > OBS_MIN_CTAS) st.obs_blocks_per_sm = OBS_MIN_CTAS;
    CU(cudaMalloc(&st.obs_ticket, sizeof(int) * 2 * OBS_TICKETS));
    CU(cudaMemset(st.obs_ticket, 0, sizeof(int) * 2 * OBS_TICKETS));
    st.topo = true;
    return JQ_OK;
}

int jq_upload_zobrist(const int64_t *piece, const int64_t *turn, const int64_t *mc, const int64_t *mslc,
                      const int64_t *winner, int64_t terminated, int64_t draw, const int64_t *seat_dead,
                      const int64_t *seat_flag, const int64_t *show_mode) {
    if (!piece || !turn || !mc || !mslc || !winner || !seat_dead || !seat_flag || !show_mode)
        return fail(JQ_ERR_ARG, "null Zobrist table");
    DeviceState *st;
    int rc = current_dev(st);
    if (rc) return rc;
    CU(cudaMemcpyToSymbol(g_zpiece, piece, sizeof(int64_t) * NP * 14 * NC));
    CU(cudaMemcpyToSymbol(g_zmc, mc, sizeof(int64_t) * 4096));
    CU(cudaMemcpyToSymbol(g_zmslc, mslc, sizeof(int64_t) * 512));
    CU(cudaMemcpyToSymbol(c_zturn, turn, sizeof(int64_t) * 4));
    CU(cudaMemcpyToSymbol(c_zwin, winner, sizeof(int64_t) * 3));
    CU(cudaMemcpyToSymbol(c_zsdead, seat_dead, sizeof(int64_t) * 4));
    CU(cudaMemcpyToSymbol(c_zsflag, seat_flag, sizeof(int64_t) * 4));
    CU(cudaMemcpyToSymbol(c_zshow, show_mode, sizeof(int64_t) * 4));
    CU(cudaMemcpyToSymbol(c_zterm, &terminated, sizeof(int64_t)));
    CU(cudaMemcpyToSymbol(c_zdraw, &draw, sizeof(int64_t)));
    st->zob = true;
    return JQ_OK;
}

int jq_upload_obs_tables(const float *prior, const float *uniform12, const float *recency) {
    if (!prior || !uniform12 || !recency) return fail(JQ_ERR_ARG, "null observation table");
    DeviceState *st;
    int rc = current_dev(st);
    if (rc) return rc;
    CU(cudaMemcpyToSymbol(g_prior, prior, sizeof(float) * 360));
    CU(cudaMemcpyToSymbol(g_uniform, uniform12, sizeof(float) * 12));
    CU(cudaMemcpyToSymbol(g_recency, recency, sizeof(float) * 4 * RECENCY_LEN));
    st->obs = true;
    return JQ_OK;
}

int jq_set_setup_pool(const int8_t *d_pool, int32_t pool_size) {
    if (!d_pool || pool_size <= 0) return fail(JQ_ERR_ARG, "empty setup pool");
    DeviceState *st;
    int rc = current_dev(st);
    if (rc) return rc;
    st->pool = d_pool;
    st->pool_size = pool_size;
    return JQ_OK;
}

int32_t jq_pool_index(uint64_t seed, uint64_t ply, int32_t env, int32_t pool_size) {
    if (pool_size <= 0) return -1;
    return (int32_t)(hash3(seed, ply, (uint64_t)env) % (uint64_t)pool_size);
}

static int rules_common(RuleArgs &a, const jq_batch *b, int mode, bool need_zob, void *stream) {
    int rc = check_batch(b);
    if (rc) return rc;
    if (mode < 0 || mode > 2) return fail(JQ_ERR_ARG, "show_mode must be 0, 1 or 2");
    DeviceState *st;
    rc = current_dev(st);
    if (rc) return rc;
    if (need_zob && !st->zob) return fail(JQ_ERR_NOT_READY, "Zobrist tables not uploaded");
    if (b->pool && b->pool_size <= 0) return fail(JQ_ERR_ARG, "jq_batch.pool given with pool_size <= 0");
    std::memset(&a, 0, sizeof a);
    a.b = *b;
    a.mode = mode;
    // the batch's own pool; the device-wide one only when it has none
    a.pool = b->pool ? b->pool : st->pool;
    a.pool_size = b->pool ? b->pool_size : st->pool_size;
    (void)stream;
    return JQ_OK;
}

int jq_reset(const jq_batch *b, uint64_t seed, uint64_t ply, int32_t all, int32_t show_mode, void *stream) {
    RuleArgs a;
    int rc = rules_common(a, b, show_mode, true, stream);
    if (rc) return rc;
    if (!a.pool) return fail(JQ_ERR_NOT_READY, "setup pool not set");
    a.flags = DO_RESET | (all ? RESET_ALL : 0);
    a.seed = seed;
    a.ply = ply;
    return launch_rules(a, (cudaStream_t)stream);
}

int jq_reset_rows(const jq_batch *b, const int32_t *d_rows, int32_t show_mode, void *stream) {
    RuleArgs a;
    int rc = rules_common(a, b, show_mode, true, stream);
    if (rc) return rc;
    if (!a.pool) return fail(JQ_ERR_NOT_READY, "setup pool not set");
    if (!d_rows) return fail(JQ_ERR_ARG, "pool rows missing");
    a.flags = DO_RESET;
    a.rows = d_rows;
    return launch_rules(a, (cudaStream_t)stream);
}

int jq_init_beliefs(const jq_batch *b, int32_t show_mode, void *stream) {
    RuleArgs a;
    int rc = rules_common(a, b, show_mode, false, stream);
    if (rc) return rc;
    a.flags = DO_BELIEF_INIT;
    return launch_rules(a, (cudaStream_t)stream);
}

int jq_legal_slots(const jq_batch *b, const int8_t *d_seats, uint8_t *d_slots, void *stream) {
    int rc = check_batch(b);
    if (rc) return rc;
    if (!d_slots) return fail(JQ_ERR_ARG, "slot mask output missing");
    if ((uintptr_t)d_slots & 15) return fail(JQ_ERR_ARG, "slot mask output must be 16-byte aligned");
    DeviceState *st;
    rc = current_dev(st);
    if (rc) return rc;
    if (!st->topo) return fail(JQ_ERR_NOT_READY, "jq_init was not called on this device");
    const size_t threads = (size_t)b->n * NP;
    slot_mask_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(*b, d_seats, d_slots);
    CU(cudaGetLastError());
    return JQ_OK;
}

int jq_rehash(const jq_batch *b, int32_t show_mode, void *stream) {
    int rc = check_batch(b);
    if (rc) return rc;
    if (show_mode < 0 || show_mode > 2) return fail(JQ_ERR_ARG, "show_mode must be 0, 1 or 2");
    DeviceState *st;
    rc = current_dev(st);
    if (rc) return rc;
    if (!st->zob) return fail(JQ_ERR_NOT_READY, "Zobrist tables not uploaded");
    rehash_kernel<<<(b->n + 7) / 8, 256, 0, (cudaStream_t)stream>>>(*b, show_mode);
    CU(cudaGetLastError());
    return JQ_OK;
}

int jq_step(const jq_batch *b, const int32_t *d_world_actions, int32_t show_mode, const jq_step_out *out,
            void *stream) {
    RuleArgs a;
    int rc = rules_common(a, b, show_mode, true, stream);
    if (rc) return rc;
    if (!d_world_actions || !out || !out->valid) return fail(JQ_ERR_ARG, "actions / outputs missing");
    a.acts = d_world_actions;
    a.out = *out;
    a.flags = DO_STEP;
    return launch_rules(a, (cudaStream_t)stream);
}

int jq_step_canonical(const jq_batch *b, const int32_t *d_compact_actions, const int8_t *d_seats,
                      int32_t show_mode, const jq_step_out *out, void *stream) {
    if (!out || !out->world_action || !d_compact_actions) return fail(JQ_ERR_ARG, "world_action output required");
    int rc = check_batch(b);
    if (rc) return rc;
    CU(launch_pdl(rotate_actions_kernel, (unsigned)((b->n + 255) / 256), 256, 0, (cudaStream_t)stream, (int)b->n,
                  d_compact_actions, d_seats, (const int8_t *)b->turn, out->world_action));
    return jq_step(b, out->world_action, show_mode, out, stream);
}

int jq_canonical_to_world(const jq_batch *b, const int32_t *d_compact_actions, const int8_t *d_seats,
                          int32_t *d_world_actions, void *stream) {
    int rc = check_batch(b);
    if (rc) return rc;
    if (!d_compact_actions || !d_world_actions) return fail(JQ_ERR_ARG, "actions missing");
    CU(launch_pdl(rotate_actions_kernel, (unsigned)((b->n + 255) / 256), 256, 0, (cudaStream_t)stream, (int)b->n,
                  d_compact_actions, d_seats, (const int8_t *)b->turn, d_world_actions));
    return JQ_OK;
}

int jq_ply(const jq_batch *b, const int32_t *d_world_actions, int32_t show_mode, const jq_step_out *out,
           int32_t autoreset, uint64_t seed, uint64_t ply, int32_t *d_counts, int32_t *d_ids, int32_t cap,
           uint8_t *d_mask, int64_t *d_stats, void *stream) {
    RuleArgs a;
    int rc = rules_common(a, b, show_mode, true, stream);
    if (rc) return rc;
    if (d_world_actions && (!out || !out->valid)) return fail(JQ_ERR_ARG, "step outputs missing");
    if (autoreset && !a.pool) return fail(JQ_ERR_NOT_READY, "setup pool not set");
    if (!d_counts || !d_ids || cap <= 0) return fail(JQ_ERR_ARG, "legal outputs missing");
    a.acts = d_world_actions;
    if (out) a.out = *out;
    a.flags = DO_LEGAL | (d_world_actions ? DO_STEP : 0) | (autoreset ? DO_RESET : 0);
    a.seed = seed;
    a.ply = ply;
    a.counts = d_counts;
    a.ids = d_ids;
    a.cap = cap;
    a.mask = d_mask;
    a.stats = d_stats;
    return launch_rules(a, (cudaStream_t)stream);
}

int32_t jq_history_record_bytes(void) { return (int32_t)sizeof(HistRec); }

int jq_history_snapshot(const jq_batch *b, const int8_t *d_seats, void *d_history, int64_t step, int64_t num_steps,
                        void *stream) {
    int rc = check_batch(b);
    if (rc) return rc;
    if (!d_history || ((uintptr_t)d_history & 15)) return fail(JQ_ERR_ARG, "history must be a 16-byte aligned buffer");
    if (step < 0 || step >= num_steps) return fail(JQ_ERR_ARG, "step outside [0, num_steps)");
    hist_snapshot_kernel<<<(b->n + 7) / 8, 256, 0, (cudaStream_t)stream>>>(*b, d_seats, static_cast<HistRec *>(d_history),
                                                                         (long long)step);
    CU(cudaGetLastError());
    return JQ_OK;
}

int jq_history_restore(const void *d_history, int64_t num_records, const int64_t *d_indices, const jq_batch *scratch,
                       int8_t *d_observers, void *stream) {
    int rc = check_batch(scratch);
    if (rc) return rc;
    if (!d_history || ((uintptr_t)d_history & 15)) return fail(JQ_ERR_ARG, "history must be a 16-byte aligned buffer");
    if (!d_indices || !d_observers || num_records < 0) return fail(JQ_ERR_ARG, "indices / observers missing");
    hist_restore_kernel<<<(scratch->n + 7) / 8, 256, 0, (cudaStream_t)stream>>>(
        *scratch, static_cast<const HistRec *>(d_history), (long long)num_records,
        reinterpret_cast<const long long *>(d_indices), d_observers);
    CU(cudaGetLastError());
    return JQ_OK;
}

static int cellbel_common(const jq_batch *b, const float *d_beliefs) {
    int rc = check_batch(b);
    if (rc) return rc;
    DeviceState *st;
    rc = current_dev(st);
    if (rc) return rc;
    if (!st->topo) return fail(JQ_ERR_NOT_READY, "jq_init was not called on this device");
    if (!d_beliefs || ((uintptr_t)d_beliefs & 15))
        return fail(JQ_ERR_ARG, "beliefs must be a 16-byte aligned (N, 4, 12, 289) float32 array");
    return JQ_OK;
}

int jq_cell_beliefs_init(const jq_batch *b, const uint8_t *d_env_mask, const float *d_prior, float *d_beliefs,
                         void *stream) {
    int rc = cellbel_common(b, d_beliefs);
    if (rc) return rc;
    if (!d_prior || ((uintptr_t)d_prior & 3)) return fail(JQ_ERR_ARG, "prior must be a 30 x 12 float32 array");
    CU(launch_pdl(cellbel_init_kernel, (unsigned)b->n, CB_INIT_THREADS, 0, (cudaStream_t)stream, *b, d_env_mask,
                  d_prior, d_beliefs));
    return JQ_OK;
}

int jq_cell_beliefs_snapshot(const jq_batch *b, uint8_t *d_prev_dead, uint8_t *d_prev_terminated, void *stream) {
    int rc = check_batch(b);
    if (rc) return rc;
    if (!d_prev_dead && !d_prev_terminated) return fail(JQ_ERR_ARG, "no snapshot output given");
    CU(launch_pdl(cellbel_snapshot_kernel, (unsigned)((b->n + 255) / 256), 256, 0, (cudaStream_t)stream, *b,
                  d_prev_dead, d_prev_terminated));
    return JQ_OK;
}

int jq_cell_beliefs_update(const jq_batch *b, const int8_t *d_event, const uint8_t *d_flag_captured,
                           const int32_t *d_world_actions, const uint8_t *d_prev_dead, const int16_t *d_strongholds,
                           float *d_beliefs, void *stream) {
    int rc = cellbel_common(b, d_beliefs);
    if (rc) return rc;
    if (!d_event || !d_flag_captured || !d_world_actions || !d_prev_dead || !d_strongholds)
        return fail(JQ_ERR_ARG, "step results, seat_dead snapshot and stronghold table are required");
    if (((uintptr_t)d_world_actions & 3) || ((uintptr_t)d_strongholds & 1))
        return fail(JQ_ERR_ARG, "world actions / strongholds misaligned");
    CU(launch_pdl(cellbel_update_kernel, (unsigned)((b->n + CB_WARPS - 1) / CB_WARPS), CB_WARPS * 32, 0,
                  (cudaStream_t)stream, *b, d_event, d_flag_captured, d_world_actions, d_prev_dead, d_strongholds,
                  d_beliefs));
    return JQ_OK;
}

int jq_legal(const jq_batch *b, const int8_t *d_seats, int32_t *d_counts, int32_t *d_ids, int32_t cap,
             uint8_t *d_mask, void *stream) {
    RuleArgs a;
    int rc = rules_common(a, b, JQ_HALF_DARK, false, stream);
    if (rc) return rc;
    if (!d_counts || cap < 0 || (cap > 0 && !d_ids)) return fail(JQ_ERR_ARG, "legal outputs missing");
    a.flags = DO_LEGAL;
    a.seats = d_seats;
    a.counts = d_counts;
    a.ids = d_ids;
    a.cap = cap;
    a.mask = d_mask;
    return launch_rules(a, (cudaStream_t)stream);
}

int32_t jq_csr_scratch_ints(int32_t n) { return n <= 0 ? 0 : (n + CSR_BLOCK - 1) / CSR_BLOCK; }

int jq_csr(int32_t n, const int32_t *d_counts, const int32_t *d_ids, int32_t cap, int32_t *d_offsets,
           int32_t *d_values, int32_t *d_block_scratch, void *stream) {
    if (n <= 0 || !d_counts || !d_ids || !d_offsets || !d_values || !d_block_scratch || cap <= 0)
        return fail(JQ_ERR_ARG, "bad CSR arguments");
    return launch_csr(n, d_counts, d_ids, cap, d_block_scratch, d_offsets, d_values, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Allocation-free CSR.  Some hosts of this library cannot allocate device
// memory: a training process whose PyTorch caching allocator has reserved
// the whole HBM budget, or a thin FFI host (a game server or evaluation
// harness calling through ctypes / cgo) that owns only the buffers it was
// handed and has no CUDA allocator of its own.  jq_csr_noalloc keeps its
// block-sum scratch in the file-scope array below instead of asking the
// caller for it, and calls no allocating routine.  The array holds one int
// per 1024 envs, so it covers up to JQ_NOALLOC_MAX_ENVS envs; every GPU that
// loads libjq.so holds these 4 KiB until the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) int32_t g_noalloc_scratch[(JQ_NOALLOC_MAX_ENVS + CSR_BLOCK - 1) / CSR_BLOCK];
static int32_t *g_noalloc_ptr[MAX_DEV];  // device address of g_noalloc_scratch, per device

int jq_csr_noalloc(int32_t n, const int32_t *d_counts, const int32_t *d_ids, int32_t cap, int32_t *d_offsets,
                   int32_t *d_values, void *stream) {
    if (n <= 0 || !d_counts || !d_ids || !d_offsets || !d_values || cap <= 0)
        return fail(JQ_ERR_ARG, "bad CSR arguments");
    if (n > JQ_NOALLOC_MAX_ENVS) return fail(JQ_ERR_CAPACITY, "jq_csr_noalloc: n exceeds JQ_NOALLOC_MAX_ENVS");
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev < 0 || dev >= MAX_DEV) return fail(JQ_ERR_ARG, "device index out of range");
    int32_t *scratch;
    {
        // First call on a device: look up the array's device address with that
        // device current.  The host-side symbol itself is only a stand-in.
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_noalloc_ptr[dev]) {
            void *p = nullptr;
            CU(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            g_noalloc_ptr[dev] = static_cast<int32_t *>(p);
        }
        scratch = g_noalloc_ptr[dev];
    }
    // csr_partial_kernel writes every block sum csr_offsets_kernel reads, so
    // the contents left by the previous call need no clearing.
    return launch_csr(n, d_counts, d_ids, cap, scratch, d_offsets, d_values, (cudaStream_t)stream);
}

// Per-CTA timestamps of the last obs_kernel / rules_kernel launch, in the
// tracing build only (JQ_TRACE, `make trace`).
int jq_trace_read(int32_t kernel, uint64_t *host, int32_t ctas) {
#ifdef JQ_TRACE
    if (kernel < 0 || kernel >= TRACE_KERNELS || !host || ctas <= 0 || ctas > TRACE_CTAS)
        return fail(JQ_ERR_ARG, "jq_trace_read: bad kernel index, output or CTA count");
    CU(cudaMemcpyFromSymbol(host, g_trace, sizeof(uint64_t) * TRACE_POINTS * ctas,
                            sizeof(uint64_t) * TRACE_POINTS * TRACE_CTAS * kernel));
    return JQ_OK;
#else
    (void)kernel, (void)host, (void)ctas;
    return fail(JQ_ERR_NOT_READY, "libjq was built without JQ_TRACE (make trace builds libjq_trace.so)");
#endif
}

static int observe_launch(const jq_batch *b, const int8_t *d_observers, int32_t seats_per_env, int32_t show_mode,
                          const float *d_beliefs, float *d_spatial, float *d_global, void *stream) {
    int rc = check_batch(b);
    if (rc) return rc;
    if (seats_per_env < 1 || seats_per_env > 4) return fail(JQ_ERR_ARG, "seats_per_env must be 1..4");
    if (show_mode < 0 || show_mode > 2) return fail(JQ_ERR_ARG, "show_mode must be 0, 1 or 2");
    if (!d_spatial || !d_global) return fail(JQ_ERR_ARG, "observation outputs missing");
    if (((uintptr_t)d_spatial & 3) || ((uintptr_t)d_global & 3))
        return fail(JQ_ERR_ARG, "observation outputs must be 4-byte aligned float arrays");
    if (!d_observers && seats_per_env != 1 && seats_per_env != 4)
        return fail(JQ_ERR_ARG, "observers required unless seats_per_env is 1 or 4");
    DeviceState *st;
    rc = current_dev(st);
    if (rc) return rc;
    if (!st->topo || !st->obs) return fail(JQ_ERR_NOT_READY, "jq_init / jq_upload_obs_tables missing");
    size_t units = (size_t)b->n * seats_per_env;
    if (units > (size_t)INT32_MAX / 2) return fail(JQ_ERR_ARG, "too many observation units for one call");
    size_t grid = (size_t)st->sms * (st->obs_blocks_per_sm > 0 ? st->obs_blocks_per_sm : 1);
    if (grid > units) grid = units;
    int *ticket = st->obs_ticket + 2 * (st->obs_calls.fetch_add(1) % OBS_TICKETS);
    CU(launch_pdl(obs_kernel, (unsigned)grid, OBS_THREADS, obs_smem(), (cudaStream_t)stream, *b, d_observers,
                  (int)seats_per_env, (int)show_mode, d_spatial, d_global, ticket, d_beliefs));
    return JQ_OK;
}

int jq_observe(const jq_batch *b, const int8_t *d_observers, int32_t seats_per_env, int32_t show_mode,
               float *d_spatial, float *d_global, void *stream) {
    return observe_launch(b, d_observers, seats_per_env, show_mode, nullptr, d_spatial, d_global, stream);
}

int jq_observe_beliefs(const jq_batch *b, const int8_t *d_observers, int32_t seats_per_env, int32_t show_mode,
                       const float *d_beliefs, float *d_spatial, float *d_global, void *stream) {
    if (!d_beliefs || ((uintptr_t)d_beliefs & 3)) return fail(JQ_ERR_ARG, "beliefs must be a float32 array");
    return observe_launch(b, d_observers, seats_per_env, show_mode, d_beliefs, d_spatial, d_global, stream);
}

int jq_sample_uniform(int32_t n, const int32_t *d_counts, const int32_t *d_ids, int32_t cap, uint64_t seed,
                      uint64_t ply, int32_t *d_actions, void *stream) {
    if (n <= 0 || !d_counts || !d_ids || !d_actions || cap <= 0) return fail(JQ_ERR_ARG, "bad sampler arguments");
    CU(launch_pdl(sample_uniform_kernel, (unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream, (int)n, d_counts,
                  d_ids, (int)cap, seed, ply, d_actions));
    return JQ_OK;
}

int jq_sample_softmax(const jq_batch *b, const int32_t *d_counts, const int32_t *d_ids, int32_t cap, uint64_t seed,
                      uint64_t ply, int32_t *d_compact_actions, int32_t *d_world_actions, void *stream) {
    if (!b || b->n <= 0 || !b->turn || !d_counts || !d_ids || cap <= 0) return fail(JQ_ERR_ARG, "bad sampler arguments");
    CU(launch_pdl(sample_softmax_kernel, (unsigned)((b->n + 127) / 128), 128, 0, (cudaStream_t)stream, (int)b->n,
                  (const int8_t *)b->turn, d_counts, d_ids, (int)cap, seed, ply, d_compact_actions, d_world_actions));
    return JQ_OK;
}

}  // extern "C"
