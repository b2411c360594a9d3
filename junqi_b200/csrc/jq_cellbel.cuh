// jq_cellbel.cuh -- per-cell float beliefs of the reference's GPU rollout
// (src/env/cuda/src/belief.cu): a (N, 4, 12, 289) float32 tensor
// [env][observer][type][world flat cell], the input jq_observe_beliefs
// reads.  These are the reference GPU path's own rules, kept beside the
// per-piece belief codes the rules kernel maintains (which follow the CPU
// BeliefTensor): a caller of the reference's GpuRollout belief calls gets
// the values that path computes.
//
// Values are only copied, set to 0 / 1, to rows of the caller's prior
// table or to 1/12; the tests on them keep the reference's float forms (a
// running float sum against 1e-8, an fmaxf chain against 1 - 1e-6).
#pragma once
#include "jq_rules.cuh"

namespace jq {

constexpr int CB_T = 12;
constexpr int CB_ENV = 4 * CB_T * NC;  // floats per env

__device__ __forceinline__ float *cb_at(float *bel, int e, int o, int cell) {
    return bel + (size_t)e * CB_ENV + (size_t)o * CB_T * NC + cell;  // type t at [t * NC]
}
__device__ __forceinline__ void cb_read(const float *p, float (&v)[CB_T]) {
#pragma unroll
    for (int t = 0; t < CB_T; ++t) v[t] = p[t * NC];
}
__device__ __forceinline__ void cb_write(float *p, const float (&v)[CB_T]) {
#pragma unroll
    for (int t = 0; t < CB_T; ++t) p[t * NC] = v[t];
}
__device__ __forceinline__ void cb_zero(float *p) {
#pragma unroll
    for (int t = 0; t < CB_T; ++t) p[t * NC] = 0.f;
}
__device__ __forceinline__ bool cb_one_hot(const float (&v)[CB_T]) {  // belief.cu:71-76
    float mx = 0.f;
#pragma unroll
    for (int t = 0; t < CB_T; ++t) mx = fmaxf(mx, v[t]);
    return mx > (1.0f - 1e-6f);
}
__device__ __forceinline__ int cb_argmax(const float (&v)[CB_T]) {  // belief.cu:79-90
    int best = 0;
    float bv = v[0];
#pragma unroll
    for (int t = 1; t < CB_T; ++t)
        if (v[t] > bv) { bv = v[t]; best = t; }
    return best;
}
__device__ __forceinline__ bool cb_is_zero(const float (&v)[CB_T]) {  // belief.cu:110-115
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < CB_T; ++t) s += v[t];
    return s < 1e-8f;
}
__device__ __forceinline__ void cb_one_hot_set(float (&v)[CB_T], int ti) {
#pragma unroll
    for (int t = 0; t < CB_T; ++t) v[t] = t == ti ? 1.f : 0.f;
}

// belief_init_kernel (belief.cu:172-248): one CTA per env.  The env's block
// is cleared, then every alive on-board piece of a tracked type gets, for
// each observer, a one-hot row when the observer owns it and its slot's
// prior row otherwise.  env_mask (N bytes, NULL: every env) selects envs.
constexpr int CB_INIT_THREADS = 256;
__global__ void __launch_bounds__(CB_INIT_THREADS) cellbel_init_kernel(jq_batch b, const uint8_t *env_mask,
                                                                       const float *prior, float *bel) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int e = blockIdx.x;
    if (e >= b.n || (env_mask && !env_mask[e])) return;
    float4 *blk = reinterpret_cast<float4 *>(bel + (size_t)e * CB_ENV);
    for (int i = threadIdx.x; i < CB_ENV / 4; i += CB_INIT_THREADS) blk[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    for (int k = threadIdx.x; k < 4 * NP; k += CB_INIT_THREADS) {
        const int p = k >> 2, o = k & 3;
        const size_t q = PI(e, p);
        if (!b.alive[q]) continue;
        const int seat = b.piece_seat[q], type = b.piece_type[q], px = b.pos_x[q], py = b.pos_y[q];
        if (px < 0 || py < 0 || px > 16 || py > 16) continue;
        const int ti = (type >= 2 && type <= 13) ? type - 2 : -1;
        if (ti < 0) continue;
        float *c = cb_at(bel, e, o, py * 17 + px);
        if (o == seat) c[ti * NC] = 1.f;
        else
#pragma unroll
            for (int t = 0; t < CB_T; ++t) c[t * NC] = prior[(p % 30) * CB_T + t];
    }
}

// seat_dead and terminated as they are before a step (snapshot_pre_step_flags,
// belief.cu:570-584); thread per env.
__global__ void cellbel_snapshot_kernel(jq_batch b, uint8_t *prev_dead, uint8_t *prev_term) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= b.n) return;
    if (prev_dead) {
#pragma unroll
        for (int s = 0; s < 4; ++s) prev_dead[(size_t)e * 4 + s] = b.seat_dead[(size_t)e * 4 + s];
    }
    if (prev_term) prev_term[e] = b.terminated[e];
}

// belief_update_kernel (belief.cu:255-565) on the post-step state: one warp
// per env.  Lane o (0..3) applies R5/R7, R1 and R6 to observer o's cells;
// then the warp sweeps the 4 x 289 (observer, cell) pairs for R4 and I5,
// which touch one cell each and read what the first phase wrote.
constexpr int CB_WARPS = 8;
__global__ void __launch_bounds__(CB_WARPS * 32) cellbel_update_kernel(jq_batch b, const int8_t *event,
                                                                      const uint8_t *flag_cap,
                                                                      const int32_t *world_actions,
                                                                      const uint8_t *prev_dead,
                                                                      const int16_t *strongholds, float *bel) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * CB_WARPS + (threadIdx.x >> 5);
    if (e >= b.n) return;
    const int ev = event[e];
    const int act = world_actions[e];
    if (b.terminated[e] || ev == 0 || act < 0 || act >= NC * NC) return;  // belief.cu:275-281
    const bool fc = flag_cap[e] != 0;
    const int src = act / NC, dst = act % NC;
    const int dstc = g_topo.f2c[dst];
    const bool dst_sh = dstc >= 0 && (g_topo.flags[dstc] & F_SH);
    // the first seat that died in this step when it captured a flag (belief.cu:363-375)
    int surrendered = -1;
    if (fc)
        for (int s = 0; s < 4; ++s)
            if (b.seat_dead[(size_t)e * 4 + s] && !prev_dead[(size_t)e * 4 + s]) { surrendered = s; break; }
    // the other stronghold of the seat whose stronghold dst is (belief.cu:380-402)
    int owner = -1, other = -1;
    if (dst_sh)
        for (int s = 0; s < 4; ++s) {
            if (strongholds[2 * s] == dst) { owner = s; other = strongholds[2 * s + 1]; break; }
            if (strongholds[2 * s + 1] == dst) { owner = s; other = strongholds[2 * s]; break; }
        }
    if (lane < 4) {
        const int o = lane;
        float vs[CB_T], vd[CB_T];
        cb_read(cb_at(bel, e, o, src), vs);
        cb_read(cb_at(bel, e, o, dst), vd);
        // R5/R7 (belief.cu:425-440): eating a known mine makes the attacker an engineer
        if (ev == EV_EAT && cb_one_hot(vd) && cb_argmax(vd) == DILEI - 2 && !cb_one_hot(vs))
            cb_one_hot_set(vs, GONGB - 2);
        // R1 migration (belief.cu:444-469)
        if (ev == EV_MOVE || ev == EV_EAT) {
            cb_write(cb_at(bel, e, o, dst), vs);
            cb_zero(cb_at(bel, e, o, src));
        } else if (ev == EV_KILLED) {
            cb_zero(cb_at(bel, e, o, src));
        } else if (ev == EV_BOMB) {
            cb_zero(cb_at(bel, e, o, src));
            cb_zero(cb_at(bel, e, o, dst));
        }
        // R6 (belief.cu:473-486): an eaten stronghold piece that is not the
        // flag puts the flag on the seat's other stronghold
        if (ev == EV_EAT && dst_sh && !fc && owner >= 0 && other >= 0 && other < NC) {
            float v[CB_T];
            cb_read(cb_at(bel, e, o, other), v);
            if (!cb_is_zero(v) && !cb_one_hot(v)) {
                cb_one_hot_set(v, JUNQI - 2);
                cb_write(cb_at(bel, e, o, other), v);
            }
        }
    }
    __syncwarp();
    const bool r4 = fc && surrendered >= 0;
    for (int k = lane; k < 4 * NC; k += 32) {
        const int o = k / NC, c = k - o * NC;
        float *cell = cb_at(bel, e, o, c);
        const int p = b.cell_pid[(size_t)e * NC + c];
        // R4 (belief.cu:490-505): after a flag capture every empty cell is cleared
        if (r4 && p < 0) {
            cb_zero(cell);
            continue;
        }
        // I5 sweep (belief.cu:518-562)
        float v[CB_T];
        cb_read(cell, v);
        if (p < 0 || p >= NP || !b.alive[PI(e, p)]) {
            if (!cb_is_zero(v)) cb_zero(cell);
        } else if (cb_is_zero(v)) {
            const int ps = b.piece_seat[PI(e, p)], pt = b.piece_type[PI(e, p)];
            const int ti = (pt >= 2 && pt <= 13) ? pt - 2 : -1;
            if ((o & 1) == (ps & 1) && ti >= 0) cb_one_hot_set(v, ti);
            else
#pragma unroll
                for (int t = 0; t < CB_T; ++t) v[t] = 1.0f / (float)CB_T;
            cb_write(cell, v);
        }
    }
}

}  // namespace jq
