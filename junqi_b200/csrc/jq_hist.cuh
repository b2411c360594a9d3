// jq_hist.cuh -- compact rollout history (the reference's DeviceRolloutHistory,
// junqi_cuda.h:186-277 and rollout_history.cu): one record per (step, env)
// holding exactly what the acting seat's observation and legal mask read,
// so a training minibatch can be rebuilt on the device later.
//
// A record keeps the env's board and piece state plus, for the acting
// observer o only, its combat-memory row, its belief codes and inventories,
// and the two opponents' views of o's own 30 pids (observation layer 2).
// Reconstruction scatters records into a scratch batch -- the observer's
// rows at their usual places, nothing else -- on which jq_legal and
// jq_observe then run unchanged.
#pragma once
#include "jq_rules.cuh"

namespace jq {

struct __align__(16) HistRec {
    uint64_t cm_direct_lo[NP], cm_direct_hi[NP], cm_chain_lo[NP], cm_chain_hi[NP];
    uint64_t cm_eaten_lo[NP], cm_eaten_hi[NP];
    uint64_t lr_direct_lo[2][30], lr_direct_hi[2][30];  // left, right observers' rows of o's own pids
    uint16_t cm_direct_type[NP], cm_chain_type[NP];
    int16_t cm_last_direct_step[NP], cm_direct_other[NP], cm_last_chain_step[NP], cm_rank_floor_step[NP];
    int16_t lr_direct_other[2][30];
    int16_t move_count[NP], active_eat[NP], passive_surv[NP], death_step[NP], death_loc[NP];
    int16_t cell_pid[NC + 1];
    int16_t hist_src[HIST], hist_dst[HIST];
    int16_t remaining[4][12];  // observer o's inventories of the four seats
    int32_t move_counter, mslc, hist_count;
    int8_t cm_rank_floor[NP];
    uint8_t cm_is_gongb[NP], cm_not_gongb[NP], cm_atk_gongb[NP];
    uint8_t lr_is_gongb[2][30], lr_atk_gongb[2][30];
    uint8_t alive[NP];
    int8_t piece_type[NP], piece_seat[NP], pos_x[NP], pos_y[NP], zero_x[NP], zero_y[NP], death_reason[NP];
    uint8_t bel_code[NP];
    uint8_t seat_dead[4], seat_flag[4], rem_tracked[4];
    int8_t turn, observer, terminated, winner, draw;
};

// Copy one field of NP (or n) entries per env between batch rows and a record,
// lanes striding over the entries.
template <typename T>
__device__ __forceinline__ void lane_copy(T *dst, const T *src, int n, int lane) {
    for (int i = lane; i < n; i += 32) dst[i] = src[i];
}

// Warp per env: record of env e for observer seats[e] (NULL: its turn) into
// hist[step * n_envs + e].
__global__ void hist_snapshot_kernel(jq_batch b, const int8_t *__restrict__ seats, HistRec *hist, long long step) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (e >= b.n) return;
    HistRec &R = hist[step * b.n + e];
    const int o = (seats ? seats[e] : b.turn[e]) & 3, left = (o + 1) & 3, right = (o + 3) & 3;
    const size_t q = PI(e, 0), k = OI(e, o, 0);
    lane_copy(R.cm_direct_lo, b.cm_direct_lo + k, NP, lane);
    lane_copy(R.cm_direct_hi, b.cm_direct_hi + k, NP, lane);
    lane_copy(R.cm_chain_lo, b.cm_chain_lo + k, NP, lane);
    lane_copy(R.cm_chain_hi, b.cm_chain_hi + k, NP, lane);
    lane_copy(R.cm_eaten_lo, b.cm_eaten_lo + k, NP, lane);
    lane_copy(R.cm_eaten_hi, b.cm_eaten_hi + k, NP, lane);
    lane_copy(R.cm_direct_type, b.cm_direct_type + k, NP, lane);
    lane_copy(R.cm_chain_type, b.cm_chain_type + k, NP, lane);
    lane_copy(R.cm_last_direct_step, b.cm_last_direct_step + k, NP, lane);
    lane_copy(R.cm_direct_other, b.cm_direct_other + k, NP, lane);
    lane_copy(R.cm_last_chain_step, b.cm_last_chain_step + k, NP, lane);
    lane_copy(R.cm_rank_floor_step, b.cm_rank_floor_step + k, NP, lane);
    lane_copy(R.cm_rank_floor, b.cm_rank_floor + k, NP, lane);
    lane_copy(R.cm_is_gongb, b.cm_is_gongb + k, NP, lane);
    lane_copy(R.cm_not_gongb, b.cm_not_gongb + k, NP, lane);
    lane_copy(R.cm_atk_gongb, b.cm_atk_gongb + k, NP, lane);
    if (lane < 30)
        for (int h = 0; h < 2; ++h) {
            const size_t kk = OI(e, h == 0 ? left : right, o * 30 + lane);
            R.lr_direct_lo[h][lane] = b.cm_direct_lo[kk];
            R.lr_direct_hi[h][lane] = b.cm_direct_hi[kk];
            R.lr_direct_other[h][lane] = b.cm_direct_other[kk];
            R.lr_is_gongb[h][lane] = b.cm_is_gongb[kk];
            R.lr_atk_gongb[h][lane] = b.cm_atk_gongb[kk];
        }
    lane_copy(R.move_count, b.move_count + q, NP, lane);
    lane_copy(R.active_eat, b.active_eat + q, NP, lane);
    lane_copy(R.passive_surv, b.passive_surv + q, NP, lane);
    lane_copy(R.death_step, b.death_step + q, NP, lane);
    lane_copy(R.death_loc, b.death_loc + q, NP, lane);
    lane_copy(R.cell_pid, b.cell_pid + (size_t)e * NC, NC, lane);
    lane_copy(R.hist_src, b.hist_src + (size_t)e * HIST, HIST, lane);
    lane_copy(R.hist_dst, b.hist_dst + (size_t)e * HIST, HIST, lane);
    lane_copy(&R.remaining[0][0], b.remaining + ((size_t)e * 4 + o) * 48, 48, lane);
    lane_copy(R.alive, b.alive + q, NP, lane);
    lane_copy(R.piece_type, b.piece_type + q, NP, lane);
    lane_copy(R.piece_seat, b.piece_seat + q, NP, lane);
    lane_copy(R.pos_x, b.pos_x + q, NP, lane);
    lane_copy(R.pos_y, b.pos_y + q, NP, lane);
    lane_copy(R.zero_x, b.zero_x + q, NP, lane);
    lane_copy(R.zero_y, b.zero_y + q, NP, lane);
    lane_copy(R.death_reason, b.death_reason + q, NP, lane);
    lane_copy(R.bel_code, b.bel_code + k, NP, lane);
    if (lane < 4) {
        R.seat_dead[lane] = b.seat_dead[(size_t)e * 4 + lane];
        R.seat_flag[lane] = b.seat_flag[(size_t)e * 4 + lane];
        R.rem_tracked[lane] = b.rem_tracked[((size_t)e * 4 + o) * 4 + lane];
    }
    if (lane == 0) {
        R.move_counter = b.move_counter[e];
        R.mslc = b.mslc[e];
        R.hist_count = b.hist_count[e];
        R.turn = b.turn[e];
        R.observer = (int8_t)o;
        R.terminated = (int8_t)b.terminated[e];
        R.winner = b.winner[e];
        R.draw = (int8_t)b.draw[e];
    }
}

// Warp per output i: record hist[index[i]] (rejected when out of range: the
// env is left empty) into env i of the scratch batch r.
__global__ void hist_restore_kernel(jq_batch r, const HistRec *hist, long long records,
                                    const long long *__restrict__ index, int8_t *observers) {
    const int lane = threadIdx.x & 31;
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (i >= r.n) return;
    const long long idx = index[i];
    const size_t q = PI(i, 0);
    if (idx < 0 || idx >= records) {  // nothing to restore: an empty, terminated env
        for (int p = lane; p < NP; p += 32) r.alive[q + p] = 0;
        for (int f = lane; f < NC; f += 32) r.cell_pid[(size_t)i * NC + f] = -1;
        if (lane == 0) {
            r.terminated[i] = 1;
            r.turn[i] = 0;
            observers[i] = 0;
        }
        return;
    }
    const HistRec &R = hist[idx];
    const int o = R.observer & 3, left = (o + 1) & 3, right = (o + 3) & 3;
    const size_t k = OI(i, o, 0);
    lane_copy(r.cm_direct_lo + k, R.cm_direct_lo, NP, lane);
    lane_copy(r.cm_direct_hi + k, R.cm_direct_hi, NP, lane);
    lane_copy(r.cm_chain_lo + k, R.cm_chain_lo, NP, lane);
    lane_copy(r.cm_chain_hi + k, R.cm_chain_hi, NP, lane);
    lane_copy(r.cm_eaten_lo + k, R.cm_eaten_lo, NP, lane);
    lane_copy(r.cm_eaten_hi + k, R.cm_eaten_hi, NP, lane);
    lane_copy(r.cm_direct_type + k, R.cm_direct_type, NP, lane);
    lane_copy(r.cm_chain_type + k, R.cm_chain_type, NP, lane);
    lane_copy(r.cm_last_direct_step + k, R.cm_last_direct_step, NP, lane);
    lane_copy(r.cm_direct_other + k, R.cm_direct_other, NP, lane);
    lane_copy(r.cm_last_chain_step + k, R.cm_last_chain_step, NP, lane);
    lane_copy(r.cm_rank_floor_step + k, R.cm_rank_floor_step, NP, lane);
    lane_copy(r.cm_rank_floor + k, R.cm_rank_floor, NP, lane);
    lane_copy(r.cm_is_gongb + k, R.cm_is_gongb, NP, lane);
    lane_copy(r.cm_not_gongb + k, R.cm_not_gongb, NP, lane);
    lane_copy(r.cm_atk_gongb + k, R.cm_atk_gongb, NP, lane);
    if (lane < 30)
        for (int h = 0; h < 2; ++h) {
            const size_t kk = OI(i, h == 0 ? left : right, o * 30 + lane);
            r.cm_direct_lo[kk] = R.lr_direct_lo[h][lane];
            r.cm_direct_hi[kk] = R.lr_direct_hi[h][lane];
            r.cm_direct_other[kk] = R.lr_direct_other[h][lane];
            r.cm_is_gongb[kk] = R.lr_is_gongb[h][lane];
            r.cm_atk_gongb[kk] = R.lr_atk_gongb[h][lane];
        }
    lane_copy(r.move_count + q, R.move_count, NP, lane);
    lane_copy(r.active_eat + q, R.active_eat, NP, lane);
    lane_copy(r.passive_surv + q, R.passive_surv, NP, lane);
    lane_copy(r.death_step + q, R.death_step, NP, lane);
    lane_copy(r.death_loc + q, R.death_loc, NP, lane);
    lane_copy(r.cell_pid + (size_t)i * NC, R.cell_pid, NC, lane);
    lane_copy(r.hist_src + (size_t)i * HIST, R.hist_src, HIST, lane);
    lane_copy(r.hist_dst + (size_t)i * HIST, R.hist_dst, HIST, lane);
    lane_copy(r.remaining + ((size_t)i * 4 + o) * 48, &R.remaining[0][0], 48, lane);
    lane_copy(r.alive + q, R.alive, NP, lane);
    lane_copy(r.piece_type + q, R.piece_type, NP, lane);
    lane_copy(r.piece_seat + q, R.piece_seat, NP, lane);
    lane_copy(r.pos_x + q, R.pos_x, NP, lane);
    lane_copy(r.pos_y + q, R.pos_y, NP, lane);
    lane_copy(r.zero_x + q, R.zero_x, NP, lane);
    lane_copy(r.zero_y + q, R.zero_y, NP, lane);
    lane_copy(r.death_reason + q, R.death_reason, NP, lane);
    lane_copy(r.bel_code + k, R.bel_code, NP, lane);
    if (lane < 4) {
        r.seat_dead[(size_t)i * 4 + lane] = R.seat_dead[lane];
        r.seat_flag[(size_t)i * 4 + lane] = R.seat_flag[lane];
        r.rem_tracked[((size_t)i * 4 + o) * 4 + lane] = R.rem_tracked[lane];
    }
    if (lane == 0) {
        r.move_counter[i] = R.move_counter;
        r.mslc[i] = R.mslc;
        r.hist_count[i] = R.hist_count;
        r.turn[i] = R.turn;
        r.terminated[i] = (uint8_t)R.terminated;
        r.winner[i] = R.winner;
        r.draw[i] = (uint8_t)R.draw;
        observers[i] = (int8_t)o;
    }
}

}  // namespace jq
