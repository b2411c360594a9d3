// jq_obs.cuh -- 317-channel observation encoder (observation.py:598-1651).
//
// One CTA per (env, observer).  The output unit is 317 planes x 289 cells of
// float32 (366,452 B) plus 28 globals, almost all zeros.  The CTA assembles
// CHUNK channels at a time in a shared-memory canvas (scatter of the sparse
// per-piece writes, plane fills for the constant groups), then streams the
// canvas to HBM with 16-byte st.global.cs stores and clears it as it reads,
// so every output byte is written exactly once and no separate zero pass
// exists.  Values are written straight to their canonical cell (the
// observer's rotation applied per cell), which equals the reference's
// world-frame build followed by rotate_planes.
#pragma once
#include "jq_rules.cuh"

namespace jq {

constexpr int OBS_THREADS = 256;
constexpr int CHUNK = 64;  // channels per canvas pass
constexpr int CANVAS_FLOATS = CHUNK * NC + 4;  // +3 floats of alignment slack

struct __align__(16) ObsSmem {
    float canvas[CANVAS_FLOATS];
    uint64_t type_lo[12], type_hi[12];  // observer-own pids of each tracked type
    int16_t rotf[NC];                   // world flat -> canonical flat for this observer
    int16_t hist_s[HIST], hist_d[HIST];
    int32_t dead_const[3], flag_const[4];
};

struct PieceView {
    int alive, seat, ti, cell, team;
    int mcnt, ae, ps;
    int zx, zy;
    int code;
};

__device__ __forceinline__ void bel_vec(int code, float *v) {
#pragma unroll
    for (int t = 0; t < 12; ++t) v[t] = 0.f;
    if (code >= 1 && code <= 12) v[code - 1] = 1.f;
    else if (code == BC_UNIFORM) {
#pragma unroll
        for (int t = 0; t < 12; ++t) v[t] = g_uniform[t];
    } else if (code >= BC_PRIOR0 && code < BC_PRIOR0 + 30) {
#pragma unroll
        for (int t = 0; t < 12; ++t) v[t] = g_prior[(code - BC_PRIOR0) * 12 + t];
    }
}

__device__ __forceinline__ bool in_back_two(int seat, int zx, int zy) {
    switch (seat) {  // observation.py:1378-1387
    case 0: return zy >= 15 && zy <= 16;
    case 2: return zy >= 0 && zy <= 1;
    case 1: return zx >= 0 && zx <= 1;
    case 3: return zx >= 15 && zx <= 16;
    }
    return false;
}

// Writes one observation unit.  `u` indexes the output rows.
__device__ void obs_unit(const jq_batch &b, int e, int o, int mode, float *__restrict__ spatial,
                         float *__restrict__ global, size_t u, ObsSmem &S) {
    const Topo &T = c_topo;
    const int tid = threadIdx.x;
    const int tm = (o + 2) & 3, left = (o + 1) & 3, right = (o + 3) & 3, oteam = o & 1;

    // ---------------- stage per-env data ----------------
    for (int f = tid; f < NC; f += OBS_THREADS) S.rotf[f] = T.rotf[o][f];
    if (tid < HIST) {
        int hc = b.hist_count[e], n = hc < HIST ? hc : HIST;
        int s = -1, d = -1;
        if (tid < n) {
            int slot = (hc - 1 - tid) & (HIST - 1);
            s = b.hist_src[(size_t)e * HIST + slot];
            d = b.hist_dst[(size_t)e * HIST + slot];
        }
        S.hist_s[tid] = (int16_t)s;
        S.hist_d[tid] = (int16_t)d;
    }
    if (tid >= 32 && tid < 44) {
        int t = tid - 32;
        uint64_t lo = 0, hi = 0;
        for (int s = 0; s < 30; ++s) {
            int p = o * 30 + s;
            if (tracked_idx(b.piece_type[PI(e, p)]) == t) set_pid_bit(lo, hi, p);
        }
        S.type_lo[t] = lo;
        S.type_hi[t] = hi;
    }
    if (tid >= 64 && tid < 67) {
        const int ord[3] = {tm, left, right};
        S.dead_const[tid - 64] = b.seat_dead[(size_t)e * 4 + ord[tid - 64]];
    }
    if (tid >= 96 && tid < 100) {
        const int ord[4] = {o, tm, left, right};
        S.flag_const[tid - 96] = b.seat_flag[(size_t)e * 4 + ord[tid - 96]];
    }
    // globals (observation.py:1623-1651)
    if (tid >= 128 && tid < 128 + OBS_GL) {
        int j = tid - 128;
        float v;
        if (j < 24) {
            int side = j < 12 ? left : right;
            v = (float)b.remaining[(size_t)e * 192 + (o * 4 + side) * 12 + (j % 12)];
        } else {
            const int ord[4] = {o, tm, left, right};
            v = b.seat_flag[(size_t)e * 4 + ord[j - 24]] ? 1.f : 0.f;
        }
        global[u * OBS_GL + j] = v;
    }

    __syncthreads();  // rotf and the staged tables are read below

    // per-piece registers (thread p < 120 owns pid p)
    PieceView pv;
    pv.alive = 0;
    pv.cell = -1;
    uint64_t dlo = 0, dhi = 0, clo = 0, chi = 0, elo = 0, ehi = 0;
    int dtype = 0, ctype = 0, other = 0, floor_ = 0, isg = 0, notg = 0, atk = 0;
    int last_d = -1, last_c = -1, last_f = -1;
    int pub = 0, my_isg = 0, my_atk = 0, dead_ch = -1, dead_cell = -1, zero_ch = -1, zero_cell = -1;
    int proj_cell = -1;
    const int cur = b.move_counter[e];
    if (tid < NP) {
        const int p = tid;
        size_t q = PI(e, p);
        pv.alive = b.alive[q];
        pv.seat = b.piece_seat[q];
        pv.team = pv.seat >= 0 ? (pv.seat & 1) : 1;
        pv.ti = tracked_idx(b.piece_type[q]);
        int x = b.pos_x[q], y = b.pos_y[q];
        pv.zx = b.zero_x[q];
        pv.zy = b.zero_y[q];
        if (pv.alive && x >= 0 && x < 17 && y >= 0 && y < 17) pv.cell = S.rotf[y * 17 + x];
        else pv.alive = 0;
        pv.mcnt = b.move_count[q];
        pv.ae = b.active_eat[q];
        pv.ps = b.passive_surv[q];
        pv.code = b.bel_code[OI(e, o, p)];
        size_t k = OI(e, o, p);
        if (pv.alive && pv.team != oteam) {
            dlo = b.cm_direct_lo[k]; dhi = b.cm_direct_hi[k];
            clo = b.cm_chain_lo[k]; chi = b.cm_chain_hi[k];
            dtype = b.cm_direct_type[k]; ctype = b.cm_chain_type[k];
            other = b.cm_direct_other[k]; floor_ = b.cm_rank_floor[k];
            isg = b.cm_is_gongb[k]; notg = b.cm_not_gongb[k]; atk = b.cm_atk_gongb[k];
            last_d = b.cm_last_direct_step[k]; last_c = b.cm_last_chain_step[k]; last_f = b.cm_rank_floor_step[k];
        }
        if (pv.alive && pv.seat == o) {
            size_t kl = OI(e, left, p), kr = OI(e, right, p);
            int lc = __popcll(b.cm_direct_lo[kl]) + __popcll(b.cm_direct_hi[kl]) + b.cm_direct_other[kl];
            int rc = __popcll(b.cm_direct_lo[kr]) + __popcll(b.cm_direct_hi[kr]) + b.cm_direct_other[kr];
            pub = lc < rc ? lc : rc;
            my_isg = b.cm_is_gongb[kl] && b.cm_is_gongb[kr];
            my_atk = b.cm_atk_gongb[kl] || b.cm_atk_gongb[kr];
        }
        if (!b.alive[q] && b.death_step[q] != -1) {  // GameState.deaths keys
            int r = b.death_reason[q];
            int ridx = (r >= 0 && r <= 2) ? r : (r == -1 ? 2 : -1);
            int s = pv.seat;
            int grp = s == o ? 0 : s == tm ? 3 : s == left ? 6 : s == right ? 9 : -1;
            if (ridx >= 0 && b.death_step[q] > 0 && grp >= 0) {
                // numpy index semantics of death_loc // 17, death_loc % 17 (-1 -> row 16, col 16)
                int fl = b.death_loc[q];
                int yy = fl >= 0 ? fl / 17 : -((-fl + 16) / 17), xx = ((fl % 17) + 17) % 17;
                if (yy < 0) yy += 17;
                if (yy >= 0 && yy < 17) { dead_ch = 90 + grp + ridx; dead_cell = S.rotf[yy * 17 + xx]; }
            }
            if (pv.zx >= 0 && pv.zy >= 0 && pv.zx < 17 && pv.zy < 17) {
                zero_ch = 102 + (pv.team == oteam ? 0 : 1);
                zero_cell = S.rotf[pv.zy * 17 + pv.zx];
            }
        }
        if (p / 30 == o) {  // layer 4: observer-own pid projected to its cell or its zero cell
            int px = b.alive[q] ? x : pv.zx, py = b.alive[q] ? y : pv.zy;
            if (px >= 0 && py >= 0 && px < 17 && py < 17) {
                proj_cell = S.rotf[py * 17 + px];
                elo = b.cm_eaten_lo[k];
                ehi = b.cm_eaten_hi[k];
            }
        }
    }
    __syncthreads();

    float *out = spatial + u * (size_t)OBS_FLOATS;
    for (int c0 = 0; c0 < OBS_CH; c0 += CHUNK) {
        const int c1 = c0 + CHUNK < OBS_CH ? c0 + CHUNK : OBS_CH;
        float *g = out + (size_t)c0 * NC;
        const int pad = (int)(((uintptr_t)g >> 2) & 3);
        float *cv = S.canvas + pad;
        auto W = [&](int ch, int cell, float v) {
            if (ch >= c0 && ch < c1) cv[(ch - c0) * NC + cell] = v;
        };
        auto inr = [&](int lo, int hi) { return lo < c1 && hi > c0; };  // group [lo,hi) overlaps chunk

        // ---- constant and static planes (cooperative) ----
        const int k_lo = c0 > 51 ? c0 : 51, k_hi = c1 < 66 ? c1 : 66;
        for (int k = tid; k < (k_hi - k_lo) * NC; k += OBS_THREADS) {
            int ch = k_lo + k / NC, cell = k % NC;
            float v = 0.f;
            if (ch >= 51 && ch < 54) v = S.dead_const[ch - 51] ? 1.f : 0.f;
            else if (ch >= 54 && ch < 58) v = S.flag_const[ch - 54] ? 1.f : 0.f;
            else if (ch == 64) {
                double dp = (double)b.mslc[e] / 200.0;
                v = (float)(dp < 1.0 ? dp : 1.0);
            } else if (ch == 65) {
                double mp = (double)cur / 4000.0;
                v = (float)(mp < 1.0 ? mp : 1.0);
            } else continue;
            if (v != 0.f) cv[(ch - c0) * NC + cell] = v;
        }
        if (inr(58, 63))
            for (int f = tid; f < NC; f += OBS_THREADS) {
                int c = T.f2c[f];
                if (c < 0) continue;
                uint8_t fl = T.flags[c];
                int cc = S.rotf[f];
                if (fl & F_CAMP) W(58, cc, 1.f);
                if (fl & F_SH) W(59, cc, 1.f);
                if (fl & F_RAIL) W(60, cc, 1.f);
                if (fl & F_NINE) W(61, cc, 1.f);
                if (fl & F_ARC) W(62, cc, 1.f);
            }
        // ---- move history (observation.py:1207-1231) ----
        if (inr(129, 161) && tid < HIST && S.hist_s[tid] >= 0 && S.hist_s[tid] < NC && S.hist_d[tid] >= 0 &&
            S.hist_d[tid] < NC) {
            W(129 + tid, S.rotf[S.hist_s[tid]], -1.f);
            W(129 + tid, S.rotf[S.hist_d[tid]], 1.f);
        }
        // ---- per-piece writers ----
        if (tid < NP) {
            if (dead_ch >= 0) W(dead_ch, dead_cell, 1.f);
            if (zero_ch >= 0) W(zero_ch, zero_cell, 1.f);
            if (proj_cell >= 0 && inr(257, 317)) {
                const int opps[2] = {left, right};
                for (int h = 0; h < 2; ++h)
                    for (int s = 0; s < 30; ++s) {
                        int gp = opps[h] * 30 + s;
                        bool on = gp < 64 ? ((elo >> gp) & 1ull) : ((ehi >> (gp - 64)) & 1ull);
                        if (on) W(257 + h * 30 + s, proj_cell, 1.f);
                    }
            }
        }
        if (tid < NP && pv.alive) {
            const int cell = pv.cell, s = pv.seat;
            float v[12];
            if (s == o && pv.ti >= 0) W(pv.ti, cell, 1.f);
            if (s == tm && inr(12, 25)) {
                bel_vec(pv.code, v);
                for (int t = 0; t < 12; ++t) if (v[t] != 0.f) W(12 + t, cell, v[t]);
                if (mode == SM_DARK) W(24, cell, 1.f);
            }
            if (s == left && inr(25, 39)) {
                W(25, cell, 1.f);
                bel_vec(pv.code, v);
                for (int t = 0; t < 12; ++t) if (v[t] != 0.f) W(27 + t, cell, v[t]);
            }
            if (s == right && inr(26, 51)) {
                W(26, cell, 1.f);
                bel_vec(pv.code, v);
                for (int t = 0; t < 12; ++t) if (v[t] != 0.f) W(39 + t, cell, v[t]);
            }
            if (inr(66, 90)) {
                int half = pv.team == oteam ? 0 : 4;
                W(66 + half + (pv.mcnt < 3 ? pv.mcnt : 3), cell, 1.f);
                int ae = pv.ae < 3 ? pv.ae : 3, ps = pv.ps < 3 ? pv.ps : 3;
                for (int k2 = 0; k2 <= ae; ++k2) W(74 + half + k2, cell, 1.f);
                for (int k2 = 0; k2 <= ps; ++k2) W(82 + half + k2, cell, 1.f);
            }
            if (inr(104, 129)) {
                int ch = T.slot_ch[tid % 30];
                W(104 + (ch < 0 ? 24 : ch), cell, 1.f);
            }
            if (pv.team != oteam && inr(161, 257)) {
                // layer 1 (observation.py:1295-1392)
                int mine = __popcll(dlo) + __popcll(dhi);
                for (int g2 = 0; g2 < 3; ++g2) if (mine >= g2 + 1) W(173 + g2, cell, 1.f);
                for (int t = 0; t < 12; ++t) if ((dtype >> t) & 1) W(161 + t, cell, 1.f);
                for (int g2 = 0; g2 < 3; ++g2) if (other >= g2 + 1) W(176 + g2, cell, 1.f);
                int chn = __popcll(clo) + __popcll(chi);
                for (int g2 = 0; g2 < 3; ++g2) if (chn >= g2 + 1) W(191 + g2, cell, 1.f);
                for (int t = 0; t < 12; ++t) if ((ctype >> t) & 1) W(179 + t, cell, 1.f);
                for (int g2 = 0; g2 < 9; ++g2) if (floor_ >= g2 + 1) W(194 + g2, cell, 1.f);
                if (isg) W(203, cell, 1.f);
                if (notg) W(204, cell, 1.f);
                if (in_back_two(s, pv.zx, pv.zy) && pv.mcnt == 0 && !atk) W(205, cell, 1.f);
                // layer 3 (observation.py:1474-1569)
                for (int sl = 0; sl < 30; ++sl) {
                    int gp = o * 30 + sl;
                    bool on = gp < 64 ? ((dlo >> gp) & 1ull) : ((dhi >> (gp - 64)) & 1ull);
                    if (on) W(223 + sl, cell, 1.f);
                }
                for (int t = 0; t < 12; ++t) {
                    int c = __popcll(dlo & S.type_lo[t]) + __popcll(dhi & S.type_hi[t]);
                    if (c > 0) {
                        float val = __fdiv_rn((float)c, 3.0f);
                        W(211 + t, cell, val < 1.f ? val : 1.f);
                    }
                }
                const int lasts[4] = {last_d, last_d, last_c, last_f};
                for (int pl = 0; pl < 4; ++pl) {
                    if (lasts[pl] < 0) continue;
                    int el = cur - lasts[pl];
                    el = el < 0 ? 0 : (el > RECENCY_LEN - 1 ? RECENCY_LEN - 1 : el);
                    float fr = g_recency[pl * RECENCY_LEN + el];
                    if (fr > 0.f) W(253 + pl, cell, fr);
                }
            }
            if (s == o && inr(206, 211)) {  // layer 2 (observation.py:1394-1459)
                for (int g2 = 0; g2 < 3; ++g2) if (pub >= g2 + 1) W(206 + g2, cell, 1.f);
                if (my_isg) W(209, cell, 1.f);
                if (in_back_two(s, pv.zx, pv.zy) && pv.mcnt == 0 && !my_atk) W(210, cell, 1.f);
            }
        }
        __syncthreads();

        // ---- stream the chunk out and clear the canvas behind the reads ----
        const int n = (c1 - c0) * NC;
        const int head = (4 - pad) & 3;
        if (tid < head && tid < n) {
            __stcs(g + tid, cv[tid]);
            cv[tid] = 0.f;
        }
        const int body = (n - head) >> 2;
        float4 *g4 = reinterpret_cast<float4 *>(g + head);
        float4 *c4 = reinterpret_cast<float4 *>(cv + head);
        const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = tid; k < body; k += OBS_THREADS) {
            float4 v4 = c4[k];
            __stcs(g4 + k, v4);
            c4[k] = z4;
        }
        for (int k = head + body * 4 + tid; k < n; k += OBS_THREADS) {
            __stcs(g + k, cv[k]);
            cv[k] = 0.f;
        }
        __syncthreads();
    }
}

// Grid: one CTA per output unit u = e * seats + k.
__global__ void __launch_bounds__(OBS_THREADS, 3) obs_kernel(jq_batch b, const int8_t *__restrict__ observers,
                                                          int seats, int mode, float *spatial, float *global) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ObsSmem &S = *reinterpret_cast<ObsSmem *>(smem_raw);
    // the canvas starts zeroed; every pass leaves it zeroed again
    for (int k = threadIdx.x; k < CANVAS_FLOATS; k += OBS_THREADS) S.canvas[k] = 0.f;
    __syncthreads();
    const size_t units = (size_t)b.n * seats;
    for (size_t u = blockIdx.x; u < units; u += gridDim.x) {
        int e = (int)(u / seats), k = (int)(u % seats);
        int o;
        if (observers) o = observers[u];
        else o = seats == 1 ? b.turn[e] : k;
        o &= 3;
        obs_unit(b, e, o, mode, spatial, global, u, S);
    }
}

}  // namespace jq
