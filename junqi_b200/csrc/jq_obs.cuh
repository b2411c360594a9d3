// jq_obs.cuh -- 317-channel observation encoder (observation.py:598-1651).
//
// One CTA per (env, observer) unit at a time, persistent grid.  A unit is
// 317 planes x 289 cells of float32 (366,452 B) plus 28 globals, almost all
// zeros.  Layout of the work:
//
//  * staging, once per unit: thread p < 120 turns piece p's state into the
//    set of channels it lights with 1.0 -- a 320-bit mask (ten 32-bit words,
//    one per 32-channel chunk) at one canonical cell -- plus the few
//    channels that carry other values (belief vectors, kill counts,
//    recency) and, for a dead piece, its death-reason cell;
//  * ten 32-channel chunks, double-buffered in shared memory: scatter a
//    chunk (one mask word per piece, plane fills for the constant groups),
//    then one thread streams the chunk's 16-byte-aligned body to HBM with a
//    TMA bulk store (cp.async.bulk ... bulk_group, L2 evict-first) while the
//    CTA scatters the next chunk into the other buffer.  The 0-3 floats
//    either side of the aligned body go out as plain stores.  A buffer is
//    cleared after its bulk store has read it (cp.async.bulk.wait_group.read).
//
// Every output byte is written once; values go straight to their canonical
// cell (the observer's rotation applied per cell), which equals the
// reference's world-frame build followed by rotate_planes.
#pragma once
#include "jq_rules.cuh"

namespace jq {

constexpr int OBS_THREADS = 256;
constexpr int CHUNK = 32;                                // channels per buffer (= one mask word)
constexpr int NCHUNK = (OBS_CH + CHUNK - 1) / CHUNK;     // 10
constexpr int BUF_FLOATS = CHUNK * NC + 4;               // +3 floats of alignment slack, 16-byte multiple
static_assert(BUF_FLOATS % 4 == 0, "buffers must keep 16-byte alignment");

struct __align__(16) ObsSmem {
    float buf[2][BUF_FLOATS];
    uint64_t type_lo[12], type_hi[12];  // observer-own pids of each tracked type
    int16_t rotf[NC];                   // world flat -> canonical flat for this observer
    int16_t hist_s[HIST], hist_d[HIST];
    int32_t dead_const[3], flag_const[4];
};

__device__ __forceinline__ void setb(uint32_t *m, int ch) { m[ch >> 5] |= 1u << (ch & 31); }

__device__ __forceinline__ bool in_back_two(int seat, int zx, int zy) {
    switch (seat) {  // observation.py:1378-1387
    case 0: return zy >= 15 && zy <= 16;
    case 2: return zy >= 0 && zy <= 1;
    case 1: return zx >= 0 && zx <= 1;
    case 3: return zx >= 15 && zx <= 16;
    }
    return false;
}

__device__ __forceinline__ float bel_value(int code, int t) {
    if (code >= 1 && code <= 12) return code - 1 == t ? 1.f : 0.f;
    if (code == BC_UNIFORM) return g_uniform[t];
    if (code >= BC_PRIOR0 && code < BC_PRIOR0 + 30) return g_prior[(code - BC_PRIOR0) * 12 + t];
    return 0.f;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void bulk_store(float *gdst, const float *ssrc, uint32_t bytes, uint64_t policy) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;"
                 :: "l"(gdst), "r"(smem_addr(ssrc)), "r"(bytes), "l"(policy) : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Per-piece write set of one unit (thread p < 120 holds piece p's).
struct PieceWrites {
    uint32_t ones[NCHUNK];  // channels lit with 1.0 at cellA
    int cellA;              // canonical cell, -1 none
    int cellB, chB;         // death-reason write of a dead piece
    int bel_base;           // 12 / 27 / 39 for teammate / left / right beliefs, -1 none
    int code;               // belief code of the piece for this observer
    uint32_t kill3;         // per tracked type: min(count, 3) in 2 bits (channels 211..222)
    float rec[4];           // recency values (channels 253..256), 0 = none
};

__device__ void stage_piece(const jq_batch &b, int e, int o, int mode, const ObsSmem &S, int p, PieceWrites &pw) {
    const int tm = (o + 2) & 3, left = (o + 1) & 3, right = (o + 3) & 3, oteam = o & 1;
#pragma unroll
    for (int i = 0; i < NCHUNK; ++i) pw.ones[i] = 0;
    pw.cellA = pw.cellB = pw.chB = pw.bel_base = -1;
    pw.code = 0;
    pw.kill3 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) pw.rec[i] = 0.f;
    const size_t q = PI(e, p), k = OI(e, o, p);
    const int alive_raw = b.alive[q];
    const int s = b.piece_seat[q];
    const int team = s >= 0 ? (s & 1) : 1;  // numpy _SEAT_TEAM[-1] is EAST's team
    const int x = b.pos_x[q], y = b.pos_y[q], zx = b.zero_x[q], zy = b.zero_y[q];
    const int mcnt = b.move_count[q];
    const bool own_pid = (p / 30) == o;
    if (alive_raw) {
        if (!(x >= 0 && x < 17 && y >= 0 && y < 17)) return;
        pw.cellA = S.rotf[y * 17 + x];
        const int ti = tracked_idx(b.piece_type[q]);
        pw.code = b.bel_code[k];
        if (s == o && ti >= 0) setb(pw.ones, ti);
        if (s == tm) {
            pw.bel_base = 12;
            if (mode == SM_DARK) setb(pw.ones, 24);
        }
        if (s == left) { setb(pw.ones, 25); pw.bel_base = 27; }
        if (s == right) { setb(pw.ones, 26); pw.bel_base = 39; }
        const int half = team == oteam ? 0 : 4;
        setb(pw.ones, 66 + half + (mcnt < 3 ? mcnt : 3));
        const int ae = b.active_eat[q] < 3 ? b.active_eat[q] : 3, ps = b.passive_surv[q] < 3 ? b.passive_surv[q] : 3;
        for (int g = 0; g <= ae; ++g) setb(pw.ones, 74 + half + g);
        for (int g = 0; g <= ps; ++g) setb(pw.ones, 82 + half + g);
        const int sch = c_topo.slot_ch[p % 30];
        setb(pw.ones, 104 + (sch < 0 ? 24 : sch));
        if (team != oteam) {
            // layer 1 + 3 (observation.py:1295-1392, 1474-1569)
            const uint64_t dlo = b.cm_direct_lo[k], dhi = b.cm_direct_hi[k];
            const uint64_t clo = b.cm_chain_lo[k], chi = b.cm_chain_hi[k];
            const int dtype = b.cm_direct_type[k], ctype = b.cm_chain_type[k];
            const int other = b.cm_direct_other[k], fl = b.cm_rank_floor[k];
            const int mine = __popcll(dlo) + __popcll(dhi), chn = __popcll(clo) + __popcll(chi);
            for (int g = 0; g < 3; ++g) {
                if (mine >= g + 1) setb(pw.ones, 173 + g);
                if (other >= g + 1) setb(pw.ones, 176 + g);
                if (chn >= g + 1) setb(pw.ones, 191 + g);
            }
            for (int t = 0; t < 12; ++t) {
                if ((dtype >> t) & 1) setb(pw.ones, 161 + t);
                if ((ctype >> t) & 1) setb(pw.ones, 179 + t);
            }
            for (int g = 0; g < 9; ++g)
                if (fl >= g + 1) setb(pw.ones, 194 + g);
            if (b.cm_is_gongb[k]) setb(pw.ones, 203);
            if (b.cm_not_gongb[k]) setb(pw.ones, 204);
            if (in_back_two(s, zx, zy) && mcnt == 0 && !b.cm_atk_gongb[k]) setb(pw.ones, 205);
            for (int sl = 0; sl < 30; ++sl) {
                const int gp = o * 30 + sl;
                const bool on = gp < 64 ? ((dlo >> gp) & 1ull) : ((dhi >> (gp - 64)) & 1ull);
                if (on) setb(pw.ones, 223 + sl);
            }
            for (int t = 0; t < 12; ++t) {
                const int c = __popcll(dlo & S.type_lo[t]) + __popcll(dhi & S.type_hi[t]);
                pw.kill3 |= (uint32_t)(c < 3 ? c : 3) << (2 * t);
            }
            const int cur = b.move_counter[e];
            const int lasts[4] = {b.cm_last_direct_step[k], b.cm_last_direct_step[k], b.cm_last_chain_step[k],
                                  b.cm_rank_floor_step[k]};
#pragma unroll
            for (int pl = 0; pl < 4; ++pl) {
                if (lasts[pl] < 0) continue;
                int el = cur - lasts[pl];
                el = el < 0 ? 0 : (el > RECENCY_LEN - 1 ? RECENCY_LEN - 1 : el);
                pw.rec[pl] = g_recency[pl * RECENCY_LEN + el];
            }
        }
        if (s == o) {  // layer 2 (observation.py:1394-1459)
            const size_t kl = OI(e, left, p), kr = OI(e, right, p);
            const int lc = __popcll(b.cm_direct_lo[kl]) + __popcll(b.cm_direct_hi[kl]) + b.cm_direct_other[kl];
            const int rc = __popcll(b.cm_direct_lo[kr]) + __popcll(b.cm_direct_hi[kr]) + b.cm_direct_other[kr];
            const int pub = lc < rc ? lc : rc;
            for (int g = 0; g < 3; ++g)
                if (pub >= g + 1) setb(pw.ones, 206 + g);
            if (b.cm_is_gongb[kl] && b.cm_is_gongb[kr]) setb(pw.ones, 209);
            const bool patk = b.cm_atk_gongb[kl] || b.cm_atk_gongb[kr];
            if (in_back_two(s, zx, zy) && mcnt == 0 && !patk) setb(pw.ones, 210);
        }
    } else {
        if (b.death_step[q] != -1) {  // GameState.deaths keys
            const int r = b.death_reason[q];
            const int ridx = (r >= 0 && r <= 2) ? r : (r == -1 ? 2 : -1);
            const int grp = s == o ? 0 : s == tm ? 3 : s == left ? 6 : s == right ? 9 : -1;
            if (ridx >= 0 && b.death_step[q] > 0 && grp >= 0) {
                // numpy index semantics of death_loc // 17, death_loc % 17 (-1 -> row 16, col 16)
                const int f = b.death_loc[q];
                int yy = f >= 0 ? f / 17 : -((-f + 16) / 17);
                const int xx = ((f % 17) + 17) % 17;
                if (yy < 0) yy += 17;
                if (yy >= 0 && yy < 17) { pw.chB = 90 + grp + ridx; pw.cellB = S.rotf[yy * 17 + xx]; }
            }
        }
        if (!(zx >= 0 && zx < 17 && zy >= 0 && zy < 17)) return;
        pw.cellA = S.rotf[zy * 17 + zx];
        if (b.death_step[q] != -1) setb(pw.ones, 102 + (team == oteam ? 0 : 1));
    }
    if (own_pid) {  // layer 4: observer-own pid at its cell (alive) or zero cell (dead)
        const uint64_t elo = b.cm_eaten_lo[k], ehi = b.cm_eaten_hi[k];
        const int opps[2] = {left, right};
        for (int h = 0; h < 2; ++h)
            for (int sl = 0; sl < 30; ++sl) {
                const int gp = opps[h] * 30 + sl;
                const bool on = gp < 64 ? ((elo >> gp) & 1ull) : ((ehi >> (gp - 64)) & 1ull);
                if (on) setb(pw.ones, 257 + h * 30 + sl);
            }
    }
}

// Grid: persistent; CTA-stride over output units u = e * seats + k.
__global__ void __launch_bounds__(OBS_THREADS, 3) obs_kernel(jq_batch b, const int8_t *__restrict__ observers,
                                                             int seats, int mode, float *spatial, float *global) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ObsSmem &S = *reinterpret_cast<ObsSmem *>(smem_raw);
    const int tid = threadIdx.x;
    uint64_t policy = 0;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    for (int k = tid; k < 2 * BUF_FLOATS; k += OBS_THREADS) (&S.buf[0][0])[k] = 0.f;
    int qn = 0;  // chunks issued by this CTA so far (selects the buffer)
    const size_t units = (size_t)b.n * seats;
    for (size_t u = blockIdx.x; u < units; u += gridDim.x) {
        const int e = (int)(u / seats);
        int o = observers ? observers[u] : (seats == 1 ? b.turn[e] : (int)(u % seats));
        o &= 3;
        const int tm = (o + 2) & 3, left = (o + 1) & 3, right = (o + 3) & 3;
        // ---------------- staging ----------------
        __syncthreads();  // previous unit's readers of the staged tables are done
        for (int f = tid; f < NC; f += OBS_THREADS) S.rotf[f] = c_topo.rotf[o][f];
        if (tid < HIST) {
            const int hc = b.hist_count[e], n = hc < HIST ? hc : HIST;
            int s = -1, d = -1;
            if (tid < n) {
                const int slot = (hc - 1 - tid) & (HIST - 1);
                s = b.hist_src[(size_t)e * HIST + slot];
                d = b.hist_dst[(size_t)e * HIST + slot];
                if (s < 0 || s >= NC || d < 0 || d >= NC) s = d = -1;
            }
            S.hist_s[tid] = (int16_t)s;
            S.hist_d[tid] = (int16_t)d;
        }
        if (tid >= 32 && tid < 44) {
            const int t = tid - 32;
            uint64_t lo = 0, hi = 0;
            for (int s = 0; s < 30; ++s)
                if (tracked_idx(b.piece_type[PI(e, o * 30 + s)]) == t) set_pid_bit(lo, hi, o * 30 + s);
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
        if (tid >= 128 && tid < 128 + OBS_GL) {  // globals (observation.py:1623-1651)
            const int j = tid - 128;
            float v;
            if (j < 24) {
                v = (float)b.remaining[(size_t)e * 192 + (o * 4 + (j < 12 ? left : right)) * 12 + (j % 12)];
            } else {
                const int ord[4] = {o, tm, left, right};
                v = b.seat_flag[(size_t)e * 4 + ord[j - 24]] ? 1.f : 0.f;
            }
            global[u * OBS_GL + j] = v;
        }
        const float prog_d = (float)fmin((double)b.mslc[e] / 200.0, 1.0);
        const float prog_m = (float)fmin((double)b.move_counter[e] / 4000.0, 1.0);
        __syncthreads();
        PieceWrites pw;
        if (tid < NP) stage_piece(b, e, o, mode, S, tid, pw);
        else pw.cellA = pw.cellB = -1;

        float *out = spatial + u * (size_t)OBS_FLOATS;
        for (int c = 0; c < NCHUNK; ++c, ++qn) {
            float *B = S.buf[qn & 1];
            const int c0 = c * CHUNK, c1 = c0 + CHUNK < OBS_CH ? c0 + CHUNK : OBS_CH;
            float *g = out + (size_t)c0 * NC;
            const int pad = (int)(((uintptr_t)g >> 2) & 3);
            float *cv = B + pad;
            // ---- buffer reuse: the bulk store issued two chunks ago from B must have read it ----
            if (qn >= 2) {
                if (tid == 0) bulk_wait_read_le1();
                __syncthreads();
                float4 *B4 = reinterpret_cast<float4 *>(B);
                const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int k2 = tid; k2 < BUF_FLOATS / 4; k2 += OBS_THREADS) B4[k2] = z4;
                __syncthreads();
            }
            // ---- scatter ----
            if (pw.cellA >= 0) {
                uint32_t m = pw.ones[c];
                while (m) {
                    const int bit = __ffs(m) - 1;
                    m &= m - 1;
                    cv[bit * NC + pw.cellA] = 1.f;
                }
                if (pw.bel_base >= 0 && pw.bel_base < c1 && pw.bel_base + 12 > c0)
                    for (int t = 0; t < 12; ++t) {
                        const int ch = pw.bel_base + t;
                        if (ch < c0 || ch >= c1) continue;
                        const float v = bel_value(pw.code, t);
                        if (v != 0.f) cv[(ch - c0) * NC + pw.cellA] = v;
                    }
                if (pw.kill3 && 211 < c1 && 223 > c0)
                    for (int t = 0; t < 12; ++t) {
                        const int ch = 211 + t, cnt = (pw.kill3 >> (2 * t)) & 3;
                        if (cnt && ch >= c0 && ch < c1) cv[(ch - c0) * NC + pw.cellA] = __fdiv_rn((float)cnt, 3.0f);
                    }
                if (253 < c1 && 257 > c0)
#pragma unroll
                    for (int pl = 0; pl < 4; ++pl) {
                        const int ch = 253 + pl;
                        if (pw.rec[pl] > 0.f && ch >= c0 && ch < c1) cv[(ch - c0) * NC + pw.cellA] = pw.rec[pl];
                    }
            }
            if (pw.cellB >= 0 && pw.chB >= c0 && pw.chB < c1) cv[(pw.chB - c0) * NC + pw.cellB] = 1.f;
            if (tid >= 128 && tid < 128 + HIST) {  // move history (observation.py:1207-1231)
                const int d = tid - 128, ch = 129 + d;
                if (ch >= c0 && ch < c1 && S.hist_s[d] >= 0) {
                    cv[(ch - c0) * NC + S.rotf[S.hist_s[d]]] = -1.f;
                    cv[(ch - c0) * NC + S.rotf[S.hist_d[d]]] = 1.f;
                }
            }
            // constant planes (observation.py:984-1021) and board statics (343-383)
            const int k_lo = c0 > 51 ? c0 : 51, k_hi = c1 < 66 ? c1 : 66;
            for (int k2 = tid; k2 < (k_hi - k_lo) * NC; k2 += OBS_THREADS) {
                const int ch = k_lo + k2 / NC, cell = k2 % NC;
                float v = 0.f;
                if (ch < 54) v = S.dead_const[ch - 51] ? 1.f : 0.f;
                else if (ch < 58) v = S.flag_const[ch - 54] ? 1.f : 0.f;
                else if (ch == 64) v = prog_d;
                else if (ch == 65) v = prog_m;
                else continue;
                if (v != 0.f) cv[(ch - c0) * NC + cell] = v;
            }
            if (58 < c1 && 63 > c0)
                for (int f = tid; f < NC; f += OBS_THREADS) {
                    const int cc = c_topo.f2c[f];
                    if (cc < 0) continue;
                    const uint8_t fl = c_topo.flags[cc];
                    const int cell = S.rotf[f];
                    const int bits[5] = {F_CAMP, F_SH, F_RAIL, F_NINE, F_ARC};
#pragma unroll
                    for (int i = 0; i < 5; ++i)
                        if ((fl & bits[i]) && 58 + i >= c0 && 58 + i < c1) cv[(58 + i - c0) * NC + cell] = 1.f;
                }
            fence_async_smem();
            __syncthreads();
            // ---- stream the chunk: aligned body by TMA bulk store, 0-3 floats each side plainly ----
            const int n = (c1 - c0) * NC;
            const int head = (4 - pad) & 3;
            const int body = ((n - head) >> 2) << 2;
            if (tid == 0 && body > 0) bulk_store(g + head, cv + head, (uint32_t)body * 4u, policy);
            if (tid >= 32 && tid < 32 + head) __stcs(g + (tid - 32), cv[tid - 32]);
            if (tid >= 64 && tid < 64 + (n - head - body)) {
                const int j = head + body + (tid - 64);
                __stcs(g + j, cv[j]);
            }
        }
    }
    if (tid == 0) bulk_wait_all();
    __syncthreads();
}

}  // namespace jq
