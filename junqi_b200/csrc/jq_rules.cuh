// jq_rules.cuh -- per-env game rules, executed by one warp per env.
//
// Semantics are those of junqi_core's BatchedGameState (the state contract):
//   step_batch / _step_single   batched_state.py:417-613, 739-980
//   _advance_turn(_vec)         batched_state.py:615-686, 1123-1169
//   _check_victory(_vec)        batched_state.py:688-733, 1171-1214
//   legal_action_ids_batch      batched_state.py:370-409 -> move_gen.py:1311-1553
//   move_requires_gongb         move_gen.py:245-296
//   apply_combat_event          combat_memory.py:354-562
//   BeliefTensor.initial/update info_model.py:218-414 (per-piece belief codes)
//   GameState.new_game          state.py:490-624 (device reset)
//
// Layout of the work: lane 0 carries the scalar part of a ply (move or
// combat, Zobrist, combat memory); the whole warp joins for the collective
// parts -- the Q12 "has any legal move" checks, seat surrenders, the belief
// sweep, resets and legal-move generation, where each of lanes 0..29 owns one
// piece of the acting seat and computes its destination set as a 129-bit
// mask over the compact board (an engineer's rail run as a frontier
// expansion over per-cell rail-neighbour masks in its own lane; the
// path-revealed-engineer check of a move, which has one walk to do, as the
// same expansion by the whole warp).
#pragma once
#include "jq_common.cuh"
#include "jq_trace.cuh"

namespace jq {

constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------------------
// Device tables (filled by the host API, see jq_api.cu)
// ---------------------------------------------------------------------------
__device__ Topo g_topo;  // same tables in global memory, for per-lane (divergent) reads
__constant__ int64_t c_zturn[4], c_zwin[3], c_zsdead[4], c_zsflag[4], c_zshow[4];
__constant__ int64_t c_zterm, c_zdraw;
__device__ int64_t g_zpiece[NP * 14 * NC];
__device__ int64_t g_zmc[4096];
__device__ int64_t g_zmslc[512];
__device__ float g_prior[30 * 12];
__device__ float g_uniform[12];
__device__ float g_recency[4 * RECENCY_LEN];

// Zobrist piece term; out-of-range arguments (only reachable from states
// written by a caller, never by the rules) contribute nothing.
__device__ __forceinline__ int64_t zpiece(int pid, int t, int f) {
    if ((unsigned)pid >= (unsigned)NP || (unsigned)t >= 14u || (unsigned)f >= (unsigned)NC) return 0;
    return g_zpiece[((size_t)pid * 14 + t) * NC + f];
}

// ---------------------------------------------------------------------------
// Per-warp shared-memory image of one env
// ---------------------------------------------------------------------------
struct StepCtx {
    int64_t z_tail;  // Zobrist keys of the post-ply move counter and no-combat counter
    int skip, ev, A, D, sf, df, acting, A_type, A_seat, D_type, D_seat;
    int mc, mslc, new_mc, new_mslc, fcap, fr_src, fr_dst, other_pid, term, win, draw;
    int new_turn, need_surrender, do_q12, combat, full_advance;
    int inv_async;  // the inventories are being copied into shared memory (cp.async)
    int cm;  // combat-memory update after the scalar part: 0 none, 1 EAT, 2 KILLED
    int died_pre[4];
};

// words of the canonical-mask bitstream: 16,641 bits, plus one zero word so
// a 16-bit window starting in the last word can read its successor
constexpr int CBW = (MASK_BYTES + 31) / 32 + 1;

struct __align__(16) WEnv {
    uint32_t cbits[CBW];     // the canonical mask as one row-major bitstream (bit j = mask byte j)
    alignas(16) uint8_t bel[4 * NP];  // belief codes (observer-major), loaded with the state for a step
    alignas(16) int16_t rem[4 * 4 * 12];  // enemy inventories (observer, seat, type), loaded when a ply changes them
    alignas(16) uint8_t rtr[16];          // their tracked flags (observer, seat)
    uint64_t cmv[4][4];      // V's combat-memory sets per observer: direct lo/hi, chain lo/hi
    int32_t scan[32];
    StepCtx x;
    int16_t cell[NC + 1];    // flat cell -> pid
    int16_t posc[NP];        // pid -> compact cell or -1
    int8_t type[NP];
    int8_t seat[NP];
    uint8_t alive[NP];
    uint8_t sdead[4];
    // the env's scalars as loaded before the ply (read by the step)
    int64_t s_zob;
    int32_t s_mc, s_mslc, s_hc;
    int8_t s_turn, s_term, s_win, s_draw;
    uint8_t sflag[4];  // seat_flag, kept in step with the global copy during the ply
};

// 16-byte global -> shared copy that does not pass through registers
// (cp.async.cg: L2 only); both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

__device__ __forceinline__ size_t PI(int e, int p) { return (size_t)e * NP + p; }
__device__ __forceinline__ size_t OI(int e, int o, int p) { return ((size_t)e * 4 + o) * NP + p; }

// Every load is issued before any shared-memory store, so the warp waits
// for global memory once.  with_bel: also the env's 480 belief codes, read
// and rewritten by the step's belief update.
__device__ void warp_load(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int lane, bool with_bel) {
    constexpr int CI = (NC + 31) / 32, PIT = (NP + 31) / 32;
    int cp[CI];
#pragma unroll
    for (int i = 0; i < CI; ++i) {
        const int f = lane + 32 * i;
        cp[i] = f < NC ? b.cell_pid[(size_t)e * NC + f] : -1;
    }
    int al[PIT], ty[PIT], se[PIT], px[PIT], py[PIT];
#pragma unroll
    for (int i = 0; i < PIT; ++i) {
        const int p = lane + 32 * i;
        if (p < NP) {
            const size_t q = PI(e, p);
            al[i] = b.alive[q];
            ty[i] = b.piece_type[q];
            se[i] = b.piece_seat[q];
            px[i] = b.pos_x[q];
            py[i] = b.pos_y[q];
        }
    }
    uint4 bel = make_uint4(0u, 0u, 0u, 0u);
    if (with_bel && lane < 4 * NP / 16) bel = reinterpret_cast<const uint4 *>(b.bel_code + OI(e, 0, 0))[lane];
    int64_t sc = 0;
    switch (lane) {
    case 0: sc = b.terminated[e]; break;
    case 1: sc = b.turn[e]; break;
    case 2: sc = b.move_counter[e]; break;
    case 3: sc = b.mslc[e]; break;
    case 4: sc = b.zobrist[e]; break;
    case 5: sc = b.hist_count[e]; break;
    case 6: sc = b.winner[e]; break;
    case 7: sc = b.draw[e]; break;
    case 8: case 9: case 10: case 11: sc = b.seat_dead[(size_t)e * 4 + lane - 8]; break;
    case 12: case 13: case 14: case 15: sc = b.seat_flag[(size_t)e * 4 + lane - 12]; break;
    default: break;
    }
#pragma unroll
    for (int i = 0; i < CI; ++i) {
        const int f = lane + 32 * i;
        if (f < NC) w.cell[f] = (int16_t)((cp[i] >= 0 && cp[i] < NP) ? cp[i] : -1);
    }
#pragma unroll
    for (int i = 0; i < PIT; ++i) {
        const int p = lane + 32 * i;
        if (p < NP) {
            w.alive[p] = (uint8_t)al[i];
            w.type[p] = (int8_t)ty[i];
            w.seat[p] = (int8_t)se[i];
            w.posc[p] = (int16_t)((px[i] >= 0 && px[i] < 17 && py[i] >= 0 && py[i] < 17) ? T.f2c[py[i] * 17 + px[i]] : -1);
        }
    }
    switch (lane) {
    case 0: w.s_term = (int8_t)sc; break;
    case 1: w.s_turn = (int8_t)sc; break;
    case 2: w.s_mc = (int32_t)sc; break;
    case 3: w.s_mslc = (int32_t)sc; break;
    case 4: w.s_zob = sc; break;
    case 5: w.s_hc = (int32_t)sc; break;
    case 6: w.s_win = (int8_t)sc; break;
    case 7: w.s_draw = (int8_t)sc; break;
    case 8: case 9: case 10: case 11: w.sdead[lane - 8] = (uint8_t)sc; break;
    case 12: case 13: case 14: case 15: w.sflag[lane - 12] = (uint8_t)sc; break;
    default: break;
    }
    if (with_bel && lane < 4 * NP / 16) reinterpret_cast<uint4 *>(w.bel)[lane] = bel;
    __syncwarp();
}

// ---------------------------------------------------------------------------
// Legal moves
// ---------------------------------------------------------------------------
// Destination mask of one piece standing on compact cell c (move_gen.py:
// 1311-1553 restricted to one candidate piece).
__device__ void piece_dsts(const TopoCore &T, int c, int t, const uint32_t (&empty)[NW], const uint32_t (&land)[NW],
                           uint32_t (&out)[NW]) {
#pragma unroll
    for (int i = 0; i < NW; ++i) out[i] = 0;
    if (c < 0 || t == JUNQI || t == DILEI || (T.flags[c] & F_SH)) return;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int nb = T.adj4[c][k];
        if (nb != NONE8 && rbit(land, nb)) rset(out, nb);
        nb = T.diag[c][k];
        if (nb != NONE8 && rbit(land, nb)) rset(out, nb);
    }
    if (!(T.flags[c] & F_RAIL)) return;
    if (t == GONGB) {
        // engineer: cells adjacent to the set reached through empty rail
        // cells, one lane per engineer (the side's engineers expand at once)
        uint32_t reach[NW], fr[NW], landing[NW];
#pragma unroll
        for (int i = 0; i < NW; ++i) reach[i] = fr[i] = landing[i] = 0;
        rset(reach, c);
        rset(fr, c);
        for (int it = 0; it < NB; ++it) {
            uint32_t nbm[NW] = {0, 0, 0, 0, 0};
#pragma unroll
            for (int wd = 0; wd < NW; ++wd) {
                uint32_t m = fr[wd];
                while (m) {
                    int v = wd * 32 + __ffs(m) - 1;
                    m &= m - 1;
                    const uint4 *row = reinterpret_cast<const uint4 *>(T.railnb[v]);
                    const uint4 r0 = row[0], r1 = row[1];
                    nbm[0] |= r0.x;
                    nbm[1] |= r0.y;
                    nbm[2] |= r0.z;
                    nbm[3] |= r0.w;
                    nbm[4] |= r1.x;
                }
            }
            uint32_t any = 0;
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                landing[i] |= nbm[i] & land[i];
                uint32_t nw = nbm[i] & empty[i] & ~reach[i];
                reach[i] |= nw;
                fr[i] = nw;
                any |= nw;
            }
            if (!any) break;
        }
#pragma unroll
        for (int i = 0; i < NW; ++i) landing[i] &= (c >> 5) == i ? ~(1u << (c & 31)) : ~0u;
#pragma unroll
        for (int i = 0; i < NW; ++i) out[i] |= landing[i];
    } else {
        // straight rays as masks: the cells up to and including the first
        // occupied one (the nearest blocker is the lowest set bit on rays of
        // increasing index, the highest on the others), then those a piece
        // may land on -- the same set as walking the ray cell by cell
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t r[NW];
#pragma unroll
            for (int i = 0; i < NW; ++i) r[i] = T.ray[c][k][i];
            int stop = (k & 1) ? -1 : (1 << 20);  // no blocker: the whole ray
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                const int ii = (k & 1) ? i : NW - 1 - i;  // the nearest blocker is seen last
                const uint32_t bl = r[ii] & ~empty[ii];
                if (bl) stop = (k & 1) ? ii * 32 + 31 - __clz(bl) : ii * 32 + __ffs(bl) - 1;
            }
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                const int lim = stop - i * 32;
                const uint32_t keep = (k & 1) ? (lim <= 0 ? ~0u : (lim > 31 ? 0u : ~((1u << lim) - 1u)))
                                              : (lim < 0 ? 0u : (lim >= 31 ? ~0u : (2u << lim) - 1u));
                out[i] |= r[i] & keep & land[i];
            }
        }
        if (T.flags[c] & F_CURVE_ACTIVE)
            for (int k = 0; k < 2; ++k)
                for (int l = 0; l < 11; ++l) {
                    int nb = T.cray[c][k][l];
                    if (nb == NONE8) break;
                    if (rbit(land, nb)) rset(out, nb);
                    if (!rbit(empty, nb)) break;
                }
    }
}

__device__ __forceinline__ void board_masks(const TopoCore &T, const WEnv &w, int lane, int team, uint32_t *empty,
                                            uint32_t *land) {
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        int c = i * 32 + lane;
        bool em = false, at = false;
        if (c < NB) {
            int p = w.cell[T.c2f[c]];
            em = p < 0;
            at = p >= 0 && team_of_pid(p) != team && !(T.flags[c] & F_CAMP);
        }
        empty[i] = __ballot_sync(FULL, em);
        land[i] = __ballot_sync(FULL, em || at);
    }
}

// Source cell of lane's piece for `seat`, or -1.
__device__ __forceinline__ int lane_source(const WEnv &w, int lane, int seat) {
    if (lane >= 30) return -1;
    int p = seat * 30 + lane;
    if (!w.alive[p] || w.seat[p] != seat) return -1;
    return w.posc[p];
}

// has_legal_moves_soa (move_gen.py:1557-1609): any legal action for `seat`,
// ignoring terminated / dead flags.
__device__ bool warp_has_moves(const TopoCore &T, const WEnv &w, int lane, int seat, int *full_scans = nullptr) {
    uint32_t empty[NW], land[NW], d[NW];
    board_masks(T, w, lane, seat & 1, empty, land);
    int src = lane_source(w, lane, seat);
    // A one-step (orthogonal or camp-diagonal) move of a movable piece is a
    // legal move on its own; only when no piece has one is the full
    // destination set (rail rays, engineer flood-fill) needed.
    bool quick = false;
    if (src >= 0) {
        const int t = w.type[seat * 30 + lane];
        if (t != JUNQI && t != DILEI && !(T.flags[src] & F_SH))
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int a = T.adj4[src][k], g = T.diag[src][k];
                quick |= (a != NONE8 && rbit(land, a)) || (g != NONE8 && rbit(land, g));
            }
    }
    if (__any_sync(FULL, quick)) return true;
    if (full_scans) ++*full_scans;
    bool any = false;
    if (src >= 0) {
        piece_dsts(T, src, w.type[seat * 30 + lane], empty, land, d);
        any = (d[0] | d[1] | d[2] | d[3] | d[4]) != 0;
    }
    return __any_sync(FULL, any);
}

// 4 mask bits -> 4 bytes of 0/1 (bit i -> byte i).
__device__ __forceinline__ uint32_t nibble_bytes(uint32_t nib) { return (nib * 0x00204081u) & 0x01010101u; }

// Mask bytes j0 .. j0 + 31 from the bitstream as one 32-byte store (p is
// 32-byte aligned).
__device__ __forceinline__ void mask_store32(uint8_t *p, const WEnv &w, int j0) {
    const int wi = j0 >> 5;
    const uint32_t bits = __funnelshift_r(w.cbits[wi], w.cbits[wi + 1], j0 & 31);
    uint32_t v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = nibble_bytes((bits >> (4 * i)) & 15u);
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// Legal actions of `seat` (empty when `skip`), ascending, written to ids
// (up to cap); optional canonical (16641) byte mask.  Returns the count on
// every lane.
__device__ int warp_legal(const TopoCore &T, WEnv &w, int lane, int seat, bool skip, int32_t *ids, int cap,
                          uint8_t *mask_env, bool traced = false) {
    uint32_t empty[NW], land[NW], d[NW] = {0, 0, 0, 0, 0};
    board_masks(T, w, lane, seat & 1, empty, land);
    int src = skip ? -1 : lane_source(w, lane, seat);
    if (src >= 0) piece_dsts(T, src, w.type[seat * 30 + lane], empty, land, d);
    int cnt = __popc(d[0]) + __popc(d[1]) + __popc(d[2]) + __popc(d[3]) + __popc(d[4]);
    if (traced) JQ_TRACE_AT(1, TR_DSTS);  // lane 0 only: no warp barrier here
#ifdef JQ_TRACE
    {  // every lane: the warp reductions stay outside the lane-0 block
        const bool eng = src >= 0 && w.type[seat * 30 + lane] == GONGB;
        const uint64_t ne = __popc(__ballot_sync(FULL, eng));
        const uint64_t em = __reduce_max_sync(FULL, eng ? (unsigned)cnt : 0u);
        const uint64_t cm = __reduce_max_sync(FULL, (unsigned)cnt);
        const uint64_t tot = __reduce_add_sync(FULL, (unsigned)cnt);
        if (traced) JQ_TRACE_COUNT(1, TR_LEGAL_SHAPE, (ne << 48) | (em << 32) | (cm << 16) | tot);
    }
#endif
    // rank of the source among all sources (compact order == flat order)
    int rank = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        uint32_t word = __reduce_or_sync(FULL, (src >= 0 && (src >> 5) == i) ? (1u << (src & 31)) : 0u);
        if (src >= 0) {
            if (i < (src >> 5)) rank += __popc(word);
            else if (i == (src >> 5)) rank += __popc(word & ((1u << (src & 31)) - 1u));
        }
    }
    w.scan[lane] = 0;
    __syncwarp();
    if (src >= 0) w.scan[rank] = cnt;
    __syncwarp();
    int v = w.scan[lane], inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc += t;
    }
    int total = __shfl_sync(FULL, inc, 31);
    __syncwarp();
    w.scan[lane] = inc - v;
    __syncwarp();
    if (traced) JQ_TRACE_AT(1, TR_RANKED);
    if (src >= 0 && ids) {
        int off = w.scan[rank];
        int base = T.c2f[src] * NC;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            uint32_t m = d[i];
            while (m) {
                int dc = i * 32 + __ffs(m) - 1;
                m &= m - 1;
                if (off < cap) ids[off] = base + T.c2f[dc];
                ++off;
            }
        }
    }
    if (traced) JQ_TRACE_AT(1, TR_IDS);
    if (mask_env) {
        for (int k = lane; k < CBW; k += 32) w.cbits[k] = 0u;
        __syncwarp();
        if (src >= 0) {
            // bit (canonical source row) * 129 + canonical destination; rows
            // of two lanes can share a word, hence the atomic
            const int rb = T.rot[seat][src] * NB;
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                uint32_t m = d[i];
                while (m) {
                    const int j = rb + T.rot[seat][i * 32 + __ffs(m) - 1];
                    m &= m - 1;
                    atomicOr(&w.cbits[j >> 5], 1u << (j & 31));
                }
            }
        }
        __syncwarp();
        // 32-byte stores from the first 32-byte boundary of the row
        const int head = (int)((32 - ((uintptr_t)mask_env & 31)) & 31);
        for (int j = lane; j < head; j += 32) mask_env[j] = (uint8_t)((w.cbits[j >> 5] >> (j & 31)) & 1u);
        const int body = (MASK_BYTES - head) >> 5;
        for (int k = lane; k < body; k += 32) mask_store32(mask_env + head + k * 32, w, head + k * 32);
        for (int j = head + body * 32 + lane; j < MASK_BYTES; j += 32)
            mask_env[j] = (uint8_t)((w.cbits[j >> 5] >> (j & 31)) & 1u);
        __syncwarp();
    }
    return total;
}

// ---------------------------------------------------------------------------
// Path-revealed engineer (move_gen.py:245-296) on the pre-move board
// ---------------------------------------------------------------------------
__device__ bool ray_clear_to(const TopoCore &T, const WEnv &w, const uint8_t *ray, int n, int dst) {
    for (int l = 0; l < n; ++l) {
        int nb = ray[l];
        if (nb == NONE8) return false;
        if (nb == dst) return true;
        if (w.cell[T.c2f[nb]] >= 0) return false;
    }
    return false;
}

// Whether an engineer on compact cell s reaches d along the railway through
// the empty cells `empty` (move_gen.py:186-224), by the whole warp (the
// result on every lane): the frontier's rail neighbours are the union of its
// cells' rows of railnb; lane l ORs the rows of the frontier cells l, l + 32,
// ... (a frontier holds a few cells, so most lanes load nothing) and one OR
// reduction per mask word gathers the union on every lane.
__device__ bool warp_engineer_reach(const TopoCore &T, int lane, int s, int d, const uint32_t (&empty)[NW],
                                    int *rounds = nullptr) {
    uint32_t reach[NW] = {0, 0, 0, 0, 0}, fr[NW] = {0, 0, 0, 0, 0};
    rset(reach, s);
    rset(fr, s);
    for (int it = 0; it < NB; ++it) {
#ifdef JQ_TRACE
        if (rounds) *rounds = it + 1;
#endif
        uint32_t nbm[NW] = {0, 0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < NW; ++i)
            if ((fr[i] >> lane) & 1u) {  // frontier bits are cells < NB
                const uint4 *row = reinterpret_cast<const uint4 *>(T.railnb[i * 32 + lane]);
                const uint4 r0 = row[0], r1 = row[1];
                nbm[0] |= r0.x;
                nbm[1] |= r0.y;
                nbm[2] |= r0.z;
                nbm[3] |= r0.w;
                nbm[4] |= r1.x;
            }
#pragma unroll
        for (int i = 0; i < NW; ++i) nbm[i] = __reduce_or_sync(FULL, nbm[i]);
        if (rbit(nbm, d)) return true;
        uint32_t any = 0;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            const uint32_t nw = nbm[i] & empty[i] & ~reach[i];
            reach[i] |= nw;
            fr[i] = nw;
            any |= nw;
        }
        if (!any) break;
    }
    return false;
}

// Whether d lies on straight rail ray k of s with every ray cell before it
// empty.  The ray's cells increase (k even) or decrease (k odd) in compact
// order, so the cells before d are the ray's cells below (above) d.
__device__ __forceinline__ bool ray_clear_mask(const TopoCore &T, int s, int k, int d, const uint32_t (&empty)[NW]) {
    bool on = false, blocked = false;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const uint32_t r = T.ray[s][k][i];
        const int lim = d - i * 32;
        const uint32_t below = lim <= 0 ? 0u : (lim >= 32 ? ~0u : (1u << lim) - 1u);
        const uint32_t dbit = (lim >= 0 && lim < 32) ? 1u << lim : 0u;
        const uint32_t before = (k & 1) ? ~(below | dbit) : below;
        on |= (r & dbit) != 0u;
        blocked |= (r & ~empty[i] & before) != 0u;
    }
    return on && !blocked;
}

// move_gen.py:245-296: whether the move sf -> df is one only an engineer's
// rail run makes.  Called by the whole warp (the board's empty cells are one
// ballot per mask word); the result is the same on every lane.
__device__ bool move_requires_gongb(const TopoCore &T, const WEnv &w, int sf, int df, int lane, int *rounds = nullptr) {
    if (sf == df) return false;
    int sx = sf % 17, sy = sf / 17, dx = df % 17, dy = df / 17;
    int adx = abs(sx - dx), ady = abs(sy - dy);
    int s = T.f2c[sf], d = T.f2c[df];
    if (s < 0 || d < 0) return false;
    if (adx + ady == 1) return false;
    if (adx == 1 && ady == 1 && ((T.flags[s] & F_CAMP) || (T.flags[d] & F_CAMP))) return false;
    if (!(T.flags[s] & F_RAIL) || !(T.flags[d] & F_RAIL)) return false;
    uint32_t empty[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int c = i * 32 + lane;
        empty[i] = __ballot_sync(FULL, c < NB && w.cell[T.c2f[c]] < 0);
    }
    if (sx == dx || sy == dy) {
        // a straight run: only the ray pointing at d can hold it
        const int k = sy == dy ? (dx > sx ? 0 : 1) : (dy > sy ? 2 : 3);
        if (ray_clear_mask(T, s, k, d, empty)) return false;
        return warp_engineer_reach(T, lane, s, d, empty, rounds);
    }
    if (T.curve[s] > 0 && T.curve[s] == T.curve[d] && (T.flags[s] & F_CURVE_ACTIVE)) {
        for (int k = 0; k < 2; ++k)
            if (ray_clear_to(T, w, T.cray[s][k], 11, d)) return false;
    }
    return warp_engineer_reach(T, lane, s, d, empty, rounds);
}

// ---------------------------------------------------------------------------
// Combat memory (combat_memory.py:354-562), scalar on global memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ void set_pid_bit(uint64_t &lo, uint64_t &hi, int pid) {
    if (pid < 64) lo |= 1ull << pid;
    else hi |= 1ull << (pid - 64);
}
__device__ __forceinline__ int next_floor(int t) {
    if (!is_ranked(t)) return 0;
    int r = 15 - t;
    return r > 9 ? 9 : r;
}

// The update touches three disjoint sets of rows, so the warp splits it:
// lanes 0..3 take observer o = lane (the attacked-by-known-engineer flag,
// chain propagation, then the direct update, all on K's row of o), and
// lanes 0..29 take the reverse projection onto pid o * 30 + lane of every
// observer o (reads V's rows, writes eaten-by rows).  The per-observer order
// of the scalar statement is kept; the three parts commute (OR / max
// updates of different rows), and none reads a row another one writes, so
// every load is issued before the first store: V's sets go through shared
// memory (one word per lane), then K's rows and the eaten-by rows are read
// together.
__device__ void warp_cm_apply(const jq_batch &b, WEnv &w, int e, int lane, bool eat, int A, int D, int A_seat,
                              int D_seat, int A_type, int D_type, int step) {
    const int K = eat ? A : D, V = eat ? D : A, V_seat = eat ? D_seat : A_seat, V_type = eat ? D_type : A_type;
    const int v_idx = tracked_idx(V_type);
    // One round of loads: V's sets (lanes 0..15, one word each), K's rows
    // (lanes 0..3) and the eaten-by rows of pid o * 30 + lane for every
    // observer o (lanes 0..29), the last before knowing which of them gain K.
    uint64_t vset = 0;
    if (lane < 16) {
        const int o = lane >> 2, f = lane & 3;
        const uint64_t *src = f == 0 ? b.cm_direct_lo : f == 1 ? b.cm_direct_hi : f == 2 ? b.cm_chain_lo : b.cm_chain_hi;
        vset = src[OI(e, o, V)];
    }
    uint64_t ea[4], eb[4];
#pragma unroll
    for (int o = 0; o < 4; ++o) {
        ea[o] = eb[o] = 0;
        if (lane < 30) {
            ea[o] = b.cm_eaten_lo[OI(e, o, o * 30 + lane)];
            eb[o] = b.cm_eaten_hi[OI(e, o, o * 30 + lane)];
        }
    }
    // K's row of observer o = lane (lanes 0..3)
    const int o4 = lane & 3;
    const size_t k = OI(e, o4, K), v = OI(e, o4, V);
    uint8_t g_v = 0;
    uint64_t ck_lo = 0, ck_hi = 0, dk_lo = 0, dk_hi = 0;
    uint16_t ck_t = 0, dv_t = 0, cv_t = 0, dk_t = 0;
    int floor_k = 0, vf = 0, dother = 0;
    if (lane < 4) {
        g_v = b.cm_is_gongb[v];
        ck_lo = b.cm_chain_lo[k];
        ck_hi = b.cm_chain_hi[k];
        ck_t = b.cm_chain_type[k];
        dv_t = b.cm_direct_type[v];
        cv_t = b.cm_chain_type[v];
        floor_k = b.cm_rank_floor[k];
        vf = b.cm_rank_floor[v];
        dother = b.cm_direct_other[k];
        dk_lo = b.cm_direct_lo[k];
        dk_hi = b.cm_direct_hi[k];
        dk_t = b.cm_direct_type[k];
    }
    if (lane < 16) w.cmv[lane >> 2][lane & 3] = vset;
    __syncwarp();
    // the eaten-by rows that gain K: pids in V's direct or chain set of
    // observer o, or V itself
    bool on[4];
#pragma unroll
    for (int o = 0; o < 4; ++o) {
        const int t = o * 30 + lane;
        const uint64_t lo = w.cmv[o][0] | w.cmv[o][2], hi = w.cmv[o][1] | w.cmv[o][3];
        on[o] = lane < 30 && ((t < 64 ? (lo >> t) & 1ull : (hi >> (t - 64)) & 1ull) || (V_seat == o && t == V));
    }
    if (lane < 4) {
        const int o = lane;
        const uint64_t dv_lo = w.cmv[o][0], dv_hi = w.cmv[o][1], cv_lo = w.cmv[o][2], cv_hi = w.cmv[o][3];
        if (!eat && (g_v || (A_type == GONGB && o == V_seat))) b.cm_atk_gongb[k] = 1;
        uint64_t lo = ck_lo | dv_lo | cv_lo;
        uint64_t hi = ck_hi | dv_hi | cv_hi;
        set_pid_bit(lo, hi, V);
        b.cm_chain_lo[k] = lo;
        b.cm_chain_hi[k] = hi;
        uint16_t ctype = (uint16_t)(ck_t | dv_t | cv_t);
        bool floor_up = false, not_g = false;
        const int prop = vf + 1 < 9 ? vf + 1 : 9;
        if (vf > 0) {
            if (prop > floor_k) { floor_k = prop; floor_up = true; }
            not_g = true;
        }
        if (V_seat != o) {
            const int c = dother + 1;
            b.cm_direct_other[k] = (int16_t)(c < 32767 ? c : 32767);
        } else {
            set_pid_bit(dk_lo, dk_hi, V);
            b.cm_direct_lo[k] = dk_lo;
            b.cm_direct_hi[k] = dk_hi;
            if (v_idx >= 0) {
                b.cm_direct_type[k] = (uint16_t)(dk_t | (1u << v_idx));
                ctype = (uint16_t)(ctype | (1u << v_idx));
            }
            if (eat) {
                if (V_type == DILEI) b.cm_is_gongb[k] = 1;
                else not_g = true;
            }
            if (is_ranked(V_type)) {  // KILLED defender lift and EAT-direct lift use the same rule
                const int pr = next_floor(V_type);
                if (pr > floor_k) { floor_k = pr; floor_up = true; }
            }
        }
        b.cm_chain_type[k] = ctype;
        b.cm_last_chain_step[k] = (int16_t)step;
        b.cm_last_direct_step[k] = (int16_t)step;
        if (floor_up) {
            b.cm_rank_floor[k] = (int8_t)floor_k;
            b.cm_rank_floor_step[k] = (int16_t)step;
        }
        if (not_g) b.cm_not_gongb[k] = 1;
    }
#pragma unroll
    for (int o = 0; o < 4; ++o) {
        if (on[o]) {
            const size_t tt = OI(e, o, o * 30 + lane);
            set_pid_bit(ea[o], eb[o], K);
            b.cm_eaten_lo[tt] = ea[o];
            b.cm_eaten_hi[tt] = eb[o];
        }
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// Beliefs (info_model.py:218-414)
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool sees_truth(int obs, int owner, int mode) {
    if (mode == SM_BRIGHT || obs == owner) return true;
    return mode == SM_HALF_DARK && ((obs & 1) == (owner & 1));
}
__device__ __forceinline__ bool bc_onehot(int c) { return c >= 1 && c <= 12; }

__device__ __forceinline__ uint8_t initial_code(const TopoCore &T, const WEnv &w, int o, int p, int mode) {
    if (!w.alive[p]) return BC_NONE;
    int s = w.seat[p];
    if (sees_truth(o, s, mode)) return (uint8_t)(tracked_idx(w.type[p]) + 1);
    if (s >= 0 && s < 4) {
        // a piece on its own setup cell (every piece right after a reset) has
        // that slot; otherwise search the seat's slots for its cell
        if (T.slot_cell[s][p % 30] == w.posc[p]) return (uint8_t)(BC_PRIOR0 + p % 30);
        for (int i = 0; i < 30; ++i)
            if (T.slot_cell[s][i] == w.posc[p]) return (uint8_t)(BC_PRIOR0 + i);
    }
    return BC_UNIFORM;
}

__device__ void warp_belief_init(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int lane, int mode) {
    for (int k = lane; k < 4 * NP; k += 32) {
        int o = k / NP, p = k - o * NP;
        const uint8_t c = initial_code(T, w, o, p, mode);
        b.bel_code[OI(e, o, p)] = c;
        w.bel[k] = c;
    }
    const int16_t counts[12] = {1, 3, 2, 1, 1, 2, 2, 2, 2, 3, 3, 3};
    for (int k = lane; k < 16 * 12; k += 32) {
        int os = k / 12, t = k - os * 12, o = os >> 2, s = os & 3;
        bool enemy = (s & 1) != (o & 1);
        b.remaining[(size_t)e * 192 + k] = enemy ? counts[t] : (int16_t)0;
        if (t == 0) b.rem_tracked[(size_t)e * 16 + os] = enemy;
    }
}

// Inventory rules on the env's shared-memory copy (observer o's rows only,
// so lanes 0..3 never touch each other's entries); returns whether it changed.
__device__ __forceinline__ bool rem_dec(WEnv &w, int o, int seat, int ti) {
    if (seat < 0 || seat > 3 || ti < 0) return false;
    const int tr = o * 4 + seat;
    if (!w.rtr[tr]) return false;
    int16_t &r = w.rem[tr * 12 + ti];
    if (r <= 0) return false;
    r = (int16_t)(r - 1);
    return true;
}
__device__ __forceinline__ bool rem_untrack(WEnv &w, int o, int seat) {
    const int tr = o * 4 + seat;
    bool changed = w.rtr[tr] != 0;
    w.rtr[tr] = 0;
    for (int t = 0; t < 12; ++t) {
        changed |= w.rem[tr * 12 + t] != 0;
        w.rem[tr * 12 + t] = 0;
    }
    return changed;
}

// Lane o (0..3) applies R3, R5/R7, R4/R6, R1 and R9 for observer o; then the
// whole warp runs the I5 sweep.  The codes are the shared-memory copy
// warp_load took; chunks the rules change are written back.
__device__ void warp_belief_update(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int lane,
                                   const StepCtx &x, int mode, const int *died) {
    bool touched = false;  // R-rules rewrote a code of this lane's observer
    bool inv = false;      // ... or an inventory entry
    // Only combat plies and seat deaths change inventories: then the env's
    // 192 entries and 16 tracked flags are in shared memory (a combat ply
    // started copying them before its combat-memory update; otherwise they
    // are loaded here in one round trip), the rules run there, and the rows
    // are written back once.
    if (x.inv_async) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncwarp();
    } else if (x.combat || died[0] || died[1] || died[2] || died[3]) {
#pragma unroll
        for (int i = 0; i < 4 * 4 * 12 / 32; ++i) w.rem[lane + 32 * i] = b.remaining[(size_t)e * 192 + lane + 32 * i];
        if (lane < 16) w.rtr[lane] = b.rem_tracked[(size_t)e * 16 + lane];
        __syncwarp();
    }
    if (lane < 4) {
        int o = lane;
        uint8_t *code = w.bel + o * NP;
        int a_bel = code[x.A];
        int d_bel = x.D >= 0 ? code[x.D] : BC_NONE;
        if (x.fr_src) inv |= rem_dec(w, o, x.acting, SILING - 2);
        if (x.fr_dst) inv |= rem_dec(w, o, x.D_seat, SILING - 2);
        if (x.ev == EV_EAT && x.D >= 0 && x.D_type == DILEI && a_bel != BC_NONE && !bc_onehot(a_bel)) {
            code[x.A] = (uint8_t)(GONGB - 1);
            touched = true;
            a_bel = code[x.A];
            inv |= rem_dec(w, o, x.acting, GONGB - 2);
        }
        if (x.fcap) {
            if (x.D_seat >= 0 && x.D_seat < 4) inv |= rem_untrack(w, o, x.D_seat);
        } else if (x.ev == EV_EAT && x.other_pid >= 0) {
            int op = x.other_pid;
            if (code[op] != BC_NONE && !bc_onehot(code[op])) {
                code[op] = (uint8_t)(JUNQI - 1);
                touched = true;
            }
        }
        a_bel = code[x.A];
        if (x.ev == EV_EAT) {
            if (bc_onehot(d_bel)) inv |= rem_dec(w, o, x.D_seat, d_bel - 1);
        } else if (x.ev == EV_KILLED) {
            if (bc_onehot(a_bel)) inv |= rem_dec(w, o, x.acting, a_bel - 1);
        } else if (x.ev == EV_BOMB) {
            if (bc_onehot(a_bel)) inv |= rem_dec(w, o, x.acting, a_bel - 1);
            if (bc_onehot(d_bel)) inv |= rem_dec(w, o, x.D_seat, d_bel - 1);
        }
        for (int s = 0; s < 4; ++s)
            if (died[s]) inv |= rem_untrack(w, o, s);
    }
    const bool any_touched = __any_sync(FULL, touched);
    if (__any_sync(FULL, inv)) {  // write the inventories back in one pass
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4 * 4 * 12 / 32; ++i)
            b.remaining[(size_t)e * 192 + lane + 32 * i] = w.rem[lane + 32 * i];
        if (lane < 16) b.rem_tracked[(size_t)e * 16 + lane] = w.rtr[lane];
    }
    // alive bits of pids 0..119 (bit p of word p >> 5)
    uint32_t am[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) am[i] = __ballot_sync(FULL, lane + 32 * i < NP && w.alive[lane + 32 * i]);
    __syncwarp();
    // I5 sweep over the env's 4 x 120 codes, 16 per lane (rows are 480 bytes,
    // 16-byte aligned: the host checks the base).  I5 rewrites a code exactly
    // when (code != NONE) differs from alive, so a chunk whose nonzero-byte
    // mask equals its pids' alive bits is left as it is.
    if (lane < 4 * NP / 16) {
        uint4 *srow = reinterpret_cast<uint4 *>(w.bel) + lane;
        uint4 v = *srow;
        uint32_t wv[4] = {v.x, v.y, v.z, v.w};
        uint32_t nz = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)  // byte b of word j nonzero -> bit 4 j + b
            nz |= ((((__vcmpne4(wv[j], 0u) & 0x01010101u) * 0x10204080u) >> 28) << (4 * j));
        // alive bits of the chunk's pids p0 .. p0 + 15, wrapping at 120 into the next observer
        const int p0 = (lane * 16) % NP;
        uint32_t al = __funnelshift_r(am[p0 >> 5], (p0 >> 5) + 1 < 4 ? am[(p0 >> 5) + 1] : 0u, p0 & 31) & 0xffffu;
        if (p0 + 16 > NP) {
            const int n1 = NP - p0;
            al = (al & ((1u << n1) - 1u)) | ((am[0] & ((1u << (16 - n1)) - 1u)) << n1);
        }
        bool changed = any_touched;
        if (nz != al)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int k = lane * 16 + i, o = k >= 3 * NP ? 3 : k >= 2 * NP ? 2 : k >= NP ? 1 : 0, p = k - o * NP;
            const uint32_t c = (wv[i >> 2] >> ((i & 3) * 8)) & 0xFFu;
            uint32_t nc = c;
            if (!w.alive[p]) nc = BC_NONE;
            else if (c == BC_NONE)
                nc = sees_truth(o, w.seat[p], mode) ? (uint32_t)(tracked_idx(w.type[p]) + 1) : (uint32_t)BC_UNIFORM;
            if (nc != c) {
                changed = true;
                wv[i >> 2] = (wv[i >> 2] & ~(0xFFu << ((i & 3) * 8))) | (nc << ((i & 3) * 8));
            }
        }
        if (changed) {
            const uint4 nv = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            *srow = nv;
            reinterpret_cast<uint4 *>(b.bel_code + OI(e, 0, 0))[lane] = nv;
        }
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// Seat surrender (batched_state.py:1078-1121), warp-parallel; returns the
// Zobrist delta on every lane.
// ---------------------------------------------------------------------------
__device__ int64_t warp_surrender(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int lane, int seat, int step) {
    int64_t d = 0;
    const bool keep_loc = b.rules == JQ_RULES_GAMESTATE;  // state.py:640-693 records the current cell
    for (int p = lane; p < NP; p += 32) {
        if (w.seat[p] != seat || !w.alive[p]) continue;
        size_t q = PI(e, p);
        int c = w.posc[p];
        b.death_loc[q] = (int16_t)(keep_loc && c >= 0 ? T.c2f[c] : -1);
        if (c >= 0) {
            int f = T.c2f[c];
            d ^= zpiece(p, w.type[p], f);
            w.cell[f] = -1;
            b.cell_pid[(size_t)e * NC + f] = -1;
        }
        w.alive[p] = 0;
        w.posc[p] = -1;
        b.alive[q] = 0;
        b.pos_x[q] = -1;
        b.pos_y[q] = -1;
        b.death_reason[q] = DR_KBE;
        b.death_step[q] = (int16_t)step;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d ^= __shfl_xor_sync(FULL, d, o);
    if (lane == 0) {
        w.sdead[seat] = 1;
        b.seat_dead[(size_t)e * 4 + seat] = 1;
    }
    __syncwarp();
    return d ^ c_zsdead[seat];
}

// ---------------------------------------------------------------------------
// Reset to GameState.new_game(lineup) (state.py:490-624), warp-parallel
// ---------------------------------------------------------------------------
__device__ void warp_reset(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int lane, const int8_t *lineup, int mode) {
    for (int f = lane; f < NC; f += 32) {
        w.cell[f] = -1;
        b.cell_pid[(size_t)e * NC + f] = -1;
    }
    __syncwarp();
    int64_t z = 0;
    for (int p = lane; p < NP; p += 32) {
        size_t q = PI(e, p);
        int t = lineup ? lineup[p] : 0;
        bool real = t != NONE;
        int s = p / 30, c = T.slot_cell[s][p % 30], f = T.c2f[c];
        int x = f % 17, y = f / 17;
        b.alive[q] = real;
        b.piece_type[q] = real ? (int8_t)t : (int8_t)-1;
        b.piece_seat[q] = real ? (int8_t)s : (int8_t)-1;
        b.pos_x[q] = b.zero_x[q] = real ? (int8_t)x : (int8_t)-1;
        b.pos_y[q] = b.zero_y[q] = real ? (int8_t)y : (int8_t)-1;
        b.move_count[q] = 0;
        b.active_eat[q] = 0;
        b.passive_surv[q] = 0;
        b.death_reason[q] = -1;
        b.death_step[q] = -1;
        b.death_loc[q] = -1;
        w.alive[p] = real;
        w.type[p] = real ? (int8_t)t : (int8_t)-1;
        w.seat[p] = real ? (int8_t)s : (int8_t)-1;
        w.posc[p] = (int16_t)(real ? c : -1);
        if (real) {
            w.cell[f] = (int16_t)p;
            b.cell_pid[(size_t)e * NC + f] = (int16_t)p;
            z ^= zpiece(p, t, f);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z ^= __shfl_xor_sync(FULL, z, o);
    if (lane < 4) {
        w.sdead[lane] = 0;
        b.seat_dead[(size_t)e * 4 + lane] = 0;
        b.seat_flag[(size_t)e * 4 + lane] = 0;
    }
    if (lane == 0) {
        b.turn[e] = 0;
        b.zobrist[e] = z ^ c_zturn[0] ^ g_zmc[0] ^ g_zmslc[0] ^ c_zwin[0] ^ c_zshow[mode & 3];
        b.move_counter[e] = 0;
        b.mslc[e] = 0;
        b.terminated[e] = 0;
        b.winner[e] = -1;
        b.draw[e] = 0;
        b.hist_count[e] = 0;
    }
    for (int k = lane; k < 4 * NP; k += 32) {
        size_t q = (size_t)e * 4 * NP + k;
        b.cm_direct_lo[q] = 0; b.cm_direct_hi[q] = 0; b.cm_direct_type[q] = 0;
        b.cm_last_direct_step[q] = -1; b.cm_direct_other[q] = 0;
        b.cm_chain_lo[q] = 0; b.cm_chain_hi[q] = 0; b.cm_chain_type[q] = 0;
        b.cm_last_chain_step[q] = -1; b.cm_eaten_lo[q] = 0; b.cm_eaten_hi[q] = 0;
        b.cm_rank_floor[q] = 0; b.cm_rank_floor_step[q] = -1;
        b.cm_is_gongb[q] = 0; b.cm_not_gongb[q] = 0; b.cm_atk_gongb[q] = 0;
    }
    b.hist_src[(size_t)e * HIST + lane] = -1;
    b.hist_dst[(size_t)e * HIST + lane] = -1;
    __syncwarp();
    warp_belief_init(b, T, w, e, lane, mode);
    __syncwarp();
}

// ---------------------------------------------------------------------------
// One ply (BatchedGameState.step_batch for one env)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int resolve_combat(int a, int d) {
    if (a <= DARK || d <= DARK || a > GONGB || d > GONGB) return 0;
    if (a == JUNQI || a == DILEI) return 0;  // the reference raises here
    if (a == ZHADAN || d == ZHADAN) return EV_BOMB;
    if (d == JUNQI) return EV_EAT;
    if (d == DILEI) return a == GONGB ? EV_EAT : EV_KILLED;
    if (a == d) return EV_BOMB;
    return a < d ? EV_EAT : EV_KILLED;
}

__device__ __forceinline__ void check_victory(const WEnv &w, int acting, int mc, int mslc, int &term, int &win,
                                              int &draw) {
    bool red = !w.sdead[0] || !w.sdead[2], blue = !w.sdead[1] || !w.sdead[3];
    term = 0; win = -1; draw = 0;
    if (!red && !blue) { term = 1; win = acting % 2; return; }
    if (!red) { term = 1; win = 1; return; }
    if (!blue) { term = 1; win = 0; return; }
    if (mc >= 4000 || mslc >= 200) { term = 1; draw = 1; }
}

__device__ __forceinline__ void kill_piece(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int pid, int cell_f,
                                           int reason, int step, int loc) {
    if (!w.alive[pid]) return;
    size_t q = PI(e, pid);
    w.alive[pid] = 0;
    w.posc[pid] = -1;
    w.cell[cell_f] = -1;
    b.alive[q] = 0;
    b.cell_pid[(size_t)e * NC + cell_f] = -1;
    b.pos_x[q] = -1;
    b.pos_y[q] = -1;
    b.death_reason[q] = (int8_t)reason;
    b.death_step[q] = (int16_t)step;
    b.death_loc[q] = (int16_t)loc;
}

__device__ __forceinline__ void move_piece(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int pid, int sf, int df) {
    size_t q = PI(e, pid);
    w.cell[sf] = -1;
    w.cell[df] = (int16_t)pid;
    w.posc[pid] = T.f2c[df];
    b.cell_pid[(size_t)e * NC + sf] = -1;
    b.cell_pid[(size_t)e * NC + df] = (int16_t)pid;
    b.pos_x[q] = (int8_t)(df % 17);
    b.pos_y[q] = (int8_t)(df / 17);
}

// Returns true on every lane when the ply was applied.
__device__ bool warp_step(const jq_batch &b, const TopoCore &T, WEnv &w, int e, int lane, int32_t act, int mode,
                          const jq_step_out &out, int64_t *stats, bool traced = false) {
    StepCtx &x = w.x;
    int64_t zob = 0;
    if (lane == 0) {
        x.skip = 1;
        int term0 = w.s_term;
        out.valid[e] = 0;
        if (out.event) out.event[e] = 0;
        if (out.terminated) out.terminated[e] = (uint8_t)term0;
        if (out.winner) out.winner[e] = w.s_win;
        if (out.draw) out.draw[e] = (uint8_t)w.s_draw;
        if (out.flag_captured) out.flag_captured[e] = 0;
        if (out.reward) out.reward[e] = 0.f;
        if (out.zobrist) out.zobrist[e] = w.s_zob;
        if (!term0 && act >= 0 && act < NC * NC) {
            int sf = act / NC, df = act % NC, A = w.cell[sf], D = w.cell[df];
            if (A >= 0 && sf != df) {
                x.sf = sf; x.df = df; x.A = A; x.D = D;
                x.A_type = w.type[A]; x.A_seat = w.seat[A];
                x.D_type = D >= 0 ? w.type[D] : 0;
                x.D_seat = D >= 0 ? w.seat[D] : -1;
                x.ev = D < 0 ? EV_MOVE : resolve_combat(x.A_type, x.D_type);
                if (x.ev) x.skip = 0;
            }
        }
    }
    __syncwarp();
    if (x.skip) return false;
    // path-revealed engineer (move_gen.py:245-296) on the pre-move board, by
    // the whole warp: a move only an engineer's rail run can make
    bool gongb_path = false;
    int path_rounds = 0;
    if (x.A_type == GONGB) {
        const int adx = abs(x.sf % 17 - x.df % 17), ady = abs(x.sf / 17 - x.df / 17);
        if (x.D >= 0 || adx + ady > 1) gongb_path = move_requires_gongb(T, w, x.sf, x.df, lane, &path_rounds);
    }
    if (traced) {
        JQ_TRACE_AT(1, TR_PATH);
        JQ_TRACE_COUNT(1, TR_PATH_ROUNDS, path_rounds);
        JQ_TRACE_COUNT(1, TR_ATYPE, x.A_type);
    }
    if (lane == 0) {
        const int sf = x.sf, df = x.df, A = x.A, D = x.D;
        x.acting = w.s_turn;
        x.mc = w.s_mc;
        x.mslc = w.s_mslc;
        x.new_mc = x.mc + 1;
        x.combat = D >= 0;
        for (int s = 0; s < 4; ++s) x.died_pre[s] = w.sdead[s];
        x.other_pid = -1;
        x.fcap = x.fr_src = x.fr_dst = 0;
        x.need_surrender = 0;
        x.cm = 0;
        if (D >= 0 && x.D_seat >= 0 && x.D_seat < 4) {
            int s0 = T.c2f[T.slot_cell[x.D_seat][26]], s1 = T.c2f[T.slot_cell[x.D_seat][28]];
            if (df == s0) x.other_pid = w.cell[s1];
            else if (df == s1) x.other_pid = w.cell[s0];
        }
        // Every global value the ply reads, loaded before its first global
        // store: the compiler cannot move a load past a store that may alias
        // it, so loads issued where they are used would each wait a full
        // round trip behind the stores before them.
        const int64_t zA_src = zpiece(A, x.A_type, sf), zA_dst = zpiece(A, x.A_type, df);
        const int64_t zD_dst = D >= 0 ? zpiece(D, x.D_type, df) : 0;
        const int64_t z_mc = g_zmc[x.mc & 0xFFF], z_mslc = g_zmslc[x.mslc & 0x1FF];
        const int64_t z_mc1 = g_zmc[(x.mc + 1) & 0xFFF], z_mslc1 = g_zmslc[D < 0 ? (x.mslc + 1) & 0x1FF : 0];
        const int cnt = D < 0 ? b.move_count[PI(e, A)]
                        : x.ev == EV_EAT ? b.active_eat[PI(e, A)]
                        : x.ev == EV_KILLED ? b.passive_surv[PI(e, D)] : 0;
        if (gongb_path)
            for (int o = 0; o < 4; ++o) b.cm_is_gongb[OI(e, o, A)] = 1;
        zob = w.s_zob ^ c_zturn[x.acting & 3] ^ z_mc ^ z_mslc;
        x.z_tail = z_mc1 ^ z_mslc1;
        if (D < 0) {
            zob ^= zA_src ^ zA_dst;
            move_piece(b, T, w, e, A, sf, df);
            b.move_count[PI(e, A)] = (int16_t)(cnt + 1);
            x.new_mslc = x.mslc + 1;
        } else {
            int ds = x.new_mc;
            x.fr_src = x.A_type == SILING && (x.ev == EV_KILLED || x.ev == EV_BOMB);
            x.fr_dst = x.D_type == SILING && (x.ev == EV_EAT || x.ev == EV_BOMB);
            if (x.fr_src && x.A_seat >= 0 && x.A_seat < 4 && !w.sflag[x.A_seat]) {
                w.sflag[x.A_seat] = 1;
                b.seat_flag[(size_t)e * 4 + x.A_seat] = 1;
                zob ^= c_zsflag[x.A_seat];
            }
            if (x.fr_dst && x.D_seat >= 0 && x.D_seat < 4 && !w.sflag[x.D_seat]) {
                w.sflag[x.D_seat] = 1;
                b.seat_flag[(size_t)e * 4 + x.D_seat] = 1;
                zob ^= c_zsflag[x.D_seat];
            }
            x.fcap = x.D_type == JUNQI;
            if (x.ev == EV_EAT) {
                zob ^= zD_dst;
                kill_piece(b, T, w, e, D, df, DR_KBE, ds, df);
                zob ^= zA_src ^ zA_dst;
                move_piece(b, T, w, e, A, sf, df);
                b.active_eat[PI(e, A)] = (int16_t)(cnt + 1);
                x.cm = 1;
            } else if (x.ev == EV_KILLED) {
                int dr = (x.D_type == DILEI || x.D_type == ZHADAN) ? DR_MINE : DR_KBE;
                zob ^= zA_src;
                kill_piece(b, T, w, e, A, sf, dr, ds, df);
                b.passive_surv[PI(e, D)] = (int16_t)(cnt + 1);
                x.cm = 2;
            } else {
                zob ^= zA_src ^ zD_dst;
                kill_piece(b, T, w, e, A, sf, DR_MUTUAL, ds, df);
                kill_piece(b, T, w, e, D, df, DR_MUTUAL, ds, df);
            }
            x.new_mslc = 0;
            if (x.fcap && x.D_seat >= 0 && x.D_seat < 4 && !w.sdead[x.D_seat]) {
                if (!w.sflag[x.D_seat]) {
                    w.sflag[x.D_seat] = 1;
                    b.seat_flag[(size_t)e * 4 + x.D_seat] = 1;
                    zob ^= c_zsflag[x.D_seat];
                }
                x.need_surrender = 1;
            }
        }
    }
    __syncwarp();
    if (traced) {
        JQ_TRACE_AT(1, TR_SCALAR);
        JQ_TRACE_COUNT(1, TR_EVENT, x.ev);
    }
    // A combat ply changes inventories: they are copied into shared memory
    // asynchronously (cp.async, no registers held) while the combat-memory
    // update runs, and the belief update waits for the copy.
    x.inv_async = x.combat && !(((uintptr_t)b.remaining | (uintptr_t)b.rem_tracked) & 15);
    if (x.inv_async) {
        if (lane < 24) cp_async16(&w.rem[lane * 8], b.remaining + (size_t)e * 192 + lane * 8);
        else if (lane == 24) cp_async16(w.rtr, b.rem_tracked + (size_t)e * 16);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (x.cm) warp_cm_apply(b, w, e, lane, x.cm == 1, x.A, x.D, x.A_seat, x.D_seat, x.A_type, x.D_type, x.new_mc);
    if (x.need_surrender) {
        int64_t d = warp_surrender(b, T, w, e, lane, x.D_seat, x.new_mc);
        if (lane == 0) zob ^= d;
    }
    if (x.combat) {
        // post-combat dead sweep (batched_state.py:893-902)
        for (int s = 0; s < 4; ++s) {
            if (w.sdead[s]) continue;
            bool any = false;
            for (int p = lane; p < NP; p += 32) any |= (w.seat[p] == s && w.alive[p]);
            if (!__any_sync(FULL, any)) {
                if (lane == 0) {
                    w.sdead[s] = 1;
                    b.seat_dead[(size_t)e * 4 + s] = 1;
                    zob ^= c_zsdead[s];
                }
                __syncwarp();
            }
        }
    }
    if (lane == 0) {
        check_victory(w, x.acting, x.new_mc, x.new_mslc, x.term, x.win, x.draw);
        int cand = (x.acting + 1) & 3;
        // Batched rules: plain moves test Q12 only past a dead next seat
        // (batched_state.py:636-684).  GameState rules and every combat ply:
        // victory first, then Q12 on every candidate (batched_state.py:
        // 905-918, state.py:595-612, 1111-1170).
        x.full_advance = x.combat || b.rules == JQ_RULES_GAMESTATE;
        x.do_q12 = x.full_advance ? !x.term : (int)w.sdead[cand];
        x.new_turn = x.full_advance ? (x.term ? x.acting : (x.acting + 1) & 3) : cand;
    }
    __syncwarp();
    if (traced) JQ_TRACE_AT(1, TR_COMBAT);
    int scans = 0;
    if (x.do_q12) {
        int cand = (x.acting + 1) & 3, chain = 0;
        bool found = false;
        while (chain < 4) {
            if (w.sdead[cand]) { cand = (cand + 1) & 3; ++chain; continue; }
            if (warp_has_moves(T, w, lane, cand, &scans)) { found = true; break; }
            int64_t d = warp_surrender(b, T, w, e, lane, cand, x.new_mc);
            if (lane == 0) zob ^= d;
            cand = (cand + 1) & 3;
            ++chain;
        }
        if (lane == 0) {
            x.new_turn = x.full_advance ? (found ? cand : (x.acting + 1) & 3) : cand;
            check_victory(w, x.acting, x.new_mc, x.new_mslc, x.term, x.win, x.draw);
        }
    }
    __syncwarp();
    if (traced) {
        JQ_TRACE_AT(1, TR_Q12);
        JQ_TRACE_COUNT(1, TR_Q12_SCANS, scans);
    }
    if (lane == 0) {
        // the caller's episode cap, after victory and Q12 (game_state.cu:1651-1655)
        if (!x.term && b.max_moves > 0 && x.new_mc >= b.max_moves) {
            x.term = 1;
            x.draw = 1;
        }
        zob ^= x.z_tail ^ c_zturn[x.new_turn & 3];  // keys of new_mc and new_mslc
        if (x.term) zob ^= c_zterm;
        if (x.draw) zob ^= c_zdraw;
        if (x.win >= 0) zob ^= c_zwin[0] ^ c_zwin[x.win + 1];
        b.move_counter[e] = x.new_mc;
        b.mslc[e] = x.new_mslc;
        b.turn[e] = (int8_t)x.new_turn;
        b.zobrist[e] = zob;
        b.terminated[e] = (uint8_t)x.term;
        b.winner[e] = (int8_t)x.win;
        b.draw[e] = (uint8_t)x.draw;
        out.valid[e] = 1;
        if (out.event) out.event[e] = (int8_t)x.ev;
        if (out.terminated) out.terminated[e] = (uint8_t)x.term;
        if (out.winner) out.winner[e] = (int8_t)x.win;
        if (out.draw) out.draw[e] = (uint8_t)x.draw;
        if (out.flag_captured) out.flag_captured[e] = (uint8_t)x.fcap;
        if (out.reward)
            out.reward[e] = (x.term && !x.draw && x.win >= 0) ? (((x.acting & 1) == x.win) ? 1.f : -1.f) : 0.f;
        if (out.zobrist) out.zobrist[e] = zob;
        int hc = w.s_hc;
        b.hist_src[(size_t)e * HIST + (hc & (HIST - 1))] = (int16_t)x.sf;
        b.hist_dst[(size_t)e * HIST + (hc & (HIST - 1))] = (int16_t)x.df;
        b.hist_count[e] = hc + 1;
        if (stats && x.term) {
            if (x.draw) atomicAdd((unsigned long long *)&stats[2], 1ull);
            else if (x.win >= 0) atomicAdd((unsigned long long *)&stats[x.win], 1ull);
            atomicAdd((unsigned long long *)&stats[3], 1ull);
            atomicAdd((unsigned long long *)&stats[4], (unsigned long long)x.new_mc);
        }
    }
    __syncwarp();
    if (traced) JQ_TRACE_AT(1, TR_COMMIT);
    int died[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) died[s] = w.sdead[s] && !x.died_pre[s];
    warp_belief_update(b, T, w, e, lane, x, mode, died);
    return true;
}

}  // namespace jq
