// jq_obs.cuh -- 317-channel observation encoder (observation.py:598-1651).
//
// A unit is one (env, observer) pair: 317 planes x 289 cells of float32
// (366,452 B) plus 28 globals, almost all zeros or ones.
//
// A unit is first described in shared memory as a bitstream with one bit per
// output float in output order (the float is 1.0, else 0.0), plus what the
// other floats need: one record per piece (cell, belief code, direct-combat
// pid set, recency values), the two progress constants, and an exception
// list (float index, value) for the -1 of each history source.  The stream
// starts 8 - head bits in, where head (0..7) is the number of floats before
// the unit's first 32-byte boundary in global memory (a unit is 91,613
// floats, so its base is only 4-byte aligned); every aligned group of 8
// floats of the output then owns one byte of a 32-bit word and is written
// with one 32-byte store.
//
// Persistent CTAs of 16 warps, specialised:
//  * 8 staging warps take units in memory order through an atomic ticket
//    and build unit k+1 in one of two shared
//    buffers: warps w and w + 4 split the 30 pieces of seat o + w, thread = piece,
//    setting the bits the piece lights at its canonical cell with shared
//    atomicOr and filling its record; then history, constant and
//    board-static planes; the globals go straight to HBM;
//  * 8 streaming warps write unit k from the other buffer: pass 1, warp w
//    one contiguous slab of the unit's aligned float4s, each float4 one
//    shared word, a shift, four selects and a 16-byte store -- no branch;
//    pass 2, after a barrier among them, over lines still in L2: belief
//    values, kill counts / 3 and recency from the piece records, the
//    progress planes, the exceptions; then they clear the bitstream.
// Named barriers hand the buffers back and forth (full / empty per buffer),
// so staging hides behind the previous unit's stream.  Taking units in
// memory order keeps the units being written at any moment in one compact
// window of the output: CTAs that drift apart under a static unit-per-CTA
// stride spread the dirty lines over the whole buffer and lose about a
// quarter of the DRAM write bandwidth (write microbenchmark on this GPU).
// The value-carrying floats are expanded by the streaming warps rather than
// queued by the staging warps because staging, not the stream, bounded the
// kernel: one shared-atomic append per belief value cost more than the
// whole record expansion.
//
// Values go straight to their canonical cell (the observer's rotation
// applied per cell), which equals the reference's world-frame build
// followed by rotate_planes.  Every output byte is written once, except
// that pass 2 overwrites the zeros pass 1 left at value-carrying floats.
#pragma once
#include "jq_rules.cuh"
#include "jq_trace.cuh"

namespace jq {

constexpr int OBS_STREAM_WARPS = 8;
constexpr int OBS_STAGE_WARPS = 8;  // two per seat relation
constexpr int OBS_STAGE_THREADS = 32 * OBS_STAGE_WARPS;                      // 256
static_assert(OBS_STAGE_WARPS % 4 == 0, "staging warps come in groups of four seat relations");
constexpr int OBS_THREADS = 32 * (OBS_STREAM_WARPS + OBS_STAGE_WARPS);      // 384
constexpr int OBS_WORDS = (OBS_FLOATS + 8 + 31) / 32;  // 2,864 words per stream
constexpr int OBS_WORDS4 = (OBS_WORDS + 3) / 4;         // in uint4
// Floats per vector store of the stream: the stream offset of a unit is 1..OBS_VEC.
constexpr int OBS_VEC = 8;
// The board-static planes 58-62 as stream words: for every stream offset
// 1..OBS_VEC they lie within the STAT_WORDS words from STAT_W0.
constexpr int STAT_W0 = (58 * NC + 1) >> 5, STAT_WORDS = ((63 * NC + OBS_VEC) >> 5) - STAT_W0 + 1;

// Built on the host once (build_static_words), copied into each CTA.
__device__ uint32_t g_statw[4][OBS_VEC][STAT_WORDS];

// The board-static bits (camp, stronghold, rail, nine-grid, arc planes
// 58-62; observation.py:343-383) for observer o and stream offset s + 1,
// as stream words from STAT_W0.
inline void build_static_words(const Topo &T, uint32_t out[4][OBS_VEC][STAT_WORDS]) {
    const uint8_t fb[5] = {F_CAMP, F_SH, F_RAIL, F_NINE, F_ARC};
    for (int o = 0; o < 4; ++o)
        for (int sh = 0; sh < OBS_VEC; ++sh) {
            for (int w = 0; w < STAT_WORDS; ++w) out[o][sh][w] = 0u;
            for (int f = 0; f < NC; ++f) {
                const int cc = T.f2c[f];
                if (cc < 0) continue;
                for (int i = 0; i < 5; ++i)
                    if (T.flags[cc] & fb[i]) {
                        const int q = (58 + i) * NC + T.rotf[o][f] + sh + 1 - STAT_W0 * 32;
                        out[o][sh][q >> 5] |= 1u << (q & 31);
                    }
            }
        }
}
// named barriers (0 is __syncthreads)
constexpr int BAR_FULL0 = 1, BAR_EMPTY0 = 3, BAR_STAGE = 5, BAR_STREAM = 6;

#ifndef OBS_MIN_CTAS
#define OBS_MIN_CTAS 2
#endif

// Exceptions per unit: the -1 of each history source.  Every other float
// that is neither 0 nor 1 comes from a per-piece record (below) or a
// per-plane constant that the streaming warps expand themselves.
constexpr int EXC_MAX = HIST;

// Pass-2 work items per unit besides the record expansions (12 per belief
// record, 16 per combat-memory record): the two progress planes.
constexpr int P2_PROG = 2 * NC;

// One staged unit.
struct __align__(16) UnitBuf {
    uint32_t bits[OBS_WORDS4 * 4];
    uint64_t pdlo[NP], pdhi[NP];        // enemy piece: its direct-combat pid set (kill-count planes 211-222)
    uint64_t type_lo[12], type_hi[12];  // observer-own pids of each tracked type
    float prec[NP][4];                  // enemy piece: recency planes 253-256 (0: none)
    int16_t pcell[NP];                  // canonical cell of an alive on-board piece, -1: none
    uint8_t pflag[NP];                  // bit 0: belief record, bit 1: combat-memory record
    uint8_t pbase[NP], pcode[NP];       // belief record: first plane (12 / 27 / 39) and belief code
    float pbel[NP][12];                 // belief record with caller-given beliefs: the 12 values at the cell
    uint8_t bel_list[NP], cm_list[NP];  // pids holding a belief / combat-memory record
    int32_t bel_off[NP];                // belief record j (list order): output float of its plane-0 value
    uint8_t bel_row[NP];                // belief record j: its row of ObsSmem::bel_tab
    int nbel, ncm;
    int32_t exc_pos[EXC_MAX];           // output float index of each exception
    float exc_val[EXC_MAX];
    float cval[2];                      // progress planes 64, 65
    int exc_n;
    int u;  // unit index, -1: no more units
    int o;  // its observer
};

struct __align__(16) ObsSmem {
    UnitBuf buf[2];
    int16_t rotf[4][NC];                // world flat -> canonical flat, per observer seat
    uint32_t statw[4][OBS_VEC][STAT_WORDS];  // board-static bits as stream words, per observer and stream offset
    int ticket[1], next_o[1];  // the staging warps' next unit and its observer
    // belief values: rows 0..29 the prior of a seat-local slot, row 30 the
    // uniform fallback (global loads here would wait behind the write stream)
    float bel_tab[31 * 12];
    int8_t slot_ch[30];
};

__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void bar_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ bool in_back_two(int seat, int zx, int zy) {
    switch (seat) {  // observation.py:1378-1387
    case 0: return zy >= 15 && zy <= 16;
    case 2: return zy >= 0 && zy <= 1;
    case 1: return zx >= 0 && zx <= 1;
    case 3: return zx >= 15 && zx <= 16;
    }
    return false;
}

__device__ __forceinline__ void set_bit(uint32_t *s, int q) { atomicOr(&s[q >> 5], 1u << (q & 31)); }

// Writes one unit's bitstream and exception list; stream position of float
// (ch, cell) is its output index ch * 289 + cell shifted by qoff = OBS_VEC - head.
struct Stager {
    UnitBuf &B;
    int qoff;
    const int16_t *rotf;  // the observer's world -> canonical cell map
    const float *ext;     // caller-given beliefs of this unit's observer, (12, 289) world frame; NULL: none
    __device__ __forceinline__ int q(int ch, int cell) const { return ch * NC + cell + qoff; }
    __device__ __forceinline__ void one(int ch, int cell) { set_bit(B.bits, q(ch, cell)); }
    __device__ __forceinline__ void exception(int j, float v) {
        // one shared atomic per group of converged lanes: a staging warp
        // works on one seat's pieces, so its lanes mostly append together
        const unsigned act = __activemask();
        const int lane = threadIdx.x & 31, leader = __ffs(act) - 1;
        int base = 0;
        if (lane == leader) base = atomicAdd(&B.exc_n, __popc(act));
        base = __shfl_sync(act, base, leader);
        const int i = base + __popc(act & ((1u << lane) - 1u));
        if (i < EXC_MAX) {
            B.exc_pos[i] = j;
            B.exc_val[i] = v;
        }
    }
    __device__ __forceinline__ void ones(int ch0, uint32_t m, int cell) {
        while (m) {
            const int i = __ffs(m) - 1;
            m &= m - 1;
            one(ch0 + i, cell);
        }
    }
    // all 289 floats of plane ch in stream s; thread k of nthreads covers some words
    __device__ __forceinline__ void fill_plane(uint32_t *s, int ch, int k, int nthreads) {
        const int q0 = q(ch, 0), q1 = q0 + NC, w0 = q0 >> 5, w1 = (q1 - 1) >> 5;
        for (int w = w0 + k; w <= w1; w += nthreads) {
            const int lo = q0 > w * 32 ? q0 - w * 32 : 0, hi = q1 < w * 32 + 32 ? q1 - w * 32 : 32;
            const uint32_t m = (hi - lo == 32 ? ~0u : ((1u << (hi - lo)) - 1u)) << lo;
            atomicOr(&s[w], m);
        }
    }
};

// Bits [pos, pos + 30) of a 120-bit pid set held as (lo, hi).
__device__ __forceinline__ uint32_t pid_field30(uint64_t lo, uint64_t hi, int pos) {
    if (pos + 30 <= 64) return (uint32_t)(lo >> pos) & 0x3FFFFFFFu;
    if (pos >= 64) return (uint32_t)(hi >> (pos - 64)) & 0x3FFFFFFFu;
    return (uint32_t)((lo >> pos) | (hi << (64 - pos))) & 0x3FFFFFFFu;
}

// The first min(max(count, 0), n) planes of a threshold group (plane g lit
// when count >= g + 1).
__device__ __forceinline__ uint32_t thresh_mask(int count, int n) {
    const int c = count < 0 ? 0 : (count > n ? n : count);
    return (1u << c) - 1u;
}

// Piece p's contribution for observer o (observation.py:1233-1569 per piece).
// Every field the piece may need is loaded up front, so the staging warps
// wait for memory once rather than once per branch.
__device__ void stage_piece(const jq_batch &b, int e, int o, int mode, const ObsSmem &S, Stager &st, int p) {
    const int tm = (o + 2) & 3, left = (o + 1) & 3, right = (o + 3) & 3, oteam = o & 1;
    const size_t q = PI(e, p), k = OI(e, o, p);
    const int alive_raw = b.alive[q];
    const int s = b.piece_seat[q];
    const int x = b.pos_x[q], y = b.pos_y[q], zx = b.zero_x[q], zy = b.zero_y[q];
    const int ptype = b.piece_type[q];
    const int mcnt = b.move_count[q], ae_raw = b.active_eat[q], ps_raw = b.passive_surv[q];
    const int dstep = b.death_step[q], dreason = b.death_reason[q], dloc = b.death_loc[q];
    const int code = b.bel_code[k];
    // an alive piece's seat is its pid / 30, so whether the observer sees it
    // as an enemy (and needs its combat-memory row) is known before any load
    const bool enemy_pid = ((p / 30) & 1) != oteam;
    uint64_t dlo = 0, dhi = 0, clo = 0, chi = 0;
    int dtype = 0, ctype = 0, other = 0, fl = 0, is_g = 0, not_g = 0, atk_g = 0, last_d = -1, last_c = -1, last_f = -1;
    if (enemy_pid) {
        dlo = b.cm_direct_lo[k];
        dhi = b.cm_direct_hi[k];
        clo = b.cm_chain_lo[k];
        chi = b.cm_chain_hi[k];
        dtype = b.cm_direct_type[k];
        ctype = b.cm_chain_type[k];
        other = b.cm_direct_other[k];
        fl = b.cm_rank_floor[k];
        is_g = b.cm_is_gongb[k];
        not_g = b.cm_not_gongb[k];
        atk_g = b.cm_atk_gongb[k];
        last_d = b.cm_last_direct_step[k];
        last_c = b.cm_last_chain_step[k];
        last_f = b.cm_rank_floor_step[k];
    }
    const int cur = b.move_counter[e];
    // recency values (observation.py:1556-1562): the table lives in global
    // memory, so the four loads are issued here, long before their use
    float recv[4] = {0.f, 0.f, 0.f, 0.f};
    if (enemy_pid && alive_raw) {
        const int lasts[4] = {last_d, last_d, last_c, last_f};
#pragma unroll
        for (int pl = 0; pl < 4; ++pl)
            if (lasts[pl] >= 0) {
                int el = cur - lasts[pl];
                el = el < 0 ? 0 : (el > RECENCY_LEN - 1 ? RECENCY_LEN - 1 : el);
                recv[pl] = g_recency[pl * RECENCY_LEN + el];
            }
    }
    // the observer's own pieces (pids o*30 .. o*30+29, one warp-aligned group
    // of lanes) also read the opponents' view of them and their eaten-by sets
    const bool own_pid = (p / 30) == o;
    int lc = 0, rc = 0, lg = 0;
    bool patk = false;
    uint64_t elo = 0, ehi = 0;
    if (own_pid) {
        const size_t kl = OI(e, left, p), kr = OI(e, right, p);
        lc = __popcll(b.cm_direct_lo[kl]) + __popcll(b.cm_direct_hi[kl]) + b.cm_direct_other[kl];
        rc = __popcll(b.cm_direct_lo[kr]) + __popcll(b.cm_direct_hi[kr]) + b.cm_direct_other[kr];
        lg = b.cm_is_gongb[kl] && b.cm_is_gongb[kr];
        patk = b.cm_atk_gongb[kl] || b.cm_atk_gongb[kr];
        elo = b.cm_eaten_lo[k];
        ehi = b.cm_eaten_hi[k];
    }

    const int team = s >= 0 ? (s & 1) : 1;  // numpy _SEAT_TEAM[-1] is EAST's team
    int cell;
    st.B.pcell[p] = -1;
    if (alive_raw) {
        if (!(x >= 0 && x < 17 && y >= 0 && y < 17)) return;
        cell = st.rotf[y * 17 + x];
        st.B.pcell[p] = (int16_t)cell;
        const int ti = tracked_idx(ptype);
        if (s == o && ti >= 0) st.one(ti, cell);
        int base = -1;
        if (s == tm) {
            base = 12;
            if (mode == SM_DARK) st.one(24, cell);
        }
        if (s == left) { st.one(25, cell); base = 27; }
        if (s == right) { st.one(26, cell); base = 39; }
        uint32_t flag = 0;
        // belief planes: a one-hot code (a known type) is a 1.0 among 0.0s,
        // so a bit of the stream; a prior or uniform code is a record the
        // streaming warps expand (any other code lights nothing); caller-given
        // beliefs are always records
        const bool bel_rec = st.ext || code == BC_UNIFORM || (code >= BC_PRIOR0 && code < BC_PRIOR0 + 30);
        if (base >= 0 && !st.ext && code >= 1 && code <= 12) st.one(base + code - 1, cell);
        if (base >= 0 && bel_rec) {
            flag = 1;
            st.B.pbase[p] = (uint8_t)base;
            st.B.pcode[p] = (uint8_t)code;
            if (st.ext) {
                float v[12];
                const float *src = st.ext + y * 17 + x;
#pragma unroll
                for (int t = 0; t < 12; ++t) v[t] = src[t * NC];
#pragma unroll
                for (int t = 0; t < 12; ++t) st.B.pbel[p][t] = v[t];
            }
        }
        const int half = team == oteam ? 0 : 4;
        st.one(66 + half + (mcnt < 3 ? mcnt : 3), cell);
        const int ae = ae_raw < 3 ? ae_raw : 3, ps = ps_raw < 3 ? ps_raw : 3;
        st.ones(74 + half, thresh_mask(ae + 1, 4), cell);
        st.ones(82 + half, thresh_mask(ps + 1, 4), cell);
        const int sch = S.slot_ch[p % 30];
        st.one(104 + (sch < 0 ? 24 : sch), cell);
        if (team != oteam) {
            // layer 1 + 3 (observation.py:1295-1392, 1474-1569)
            const int mine = __popcll(dlo) + __popcll(dhi), chn = __popcll(clo) + __popcll(chi);
            st.ones(173, thresh_mask(mine, 3), cell);
            st.ones(176, thresh_mask(other, 3), cell);
            st.ones(191, thresh_mask(chn, 3), cell);
            st.ones(161, (uint32_t)dtype & 0xFFFu, cell);
            st.ones(179, (uint32_t)ctype & 0xFFFu, cell);
            st.ones(194, thresh_mask(fl, 9), cell);
            if (is_g) st.one(203, cell);
            if (not_g) st.one(204, cell);
            if (in_back_two(s, zx, zy) && mcnt == 0 && !atk_g) st.one(205, cell);
            st.ones(223, pid_field30(dlo, dhi, o * 30), cell);
            // kill-count and recency planes: expanded from this record
            flag |= 2;
            st.B.pdlo[p] = dlo;
            st.B.pdhi[p] = dhi;
            *reinterpret_cast<float4 *>(st.B.prec[p]) = make_float4(recv[0], recv[1], recv[2], recv[3]);
        }
        st.B.pflag[p] = (uint8_t)flag;
        if (s == o) {  // layer 2 (observation.py:1394-1459)
            st.ones(206, thresh_mask(lc < rc ? lc : rc, 3), cell);
            if (lg) st.one(209, cell);
            if (in_back_two(s, zx, zy) && mcnt == 0 && !patk) st.one(210, cell);
        }
    } else {
        if (dstep != -1) {  // GameState.deaths keys
            const int ridx = (dreason >= 0 && dreason <= 2) ? dreason : (dreason == -1 ? 2 : -1);
            const int grp = s == o ? 0 : s == tm ? 3 : s == left ? 6 : s == right ? 9 : -1;
            if (ridx >= 0 && dstep > 0 && grp >= 0) {
                // numpy index semantics of death_loc // 17, death_loc % 17 (-1 -> row 16, col 16)
                int yy = dloc >= 0 ? dloc / 17 : -((-dloc + 16) / 17);
                const int xx = ((dloc % 17) + 17) % 17;
                if (yy < 0) yy += 17;
                if (yy >= 0 && yy < 17) st.one(90 + grp + ridx, st.rotf[yy * 17 + xx]);
            }
        }
        if (!(zx >= 0 && zx < 17 && zy >= 0 && zy < 17)) return;
        cell = st.rotf[zy * 17 + zx];
        if (dstep != -1) st.one(102 + (team == oteam ? 0 : 1), cell);
    }
    if (own_pid) {  // layer 4: observer-own pid at its cell (alive) or zero cell (dead)
        st.ones(257, pid_field30(elo, ehi, left * 30), cell);
        st.ones(287, pid_field30(elo, ehi, right * 30), cell);
    }
}

__device__ __forceinline__ float bit_value(const UnitBuf &B, int j, int qoff) {
    const int qq = j + qoff;
    return ((B.bits[qq >> 5] >> (qq & 31)) & 1u) ? 1.f : 0.f;
}

__device__ __forceinline__ int unit_head(const float *spatial, int u) {
    const float *out = spatial + (size_t)u * OBS_FLOATS;
    return (int)((OBS_VEC - (((uintptr_t)out >> 2) & (OBS_VEC - 1))) & (OBS_VEC - 1));
}

// Eight floats, bit i of `by` -> 1.0 else 0.0, as one 32-byte store (p is
// 32-byte aligned).
__device__ __forceinline__ void st_bits8(float *p, uint32_t by) {
    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p),
                 "f"((by & 1u) ? 1.f : 0.f), "f"((by & 2u) ? 1.f : 0.f), "f"((by & 4u) ? 1.f : 0.f),
                 "f"((by & 8u) ? 1.f : 0.f), "f"((by & 16u) ? 1.f : 0.f), "f"((by & 32u) ? 1.f : 0.f),
                 "f"((by & 64u) ? 1.f : 0.f), "f"((by & 128u) ? 1.f : 0.f)
                 : "memory");
}

// Staging warps: build unit u (observer o of env e) into B.  t = thread in 0..127.
__device__ __forceinline__ int unit_observer(const jq_batch &b, const int8_t *observers, int seats, int u) {
    const int e = u / seats;
    return (observers ? observers[u] : (seats == 1 ? b.turn[e] : u % seats)) & 3;
}

__device__ void stage_unit(const jq_batch &b, int seats, int mode, const float *ext_bel, float *global, ObsSmem &S,
                           UnitBuf &B, int u, int o, int head, int t, int bar_stage) {
    const int e = u / seats;
    const int tm = (o + 2) & 3, left = (o + 1) & 3, right = (o + 3) & 3;
    // B.bits arrive zeroed by the streaming warps
    Stager st{B, OBS_VEC - head, S.rotf[o], ext_bel ? ext_bel + ((size_t)e * 4 + o) * 12 * NC : nullptr};
    if (t < 32) {  // observer-own pids per tracked type: one load per lane, one ballot per type
        const int ti = t < 30 ? tracked_idx(b.piece_type[PI(e, o * 30 + t)]) : -1;
        const int pos = o * 30;
#pragma unroll
        for (int tt = 0; tt < 12; ++tt) {
            const uint64_t m = __ballot_sync(0xffffffffu, ti == tt) & 0x3FFFFFFFu;
            if (t == tt) {
                B.type_lo[tt] = pos < 64 ? m << pos : 0ull;
                B.type_hi[tt] = pos >= 64 ? m << (pos - 64) : (pos + 30 > 64 ? m >> (64 - pos) : 0ull);
            }
        }
    }
    if (t == 32) B.cval[0] = (float)fmin((double)b.mslc[e] / 200.0, 1.0);
    if (t == 33) B.cval[1] = (float)fmin((double)b.move_counter[e] / 4000.0, 1.0);
    // globals (observation.py:1623-1651); with caller-given beliefs the
    // streaming warps write global[0:24] from the belief records
    if (t >= 64 + (ext_bel ? 24 : 0) && t < 64 + OBS_GL) {
        const int j = t - 64;
        float v;
        if (j < 24) {
            v = (float)b.remaining[(size_t)e * 192 + (o * 4 + (j < 12 ? left : right)) * 12 + (j % 12)];
        } else {
            const int sf = j == 24 ? o : j == 25 ? tm : j == 26 ? left : right;
            v = b.seat_flag[(size_t)e * 4 + sf] ? 1.f : 0.f;
        }
        global[(size_t)u * OBS_GL + j] = v;
    }
    if (t == 0) {
        B.u = u;
        B.o = o;
        B.exc_n = 0;
        B.nbel = 0;
        B.ncm = 0;
    }
    bar_sync(bar_stage, OBS_STAGE_THREADS);
    // pieces, then history / constants / statics (all bit writes are atomic)
    {  // staging warp w takes a share of the pieces of seat o + w % 4: one seat relation per warp
        constexpr int wps = OBS_STAGE_WARPS / 4, per = (30 + wps - 1) / wps;
        const int ln = t & 31, wi = t >> 5, slot = (wi >> 2) * per + ln;
        const bool mine = ln < per && slot < 30;
        const int p = ((o + (wi & 3)) & 3) * 30 + (mine ? slot : 0);
        if (mine) stage_piece(b, e, o, mode, S, st, p);
        // list the pieces holding records, one shared atomic per warp and list
        const bool rec = mine && B.pcell[p] >= 0;
        const uint32_t fl = rec ? B.pflag[p] : 0u, below = (1u << ln) - 1u;
        const uint32_t mb = __ballot_sync(0xffffffffu, fl & 1u), mc = __ballot_sync(0xffffffffu, fl & 2u);
        int bb = 0, bc = 0;
        if (ln == 0) {
            bb = mb ? atomicAdd(&B.nbel, __popc(mb)) : 0;
            bc = mc ? atomicAdd(&B.ncm, __popc(mc)) : 0;
        }
        bb = __shfl_sync(0xffffffffu, bb, 0);
        bc = __shfl_sync(0xffffffffu, bc, 0);
        if (fl & 1u) {
            const int j = bb + __popc(mb & below), code = B.pcode[p];
            B.bel_list[j] = (uint8_t)p;
            B.bel_off[j] = B.pbase[p] * NC + B.pcell[p];
            B.bel_row[j] = (uint8_t)(code == BC_UNIFORM ? 30 : code - BC_PRIOR0);
        }
        if (fl & 2u) B.cm_list[bc + __popc(mc & below)] = (uint8_t)p;
    }
    if (t < HIST) {  // move history (observation.py:1207-1231)
        const int hc = b.hist_count[e], n = hc < HIST ? hc : HIST;
        if (t < n) {
            const int slot = (hc - 1 - t) & (HIST - 1);
            const int s = b.hist_src[(size_t)e * HIST + slot], d = b.hist_dst[(size_t)e * HIST + slot];
            if (s >= 0 && s < NC && d >= 0 && d < NC) {
                const int cs = st.rotf[s], cd = st.rotf[d];
                st.one(129 + t, cd);
                if (cs != cd) st.exception((129 + t) * NC + cs, -1.f);  // the destination's +1 wins
            }
        }
    } else {  // constant planes (observation.py:984-1021) and board statics (343-383)
        const int k = t - HIST, nk = OBS_STAGE_THREADS - HIST;
        uint32_t dead4 = 0, flag4 = 0;  // one load each: the env's four seat bytes
        {
            const uint8_t *sdp = b.seat_dead + (size_t)e * 4, *sfp = b.seat_flag + (size_t)e * 4;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                dead4 |= (sdp[i] ? 1u : 0u) << i;
                flag4 |= (sfp[i] ? 1u : 0u) << i;
            }
        }
#pragma unroll
        for (int j = 0; j < 7; ++j) {
            const int sd = j == 0 ? tm : j == 1 ? left : j == 2 ? right : j == 3 ? o : j == 4 ? tm : j == 5 ? left : right;
            const uint32_t on = ((j < 3 ? dead4 : flag4) >> sd) & 1u;
            if (on) st.fill_plane(B.bits, 51 + j, k, nk);
        }
        const uint32_t *sw = S.statw[o][st.qoff - 1];
        for (int w = k; w < STAT_WORDS; w += nk)
            if (sw[w]) atomicOr(&B.bits[STAT_W0 + w], sw[w]);
    }
}

// Streaming warps: write unit B.u.  w = streaming warp 0..nwarps-1, t = its thread;
// bar_stream is a named barrier of the nwarps streaming warps.
__device__ void stream_unit(UnitBuf &B, const float *bel_tab, bool ext, float *spatial,
                            float *global, int w, int lane, int nwarps, int bar_stream) {
    const int u = B.u, t = w * 32 + lane;
    float *out = spatial + (size_t)u * OBS_FLOATS;
    const int head = unit_head(spatial, u), qoff = OBS_VEC - head;
    const int body8 = (OBS_FLOATS - head) >> 3;
    // pass 1: every float as 0 / 1 -- the head and tail floats one by one, the
    // aligned body in groups of 8 (warp w: one contiguous slab), branch-free
    if (t < head) out[t] = bit_value(B, t, qoff);
    if (t >= 32 && t < 32 + OBS_VEC) {
        const int j = head + body8 * 8 + (t - 32);
        if (j < OBS_FLOATS) out[j] = bit_value(B, j, qoff);
    }
    float *out8 = out + head;
    const int per = (body8 + nwarps - 1) / nwarps;
    const int g0 = w * per, g1 = g0 + per < body8 ? g0 + per : body8;
    // group g holds output floats head + 8g .. +7 = stream bits 8g + 8 .. 8g
    // + 15, byte g + 1 of the stream; four groups per lane and pass, their
    // bytes loaded before the stores
    for (int g = g0 + lane; g < g1; g += 128) {
        uint32_t by[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int gi = g + 32 * i;
            by[i] = gi < g1 ? (B.bits[(gi + 1) >> 2] >> (((gi + 1) & 3) << 3)) & 0xffu : 0u;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (g + 32 * i < g1) st_bits8(out8 + 8 * (g + 32 * i), by[i]);
    }
    // pass 2, ordered after pass 1 by the streaming warps' barrier: the
    // floats that are neither 0 nor 1, over lines still in L2 -- exceptions,
    // then the values the per-piece records and the progress constants
    // expand to (observation.py:937-962, 1014-1021, 1541-1562); then the
    // bitstream is cleared for the unit staged next in B
    bar_sync(bar_stream, 32 * nwarps);
    const int nthr = 32 * nwarps;
    const int n = B.exc_n < EXC_MAX ? B.exc_n : EXC_MAX;
    for (int i = t; i < n; i += nthr) out[B.exc_pos[i]] = B.exc_val[i];
    const int nb = B.nbel * 12, nc = B.ncm * 16;
    for (int i = t; i < nb; i += nthr) {
        const int j = i / 12, k = i - j * 12;
        // caller-given beliefs are written where > 0 (observation.cu:330-370)
        const float v = ext ? B.pbel[B.bel_list[j]][k] : bel_tab[B.bel_row[j] * 12 + k];
        if (v > 0.f) out[B.bel_off[j] + k * NC] = v;
    }
    if (ext && t < 24) {
        // global[0:24] from caller-given beliefs: their sums over the left /
        // right enemy pieces' cells (observation.cu:417-424, 533-544), added
        // in ascending pid order (the reference's float atomics have none)
        const int base = t < 12 ? 27 : 39, k = t < 12 ? t : t - 12;
        float acc = 0.f;
        for (int p = 0; p < NP; ++p)
            if (B.pcell[p] >= 0 && (B.pflag[p] & 1) && B.pbase[p] == base) acc += B.pbel[p][k];
        global[(size_t)B.u * OBS_GL + t] = acc;
    }
    for (int i = t; i < nc; i += nthr) {
        const int j = i >> 4, k = i & 15, p = B.cm_list[j], cell = B.pcell[p];
        if (k < 12) {
            const int c = __popcll(B.pdlo[p] & B.type_lo[k]) + __popcll(B.pdhi[p] & B.type_hi[k]);
            if (c) out[(211 + k) * NC + cell] = __fdiv_rn((float)(c < 3 ? c : 3), 3.0f);
        } else {
            const float r = B.prec[p][k - 12];
            if (r > 0.f) out[(253 + k - 12) * NC + cell] = r;
        }
    }
    for (int i = t; i < P2_PROG; i += nthr) {
        const int j = i >= NC ? 1 : 0;
        const float v = B.cval[j];
        if (v != 0.f) out[(64 + j) * NC + i - j * NC] = v;
    }
    uint4 *b4 = reinterpret_cast<uint4 *>(B.bits);
    for (int k = t; k < OBS_WORDS4; k += nthr) b4[k] = make_uint4(0u, 0u, 0u, 0u);
}

// Grid: persistent.  ticket[0] hands out units u = e * seats + k in order;
// ticket[1] counts finished CTAs, and the last one resets both to zero for
// the next launch that uses this ticket.
__global__ void __launch_bounds__(OBS_THREADS, OBS_MIN_CTAS) obs_kernel(jq_batch b, const int8_t *__restrict__ observers,
                                                                        int seats, int mode, float *spatial,
                                                                        float *global, int *ticket,
                                                                        const float *__restrict__ ext_bel) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ObsSmem &S = *reinterpret_cast<ObsSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) JQ_TRACE_AT(0, TO_ENTRY);
    asm volatile("griddepcontrol.launch_dependents;");
    // once per CTA: observer rotations, belief tables and board-static words
    // into shared memory; both bitstreams cleared
    for (int i = tid; i < 4 * NC; i += OBS_THREADS) (&S.rotf[0][0])[i] = (&g_topo.rotf[0][0])[i];
    for (int i = tid; i < 30 * 12; i += OBS_THREADS) S.bel_tab[i] = g_prior[i];
    if (tid < 12) S.bel_tab[30 * 12 + tid] = g_uniform[tid];
    if (tid < 30) S.slot_ch[tid] = g_topo.slot_ch[tid];
    for (int i = tid; i < 2 * OBS_WORDS4; i += OBS_THREADS)
        reinterpret_cast<uint4 *>(S.buf[i / OBS_WORDS4].bits)[i % OBS_WORDS4] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid; i < 4 * OBS_VEC * STAT_WORDS; i += OBS_THREADS) (&S.statw[0][0][0])[i] = (&g_statw[0][0][0])[i];
    // launched as a programmatic dependent (see the rules kernel): caller
    // memory -- tickets, state, outputs -- only after the previous kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __syncthreads();
    if (tid == 0) JQ_TRACE_AT(0, TO_WAITED);
    const int units = b.n * seats;
    if (warp < OBS_STREAM_WARPS) {
        for (int k = 0;; ++k) {
            const int bi = k & 1;
            bar_sync(BAR_FULL0 + bi, OBS_THREADS);  // buffer bi staged
            if (tid == 0 && k < 3) JQ_TRACE_AT(0, TO_UNIT_STREAM0 + 2 * k);
            UnitBuf &B = S.buf[bi];
            if (B.u < 0) break;
            if (k == 0 && tid == 0) JQ_TRACE_AT(0, TO_FIRST_STREAM);
            stream_unit(B, S.bel_tab, ext_bel != nullptr, spatial, global, warp, lane, OBS_STREAM_WARPS,
                        BAR_STREAM);
            if (tid == 0 && k < 3) JQ_TRACE_AT(0, TO_UNIT_STREAM0 + 2 * k + 1);
            if (tid == 0) JQ_TRACE_AT(0, TO_LAST_STREAMED);
            bar_arrive(BAR_EMPTY0 + bi, OBS_THREADS);  // buffer bi free again
        }
    } else {
        const int t = tid - 32 * OBS_STREAM_WARPS;
        // A unit is taken only when the staging warps are ready to build it:
        // the units being written at any moment then stay in the tightest
        // window of the output, and no CTA holds a unit it has not started
        // when the tickets run out (a reservation one unit ahead measured
        // 1 % slower at both 4,096 and 65,536 units).
        if (t == 0) {
            const int u0 = atomicAdd(&ticket[0], 1);
            S.ticket[0] = u0;
            S.next_o[0] = u0 < units ? unit_observer(b, observers, seats, u0) : 0;
        }
        bar_sync(BAR_STAGE, OBS_STAGE_THREADS);
        int u = S.ticket[0], o = S.next_o[0];
        int k = 0;
        for (;; ++k) {
            const int bi = k & 1;
            UnitBuf &B = S.buf[bi];
            if (k >= 2) bar_sync(BAR_EMPTY0 + bi, OBS_THREADS);  // unit k - 2 streamed out of buffer bi
            if (t == 0 && (k == 2 || k == 3)) JQ_TRACE_AT(0, TO_UNIT_STAGE_START2 + k - 2);
            if (u >= units) {
                if (t == 0) B.u = -1;
                bar_arrive(BAR_FULL0 + bi, OBS_THREADS);
                break;
            }
            stage_unit(b, seats, mode, ext_bel, global, S, B, u, o, unit_head(spatial, u), t, BAR_STAGE);
            bar_sync(BAR_STAGE, OBS_STAGE_THREADS);    // unit staged by every staging thread
            if (k == 0 && t == 0) JQ_TRACE_AT(0, TO_FIRST_STAGED);
            if (t == 0) JQ_TRACE_AT(0, TO_LAST_STAGED);
            if (t == 0 && k < 3) JQ_TRACE_AT(0, TO_UNIT_STAGED0 + k);
            bar_arrive(BAR_FULL0 + bi, OBS_THREADS);  // hand it to the streaming warps
            if (t == 0) {
                const int un = atomicAdd(&ticket[0], 1);
                S.ticket[0] = un;
                S.next_o[0] = un < units ? unit_observer(b, observers, seats, un) : 0;
                if (un < units) JQ_TRACE_AT(0, TO_LAST_TICKET);
            }
            bar_sync(BAR_STAGE, OBS_STAGE_THREADS);  // next ticket published
            u = S.ticket[0];
            o = S.next_o[0];
        }
        if (k >= 1) bar_sync(BAR_EMPTY0 + ((k - 1) & 1), OBS_THREADS);  // the last unit has been streamed
        if (t == 0) {
            JQ_TRACE_AT(0, TO_EXIT);
            JQ_TRACE_COUNT(0, TO_UNITS, k);
            __threadfence();
            if (atomicAdd(&ticket[1], 1) == (int)gridDim.x - 1) {
                ticket[0] = 0;
                ticket[1] = 0;
            }
        }
    }
}

}  // namespace jq
