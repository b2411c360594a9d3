/*
 * jq_oracle.c -- scalar CPU restatement of the JunQi reference rules.
 *
 * TEST INFRASTRUCTURE ONLY (see jq_oracle.h).  Every function cites the
 * junqi_core file:line it restates.  Nothing here is shared with the CUDA
 * product code: the tables below are rebuilt independently so that a
 * topology mistake in either copy shows up as a parity failure.
 */
#include "jq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* junqi_core/rules.py:57-74 PieceType values */
enum { T_NONE = 0, T_DARK = 1, T_JUNQI = 2, T_DILEI = 3, T_ZHADAN = 4, T_SILING = 5,
       T_JUNZH = 6, T_SHIZH = 7, T_LVZH = 8, T_TUANZH = 9, T_YINGZH = 10, T_LIANZH = 11,
       T_PAIZH = 12, T_GONGB = 13 };
/* rules.py:255-261 Event */
enum { EV_MOVE = 1, EV_EAT = 2, EV_BOMB = 3, EV_KILLED = 4 };
/* rules.py:281-286 DeathReason */
enum { DR_KBE = 0, DR_MINE = 1, DR_MUTUAL = 2 };
/* rules.py:598-603 ShowMode */
enum { SM_BRIGHT = 0, SM_DARK = 1, SM_HALF_DARK = 2 };

#define NC 289
#define NP 120

/* ======================================================================
 * Topology (junqi_core/board.py:80-255, rail_topology.py:91-262,
 * _movegen_tables.py:130-470)
 * ====================================================================== */
static int T_on[NC], T_camp[NC], T_sh[NC], T_rail[NC], T_nine[NC], T_curve[NC];
static int T_adj[NC][4];
static int T_diag[NC][4], T_ndiag[NC];
static int T_radj[NC][4], T_nradj[NC];
static int T_sray[NC][4][12], T_nsray[NC][4];
static int T_cray[NC][2][11], T_ncray[NC][2];
static int T_curve_active[NC];
static int T_c2f[129], T_f2c[NC];
static int T_rot[4][NC];
static int T_arc[NC];
static int T_ready = 0;

/* board.py:80-99 index_to_pos */
static void index_to_pos(int seat, int i, int *x, int *y) {
    int col = i % 5, row = i / 5;
    switch (seat) {
    case 0: *x = 10 - col; *y = 11 + row; break;
    case 1: *x = 5 - row; *y = 10 - col; break;
    case 2: *x = 6 + col; *y = 5 - row; break;
    default: *x = 11 + row; *y = 6 + col; break;
    }
}

static int is_camp_slot(int i) { return i == 6 || i == 8 || i == 12 || i == 16 || i == 18; }

static void build_topology(void) {
    if (T_ready) return;
    int x, y;
    memset(T_on, 0, sizeof T_on);
    memset(T_camp, 0, sizeof T_camp);
    memset(T_sh, 0, sizeof T_sh);
    memset(T_rail, 0, sizeof T_rail);
    memset(T_nine, 0, sizeof T_nine);
    memset(T_curve, 0, sizeof T_curve);
    /* rail_topology.py:172-188 curve ids, last write wins */
    for (int cid = 1; cid <= 4; ++cid) {
        int sa = cid - 1, sb = cid % 4;
        for (int j = 0; j < 30; ++j) {
            if (j % 5 != 4) continue;
            index_to_pos(sa, j, &x, &y);
            T_curve[y * 17 + x] = cid;
            index_to_pos(sb, j - 4, &x, &y);
            T_curve[y * 17 + x] = cid;
        }
    }
    /* board.py:139-169 seat zones, rail rule i<25 && (row in {0,4} || col in {0,4}) */
    for (int s = 0; s < 4; ++s)
        for (int i = 0; i < 30; ++i) {
            index_to_pos(s, i, &x, &y);
            int f = y * 17 + x, row = i / 5, col = i % 5;
            T_on[f] = 1;
            T_camp[f] = is_camp_slot(i);
            T_sh[f] = (i == 26 || i == 28);
            T_rail[f] = (i < 25) && (row == 0 || row == 4 || col == 0 || col == 4);
        }
    /* board.py:178-196 nine grid cells are rail */
    for (int i = 0; i < 9; ++i) {
        x = 10 - (i % 3) * 2;
        y = 6 + (i / 3) * 2;
        T_on[y * 17 + x] = 1;
        T_rail[y * 17 + x] = 1;
        T_nine[y * 17 + x] = 1;
    }
    /* rail_topology.py:199-238 adjacency: ortho rail, nine-grid 2-steps, 4 corner arcs */
    static unsigned char A[NC][NC];
    memset(A, 0, sizeof A);
    for (int f = 0; f < NC; ++f) {
        if (!T_rail[f]) continue;
        int fx = f % 17, fy = f / 17;
        static const int d4[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
        for (int k = 0; k < 4; ++k) {
            int nx = fx + d4[k][0], ny = fy + d4[k][1];
            if (nx < 0 || nx > 16 || ny < 0 || ny > 16) continue;
            int g = ny * 17 + nx;
            if (T_rail[g]) A[f][g] = A[g][f] = 1;
        }
        if (T_nine[f])
            for (int k = 0; k < 4; ++k) {
                int nx = fx + 2 * d4[k][0], ny = fy + 2 * d4[k][1];
                if (nx < 0 || nx > 16 || ny < 0 || ny > 16) continue;
                int g = ny * 17 + nx;
                if (T_nine[g]) A[f][g] = A[g][f] = 1;
            }
    }
    static const int spc[4][4] = {{10, 11, 11, 10}, {6, 11, 5, 10}, {6, 5, 5, 6}, {11, 6, 10, 5}};
    for (int k = 0; k < 4; ++k) {
        int a = spc[k][1] * 17 + spc[k][0], b = spc[k][3] * 17 + spc[k][2];
        A[a][b] = A[b][a] = 1;
    }
    for (int f = 0; f < NC; ++f) {
        T_nradj[f] = 0;
        for (int g = 0; g < NC; ++g)
            if (A[f][g]) T_radj[f][T_nradj[f]++] = g; /* ascending, rail_topology.py:238 */
    }
    /* _movegen_tables.py:164-180 ADJ_STRAIGHT (+x,-x,+y,-y) */
    static const int dirs[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
    for (int f = 0; f < NC; ++f) {
        int fx = f % 17, fy = f / 17;
        for (int k = 0; k < 4; ++k) {
            T_adj[f][k] = -1;
            if (!T_on[f]) continue;
            int nx = fx + dirs[k][0], ny = fy + dirs[k][1];
            if (nx < 0 || nx > 16 || ny < 0 || ny > 16) continue;
            if (T_on[ny * 17 + nx]) T_adj[f][k] = ny * 17 + nx;
        }
    }
    /* _movegen_tables.py:190-208 ADJ_DIAG_INTO_CAMP order (1,1),(1,-1),(-1,1),(-1,-1) */
    static const int dg[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
    for (int f = 0; f < NC; ++f) {
        T_ndiag[f] = 0;
        if (!T_on[f]) continue;
        int fx = f % 17, fy = f / 17;
        for (int k = 0; k < 4; ++k) {
            int nx = fx + dg[k][0], ny = fy + dg[k][1];
            if (nx < 0 || nx > 16 || ny < 0 || ny > 16) continue;
            int g = ny * 17 + nx;
            if (!T_on[g]) continue;
            if (T_camp[f] || T_camp[g]) T_diag[f][T_ndiag[f]++] = g;
        }
    }
    /* _movegen_tables.py:230-284 straight rail rays: graph walk along the axis */
    for (int f = 0; f < NC; ++f) {
        for (int k = 0; k < 4; ++k) T_nsray[f][k] = 0;
        if (!T_rail[f]) continue;
        int sx = f % 17, sy = f / 17;
        for (int k = 0; k < 4; ++k) {
            int dx = dirs[k][0], dy = dirs[k][1];
            int px = sx, py = sy;
            for (;;) {
                int nxt = -1;
                int cur = py * 17 + px;
                for (int j = 0; j < T_nradj[cur]; ++j) {
                    int nb = T_radj[cur][j], nx = nb % 17, ny = nb / 17;
                    if (dx != 0) {
                        if (ny != sy) continue;
                        if ((nx - px) * dx <= 0) continue;
                    } else {
                        if (nx != sx) continue;
                        if ((ny - py) * dy <= 0) continue;
                    }
                    if (nb == f) continue;
                    nxt = nb;
                }
                if (nxt < 0) break;
                T_sray[f][k][T_nsray[f][k]++] = nxt;
                px = nxt % 17;
                py = nxt / 17;
            }
        }
    }
    /* _movegen_tables.py:375-470 curve chains and their per-cell rays */
    static int cnb[NC][4], ncnb[NC];
    for (int f = 0; f < NC; ++f) {
        ncnb[f] = 0;
        if (!T_curve[f]) continue;
        for (int j = 0; j < T_nradj[f]; ++j)
            if (T_curve[T_radj[f][j]] == T_curve[f]) cnb[f][ncnb[f]++] = T_radj[f][j];
    }
    for (int f = 0; f < NC; ++f) {
        T_ncray[f][0] = T_ncray[f][1] = 0;
        T_curve_active[f] = (T_curve[f] > 0 && ncnb[f] > 0);
    }
    for (int cid = 1; cid <= 4; ++cid) {
        int active[NC], na = 0, start = -1;
        for (int f = 0; f < NC; ++f)
            if (T_curve[f] == cid && ncnb[f] > 0) active[na++] = f;
        for (int i = 0; i < na; ++i)
            if (ncnb[active[i]] == 1) { start = active[i]; break; }
        int chain[NC], nch = 0;
        if (start < 0) {
            for (int i = 0; i < na; ++i) chain[nch++] = active[i];
        } else {
            unsigned char vis[NC];
            memset(vis, 0, sizeof vis);
            chain[nch++] = start;
            vis[start] = 1;
            for (;;) {
                int cur = chain[nch - 1], found = 0;
                for (int j = 0; j < ncnb[cur]; ++j) {
                    int nb = cnb[cur][j];
                    if (!vis[nb]) { chain[nch++] = nb; vis[nb] = 1; found = 1; break; }
                }
                if (!found) break;
            }
        }
        for (int i = 0; i < nch; ++i) {
            int f = chain[i];
            for (int j = i + 1; j < nch && T_ncray[f][0] < 11; ++j) T_cray[f][0][T_ncray[f][0]++] = chain[j];
            for (int j = i - 1; j >= 0 && T_ncray[f][1] < 11; --j) T_cray[f][1][T_ncray[f][1]++] = chain[j];
        }
    }
    /* board.py:263-280 compact maps */
    int c = 0;
    for (int f = 0; f < NC; ++f) {
        T_f2c[f] = -1;
        if (T_on[f]) { T_f2c[f] = c; T_c2f[c++] = f; }
    }
    /* rotation.py:44-65 world_to_canonical */
    for (int s = 0; s < 4; ++s)
        for (int f = 0; f < NC; ++f) {
            int wx = f % 17, wy = f / 17, cx, cy;
            switch (s) {
            case 0: cx = wx; cy = wy; break;
            case 1: cx = wy; cy = 16 - wx; break;
            case 2: cx = 16 - wx; cy = 16 - wy; break;
            default: cx = 16 - wy; cy = wx; break;
            }
            T_rot[s][f] = cy * 17 + cx;
        }
    /* rail_topology.py:245-262 CURVE_ARC_CELLS */
    for (int f = 0; f < NC; ++f) {
        T_arc[f] = 0;
        int fx = f % 17, fy = f / 17;
        for (int j = 0; j < T_nradj[f]; ++j) {
            int nb = T_radj[f][j], nx = nb % 17, ny = nb / 17;
            if (abs(fx - nx) == 1 && abs(fy - ny) == 1) { T_arc[f] = 1; break; }
        }
    }
    T_ready = 1;
}

int jqo_topology(int32_t *on_board, int32_t *rail, int32_t *curve, int32_t *rail_adj,
                 int32_t *srays, int32_t *crays, int32_t *c2f) {
    build_topology();
    for (int f = 0; f < NC; ++f) {
        on_board[f] = T_on[f];
        rail[f] = T_rail[f];
        curve[f] = T_curve[f];
        for (int k = 0; k < 4; ++k) rail_adj[f * 4 + k] = k < T_nradj[f] ? T_radj[f][k] : -1;
        for (int k = 0; k < 4; ++k)
            for (int l = 0; l < 12; ++l)
                srays[(f * 4 + k) * 12 + l] = l < T_nsray[f][k] ? T_sray[f][k][l] : -1;
        for (int k = 0; k < 2; ++k)
            for (int l = 0; l < 11; ++l)
                crays[(f * 2 + k) * 11 + l] = l < T_ncray[f][k] ? T_cray[f][k][l] : -1;
    }
    for (int i = 0; i < 129; ++i) c2f[i] = T_c2f[i];
    return 0;
}

/* ======================================================================
 * Tables supplied by the host (generated with numpy exactly as the
 * reference does: _zobrist.py:80-122, info_model.py:126-146,
 * observation.py:1560-1562)
 * ====================================================================== */
static int64_t Z_piece[NP * 14 * NC], Z_turn[4], Z_mc[4096], Z_mslc[512], Z_term, Z_win[3],
    Z_draw, Z_sdead[4], Z_sflag[4], Z_show[4];
static float P_prior[30 * 12], P_uniform[12], P_recency[4 * 4097];

int jqo_set_tables(const int64_t *zp, const int64_t *zt, const int64_t *zmc, const int64_t *zms,
                   int64_t zterm, const int64_t *zw, int64_t zdraw, const int64_t *zsd,
                   const int64_t *zsf, const int64_t *zsm, const float *prior,
                   const float *uniform12, const float *recency) {
    build_topology();
    memcpy(Z_piece, zp, sizeof Z_piece);
    memcpy(Z_turn, zt, sizeof Z_turn);
    memcpy(Z_mc, zmc, sizeof Z_mc);
    memcpy(Z_mslc, zms, sizeof Z_mslc);
    Z_term = zterm;
    memcpy(Z_win, zw, sizeof Z_win);
    Z_draw = zdraw;
    memcpy(Z_sdead, zsd, sizeof Z_sdead);
    memcpy(Z_sflag, zsf, sizeof Z_sflag);
    memcpy(Z_show, zsm, sizeof Z_show);
    memcpy(P_prior, prior, sizeof P_prior);
    memcpy(P_uniform, uniform12, sizeof P_uniform);
    memcpy(P_recency, recency, sizeof P_recency);
    return 0;
}

#define ZP(pid, t, f) Z_piece[((pid) * 14 + (t)) * NC + (f)]

/* ======================================================================
 * Per-env accessors
 * ====================================================================== */
#define PI(e, p) ((size_t)(e) * NP + (p))
#define CI(e, f) ((size_t)(e) * NC + (f))
#define SI(e, s) ((size_t)(e) * 4 + (s))
#define OI(e, o, p) (((size_t)(e) * 4 + (o)) * NP + (p))

static inline int team_of_pid(int pid) { return (pid / 30) & 1; } /* move_gen.py:1003 */

/* ======================================================================
 * Legal generation (move_gen.py:1311-1553 generate_legal_action_ids_n,
 * per env; move_gen.py:870-890 _engineer_dests_soa)
 * ====================================================================== */
static int cmp_i32(const void *a, const void *b) {
    int32_t x = *(const int32_t *)a, y = *(const int32_t *)b;
    return (x > y) - (x < y);
}

/* Emits sorted, de-duplicated ids into out (up to cap); returns the count
 * (which may exceed cap, in which case only cap ids were written). */
static int legal_env(const jqo_batch *b, int e, int seat, int32_t *out, int cap) {
    const int16_t *cp = b->cell_pid + CI(e, 0);
    unsigned char empty[NC], att[NC], land[NC];
    int at = seat & 1;
    for (int f = 0; f < NC; ++f) {
        int pid = cp[f];
        empty[f] = pid < 0;
        att[f] = pid >= 0 && team_of_pid(pid) != at && !T_camp[f];
        land[f] = empty[f] | att[f];
    }
    int32_t tmp[2048];
    int n = 0;
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        if (!b->alive[q] || b->piece_seat[q] != seat) continue;
        int t = b->piece_type[q];
        if (t == T_JUNQI || t == T_DILEI) continue; /* _movegen_tables.py:146 IS_IMMOBILE_TYPE */
        int px = b->pos_x[q], py = b->pos_y[q];
        if (px < 0 || py < 0) continue;
        int sf = py * 17 + px;
        if (sf >= NC || T_sh[sf]) continue;
        int base = sf * NC;
        for (int k = 0; k < 4; ++k) {
            int nb = T_adj[sf][k];
            if (nb >= 0 && land[nb]) tmp[n++] = base + nb;
        }
        for (int k = 0; k < T_ndiag[sf]; ++k) {
            int nb = T_diag[sf][k];
            if (land[nb]) tmp[n++] = base + nb;
        }
        if (!T_rail[sf]) continue;
        if (t == T_GONGB) {
            unsigned char vis[NC];
            int queue[NC], qh = 0, qt = 0;
            memset(vis, 0, sizeof vis);
            vis[sf] = 1;
            queue[qt++] = sf;
            while (qh < qt) {
                int cur = queue[qh++];
                for (int j = 0; j < T_nradj[cur]; ++j) {
                    int nb = T_radj[cur][j];
                    if (vis[nb]) continue;
                    vis[nb] = 1;
                    if (empty[nb]) { tmp[n++] = base + nb; queue[qt++] = nb; }
                    else if (att[nb]) tmp[n++] = base + nb;
                }
            }
        } else {
            for (int k = 0; k < 4; ++k)
                for (int l = 0; l < T_nsray[sf][k]; ++l) {
                    int nb = T_sray[sf][k][l];
                    if (land[nb]) tmp[n++] = base + nb;
                    if (!empty[nb]) break;
                }
            if (T_curve[sf] > 0 && T_curve_active[sf])
                for (int k = 0; k < 2; ++k)
                    for (int l = 0; l < T_ncray[sf][k]; ++l) {
                        int nb = T_cray[sf][k][l];
                        if (land[nb]) tmp[n++] = base + nb;
                        if (!empty[nb]) break;
                    }
        }
    }
    qsort(tmp, (size_t)n, sizeof(int32_t), cmp_i32);
    int m = 0;
    for (int i = 0; i < n; ++i) {
        if (i > 0 && tmp[i] == tmp[i - 1]) continue;
        if (m < cap) out[m] = tmp[i];
        ++m;
    }
    return m;
}

/* batched_state.py:370-409 legal_action_ids_batch: empty when terminated or
 * the seat is dead. */
int jqo_legal(const jqo_batch *b, int e, int seat, int ignore_skip, int32_t *out, int cap) {
    build_topology();
    if (seat < 0 || seat > 3) return 0;
    if (!ignore_skip && (b->terminated[e] || b->seat_dead[SI(e, seat)])) return 0;
    return legal_env(b, e, seat, out, cap);
}

int jqo_legal_batch(const jqo_batch *b, const int8_t *seats, int32_t *counts, int32_t *ids,
                    int cap, int nthreads) {
    build_topology();
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads > 0 ? nthreads : 1)
    for (int e = 0; e < b->n; ++e)
        counts[e] = jqo_legal(b, e, seats[e], 0, ids + (size_t)e * cap, cap);
    return 0;
}

/* move_gen.py:1557-1609 has_legal_moves_soa (no terminated / dead check) */
static int has_moves(const jqo_batch *b, int e, int seat) {
    int32_t tmp[1];
    return legal_env(b, e, seat, tmp, 0) > 0;
}

/* action_lut.py:174-212 world ids -> compact canonical mask */
int jqo_canonical_mask(const int32_t *ids, int count, int seat, uint8_t *mask) {
    build_topology();
    memset(mask, 0, JQO_ACTIONS_COMPACT);
    for (int i = 0; i < count; ++i) {
        int sf = ids[i] / NC, df = ids[i] % NC;
        int cs = T_f2c[T_rot[seat][sf]], cd = T_f2c[T_rot[seat][df]];
        if (cs >= 0 && cd >= 0) mask[cs * 129 + cd] = 1;
    }
    return 0;
}

/* ======================================================================
 * Per-piece 80-slot legal mask: the reference GPU format of
 * legal_action_mask_batch (src/env/cuda/src/game_state.cu:1985-2197, tables
 * from tables.cu:176-350).  junqi_core has no counterpart; this restates the
 * kernel's algorithm so the CUDA path has a checker, and additionally
 * reports the destination cell of every set slot.
 * ====================================================================== */
static int S_adj8[NC][8];      /* tables.cu:176-211: 4 ortho (+x,-x,+y,-y), then camp diagonals compacted */
static int S_ri[NC];           /* flat -> rail index (rail cells in flat order) */
static int S_rcell[NC];        /* rail index -> flat */
static int S_nrail;
static int S_rn[NC][8], S_nrn[NC]; /* rail-index adjacency, ascending (tables.cu:291) */
static int S_sray[NC][4][12];  /* tables.cu:303-350 straight rays, -1 padded */
static int S_ready = 0;

static void build_slot_tables(void) {
    if (S_ready) return;
    build_topology();
    static const int dd[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
    for (int f = 0; f < NC; ++f) {
        for (int k = 0; k < 8; ++k) S_adj8[f][k] = -1;
        if (!T_on[f]) continue;
        for (int k = 0; k < 4; ++k) S_adj8[f][k] = T_adj[f][k];
        int fx = f % 17, fy = f / 17, slot = 4;
        for (int k = 0; k < 4 && slot < 8; ++k) {
            int nx = fx + dd[k][0], ny = fy + dd[k][1];
            if (nx < 0 || nx > 16 || ny < 0 || ny > 16) continue;
            int g = ny * 17 + nx;
            if (!T_on[g]) continue;
            if (T_camp[f] || T_camp[g]) S_adj8[f][slot++] = g;
        }
    }
    S_nrail = 0;
    for (int f = 0; f < NC; ++f) {
        S_ri[f] = -1;
        if (T_rail[f]) { S_ri[f] = S_nrail; S_rcell[S_nrail++] = f; }
    }
    for (int r = 0; r < S_nrail; ++r) {
        int f = S_rcell[r];
        S_nrn[r] = 0;
        for (int k = 0; k < T_nradj[f] && S_nrn[r] < 8; ++k) S_rn[r][S_nrn[r]++] = S_ri[T_radj[f][k]];
    }
    static const int d4[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
    for (int f = 0; f < NC; ++f)
        for (int d = 0; d < 4; ++d)
            for (int k = 0; k < 12; ++k) S_sray[f][d][k] = -1;
    for (int r = 0; r < S_nrail; ++r) {
        int src = S_rcell[r], sx = src % 17, sy = src / 17;
        for (int d = 0; d < 4; ++d) {
            int k = 0, cur = src, prev = -1;
            while (k < 12) {
                int cr = S_ri[cur], next = -1;
                if (cr < 0) break;
                for (int i = 0; i < S_nrn[cr]; ++i) {
                    int nb = S_rcell[S_rn[cr][i]];
                    if (nb == prev) continue;
                    int nx = nb % 17, ny = nb / 17;
                    if (d4[d][0] != 0) {
                        if (ny != sy || (nx - cur % 17) * d4[d][0] <= 0) continue;
                    } else {
                        if (nx != sx || (ny - cur / 17) * d4[d][1] <= 0) continue;
                    }
                    next = nb;
                    break; /* the chain is simple: first match wins */
                }
                if (next < 0) break;
                S_sray[src][d][k++] = next;
                prev = cur;
                cur = next;
            }
        }
    }
    S_ready = 1;
}

int jqo_slot_tables(int32_t *adj8 /*289x8*/, int32_t *srays /*289x4x12*/, int32_t *rail_adj /*289x8 flat*/) {
    build_slot_tables();
    for (int f = 0; f < NC; ++f) {
        for (int k = 0; k < 8; ++k) {
            adj8[f * 8 + k] = S_adj8[f][k];
            rail_adj[f * 8 + k] = (S_ri[f] >= 0 && k < S_nrn[S_ri[f]]) ? S_rcell[S_rn[S_ri[f]][k]] : -1;
        }
        for (int d = 0; d < 4; ++d)
            for (int k = 0; k < 12; ++k) srays[(f * 4 + d) * 12 + k] = S_sray[f][d][k];
    }
    return 0;
}

/* game_state.cu:1985-2197, one (env, pid) row per piece of `seat`. */
int jqo_slot_mask(const jqo_batch *b, int env, int seat, uint8_t *mask /*120x80*/, int16_t *dst /*120x80*/) {
    build_slot_tables();
    memset(mask, 0, NP * JQO_SLOTS);
    if (dst)
        for (int i = 0; i < NP * JQO_SLOTS; ++i) dst[i] = -1;
    const size_t q0 = (size_t)env * NP;
    const int16_t *cp = b->cell_pid + (size_t)env * NC;
    const int team = seat & 1;
#define SLOT_SET(slot, cell)                                    \
    do {                                                        \
        mask[pid * JQO_SLOTS + (slot)] = 1;                     \
        if (dst) dst[pid * JQO_SLOTS + (slot)] = (int16_t)(cell); \
    } while (0)
    for (int pid = 0; pid < NP; ++pid) {
        if (b->piece_seat[q0 + pid] != seat || !b->alive[q0 + pid]) continue;
        int t = b->piece_type[q0 + pid];
        if (t == T_JUNQI || t == T_DILEI) continue;
        int sx = b->pos_x[q0 + pid], sy = b->pos_y[q0 + pid];
        if (sx < 0 || sy < 0) continue;
        int src = sy * 17 + sx;
        if (src >= NC || !T_on[src] || T_sh[src]) continue;
#define ENEMY_AT(cell, occ) ((((int)b->piece_seat[q0 + (occ)]) & 1) != team && !T_camp[cell])
        for (int k = 0; k < 8; ++k) {
            int nb = S_adj8[src][k];
            if (nb < 0) continue;
            int occ = cp[nb];
            if (occ < 0 || ENEMY_AT(nb, occ)) SLOT_SET(k, nb);
        }
        if (!T_rail[src]) continue;
        const int o0 = S_adj8[src][0], o1 = S_adj8[src][1], o2 = S_adj8[src][2], o3 = S_adj8[src][3];
#define IS_ORTHO(c) ((c) == o0 || (c) == o1 || (c) == o2 || (c) == o3)
        unsigned char vis[NC];
        int qu[NC], qh = 0, qt = 0;
        if (t != T_GONGB) {
            for (int d = 0; d < 4; ++d)
                for (int k = 0; k < 12; ++k) {
                    int nb = S_sray[src][d][k];
                    if (nb < 0) break;
                    int occ = cp[nb], slot = 8 + d * 12 + k;
                    if (occ < 0) {
                        if (!IS_ORTHO(nb)) SLOT_SET(slot, nb);
                    } else {
                        if (!IS_ORTHO(nb) && ENEMY_AT(nb, occ)) SLOT_SET(slot, nb);
                        break;
                    }
                }
            int sc = T_curve[src], sr = S_ri[src];
            if (sc > 0 && sr >= 0) {
                memset(vis, 0, sizeof vis);
                vis[sr] = 1;
                qu[qt++] = sr;
                int cs = 56;
                while (qh < qt) {
                    int cur = qu[qh++];
                    for (int i = 0; i < S_nrn[cur]; ++i) {
                        int nr = S_rn[cur][i];
                        if (vis[nr]) continue;
                        vis[nr] = 1;
                        int nf = S_rcell[nr];
                        if (T_curve[nf] != sc) continue;
                        int same_axis = (nf % 17 == sx) || (nf / 17 == sy);
                        int occ = cp[nf];
                        if (occ < 0) {
                            if (!same_axis && cs < 68) { SLOT_SET(cs, nf); ++cs; }
                            qu[qt++] = nr;
                        } else if (!same_axis && cs < 68 && ENEMY_AT(nf, occ)) {
                            SLOT_SET(cs, nf);
                            ++cs;
                        }
                    }
                }
            }
        } else {
            int sr = S_ri[src];
            if (sr < 0) continue;
            memset(vis, 0, sizeof vis);
            vis[sr] = 1;
            qu[qt++] = sr;
            int cs = 8;
            while (qh < qt) {
                int cur = qu[qh++];
                for (int i = 0; i < S_nrn[cur]; ++i) {
                    int nr = S_rn[cur][i];
                    if (vis[nr]) continue;
                    vis[nr] = 1;
                    int nf = S_rcell[nr], occ = cp[nf];
                    if (occ < 0) {
                        if (!IS_ORTHO(nf) && cs < JQO_SLOTS) { SLOT_SET(cs, nf); ++cs; }
                        qu[qt++] = nr;
                    } else if (!IS_ORTHO(nf) && cs < JQO_SLOTS && ENEMY_AT(nf, occ)) {
                        SLOT_SET(cs, nf);
                        ++cs;
                    }
                }
            }
        }
#undef IS_ORTHO
#undef ENEMY_AT
    }
#undef SLOT_SET
    return 0;
}

/* ======================================================================
 * move_requires_gongb (move_gen.py:245-296) on the pre-move board
 * ====================================================================== */
/* move_gen.py:127-165 _straight_rail_clear */
static int straight_rail_clear(const int16_t *cp, int s, int d) {
    if (s == d) return 0;
    int sx = s % 17, sy = s / 17, dx = d % 17, dy = d / 17;
    if (sx != dx && sy != dy) return 0;
    unsigned char vis[NC];
    int q[NC], qh = 0, qt = 0;
    memset(vis, 0, sizeof vis);
    vis[s] = 1;
    q[qt++] = s;
    while (qh < qt) {
        int cur = q[qh++];
        for (int j = 0; j < T_nradj[cur]; ++j) {
            int nb = T_radj[cur][j];
            if (vis[nb]) continue;
            int nx = nb % 17, ny = nb / 17;
            if (sx == dx && nx != sx) continue;
            if (sy == dy && ny != sy) continue;
            if (nb == d) return 1;
            if (cp[nb] >= 0) continue;
            vis[nb] = 1;
            q[qt++] = nb;
        }
    }
    return 0;
}

/* move_gen.py:186-224 _engineer_can_reach */
static int engineer_can_reach(const int16_t *cp, int s, int d) {
    if (!T_rail[s] || !T_rail[d] || s == d) return 0;
    unsigned char vis[NC];
    int q[NC], qh = 0, qt = 0;
    memset(vis, 0, sizeof vis);
    vis[s] = 1;
    q[qt++] = s;
    while (qh < qt) {
        int cur = q[qh++];
        for (int j = 0; j < T_nradj[cur]; ++j) {
            int nb = T_radj[cur][j];
            if (vis[nb]) continue;
            if (nb == d) return 1;
            if (cp[nb] >= 0) continue;
            vis[nb] = 1;
            q[qt++] = nb;
        }
    }
    return 0;
}

/* move_gen.py:384-423 _curve_rail_clear: BFS restricted to the cells that
 * carry the same curve id (including the two non-rail headquarters cells). */
static int curve_rail_clear(const int16_t *cp, int s, int d) {
    int cid = T_curve[s];
    if (cid <= 0 || T_curve[d] != cid) return 0;
    unsigned char vis[NC];
    int q[NC], qh = 0, qt = 0;
    memset(vis, 0, sizeof vis);
    vis[s] = 1;
    q[qt++] = s;
    while (qh < qt) {
        int cur = q[qh++];
        for (int j = 0; j < T_nradj[cur]; ++j) {
            int nb = T_radj[cur][j];
            if (vis[nb] || T_curve[nb] != cid) continue;
            if (nb == d) return 1;
            if (cp[nb] >= 0) continue;
            vis[nb] = 1;
            q[qt++] = nb;
        }
    }
    return 0;
}

static int move_requires_gongb(const int16_t *cp, int s, int d) {
    if (s == d) return 0;
    int sx = s % 17, sy = s / 17, dx = d % 17, dy = d / 17;
    int adx = abs(sx - dx), ady = abs(sy - dy);
    if (adx + ady == 1) return 0;
    if (adx == 1 && ady == 1 && (T_camp[s] || T_camp[d])) return 0;
    if (!(T_rail[s] && T_rail[d])) return 0;
    if (sx == dx || sy == dy) {
        if (straight_rail_clear(cp, s, d)) return 0;
        return engineer_can_reach(cp, s, d);
    }
    if (T_curve[s] > 0 && T_curve[s] == T_curve[d] && curve_rail_clear(cp, s, d)) return 0;
    return engineer_can_reach(cp, s, d);
}

/* ======================================================================
 * Combat memory (combat_memory.py:321-562)
 * ====================================================================== */
static inline int tracked_idx(int t) { return (t >= 2 && t <= 13) ? t - 2 : -1; }
static inline int is_ranked(int t) { return t >= T_SILING && t <= T_GONGB; }
/* combat_memory.py:139-151 next_floor_after_eat: rank = 14 - t for ranked */
static inline int next_floor(int t) {
    if (!is_ranked(t)) return 0;
    int r = 14 - t + 1;
    return r > 9 ? 9 : r;
}
static inline void set_bit(uint64_t *lo, uint64_t *hi, int pid) {
    if (pid < 64) *lo |= (uint64_t)1 << pid;
    else *hi |= (uint64_t)1 << (pid - 64);
}

static void cm_apply(jqo_batch *b, int e, int eat, int A, int D, int A_seat, int D_seat,
                     int A_type, int D_type, int step) {
    int K, V, V_seat, V_type;
    if (eat) { K = A; V = D; V_seat = D_seat; V_type = D_type; }
    else { K = D; V = A; V_seat = A_seat; V_type = A_type; }
    if (K < 0 || V < 0) return;
    int v_idx = tracked_idx(V_type);
    /* combat_memory.py:425-433 KILLED preflight */
    if (!eat) {
        for (int o = 0; o < 4; ++o) {
            int known = b->cm_is_gongb[OI(e, o, V)] || (A_type == T_GONGB && o == V_seat);
            if (known) b->cm_atk_gongb[OI(e, o, K)] = 1;
        }
    }
    /* combat_memory.py:435-461 chain propagation + chain floor */
    for (int o = 0; o < 4; ++o) {
        size_t k = OI(e, o, K), v = OI(e, o, V);
        b->cm_chain_lo[k] |= b->cm_direct_lo[v] | b->cm_chain_lo[v];
        b->cm_chain_hi[k] |= b->cm_direct_hi[v] | b->cm_chain_hi[v];
        set_bit(&b->cm_chain_lo[k], &b->cm_chain_hi[k], V);
        b->cm_chain_type[k] |= (uint16_t)(b->cm_direct_type[v] | b->cm_chain_type[v]);
        b->cm_last_chain_step[k] = (int16_t)step;
        int vf = b->cm_rank_floor[v];
        int proposed = vf + 1 < 9 ? vf + 1 : 9;
        int has = vf > 0;
        if (has && proposed > b->cm_rank_floor[k]) {
            b->cm_rank_floor[k] = (int8_t)proposed;
            b->cm_rank_floor_step[k] = (int16_t)step;
        }
        if (has) b->cm_not_gongb[k] = 1;
    }
    /* combat_memory.py:463-509 reverse projection onto observer-own pids */
    for (int o = 0; o < 4; ++o) {
        size_t v = OI(e, o, V);
        uint64_t mlo = 0, mhi = 0;
        for (int s = 0; s < 30; ++s) set_bit(&mlo, &mhi, o * 30 + s);
        uint64_t vlo = (b->cm_direct_lo[v] | b->cm_chain_lo[v]) & mlo;
        uint64_t vhi = (b->cm_direct_hi[v] | b->cm_chain_hi[v]) & mhi;
        if (V_seat == o) set_bit(&vlo, &vhi, V);
        for (int t = 0; t < 128; ++t) {
            int on = t < 64 ? (int)((vlo >> t) & 1) : (int)((vhi >> (t - 64)) & 1);
            if (!on || t >= NP) continue;
            size_t tt = OI(e, o, t);
            set_bit(&b->cm_eaten_lo[tt], &b->cm_eaten_hi[tt], K);
        }
    }
    /* combat_memory.py:511-562 per-observer dispatch */
    for (int o = 0; o < 4; ++o) {
        size_t k = OI(e, o, K);
        if (V_seat != o) {
            int c = b->cm_direct_other[k] + 1;
            b->cm_direct_other[k] = (int16_t)(c < 32767 ? c : 32767);
            b->cm_last_direct_step[k] = (int16_t)step;
            continue;
        }
        set_bit(&b->cm_direct_lo[k], &b->cm_direct_hi[k], V);
        if (v_idx >= 0) {
            b->cm_direct_type[k] |= (uint16_t)(1u << v_idx);
            b->cm_chain_type[k] |= (uint16_t)(1u << v_idx);
        }
        b->cm_last_direct_step[k] = (int16_t)step;
        if (eat) {
            if (V_type == T_DILEI) b->cm_is_gongb[k] = 1;
            else b->cm_not_gongb[k] = 1;
        } else if (is_ranked(V_type)) {
            int pr = next_floor(V_type);
            if (pr > b->cm_rank_floor[k]) {
                b->cm_rank_floor[k] = (int8_t)pr;
                b->cm_rank_floor_step[k] = (int16_t)step;
            }
        }
        if (eat && is_ranked(V_type)) {
            int pr = next_floor(V_type);
            if (pr > b->cm_rank_floor[k]) {
                b->cm_rank_floor[k] = (int8_t)pr;
                b->cm_rank_floor_step[k] = (int16_t)step;
            }
        }
    }
}

/* ======================================================================
 * Beliefs (info_model.py:165-520), one byte per (observer, pid):
 *   0 = no entry, 1..12 = one-hot tracked type (idx+1), 14 = uniform
 *   fallback, 32+slot = per-slot prior of seat-local slot (0..29).
 * ====================================================================== */
enum { BC_NONE = 0, BC_UNIFORM = 14, BC_PRIOR0 = 32 };
static const int16_t PIECE_COUNTS12[12] = {1, 3, 2, 1, 1, 2, 2, 2, 2, 3, 3, 3};

static inline int bc_onehot(int code) { return code >= 1 && code <= 12; }

/* info_model.py:607-618 _observer_sees_truth */
static inline int sees_truth(int obs, int owner, int mode) {
    if (mode == SM_BRIGHT) return 1;
    if (obs == owner) return 1;
    return mode == SM_HALF_DARK && ((obs & 1) == (owner & 1));
}

static void bel_dec(jqo_batch *b, int e, int o, int seat, int ti) {
    if (seat < 0 || seat > 3 || ti < 0) return;
    size_t tr = ((size_t)e * 4 + o) * 4 + seat;
    if (!b->rem_tracked[tr]) return;
    int16_t *r = &b->remaining[tr * 12 + ti];
    if (*r > 0) (*r)--;
}

static void bel_untrack(jqo_batch *b, int e, int o, int seat) {
    size_t tr = ((size_t)e * 4 + o) * 4 + seat;
    b->rem_tracked[tr] = 0;
    for (int t = 0; t < 12; ++t) b->remaining[tr * 12 + t] = 0;
}

/* info_model.py:218-270 BeliefTensor.initial for every observer */
static void bel_initial(jqo_batch *b, int e, int mode) {
    for (int o = 0; o < 4; ++o) {
        for (int p = 0; p < NP; ++p) {
            size_t q = PI(e, p);
            uint8_t code = BC_NONE;
            if (b->alive[q]) {
                int s = b->piece_seat[q];
                if (sees_truth(o, s, mode)) {
                    code = (uint8_t)(tracked_idx(b->piece_type[q]) + 1);
                } else {
                    /* info_model.py:155-162,240-252: prior of the seat-local slot the
                       piece stands on, uniform when it is outside its own zone */
                    code = BC_UNIFORM;
                    int f = b->pos_y[q] * 17 + b->pos_x[q];
                    for (int i = 0; i < 30 && s >= 0; ++i) {
                        int x, y;
                        index_to_pos(s, i, &x, &y);
                        if (y * 17 + x == f) { code = (uint8_t)(BC_PRIOR0 + i); break; }
                    }
                }
            }
            b->bel_code[OI(e, o, p)] = code;
        }
        for (int s = 0; s < 4; ++s) {
            size_t tr = ((size_t)e * 4 + o) * 4 + s;
            int enemy = (s & 1) != (o & 1);
            b->rem_tracked[tr] = (uint8_t)enemy;
            for (int t = 0; t < 12; ++t) b->remaining[tr * 12 + t] = enemy ? PIECE_COUNTS12[t] : 0;
        }
    }
}

typedef struct {
    int event, A, D, A_seat, D_seat, A_type, D_type, sf, df;
    int fr_src, fr_dst, flag_captured;
    int other_pid; /* pid on the defender's other stronghold before the step */
    int died[4];
} bel_edge;

/* info_model.py:272-414 BeliefTensor.update (R3, R5/R7, R4/R6, R1, R9, I5) */
static void bel_update(jqo_batch *b, int e, const bel_edge *x, int mode) {
    static const int sh_slot[2] = {26, 28};
    for (int o = 0; o < 4; ++o) {
        uint8_t *code = b->bel_code + OI(e, o, 0);
        int a_bel = code[x->A];
        int d_bel = x->D >= 0 ? code[x->D] : BC_NONE;
        if (x->fr_src) bel_dec(b, e, o, x->A_seat, T_SILING - 2);
        if (x->fr_dst) bel_dec(b, e, o, x->D_seat, T_SILING - 2);
        if (x->event == EV_EAT && x->D >= 0 && x->D_type == T_DILEI && a_bel != BC_NONE &&
            !bc_onehot(a_bel)) {
            code[x->A] = (uint8_t)(T_GONGB - 2 + 1);
            a_bel = code[x->A];
            bel_dec(b, e, o, x->A_seat, T_GONGB - 2);
        }
        if (x->flag_captured) {
            bel_untrack(b, e, o, x->D_seat);
        } else if (x->event == EV_EAT && x->D >= 0 && x->D_seat >= 0) {
            int sx, sy, s0, s1;
            index_to_pos(x->D_seat, sh_slot[0], &sx, &sy);
            s0 = sy * 17 + sx;
            index_to_pos(x->D_seat, sh_slot[1], &sx, &sy);
            s1 = sy * 17 + sx;
            if (x->df == s0 || x->df == s1) {
                int op = x->other_pid;
                if (op >= 0 && code[op] != BC_NONE && !bc_onehot(code[op]))
                    code[op] = (uint8_t)(T_JUNQI - 2 + 1);
            }
        }
        a_bel = code[x->A];
        if (x->event == EV_EAT) {
            if (d_bel != BC_NONE && bc_onehot(d_bel)) bel_dec(b, e, o, x->D_seat, d_bel - 1);
        } else if (x->event == EV_KILLED) {
            if (a_bel != BC_NONE && bc_onehot(a_bel)) bel_dec(b, e, o, x->A_seat, a_bel - 1);
        } else if (x->event == EV_BOMB) {
            if (a_bel != BC_NONE && bc_onehot(a_bel)) bel_dec(b, e, o, x->A_seat, a_bel - 1);
            if (d_bel != BC_NONE && bc_onehot(d_bel)) bel_dec(b, e, o, x->D_seat, d_bel - 1);
        }
        for (int s = 0; s < 4; ++s)
            if (x->died[s]) bel_untrack(b, e, o, s);
        for (int p = 0; p < NP; ++p) {
            size_t q = PI(e, p);
            if (!b->alive[q]) { code[p] = BC_NONE; continue; }
            if (code[p] == BC_NONE)
                code[p] = sees_truth(o, b->piece_seat[q], mode)
                              ? (uint8_t)(tracked_idx(b->piece_type[q]) + 1)
                              : (uint8_t)BC_UNIFORM;
        }
    }
}

/* ======================================================================
 * Step (batched_state.py:417-613 step_batch, 739-980 _step_single)
 * ====================================================================== */
static void kill_piece(jqo_batch *b, int e, int pid, int cell, int reason, int step, int loc) {
    size_t q = PI(e, pid);
    if (!b->alive[q]) return;
    b->alive[q] = 0;
    b->cell_pid[CI(e, cell)] = -1;
    b->pos_x[q] = -1;
    b->pos_y[q] = -1;
    b->death_reason[q] = (int8_t)reason;
    b->death_step[q] = (int16_t)step;
    b->death_loc[q] = (int16_t)loc;
}

static int64_t flag_reveal_delta(jqo_batch *b, int e, int seat) {
    if (!b->seat_flag[SI(e, seat)]) {
        b->seat_flag[SI(e, seat)] = 1;
        return Z_sflag[seat];
    }
    return 0;
}

/* batched_state.py:1078-1121 (death_loc -1); with GameState rules the
 * current cell is kept as death_loc (state.py:640-693). */
static int64_t surrender_delta(jqo_batch *b, int e, int seat, int step) {
    int64_t d = 0;
    int keep_loc = b->rules == 1;
    b->seat_dead[SI(e, seat)] = 1;
    d ^= Z_sdead[seat];
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        if (b->piece_seat[q] != seat || !b->alive[q]) continue;
        int px = b->pos_x[q], py = b->pos_y[q];
        if (px >= 0 && py >= 0) {
            int f = py * 17 + px;
            d ^= ZP(p, b->piece_type[q], f);
            b->cell_pid[CI(e, f)] = -1;
        }
        b->alive[q] = 0;
        b->pos_x[q] = -1;
        b->pos_y[q] = -1;
        b->death_reason[q] = DR_KBE;
        b->death_step[q] = (int16_t)step;
        b->death_loc[q] = (int16_t)(keep_loc && px >= 0 && py >= 0 ? py * 17 + px : -1);
    }
    return d;
}

/* batched_state.py:1187-1231 _check_victory (draw threshold = max_moves) */
static void check_victory(const jqo_batch *b, int e, int acting, int mc, int mslc, int *term,
                          int *win, int *draw) {
    const uint8_t *sd = b->seat_dead + SI(e, 0);
    int red = !sd[0] || !sd[2], blue = !sd[1] || !sd[3];
    *term = 0; *win = -1; *draw = 0;
    if (!red && !blue) { *term = 1; *win = acting % 2; return; }
    if (!red) { *term = 1; *win = 1; return; }
    if (!blue) { *term = 1; *win = 0; return; }
    if (mc >= 4000 || mslc >= 200) { *term = 1; *draw = 1; }
}

/* combat: rules.py:466-516 resolve_combat (returns 0 where it raises) */
static int resolve_combat(int a, int d) {
    if (a <= T_DARK || d <= T_DARK) return 0;
    if (a == T_JUNQI || a == T_DILEI) return 0;
    if (a == T_ZHADAN || d == T_ZHADAN) return EV_BOMB;
    if (d == T_JUNQI) return EV_EAT;
    if (d == T_DILEI) return a == T_GONGB ? EV_EAT : EV_KILLED;
    if (a == d) return EV_BOMB;
    return a < d ? EV_EAT : EV_KILLED;
}

static void step_env(jqo_batch *b, int e, int32_t act, int mode, jqo_step_out *out) {
    out->valid[e] = 0;
    out->event[e] = 0;
    out->flag_captured[e] = 0;
    out->reward[e] = 0.f;
    out->terminated[e] = b->terminated[e];
    out->winner[e] = b->winner[e];
    out->draw[e] = b->draw[e];
    if (b->terminated[e]) return;
    if (act < 0 || act >= NC * NC) return;
    int sf = act / NC, df = act % NC;
    int16_t *cp = b->cell_pid + CI(e, 0);
    int A = cp[sf], D = cp[df];
    if (A < 0 || sf == df) return;
    int acting = b->turn[e], mc = b->move_counter[e], mslc = b->mslc[e];
    int A_type = b->piece_type[PI(e, A)], A_seat = b->piece_seat[PI(e, A)];
    int D_type = D >= 0 ? b->piece_type[PI(e, D)] : 0, D_seat = D >= 0 ? b->piece_seat[PI(e, D)] : -1;
    int ev = EV_MOVE;
    if (D >= 0) {
        ev = resolve_combat(A_type, D_type);
        if (!ev) return; /* the reference raises for these attacker types */
    }
    int64_t zob = b->zobrist[e];
    int died_pre[4];
    for (int s = 0; s < 4; ++s) died_pre[s] = b->seat_dead[SI(e, s)];
    bel_edge x;
    memset(&x, 0, sizeof x);
    x.event = ev; x.A = A; x.D = D; x.A_seat = acting; x.D_seat = D_seat;
    x.A_type = A_type; x.D_type = D_type; x.sf = sf; x.df = df; x.other_pid = -1;
    if (D >= 0 && D_seat >= 0) {
        int sx, sy, s0, s1;
        index_to_pos(D_seat, 26, &sx, &sy); s0 = sy * 17 + sx;
        index_to_pos(D_seat, 28, &sx, &sy); s1 = sy * 17 + sx;
        if (df == s0) x.other_pid = cp[s1];
        else if (df == s1) x.other_pid = cp[s0];
    }
    /* path-revealed engineer (batched_state.py:487-512, 819-828) on the pre-move board */
    if (A_type == T_GONGB) {
        int adx = abs(sf % 17 - df % 17), ady = abs(sf / 17 - df / 17);
        if (D >= 0 || adx + ady > 1) {
            if (move_requires_gongb(cp, sf, df))
                for (int o = 0; o < 4; ++o) b->cm_is_gongb[OI(e, o, A)] = 1;
        }
    }
    int new_mc = mc + 1, new_mslc, new_turn, term, win, draw, fcap = 0;
    zob ^= Z_turn[acting] ^ Z_mc[mc & 0xFFF] ^ Z_mslc[mslc & 0x1FF];
    if (D < 0) {
        /* plain path (batched_state.py:468-575) */
        zob ^= ZP(A, A_type, sf) ^ ZP(A, A_type, df);
        cp[sf] = -1;
        cp[df] = (int16_t)A;
        b->pos_x[PI(e, A)] = (int8_t)(df % 17);
        b->pos_y[PI(e, A)] = (int8_t)(df / 17);
        b->move_count[PI(e, A)]++;
        new_mslc = mslc + 1;
    }
    if (D < 0 && b->rules != 1) {
        /* _advance_turn_vec (batched_state.py:615-686): Q12 only past a dead seat */
        int cand = (acting + 1) % 4;
        if (b->seat_dead[SI(e, cand)]) {
            int chain = 0;
            int64_t delta = 0;
            while (chain < 4) {
                if (b->seat_dead[SI(e, cand)]) { cand = (cand + 1) % 4; ++chain; continue; }
                if (has_moves(b, e, cand)) break;
                delta ^= surrender_delta(b, e, cand, new_mc);
                cand = (cand + 1) % 4;
                ++chain;
            }
            zob ^= delta;
        }
        new_turn = cand;
        check_victory(b, e, acting, new_mc, new_mslc, &term, &win, &draw);
    } else {
        /* combat path (_step_single); plain moves too under GameState rules
           (state.py:309-669 runs the same sequence for every ply) */
        int death_step = mc + 1;
      if (D >= 0) {
        int fr_src = (A_type == T_SILING) && (ev == EV_KILLED || ev == EV_BOMB);
        int fr_dst = (D_type == T_SILING) && (ev == EV_EAT || ev == EV_BOMB);
        if (fr_src) zob ^= flag_reveal_delta(b, e, A_seat);
        if (fr_dst) zob ^= flag_reveal_delta(b, e, D_seat);
        x.fr_src = fr_src;
        x.fr_dst = fr_dst;
        fcap = D_type == T_JUNQI;
        if (ev == EV_EAT) {
            zob ^= ZP(D, D_type, df);
            kill_piece(b, e, D, df, DR_KBE, death_step, df);
            zob ^= ZP(A, A_type, sf) ^ ZP(A, A_type, df);
            cp[sf] = -1;
            cp[df] = (int16_t)A;
            b->pos_x[PI(e, A)] = (int8_t)(df % 17);
            b->pos_y[PI(e, A)] = (int8_t)(df / 17);
            b->active_eat[PI(e, A)]++;
            cm_apply(b, e, 1, A, D, A_seat, D_seat, A_type, D_type, death_step);
        } else if (ev == EV_KILLED) {
            int dr = (D_type == T_DILEI || D_type == T_ZHADAN) ? DR_MINE : DR_KBE;
            zob ^= ZP(A, A_type, sf);
            kill_piece(b, e, A, sf, dr, death_step, df);
            b->passive_surv[PI(e, D)]++;
            cm_apply(b, e, 0, A, D, A_seat, D_seat, A_type, D_type, death_step);
        } else {
            zob ^= ZP(A, A_type, sf) ^ ZP(D, D_type, df);
            kill_piece(b, e, A, sf, DR_MUTUAL, death_step, df);
            kill_piece(b, e, D, df, DR_MUTUAL, death_step, df);
        }
        new_mslc = 0;
      }
        if (fcap && !b->seat_dead[SI(e, D_seat)]) {
            zob ^= flag_reveal_delta(b, e, D_seat);
            zob ^= surrender_delta(b, e, D_seat, death_step);
        }
        for (int s = 0; s < 4; ++s) {
            if (b->seat_dead[SI(e, s)]) continue;
            int any = 0;
            for (int p = 0; p < NP && !any; ++p)
                any = b->piece_seat[PI(e, p)] == s && b->alive[PI(e, p)];
            if (!any) { b->seat_dead[SI(e, s)] = 1; zob ^= Z_sdead[s]; }
        }
        check_victory(b, e, acting, new_mc, new_mslc, &term, &win, &draw);
        if (!term) {
            /* _advance_turn (batched_state.py:1123-1169): Q12 on every candidate */
            int cand = (acting + 1) % 4, chain = 0, found = 0;
            int64_t delta = 0;
            while (chain < 4) {
                if (b->seat_dead[SI(e, cand)]) { cand = (cand + 1) % 4; ++chain; continue; }
                if (has_moves(b, e, cand)) { found = 1; break; }
                delta ^= surrender_delta(b, e, cand, new_mc);
                cand = (cand + 1) % 4;
                ++chain;
            }
            new_turn = found ? cand : (acting + 1) % 4;
            zob ^= delta;
            check_victory(b, e, acting, new_mc, new_mslc, &term, &win, &draw);
        } else {
            new_turn = acting;
        }
    }
    /* the caller's episode cap, after victory and Q12 (game_state.cu:1651-1655) */
    if (!term && b->max_moves > 0 && new_mc >= b->max_moves) { term = 1; draw = 1; }
    zob ^= Z_mc[new_mc & 0xFFF] ^ Z_mslc[new_mslc & 0x1FF] ^ Z_turn[new_turn];
    if (term) zob ^= Z_term;
    if (draw) zob ^= Z_draw;
    if (win >= 0) zob ^= Z_win[0] ^ Z_win[win + 1];
    b->move_counter[e] = new_mc;
    b->mslc[e] = new_mslc;
    b->turn[e] = (int8_t)new_turn;
    b->zobrist[e] = zob;
    b->terminated[e] = (uint8_t)term;
    b->winner[e] = (int8_t)win;
    b->draw[e] = (uint8_t)draw;
    out->valid[e] = 1;
    out->event[e] = (int8_t)ev;
    out->terminated[e] = (uint8_t)term;
    out->winner[e] = (int8_t)win;
    out->draw[e] = (uint8_t)draw;
    out->flag_captured[e] = (uint8_t)fcap;
    /* game_state.cu compute_rewards semantics: terminal +-1 for the acting team */
    if (term && !draw && win >= 0) out->reward[e] = ((acting & 1) == win) ? 1.f : -1.f;
    /* state.py:344-349 move history ring (most recent last, capped at 32) */
    int hc = b->hist_count[e];
    b->hist_src[(size_t)e * JQO_HIST + (hc % JQO_HIST)] = (int16_t)sf;
    b->hist_dst[(size_t)e * JQO_HIST + (hc % JQO_HIST)] = (int16_t)df;
    b->hist_count[e] = hc + 1;
    /* beliefs of all four observers (junqi_rl/env.py:298-300) */
    x.flag_captured = fcap;
    for (int s = 0; s < 4; ++s) x.died[s] = b->seat_dead[SI(e, s)] && !died_pre[s];
    bel_update(b, e, &x, mode);
}

int jqo_step(jqo_batch *b, const int32_t *actions, int mode, jqo_step_out *out, int nthreads) {
    build_topology();
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads > 0 ? nthreads : 1)
    for (int e = 0; e < b->n; ++e) step_env(b, e, actions[e], mode, out);
    return 0;
}

/* ======================================================================
 * Reset: state.py:490-624 GameState.new_game on a pool lineup, plus the
 * initial beliefs, zeroed combat memory and an empty move history.
 * ====================================================================== */
int jqo_reset_env(jqo_batch *b, int e, const int8_t *lineup, int mode) {
    build_topology();
    int64_t zob = 0;
    for (int f = 0; f < NC; ++f) b->cell_pid[CI(e, f)] = -1;
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        int t = lineup[p];
        b->alive[q] = 0;
        b->piece_type[q] = -1; b->piece_seat[q] = -1;
        b->pos_x[q] = -1; b->pos_y[q] = -1; b->zero_x[q] = -1; b->zero_y[q] = -1;
        b->move_count[q] = 0; b->active_eat[q] = 0; b->passive_surv[q] = 0;
        b->death_reason[q] = -1; b->death_step[q] = -1; b->death_loc[q] = -1;
        if (t == T_NONE) continue;
        int x, y, s = p / 30;
        index_to_pos(s, p % 30, &x, &y);
        int f = y * 17 + x;
        b->alive[q] = 1;
        b->piece_type[q] = (int8_t)t;
        b->piece_seat[q] = (int8_t)s;
        b->pos_x[q] = b->zero_x[q] = (int8_t)x;
        b->pos_y[q] = b->zero_y[q] = (int8_t)y;
        b->cell_pid[CI(e, f)] = (int16_t)p;
        zob ^= ZP(p, t, f);
    }
    for (int s = 0; s < 4; ++s) { b->seat_dead[SI(e, s)] = 0; b->seat_flag[SI(e, s)] = 0; }
    zob ^= Z_turn[0] ^ Z_mc[0] ^ Z_mslc[0] ^ Z_win[0] ^ Z_show[mode & 3];
    b->turn[e] = 0; b->zobrist[e] = zob; b->move_counter[e] = 0; b->mslc[e] = 0;
    b->terminated[e] = 0; b->winner[e] = -1; b->draw[e] = 0;
    for (int o = 0; o < 4; ++o)
        for (int p = 0; p < NP; ++p) {
            size_t k = OI(e, o, p);
            b->cm_direct_lo[k] = b->cm_direct_hi[k] = 0; b->cm_direct_type[k] = 0;
            b->cm_last_direct_step[k] = -1; b->cm_direct_other[k] = 0;
            b->cm_chain_lo[k] = b->cm_chain_hi[k] = 0; b->cm_chain_type[k] = 0;
            b->cm_last_chain_step[k] = -1;
            b->cm_eaten_lo[k] = b->cm_eaten_hi[k] = 0;
            b->cm_rank_floor[k] = 0; b->cm_rank_floor_step[k] = -1;
            b->cm_is_gongb[k] = b->cm_not_gongb[k] = b->cm_atk_gongb[k] = 0;
        }
    for (int i = 0; i < JQO_HIST; ++i) {
        b->hist_src[(size_t)e * JQO_HIST + i] = -1;
        b->hist_dst[(size_t)e * JQO_HIST + i] = -1;
    }
    b->hist_count[e] = 0;
    bel_initial(b, e, mode);
    return 0;
}

/* ======================================================================
 * Observation (observation.py:598-858 _fill_into and writers 908-1651).
 * World-frame values are written straight to their canonical cell, which
 * equals building the world frame and applying rotate_planes afterwards.
 * ====================================================================== */
static inline int popc64(uint64_t v) { return __builtin_popcountll(v); }

static void bel_vec(int code, int pid, float *v) {
    for (int t = 0; t < 12; ++t) v[t] = 0.f;
    if (code >= 1 && code <= 12) v[code - 1] = 1.f;
    else if (code >= BC_PRIOR0 && code < BC_PRIOR0 + 30) memcpy(v, P_prior + (code - BC_PRIOR0) * 12, 12 * sizeof(float));
    else if (code == BC_UNIFORM) memcpy(v, P_uniform, 12 * sizeof(float));
}

static int in_back_two(int seat, int zx, int zy) {
    /* observation.py:1378-1387 */
    switch (seat) {
    case 0: return zy >= 15 && zy <= 16;
    case 2: return zy >= 0 && zy <= 1;
    case 1: return zx >= 0 && zx <= 1;
    case 3: return zx >= 15 && zx <= 16;
    }
    return 0;
}

int jqo_obs(const jqo_batch *b, int e, int o, int mode, float *sp, float *gl) {
    build_topology();
    const int *rot = T_rot[o];
#define W(ch, f) sp[(size_t)(ch) * NC + rot[(f)]]
    memset(sp, 0, sizeof(float) * JQO_OBS_CH * NC);
    memset(gl, 0, sizeof(float) * JQO_OBS_GLOBAL);
    int tm = (o + 2) % 4, left = (o + 1) % 4, right = (o + 3) % 4, oteam = o & 1;
    const uint8_t *code = b->bel_code + OI(e, o, 0);
    float v[12];
    /* groups 1-7: pieces, teammate probs, dark teammate, enemy masks/beliefs */
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        if (!b->alive[q]) continue;
        int f = b->pos_y[q] * 17 + b->pos_x[q], s = b->piece_seat[q], ti = tracked_idx(b->piece_type[q]);
        if (s == o && ti >= 0) W(ti, f) = 1.f;
        if (s == tm) {
            bel_vec(code[p], p, v);
            for (int t = 0; t < 12; ++t) W(12 + t, f) = v[t];
            if (mode == SM_DARK) W(24, f) = 1.f;
        }
        if (s == left) {
            W(25, f) = 1.f;
            bel_vec(code[p], p, v);
            for (int t = 0; t < 12; ++t) W(27 + t, f) = v[t];
        }
        if (s == right) {
            W(26, f) = 1.f;
            bel_vec(code[p], p, v);
            for (int t = 0; t < 12; ++t) W(39 + t, f) = v[t];
        }
    }
    /* 8-9: constant planes (observation.py:984-997) */
    const int dead_order[3] = {tm, left, right}, flag_order[4] = {o, tm, left, right};
    for (int k = 0; k < 3; ++k)
        if (b->seat_dead[SI(e, dead_order[k])])
            for (int c = 0; c < NC; ++c) sp[(size_t)(51 + k) * NC + c] = 1.f;
    for (int k = 0; k < 4; ++k)
        if (b->seat_flag[SI(e, flag_order[k])])
            for (int c = 0; c < NC; ++c) sp[(size_t)(54 + k) * NC + c] = 1.f;
    /* 10: board statics (observation.py:343-383) */
    for (int f = 0; f < NC; ++f) {
        if (T_camp[f]) W(58, f) = 1.f;
        if (T_sh[f]) W(59, f) = 1.f;
        if (T_rail[f]) W(60, f) = 1.f;
        if (T_nine[f]) W(61, f) = 1.f;
        if (T_arc[f]) W(62, f) = 1.f;
    }
    /* 11: turn history (observation.py:1000-1021): double division then float32 */
    {
        double dp = (double)b->mslc[e] / 200.0, mp = (double)b->move_counter[e] / 4000.0;
        float d32 = (float)(dp < 1.0 ? dp : 1.0), m32 = (float)(mp < 1.0 ? mp : 1.0);
        for (int c = 0; c < NC; ++c) { sp[64 * NC + c] = d32; sp[65 * NC + c] = m32; }
    }
    /* 12-14: buckets (observation.py:1027-1100) */
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        if (!b->alive[q]) continue;
        int f = b->pos_y[q] * 17 + b->pos_x[q];
        int half = ((b->piece_seat[q] & 1) == oteam) ? 0 : 4;
        int mcnt = b->move_count[q] < 3 ? b->move_count[q] : 3;
        W(66 + half + mcnt, f) = 1.f;
        int ae = b->active_eat[q] < 3 ? b->active_eat[q] : 3;
        int ps = b->passive_surv[q] < 3 ? b->passive_surv[q] : 3;
        for (int k = 0; k <= ae; ++k) W(74 + half + k, f) = 1.f;
        for (int k = 0; k <= ps; ++k) W(82 + half + k, f) = 1.f;
    }
    /* 15-16: death reason + dead at zero (observation.py:1103-1180) */
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        if (b->alive[q] || b->death_step[q] == -1) continue; /* GameState.deaths keys */
        int s = b->piece_seat[q];
        int r = b->death_reason[q];
        int ridx = (r >= 0 && r <= 2) ? r : (r == -1 ? 2 : -1);
        if (ridx >= 0 && b->death_step[q] > 0) {
            int grp = s == o ? 0 : s == tm ? 3 : s == left ? 6 : s == right ? 9 : -1;
            int fl = b->death_loc[q];
            int yy = fl >= 0 ? fl / 17 : -((-fl + 16) / 17), xx = ((fl % 17) + 17) % 17;
            if (yy < 0) yy += 17;
            if (grp >= 0 && yy >= 0 && yy < 17) W(90 + grp + ridx, yy * 17 + xx) = 1.f;
        }
        int zx = b->zero_x[q], zy = b->zero_y[q];
        if (zx >= 0 && zy >= 0) {
            int steam = s >= 0 ? (s & 1) : 1;
            W(102 + (steam == oteam ? 0 : 1), zy * 17 + zx) = 1.f;
        }
    }
    /* 17: piece slot (observation.py:1183-1204) */
    {
        int slot_ch[30], nx = 0;
        for (int s = 0; s < 30; ++s) slot_ch[s] = is_camp_slot(s) ? -1 : nx++;
        for (int p = 0; p < NP; ++p) {
            size_t q = PI(e, p);
            if (!b->alive[q]) continue;
            int ch = slot_ch[p % 30];
            if (ch < 0) ch = 24;
            W(104 + ch, b->pos_y[q] * 17 + b->pos_x[q]) = 1.f;
        }
    }
    /* 18: move history (observation.py:1207-1231) */
    {
        int hc = b->hist_count[e], n = hc < JQO_HIST ? hc : JQO_HIST;
        for (int d = 0; d < n; ++d) {
            int slot = (hc - 1 - d) % JQO_HIST;
            int s = b->hist_src[(size_t)e * JQO_HIST + slot], t = b->hist_dst[(size_t)e * JQO_HIST + slot];
            W(129 + d, s) = -1.f;
            W(129 + d, t) = 1.f;
        }
    }
    /* 19: combat memory tail (observation.py:1234-1620) */
    int lo_opp = (o + 1) % 4, ro_opp = (o + 3) % 4;
    uint64_t type_lo[12], type_hi[12];
    for (int t = 0; t < 12; ++t) type_lo[t] = type_hi[t] = 0;
    for (int s = 0; s < 30; ++s) {
        int ti = tracked_idx(b->piece_type[PI(e, o * 30 + s)]);
        if (ti >= 0) set_bit(&type_lo[ti], &type_hi[ti], o * 30 + s);
    }
    int cur = b->move_counter[e];
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        if (!b->alive[q]) continue;
        int f = b->pos_y[q] * 17 + b->pos_x[q], s = b->piece_seat[q];
        int steam = s >= 0 ? (s & 1) : 1;
        if (steam != oteam) {
            size_t k = OI(e, o, p);
            uint64_t dlo = b->cm_direct_lo[k], dhi = b->cm_direct_hi[k];
            int mine = popc64(dlo) + popc64(dhi);
            for (int g = 0; g < 3; ++g) if (mine >= g + 1) W(173 + g, f) = 1.f;
            for (int t = 0; t < 12; ++t) if ((b->cm_direct_type[k] >> t) & 1) W(161 + t, f) = 1.f;
            for (int g = 0; g < 3; ++g) if (b->cm_direct_other[k] >= g + 1) W(176 + g, f) = 1.f;
            int ch = popc64(b->cm_chain_lo[k]) + popc64(b->cm_chain_hi[k]);
            for (int g = 0; g < 3; ++g) if (ch >= g + 1) W(191 + g, f) = 1.f;
            for (int t = 0; t < 12; ++t) if ((b->cm_chain_type[k] >> t) & 1) W(179 + t, f) = 1.f;
            for (int g = 0; g < 9; ++g) if (b->cm_rank_floor[k] >= g + 1) W(194 + g, f) = 1.f;
            if (b->cm_is_gongb[k]) W(203, f) = 1.f;
            if (b->cm_not_gongb[k]) W(204, f) = 1.f;
            if (in_back_two(s, b->zero_x[q], b->zero_y[q]) && b->move_count[q] == 0 && !b->cm_atk_gongb[k])
                W(205, f) = 1.f;
            /* layer 3 */
            for (int sl = 0; sl < 30; ++sl) {
                int gp = o * 30 + sl;
                int on = gp < 64 ? (int)((dlo >> gp) & 1) : (int)((dhi >> (gp - 64)) & 1);
                if (on) W(223 + sl, f) = 1.f;
            }
            for (int t = 0; t < 12; ++t) {
                int c = popc64(dlo & type_lo[t]) + popc64(dhi & type_hi[t]);
                if (c > 0) {
                    float val = (float)c / 3.0f;
                    W(211 + t, f) = val < 1.f ? val : 1.f;
                }
            }
            int lasts[4] = {b->cm_last_direct_step[k], b->cm_last_direct_step[k], b->cm_last_chain_step[k],
                            b->cm_rank_floor_step[k]};
            for (int pl = 0; pl < 4; ++pl) {
                if (lasts[pl] < 0) continue;
                int el = cur - lasts[pl];
                if (el < 0) el = 0;
                if (el > 4096) el = 4096;
                float fr = P_recency[pl * 4097 + el];
                if (fr > 0.f) W(253 + pl, f) = fr;
            }
        }
        if (s == o) {
            size_t kl = OI(e, lo_opp, p), kr = OI(e, ro_opp, p);
            int lc = popc64(b->cm_direct_lo[kl]) + popc64(b->cm_direct_hi[kl]) + b->cm_direct_other[kl];
            int rc = popc64(b->cm_direct_lo[kr]) + popc64(b->cm_direct_hi[kr]) + b->cm_direct_other[kr];
            int pub = lc < rc ? lc : rc;
            for (int g = 0; g < 3; ++g) if (pub >= g + 1) W(206 + g, f) = 1.f;
            if (b->cm_is_gongb[kl] && b->cm_is_gongb[kr]) W(209, f) = 1.f;
            int patk = b->cm_atk_gongb[kl] || b->cm_atk_gongb[kr];
            if (in_back_two(s, b->zero_x[q], b->zero_y[q]) && b->move_count[q] == 0 && !patk)
                W(210, f) = 1.f;
        }
    }
    /* layer 4: reverse projection onto observer-own pids */
    for (int sl = 0; sl < 30; ++sl) {
        int mp = o * 30 + sl;
        size_t q = PI(e, mp);
        int px = b->alive[q] ? b->pos_x[q] : b->zero_x[q];
        int py = b->alive[q] ? b->pos_y[q] : b->zero_y[q];
        if (px < 0 || py < 0) continue;
        size_t k = OI(e, o, mp);
        uint64_t elo = b->cm_eaten_lo[k], ehi = b->cm_eaten_hi[k];
        const int opps[2] = {lo_opp, ro_opp};
        for (int h = 0; h < 2; ++h)
            for (int s = 0; s < 30; ++s) {
                int gp = opps[h] * 30 + s;
                int on = gp < 64 ? (int)((elo >> gp) & 1) : (int)((ehi >> (gp - 64)) & 1);
                if (on) W(257 + h * 30 + s, py * 17 + px) = 1.f;
            }
    }
    /* globals (observation.py:1623-1651) */
    const int16_t *rem = b->remaining + ((size_t)e * 4 + o) * 4 * 12;
    for (int t = 0; t < 12; ++t) {
        gl[t] = (float)rem[left * 12 + t];
        gl[12 + t] = (float)rem[right * 12 + t];
    }
    for (int k = 0; k < 4; ++k) gl[24 + k] = b->seat_flag[SI(e, flag_order[k])] ? 1.f : 0.f;
#undef W
    return 0;
}

/* Initial beliefs and an empty move history for an env whose state was
 * loaded directly (for fixtures that start from an arbitrary position). */
int jqo_init_beliefs(jqo_batch *b, int e, int mode) {
    build_topology();
    bel_initial(b, e, mode);
    for (int i = 0; i < JQO_HIST; ++i) {
        b->hist_src[(size_t)e * JQO_HIST + i] = -1;
        b->hist_dst[(size_t)e * JQO_HIST + i] = -1;
    }
    b->hist_count[e] = 0;
    return 0;
}

/* Observation with caller-given per-cell float beliefs, restating the
 * reference GPU encoder's belief input (src/env/cuda/src/observation.cu):
 * the observer's (12, 289) slice of bel (246-253) is written at each alive
 * teammate / left / right piece's cell, in channels 12-23 / 27-38 / 39-50,
 * where it is > 0 (330-370); global[0:12] and [12:24] are its sums over the
 * left and right enemy pieces' cells (417-424, 533-544).  The reference adds
 * those per-piece values with float atomics in no fixed order; here they are
 * added in ascending pid order.  Everything else is jqo_obs.  bel is this
 * env's (4, 12, 289) float32 block: [observer][type][world flat]. */
int jqo_obs_ext(const jqo_batch *b, int e, int o, int mode, const float *bel, float *sp, float *gl) {
    jqo_obs(b, e, o, mode, sp, gl);
    const int *rot = T_rot[o];
    const float *bo = bel + (size_t)o * 12 * NC;
    const int tm = (o + 2) % 4, left = (o + 1) % 4, right = (o + 3) % 4;
    float rl[12], rr[12];
    for (int t = 0; t < 12; ++t) rl[t] = rr[t] = 0.f;
    for (int p = 0; p < NP; ++p) {
        size_t q = PI(e, p);
        if (!b->alive[q]) continue;
        const int f = b->pos_y[q] * 17 + b->pos_x[q], s = b->piece_seat[q];
        const int base = s == tm ? 12 : s == left ? 27 : s == right ? 39 : -1;
        if (base < 0) continue;
        for (int t = 0; t < 12; ++t) {
            const float x = bo[(size_t)t * NC + f];
            sp[(size_t)(base + t) * NC + rot[f]] = x > 0.f ? x : 0.f;
            if (s == left) rl[t] += x;
            if (s == right) rr[t] += x;
        }
    }
    for (int t = 0; t < 12; ++t) {
        gl[t] = rl[t];
        gl[12 + t] = rr[t];
    }
    return 0;
}

int jqo_obs_ext_batch(const jqo_batch *b, const int8_t *observers, int mode, const float *bel, float *sp,
                      float *gl, int nthreads) {
    build_topology();
#pragma omp parallel for schedule(dynamic, 8) num_threads(nthreads > 0 ? nthreads : 1)
    for (int e = 0; e < b->n; ++e)
        jqo_obs_ext(b, e, observers[e], mode, bel + (size_t)e * 4 * 12 * NC, sp + (size_t)e * JQO_OBS_CH * NC,
                    gl + (size_t)e * JQO_OBS_GLOBAL);
    return 0;
}

int jqo_obs_batch(const jqo_batch *b, const int8_t *observers, int mode, float *sp, float *gl,
                  int nthreads) {
    build_topology();
#pragma omp parallel for schedule(dynamic, 8) num_threads(nthreads > 0 ? nthreads : 1)
    for (int e = 0; e < b->n; ++e)
        jqo_obs(b, e, observers[e], mode, sp + (size_t)e * JQO_OBS_CH * NC, gl + (size_t)e * JQO_OBS_GLOBAL);
    return 0;
}

/* ------------------------------------------------------------------------
 * Per-cell float beliefs of the reference GPU rollout (belief.cu).  Values
 * are copied, set to 0 / 1, to prior rows or to 1/12; the tests on them use
 * the reference's float forms (running float sum, fmaxf chain).
 * ------------------------------------------------------------------------ */
#define CB_T 12
static float *cb_at(float *bel, int env, int o, int cell) {
    return bel + ((size_t)env * 4 + o) * CB_T * NC + cell; /* type t at [t * NC] */
}
static void cb_read(float *bel, int env, int o, int cell, float *v) {
    const float *p = cb_at(bel, env, o, cell);
    for (int t = 0; t < CB_T; ++t) v[t] = p[t * NC];
}
static void cb_write(float *bel, int env, int o, int cell, const float *v) {
    float *p = cb_at(bel, env, o, cell);
    for (int t = 0; t < CB_T; ++t) p[t * NC] = v[t];
}
static void cb_zero(float *bel, int env, int o, int cell) {
    float *p = cb_at(bel, env, o, cell);
    for (int t = 0; t < CB_T; ++t) p[t * NC] = 0.f;
}
static int cb_one_hot(const float *v) { /* belief.cu:71-76 */
    float mx = 0.f;
    for (int t = 0; t < CB_T; ++t) mx = fmaxf(mx, v[t]);
    return mx > (1.0f - 1e-6f);
}
static int cb_argmax(const float *v) { /* belief.cu:79-90 */
    int best = 0;
    float bv = v[0];
    for (int t = 1; t < CB_T; ++t)
        if (v[t] > bv) { bv = v[t]; best = t; }
    return best;
}
static int cb_is_zero(const float *v) { /* belief.cu:110-115 */
    float s = 0.f;
    for (int t = 0; t < CB_T; ++t) s += v[t];
    return s < 1e-8f;
}
static void cb_set_one_hot(float *v, int ti) {
    for (int t = 0; t < CB_T; ++t) v[t] = t == ti ? 1.f : 0.f;
}

int jqo_cellbel_init(const jqo_batch *b, int env, const float *prior, float *bel) {
    memset(cb_at(bel, env, 0, 0), 0, sizeof(float) * 4 * CB_T * NC);
    for (int p = 0; p < NP; ++p) { /* belief.cu:208-247 */
        const size_t q = (size_t)env * NP + p;
        if (!b->alive[q]) continue;
        const int seat = b->piece_seat[q], type = b->piece_type[q], px = b->pos_x[q], py = b->pos_y[q];
        if (px < 0 || py < 0 || px > 16 || py > 16) continue;
        const int cell = py * 17 + px, ti = (type >= 2 && type <= 13) ? type - 2 : -1;
        if (ti < 0) continue;
        for (int o = 0; o < 4; ++o) {
            float *c = cb_at(bel, env, o, cell);
            if (o == seat) c[ti * NC] = 1.f;
            else
                for (int t = 0; t < CB_T; ++t) c[t * NC] = prior[(p % 30) * CB_T + t];
        }
    }
    return 0;
}

int jqo_cellbel_update(const jqo_batch *b, int env, int event, int flag_cap, int32_t act, const uint8_t *prev_dead,
                       const int16_t *sh, float *bel) {
    build_topology();
    if (b->terminated[env] || event == 0) return 0; /* belief.cu:275-281 */
    if (act < 0 || act >= NC * NC) return 0;
    const int src = act / NC, dst = act % NC;
    const int16_t *cpid = b->cell_pid + (size_t)env * NC;
    const uint8_t *sdead = b->seat_dead + (size_t)env * 4;
    int surrendered = -1; /* belief.cu:363-375: the first newly dead seat of a flag capture */
    if (flag_cap)
        for (int s = 0; s < 4; ++s)
            if (sdead[s] && !prev_dead[s]) { surrendered = s; break; }
    int owner = -1, other = -1; /* belief.cu:380-402 */
    if (T_sh[dst])
        for (int s = 0; s < 4; ++s) {
            if (sh[2 * s] == dst) { owner = s; other = sh[2 * s + 1]; break; }
            if (sh[2 * s + 1] == dst) { owner = s; other = sh[2 * s]; break; }
        }
    for (int o = 0; o < 4; ++o) {
        float vs[CB_T], vd[CB_T];
        cb_read(bel, env, o, src, vs);
        cb_read(bel, env, o, dst, vd);
        /* R5/R7 (belief.cu:425-440): eating a known mine makes the attacker an engineer */
        if (event == 2 && cb_one_hot(vd) && cb_argmax(vd) == 1 && !cb_one_hot(vs)) cb_set_one_hot(vs, 11);
        /* R1 migration (belief.cu:444-469) */
        if (event == 1 || event == 2) {
            cb_write(bel, env, o, dst, vs);
            cb_zero(bel, env, o, src);
        } else if (event == 4) {
            cb_zero(bel, env, o, src);
        } else if (event == 3) {
            cb_zero(bel, env, o, src);
            cb_zero(bel, env, o, dst);
        }
        /* R6 (belief.cu:473-486): an eaten stronghold piece that is not the
         * flag puts the flag on the seat's other stronghold */
        if (event == 2 && T_sh[dst] && !flag_cap && owner >= 0 && other >= 0 && other < NC) {
            float v[CB_T];
            cb_read(bel, env, o, other, v);
            if (!cb_is_zero(v) && !cb_one_hot(v)) {
                cb_set_one_hot(v, 0);
                cb_write(bel, env, o, other, v);
            }
        }
        /* R4 (belief.cu:490-505): after a flag capture every empty cell is cleared */
        if (flag_cap && surrendered >= 0)
            for (int c = 0; c < NC; ++c)
                if (cpid[c] < 0) cb_zero(bel, env, o, c);
        /* I5 sweep (belief.cu:518-562) */
        for (int c = 0; c < NC; ++c) {
            const int p = cpid[c];
            float v[CB_T];
            cb_read(bel, env, o, c, v);
            if (p < 0 || p >= NP || !b->alive[(size_t)env * NP + p]) {
                if (!cb_is_zero(v)) cb_zero(bel, env, o, c);
            } else if (cb_is_zero(v)) {
                const int ps = b->piece_seat[(size_t)env * NP + p], pt = b->piece_type[(size_t)env * NP + p];
                const int ti = (pt >= 2 && pt <= 13) ? pt - 2 : -1;
                if ((o & 1) == (ps & 1) && ti >= 0) cb_set_one_hot(v, ti);
                else
                    for (int t = 0; t < CB_T; ++t) v[t] = 1.0f / (float)CB_T;
                cb_write(bel, env, o, c, v);
            }
        }
    }
    return 0;
}
