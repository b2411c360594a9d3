// jq_topo_build.h -- host-side construction of the compact board tables.
//
// Geometry follows junqi_core: seat zones and camps (board.py:80-196), the
// rail graph = orthogonal rail links + nine-grid two-steps + the four corner
// arcs (rail_topology.py:199-238), straight rays as axis-monotone walks on
// that graph (_movegen_tables.py:230-284) and the curve chains linearised
// from their first degree-1 end (_movegen_tables.py:375-470).
#pragma once
#include <cstdlib>
#include <cstring>
#include <vector>

#include "jq_common.cuh"

namespace jq {

inline void build_topo(Topo &T) {
    std::memset(&T, 0, sizeof T);
    // ---- flat-space cell properties ----
    bool on[NC] = {}, camp[NC] = {}, sh[NC] = {}, rail[NC] = {}, nine[NC] = {};
    int curve[NC] = {};
    for (int seat = 0; seat < 4; ++seat)
        for (int i = 0; i < 30; ++i) {
            int x, y;
            slot_xy(seat, i, x, y);
            int f = y * 17 + x, row = i / 5, col = i % 5;
            on[f] = true;
            camp[f] = (i == 6 || i == 8 || i == 12 || i == 16 || i == 18);
            sh[f] = (i == 26 || i == 28);
            rail[f] = i < 25 && (row == 0 || row == 4 || col == 0 || col == 4);
        }
    for (int i = 0; i < 9; ++i) {
        int f = (6 + (i / 3) * 2) * 17 + (10 - (i % 3) * 2);
        on[f] = rail[f] = nine[f] = true;
    }
    // legacy InitCurveRail ids: column 4 of seat (id-1) with column 0 of seat id%4
    for (int id = 1; id <= 4; ++id)
        for (int j = 4; j < 30; j += 5) {
            int x, y;
            slot_xy(id - 1, j, x, y);
            curve[y * 17 + x] = id;
            slot_xy(id % 4, j - 4, x, y);
            curve[y * 17 + x] = id;
        }
    // ---- rail adjacency (flat), neighbour lists kept ascending ----
    std::vector<std::vector<int>> radj(NC);
    auto link = [&](int a, int b) {
        for (int v : radj[a]) if (v == b) return;
        radj[a].push_back(b);
        radj[b].push_back(a);
    };
    auto inb = [](int x, int y) { return x >= 0 && x < 17 && y >= 0 && y < 17; };
    for (int f = 0; f < NC; ++f) {
        if (!rail[f]) continue;
        int x = f % 17, y = f / 17;
        const int d[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
        for (auto &dd : d) {
            if (inb(x + dd[0], y + dd[1]) && rail[(y + dd[1]) * 17 + x + dd[0]]) link(f, (y + dd[1]) * 17 + x + dd[0]);
            if (nine[f] && inb(x + 2 * dd[0], y + 2 * dd[1]) && nine[(y + 2 * dd[1]) * 17 + x + 2 * dd[0]])
                link(f, (y + 2 * dd[1]) * 17 + x + 2 * dd[0]);
        }
    }
    const int arcs[4][4] = {{10, 11, 11, 10}, {6, 11, 5, 10}, {6, 5, 5, 6}, {11, 6, 10, 5}};
    for (auto &a : arcs) link(a[1] * 17 + a[0], a[3] * 17 + a[2]);
    for (auto &v : radj) {
        for (size_t i = 1; i < v.size(); ++i)
            for (size_t j = i; j > 0 && v[j - 1] > v[j]; --j) std::swap(v[j - 1], v[j]);
    }
    // ---- compact numbering ----
    int nb = 0;
    for (int f = 0; f < NC; ++f) {
        T.f2c[f] = on[f] ? (int16_t)nb : (int16_t)-1;
        if (on[f]) T.c2f[nb++] = (int16_t)f;
    }
    auto C = [&](int f) -> uint8_t { return f < 0 ? NONE8 : (uint8_t)T.f2c[f]; };
    for (int c = 0; c < NB; ++c) {
        int f = T.c2f[c], x = f % 17, y = f / 17;
        uint8_t fl = 0;
        if (camp[f]) fl |= F_CAMP;
        if (sh[f]) fl |= F_SH;
        if (rail[f]) fl |= F_RAIL;
        if (nine[f]) fl |= F_NINE;
        for (int v : radj[f])
            if (std::abs(v % 17 - x) == 1 && std::abs(v / 17 - y) == 1) fl |= F_ARC;
        T.flags[c] = fl;
        T.curve[c] = (uint8_t)curve[f];
        const int d4[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
        for (int k = 0; k < 4; ++k) {
            int nx = x + d4[k][0], ny = y + d4[k][1];
            T.adj4[c][k] = (inb(nx, ny) && on[ny * 17 + nx]) ? C(ny * 17 + nx) : NONE8;
        }
        const int dg[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
        int nd = 0;
        for (int k = 0; k < 4; ++k) T.diag[c][k] = NONE8;
        for (auto &dd : dg) {
            int nx = x + dd[0], ny = y + dd[1];
            if (!inb(nx, ny) || !on[ny * 17 + nx]) continue;
            if (camp[f] || camp[ny * 17 + nx]) T.diag[c][nd++] = C(ny * 17 + nx);
        }
        for (int v : radj[f]) T.railnb[c][T.f2c[v] >> 5] |= 1u << (T.f2c[v] & 31);
        // straight rays: keep stepping to the rail neighbour that stays on the
        // axis and moves strictly forward
        for (int k = 0; k < 4; ++k) {
            for (int l = 0; l < 12; ++l) T.sray[c][k][l] = NONE8;
            if (!rail[f]) continue;
            int cur = f, n = 0;
            while (n < 12) {
                int nxt = -1;
                for (int v : radj[cur]) {
                    int vx = v % 17, vy = v / 17, cx = cur % 17, cy = cur / 17;
                    bool ok = d4[k][0] ? (vy == y && (vx - cx) * d4[k][0] > 0)
                                       : (vx == x && (vy - cy) * d4[k][1] > 0);
                    if (ok) nxt = v;
                }
                if (nxt < 0) break;
                T.sray[c][k][n++] = C(nxt);
                cur = nxt;
            }
        }
        for (int k = 0; k < 2; ++k)
            for (int l = 0; l < 11; ++l) T.cray[c][k][l] = NONE8;
    }
    // ---- curve chains: rail neighbours sharing the id, walked end to end ----
    for (int id = 1; id <= 4; ++id) {
        auto deg = [&](int f) {
            int d = 0;
            for (int v : radj[f]) d += curve[v] == id;
            return d;
        };
        int start = -1;
        std::vector<int> act;
        for (int f = 0; f < NC; ++f)
            if (curve[f] == id && deg(f) > 0) act.push_back(f);
        for (int f : act) {
            T.flags[T.f2c[f]] |= F_CURVE_ACTIVE;  // IS_CURVE_ACTIVE: id > 0 and degree > 0
            if (start < 0 && deg(f) == 1) start = f;
        }
        std::vector<int> chain;
        if (start < 0) chain = act;
        else {
            std::vector<char> seen(NC, 0);
            chain.push_back(start);
            seen[start] = 1;
            for (bool grew = true; grew;) {
                grew = false;
                for (int v : radj[chain.back()])
                    if (curve[v] == id && !seen[v]) { chain.push_back(v); seen[v] = 1; grew = true; break; }
            }
        }
        for (size_t i = 0; i < chain.size(); ++i) {
            int c = T.f2c[chain[i]];
            int n0 = 0, n1 = 0;
            for (size_t j = i + 1; j < chain.size() && n0 < 11; ++j) T.cray[c][0][n0++] = C(chain[j]);
            for (int j = (int)i - 1; j >= 0 && n1 < 11; --j) T.cray[c][1][n1++] = C(chain[j]);
        }
    }
    // ---- rotations (rotation.py:44-65) ----
    for (int s = 0; s < 4; ++s)
        for (int f = 0; f < NC; ++f) {
            int x = f % 17, y = f / 17, cx, cy;
            switch (s) {
            case 0: cx = x; cy = y; break;
            case 1: cx = y; cy = 16 - x; break;
            case 2: cx = 16 - x; cy = 16 - y; break;
            default: cx = 16 - y; cy = x; break;
            }
            T.rotf[s][f] = (int16_t)(cy * 17 + cx);
            if (on[f]) T.rot[s][T.f2c[f]] = (uint8_t)T.f2c[cy * 17 + cx];
        }
    for (int s = 0; s < 4; ++s)
        for (int i = 0; i < 30; ++i) {
            int x, y;
            slot_xy(s, i, x, y);
            T.slot_cell[s][i] = (uint8_t)T.f2c[y * 17 + x];
        }
    for (int i = 0, ch = 0; i < 30; ++i) {
        bool cp = (i == 6 || i == 8 || i == 12 || i == 16 || i == 18);
        T.slot_ch[i] = cp ? (int8_t)-1 : (int8_t)ch++;
    }
}

// The 80-slot mask's tables, derived from the compact tables above in the
// order that format numbers its slots (tables.cu:176-211, 240-297 of the
// reference CUDA extension).
inline void build_slot_topo(const Topo &T, SlotTopo &S) {
    std::memset(&S, 0xff, sizeof S);  // -1 everywhere
    auto on = [&](int f) { return T.f2c[f] >= 0; };
    auto camp = [&](int f) { return T.f2c[f] >= 0 && (T.flags[T.f2c[f]] & F_CAMP); };
    const int od[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}}, dd[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
    for (int f = 0; f < NC; ++f) {
        if (!on(f)) continue;
        const int x = f % 17, y = f / 17;
        for (int k = 0; k < 4; ++k) {
            const int nx = x + od[k][0], ny = y + od[k][1];
            if (nx >= 0 && nx < 17 && ny >= 0 && ny < 17 && on(ny * 17 + nx)) S.adj8[f][k] = (int16_t)(ny * 17 + nx);
        }
        int slot = 4;
        for (int k = 0; k < 4; ++k) {
            const int nx = x + dd[k][0], ny = y + dd[k][1];
            if (nx < 0 || nx >= 17 || ny < 0 || ny >= 17) continue;
            const int g = ny * 17 + nx;
            if (on(g) && (camp(f) || camp(g))) S.adj8[f][slot++] = (int16_t)g;
        }
    }
    int n = 0;
    for (int f = 0; f < NC; ++f)
        if (on(f) && (T.flags[T.f2c[f]] & F_RAIL)) {
            S.ri[f] = (int8_t)n;
            S.rcell[n++] = (int16_t)f;
        }
    for (int r = 0; r < n; ++r) {
        const int c = T.f2c[S.rcell[r]];
        int k = 0;
        for (int v = 0; v < NB && k < 8; ++v)  // compact order is flat order, so this is ascending
            if ((T.railnb[c][v >> 5] >> (v & 31)) & 1u) S.rn[r][k++] = S.ri[T.c2f[v]];
    }
}

// Straight rail rays as cell masks: ray k of cell c (directions +x, -x, +y,
// -y) holds the cells of T.sray[c][k].  Those cells lie on one axis in strictly
// increasing (k = 0, 2) or decreasing (k = 1, 3) flat, hence compact, order,
// which lets a kernel find the first blocker with one bit scan.  Returns
// false if a ray breaks that order.
inline bool build_ray_masks(const Topo &T, uint32_t out[NB][4][NW]) {
    for (int c = 0; c < NB; ++c)
        for (int k = 0; k < 4; ++k) {
            for (int i = 0; i < NW; ++i) out[c][k][i] = 0u;
            int prev = c;
            for (int l = 0; l < 12 && T.sray[c][k][l] != NONE8; ++l) {
                const int v = T.sray[c][k][l];
                if ((k & 1) ? v >= prev : v <= prev) return false;
                out[c][k][v >> 5] |= 1u << (v & 31);
                prev = v;
            }
        }
    return true;
}

}  // namespace jq
