// jq_slots.cuh -- per-piece 80-slot legal-action mask, the reference GPU
// format of legal_action_mask_batch (src/env/cuda/src/game_state.cu:
// 1985-2197; slot layout in bindings.cpp:979-1000).
//
// Row (env, pid) has 80 slots; only pieces of the given seat have set slots:
//   0..3   orthogonal one-steps (+x, -x, +y, -y)
//   4..7   camp-diagonal one-steps, compacted in (+1,+1), (+1,-1), (-1,+1),
//          (-1,-1) order
//   8..55  non-engineers: straight rail ray d (0..3 = +x, -x, +y, -y) cell k
//          at slot 8 + 12 d + k, a cell that is also an orthogonal neighbour
//          left to slots 0..3
//   56..67 non-engineers: the curve rail of the source, breadth-first over
//          the rail graph, cells on neither the source's row nor its column,
//          packed in visiting order
//   8..79  engineers: rail cells reachable through empty rail cells,
//          breadth-first, orthogonal neighbours excluded, packed in visiting
//          order
// A slot is set when the cell is empty or holds an enemy outside a camp.
// One thread per (env, pid); the row is built as 80 bits and written as
// five 16-byte words of 0/1 bytes.
#pragma once
#include "jq_rules.cuh"

namespace jq {

__device__ SlotTopo g_slot;

__device__ __forceinline__ void slot_set(uint32_t &m0, uint32_t &m1, uint32_t &m2, int s) {
    const uint32_t bit = 1u << (s & 31);
    if (s < 32) m0 |= bit;
    else if (s < 64) m1 |= bit;
    else m2 |= bit;
}

__global__ void slot_mask_kernel(jq_batch b, const int8_t *__restrict__ seats, uint8_t *__restrict__ out) {
    const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (t >= (size_t)b.n * NP) return;
    const int e = (int)(t / NP), pid = (int)(t % NP);
    const SlotTopo &S = g_slot;
    uint32_t m0 = 0, m1 = 0, m2 = 0;
    const int seat = seats ? seats[e] : b.turn[e];
    const size_t q = PI(e, pid);
    const int t_pid = b.piece_type[q], sx = b.pos_x[q], sy = b.pos_y[q];
    const int src = (sx >= 0 && sx < 17 && sy >= 0 && sy < 17) ? sy * 17 + sx : -1;
    const int sc = src >= 0 ? g_topo.f2c[src] : -1;
    if (b.piece_seat[q] == seat && b.alive[q] && t_pid != JUNQI && t_pid != DILEI && sc >= 0 &&
        !(g_topo.flags[sc] & F_SH)) {
        const int16_t *cp = b.cell_pid + (size_t)e * NC;
        const int team = seat & 1;
        // the cell is a landing: empty, or an enemy not in a camp
        auto enemy_at = [&](int f, int occ) {
            if (occ < 0 || occ >= NP) return false;
            const int c = g_topo.f2c[f];
            return ((int)b.piece_seat[PI(e, occ)] & 1) != team && !(c >= 0 && (g_topo.flags[c] & F_CAMP));
        };
        for (int k = 0; k < 8; ++k) {
            const int nb = S.adj8[src][k];
            if (nb < 0) continue;
            const int occ = cp[nb];
            if (occ < 0 || enemy_at(nb, occ)) slot_set(m0, m1, m2, k);
        }
        if (g_topo.flags[sc] & F_RAIL) {
            const int o0 = S.adj8[src][0], o1 = S.adj8[src][1], o2 = S.adj8[src][2], o3 = S.adj8[src][3];
            auto is_ortho = [&](int f) { return f == o0 || f == o1 || f == o2 || f == o3; };
            uint8_t queue[80];
            uint64_t v0 = 0, v1 = 0;
            auto visit = [&](int r) {  // true the first time rail index r is seen
                uint64_t &v = r < 64 ? v0 : v1;
                const uint64_t bit = 1ull << (r & 63);
                if (v & bit) return false;
                v |= bit;
                return true;
            };
            const int sr = S.ri[src];
            if (t_pid != GONGB) {
                for (int d = 0; d < 4; ++d)
                    for (int k = 0; k < 12; ++k) {
                        const int c = g_topo.sray[sc][d][k];
                        if (c == NONE8) break;
                        const int nb = g_topo.c2f[c], occ = cp[nb];
                        if (occ < 0) {
                            if (!is_ortho(nb)) slot_set(m0, m1, m2, 8 + 12 * d + k);
                        } else {
                            if (!is_ortho(nb) && enemy_at(nb, occ)) slot_set(m0, m1, m2, 8 + 12 * d + k);
                            break;
                        }
                    }
                const int curve = g_topo.curve[sc];
                if (curve > 0 && sr >= 0) {
                    int qh = 0, qt = 0, slot = 56;
                    visit(sr);
                    queue[qt++] = (uint8_t)sr;
                    while (qh < qt) {
                        const int cur = queue[qh++];
                        for (int i = 0; i < 8; ++i) {
                            const int nr = S.rn[cur][i];
                            if (nr < 0) break;
                            if (!visit(nr)) continue;
                            const int nf = S.rcell[nr], ncomp = g_topo.f2c[nf];
                            if (ncomp < 0 || g_topo.curve[ncomp] != curve) continue;
                            const bool same_axis = (nf % 17 == sx) || (nf / 17 == sy);
                            const int occ = cp[nf];
                            if (occ < 0) {
                                if (!same_axis && slot < 68) slot_set(m0, m1, m2, slot++);
                                if (qt < 80) queue[qt++] = (uint8_t)nr;
                            } else if (!same_axis && slot < 68 && enemy_at(nf, occ)) {
                                slot_set(m0, m1, m2, slot++);
                            }
                        }
                    }
                }
            } else if (sr >= 0) {
                int qh = 0, qt = 0, slot = 8;
                visit(sr);
                queue[qt++] = (uint8_t)sr;
                while (qh < qt) {
                    const int cur = queue[qh++];
                    for (int i = 0; i < 8; ++i) {
                        const int nr = S.rn[cur][i];
                        if (nr < 0) break;
                        if (!visit(nr)) continue;
                        const int nf = S.rcell[nr], occ = cp[nf];
                        if (occ < 0) {
                            if (!is_ortho(nf) && slot < 80) slot_set(m0, m1, m2, slot++);
                            if (qt < 80) queue[qt++] = (uint8_t)nr;
                        } else if (!is_ortho(nf) && slot < 80 && enemy_at(nf, occ)) {
                            slot_set(m0, m1, m2, slot++);
                        }
                    }
                }
            }
        }
    }
    // 80 bits -> 80 bytes of 0 / 1, five aligned 16-byte words
    uint4 *row = reinterpret_cast<uint4 *>(out + t * 80);
    const uint32_t w[3] = {m0, m1, m2};
#pragma unroll
    for (int i = 0; i < 5; ++i) {
        const uint32_t bits = (w[(i * 16) >> 5] >> ((i * 16) & 31)) & 0xFFFFu;
        row[i] = make_uint4(nibble_bytes(bits & 15u), nibble_bytes((bits >> 4) & 15u), nibble_bytes((bits >> 8) & 15u),
                            nibble_bytes(bits >> 12));
    }
}

}  // namespace jq
