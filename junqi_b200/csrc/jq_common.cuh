// jq_common.cuh -- shared definitions for the sm_100a JunQi kernels.
//
// Board geometry is held in "compact" cell space: the 129 on-board cells of
// the 17x17 grid numbered in ascending flat order (junqi_core/board.py:263-
// 280), so compact order equals flat order and a 129-bit mask (five 32-bit
// words) covers the whole board.  All per-cell tables below are built once on
// the host (jq_topo_build.h) and copied to __constant__ memory; kernels that
// index them per lane stage a copy in shared memory.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/jq.h"

namespace jq {

constexpr int NP = 120;           // piece ids, seat*30 + slot
constexpr int NC = 289;           // flat cells
constexpr int NB = 129;           // on-board (compact) cells
constexpr int NW = 5;             // 32-bit words of a compact cell mask
constexpr int OBS_CH = 317;
constexpr int OBS_PLANE = 289;
constexpr int OBS_FLOATS = OBS_CH * OBS_PLANE;  // 91613
constexpr int OBS_GL = 28;
constexpr int HIST = 32;
constexpr int MASK_BYTES = 16641;
constexpr int RECENCY_LEN = 4097;
constexpr uint8_t NONE8 = 255;

// junqi_core/rules.py:57-74
enum PieceT : int { NONE = 0, DARK = 1, JUNQI = 2, DILEI = 3, ZHADAN = 4, SILING = 5, JUNZH = 6,
                    SHIZH = 7, LVZH = 8, TUANZH = 9, YINGZH = 10, LIANZH = 11, PAIZH = 12,
                    GONGB = 13 };
enum EventT : int { EV_MOVE = 1, EV_EAT = 2, EV_BOMB = 3, EV_KILLED = 4 };
enum DeathT : int { DR_KBE = 0, DR_MINE = 1, DR_MUTUAL = 2 };
enum ShowT : int { SM_BRIGHT = 0, SM_DARK = 1, SM_HALF_DARK = 2 };

// cell flag bits
enum : uint8_t { F_CAMP = 1, F_SH = 2, F_RAIL = 4, F_NINE = 8, F_ARC = 16, F_CURVE_ACTIVE = 32 };

// Belief codes, one byte per (observer, pid): 0 no entry, 1..12 one-hot of
// tracked type (idx+1), 14 uniform fallback, 32+slot prior of seat-local slot.
enum : uint8_t { BC_NONE = 0, BC_UNIFORM = 14, BC_PRIOR0 = 32 };

// The board tables the rules kernel reads; each of its CTAs holds a copy in
// shared memory.
struct __align__(16) TopoCore {
    int16_t c2f[NB];           // compact -> flat
    int16_t f2c[NC];           // flat -> compact, -1 off board
    uint8_t flags[NB];
    uint8_t curve[NB];         // legacy curve-rail id 0..4 (all cells carrying one)
    uint8_t adj4[NB][4];       // orthogonal neighbours (+x,-x,+y,-y)
    uint8_t diag[NB][4];       // diagonal steps into / out of a camp
    uint8_t cray[NB][2][11];   // curve-chain rays (forward, backward)
    alignas(16) uint32_t railnb[NB][8];  // rail-graph neighbours as a mask; words NW.. are zero, so a
                                         // row loads as two 16-byte words
    alignas(16) uint32_t ray[NB][4][NW];  // straight rail rays (+x,-x,+y,-y) as cell masks (build_ray_masks)
    uint8_t rot[4][NB];        // world compact -> canonical compact, per seat
    uint8_t slot_cell[4][30];  // compact cell of (seat, slot)
};

// All board tables: the rules kernel's, and those only the host, the
// observation encoder and the 80-slot mask read.
struct __align__(16) Topo : TopoCore {
    uint8_t sray[NB][4][12];   // straight rail rays (+x,-x,+y,-y) as cell lists
    int16_t rotf[4][NC];       // world flat -> canonical flat, per seat
    int8_t slot_ch[30];        // piece-slot channel of a seat-local slot, -1 camp
};

// Tables of the per-piece 80-slot legal mask (the reference GPU format of
// legal_action_mask_batch): flat-space neighbours in the order that format
// numbers its slots, and the rail graph in rail-index space (rail cells in
// flat order, neighbours ascending).
struct __align__(16) SlotTopo {
    int16_t adj8[NC][8];   // 0..3 orthogonal (+x, -x, +y, -y), 4..7 camp diagonals compacted; -1 none
    int16_t rcell[80];     // rail index -> flat
    int8_t ri[NC];         // flat -> rail index, -1 off the railway
    int8_t rn[80][8];      // rail-index neighbours, ascending, -1 padded
};

__host__ __device__ inline int tracked_idx(int t) { return (t >= 2 && t <= 13) ? t - 2 : -1; }
__host__ __device__ inline bool is_ranked(int t) { return t >= SILING && t <= GONGB; }
__host__ __device__ inline int team_of_pid(int pid) { return (pid / 30) & 1; }

// board.py:80-99 (legacy SetChess) seat-local slot -> world (x, y)
__host__ __device__ inline void slot_xy(int seat, int i, int &x, int &y) {
    int col = i % 5, row = i / 5;
    switch (seat) {
    case 0: x = 10 - col; y = 11 + row; break;
    case 1: x = 5 - row; y = 10 - col; break;
    case 2: x = 6 + col; y = 5 - row; break;
    default: x = 11 + row; y = 6 + col; break;
    }
}

// SplitMix64 finaliser (Steele, Lea, Flood 2014) used as a counter-based
// hash for pool selection and sampling.
__host__ __device__ inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t hash3(uint64_t a, uint64_t b, uint64_t c) {
    return mix64(mix64(mix64(a) ^ b) ^ c);
}

__device__ __forceinline__ bool mbit(const uint32_t *m, int c) { return (m[c >> 5] >> (c & 31)) & 1u; }
__device__ __forceinline__ void mset(uint32_t *m, int c) { m[c >> 5] |= 1u << (c & 31); }
// The same on a 5-word mask held in registers: select instead of a dynamic
// index, so the array stays in registers rather than local memory.
__device__ __forceinline__ bool rbit(const uint32_t (&m)[5], int c) {
    const uint32_t wd = c < 64 ? (c < 32 ? m[0] : m[1]) : (c < 96 ? m[2] : (c < 128 ? m[3] : m[4]));
    return (wd >> (c & 31)) & 1u;
}
__device__ __forceinline__ void rset(uint32_t (&m)[5], int c) {
    const uint32_t bit = 1u << (c & 31), wi = (uint32_t)c >> 5;
#pragma unroll
    for (uint32_t i = 0; i < 5; ++i) m[i] |= wi == i ? bit : 0u;
}

}  // namespace jq
