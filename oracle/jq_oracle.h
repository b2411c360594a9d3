/*
 * jq_oracle.h -- CPU restatement of the JunQi reference rules.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * kernels in junqi_b200/csrc: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py may load it.  The product path
 * never links or calls it.
 *
 * It restates, function by function, the reference's authoritative CPU
 * rules (junqi_core, file:line cited at each function in jq_oracle.c):
 *   batched_state.py   step_batch / _step_single / _advance_turn(_vec) /
 *                      _check_victory(_vec) / _surrender_seat_delta
 *   move_gen.py        generate_legal_action_ids_n, has_legal_moves_soa,
 *                      move_requires_gongb and its BFS helpers
 *   combat_memory.py   apply_combat_event / apply_path_revealed_gongb
 *   info_model.py      BeliefTensor.initial / update (per-piece codes)
 *   observation.py     ObservationBuilder._fill_into and its writers
 *   state.py           GameState.new_game (device reset semantics)
 * Parity against the reference itself is pinned by the golden fixtures
 * under tests/golden/ (generated from junqi_core by tests/golden/make_golden.py).
 */
#ifndef JQ_ORACLE_H
#define JQ_ORACLE_H
#include <stdint.h>

#define JQO_PIECES 120
#define JQO_CELLS 289
#define JQO_OBS_CH 317
#define JQO_OBS_GLOBAL 28
#define JQO_HIST 32
#define JQO_ACTIONS_COMPACT 16641

/* Field-major SoA batch, same layout as the device batch (include/jq.h). */
typedef struct {
    int32_t n;
    /* piece-indexed (n,120) */
    uint8_t *alive;
    int8_t *piece_type, *piece_seat, *pos_x, *pos_y, *zero_x, *zero_y;
    int16_t *move_count, *active_eat, *passive_surv;
    int8_t *death_reason;
    int16_t *death_step, *death_loc;
    /* cell-indexed (n,289) */
    int16_t *cell_pid;
    /* seat-indexed (n,4) */
    uint8_t *seat_dead, *seat_flag;
    /* scalars (n,) */
    int8_t *turn;
    int64_t *zobrist;
    int32_t *move_counter, *mslc;
    uint8_t *terminated;
    int8_t *winner;
    uint8_t *draw;
    /* combat memory (n,4,120) */
    uint64_t *cm_direct_lo, *cm_direct_hi;
    uint16_t *cm_direct_type;
    int16_t *cm_last_direct_step, *cm_direct_other;
    uint64_t *cm_chain_lo, *cm_chain_hi;
    uint16_t *cm_chain_type;
    int16_t *cm_last_chain_step;
    uint64_t *cm_eaten_lo, *cm_eaten_hi;
    int8_t *cm_rank_floor;
    int16_t *cm_rank_floor_step;
    uint8_t *cm_is_gongb, *cm_not_gongb, *cm_atk_gongb;
    /* move-history ring (n,32) + total count (n,) */
    int16_t *hist_src, *hist_dst;
    int32_t *hist_count;
    /* beliefs: per (observer, pid) code (n,4,120); remaining (n,4,4,12);
       tracked (n,4,4) */
    uint8_t *bel_code;
    int16_t *remaining;
    uint8_t *rem_tracked;
    int32_t rules; /* 0: BatchedGameState rules, 1: GameState rules */
    int32_t max_moves; /* episode cap in plies (draw), 0: none beyond the rules' 4000 */
} jqo_batch;

/* Per-step outputs (n,) */
typedef struct {
    uint8_t *valid;
    int8_t *event;
    uint8_t *terminated;
    int8_t *winner;
    uint8_t *draw;
    uint8_t *flag_captured;
    float *reward;
} jqo_step_out;

#ifdef __cplusplus
extern "C" {
#endif
int jqo_set_tables(const int64_t *zob_piece, const int64_t *zob_turn,
                   const int64_t *zob_mc, const int64_t *zob_mslc,
                   int64_t zob_terminated, const int64_t *zob_winner,
                   int64_t zob_draw, const int64_t *zob_seat_dead,
                   const int64_t *zob_seat_flag, const int64_t *zob_show_mode,
                   const float *prior_table /*30x12*/, const float *uniform12,
                   const float *recency_lut /*4x4097*/);
int jqo_topology(int32_t *out_on_board, int32_t *out_rail, int32_t *out_curve,
                 int32_t *out_rail_adj /*289x4*/, int32_t *out_srays /*289x4x12*/,
                 int32_t *out_crays /*289x2x11*/, int32_t *out_compact_to_flat);
int jqo_reset_env(jqo_batch *b, int env, const int8_t *lineup120, int show_mode);
int jqo_init_beliefs(jqo_batch *b, int env, int show_mode);
int jqo_step(jqo_batch *b, const int32_t *actions, int show_mode, jqo_step_out *out,
             int nthreads);
int jqo_legal(const jqo_batch *b, int env, int seat, int ignore_skip, int32_t *out_ids,
              int cap);
int jqo_legal_batch(const jqo_batch *b, const int8_t *seats, int32_t *counts,
                    int32_t *ids /* n x cap */, int cap, int nthreads);
int jqo_canonical_mask(const int32_t *ids, int count, int seat, uint8_t *mask16641);
#define JQO_SLOTS 80
int jqo_slot_tables(int32_t *adj8 /*289x8*/, int32_t *srays /*289x4x12*/, int32_t *rail_adj /*289x8*/);
int jqo_slot_mask(const jqo_batch *b, int env, int seat, uint8_t *mask /*120x80*/, int16_t *dst /*120x80, or NULL*/);
int jqo_obs(const jqo_batch *b, int env, int observer, int show_mode, float *spatial,
            float *global);
int jqo_obs_batch(const jqo_batch *b, const int8_t *observers, int show_mode,
                  float *spatial, float *global, int nthreads);
/* As jqo_obs / jqo_obs_batch, with caller-given per-cell float beliefs
 * bel (N, 4, 12, 289) in the belief planes and global[0:24]. */
int jqo_obs_ext(const jqo_batch *b, int env, int observer, int show_mode, const float *bel, float *spatial,
                float *global);
int jqo_obs_ext_batch(const jqo_batch *b, const int8_t *observers, int show_mode, const float *bel,
                      float *spatial, float *global, int nthreads);
/* Per-cell float beliefs of the reference's GPU rollout (belief.cu), in
 * bel (N, 4, 12, 289) [env][observer][type][world cell]:
 * jqo_cellbel_init -- belief_init_kernel (belief.cu:172-248) for one env,
 * prior = the 30 x 12 per-slot table the caller uploads;
 * jqo_cellbel_update -- belief_update_kernel (belief.cu:255-565) for one env
 * on its post-step state, with the step's event / flag capture / world
 * action, the seat_dead snapshot prev_dead (4) and the 4 x 2 stronghold
 * cells of each seat. */
int jqo_cellbel_init(const jqo_batch *b, int env, const float *prior, float *bel);
int jqo_cellbel_update(const jqo_batch *b, int env, int event, int flag_captured, int32_t world_action,
                       const uint8_t *prev_dead, const int16_t *strongholds, float *bel);
#ifdef __cplusplus
}
#endif
#endif
