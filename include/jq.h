/*
 * jq.h -- C ABI of the B200 JunQi environment library (libjq.so).
 *
 * One process drives one GPU.  All state lives in caller-owned device memory
 * described by `jq_batch` (field-major SoA, one row per env); every entry
 * point takes plain device pointers, sizes and a cudaStream_t (passed as
 * void*), launches asynchronously on that stream and returns a status code.
 * Nothing here synchronises the device or calls exit().
 *
 * Each entry point names the reference interface it replaces
 * (freezeng123456/JunQi, src/env/cuda/src/bindings.cpp and
 * src/env/cuda/include/junqi_cuda.h).
 */
#ifndef JQ_H
#define JQ_H
#include <stddef.h>
#include <stdint.h>

#define JQ_ABI_VERSION 7

#define JQ_NUM_PIECES 120
#define JQ_NUM_CELLS 289
#define JQ_BOARD_SIZE 17
#define JQ_NUM_SEATS 4
#define JQ_NUM_OBS_CHANNELS 317
#define JQ_NUM_GLOBAL_DIMS 28
#define JQ_NUM_TRACKED_TYPES 12
#define JQ_FLAT_ACTION_SPACE 16641 /* 129 x 129 compact canonical actions */
#define JQ_HISTORY 32
#define JQ_MAX_LEGAL 512
#define JQ_RECENCY_LEN 4097

/* Status codes. */
enum {
    JQ_OK = 0,
    JQ_ERR_ARG = 1,       /* bad size / null pointer / out-of-range argument */
    JQ_ERR_CUDA = 2,      /* a CUDA runtime call failed; see jq_last_error() */
    JQ_ERR_NOT_READY = 3, /* jq_init / table uploads missing on this device */
    JQ_ERR_CAPACITY = 4   /* an output buffer is too small */
};

/* Rule sets (jq_batch.rules).  JQ_RULES_BATCHED follows BatchedGameState
 * (batched_state.py): after a plain move the Q12 "no legal move -> seat
 * dies" test only runs past an already-dead next seat, and surrendered
 * pieces get death_loc -1.  JQ_RULES_GAMESTATE follows GameState.step_inplace
 * (state.py:309-669), which the single-env JunqiEnv and the reference's GPU
 * rollout also follow: Q12 after every ply, victory checked before the turn
 * advances, surrendered pieces keep their current cell as death_loc. */
enum { JQ_RULES_BATCHED = 0, JQ_RULES_GAMESTATE = 1 };

/* Show modes (junqi_core/rules.py:598-603). */
enum { JQ_BRIGHT = 0, JQ_DARK = 1, JQ_HALF_DARK = 2 };

/*
 * Batch of N envs.  Shapes are per env; every array is contiguous with the
 * env index outermost and aligned to its element size; bel_code must be
 * 16-byte aligned (the kernels move it in 16-byte words).  Entry points
 * taking a batch return JQ_ERR_ARG otherwise.  Replaces DeviceGameStateBatch (junqi_cuda.h:48-111)
 * plus the CombatMemory, move-history and belief buffers the reference keeps
 * in process-global scratch.
 */
typedef struct jq_batch {
    int32_t n;
    uint8_t *alive;                    /* (120)  bool */
    int8_t *piece_type, *piece_seat;   /* (120)  -1 for empty camp slots */
    int8_t *pos_x, *pos_y;             /* (120)  -1 when dead */
    int8_t *zero_x, *zero_y;           /* (120)  initial cell */
    int16_t *move_count, *active_eat, *passive_surv; /* (120) */
    int8_t *death_reason;              /* (120)  -1 alive */
    int16_t *death_step, *death_loc;   /* (120)  -1 alive */
    int16_t *cell_pid;                 /* (289)  -1 empty */
    uint8_t *seat_dead, *seat_flag;    /* (4)    bool */
    int8_t *turn;                      /* ()     */
    int64_t *zobrist;                  /* ()     */
    int32_t *move_counter, *mslc;      /* ()     */
    uint8_t *terminated;               /* ()     bool */
    int8_t *winner;                    /* ()     -1 none */
    uint8_t *draw;                     /* ()     bool */
    uint64_t *cm_direct_lo, *cm_direct_hi;      /* (4,120) */
    uint16_t *cm_direct_type;                   /* (4,120) */
    int16_t *cm_last_direct_step, *cm_direct_other; /* (4,120) */
    uint64_t *cm_chain_lo, *cm_chain_hi;        /* (4,120) */
    uint16_t *cm_chain_type;                    /* (4,120) */
    int16_t *cm_last_chain_step;                /* (4,120) */
    uint64_t *cm_eaten_lo, *cm_eaten_hi;        /* (4,120) */
    int8_t *cm_rank_floor;                      /* (4,120) */
    int16_t *cm_rank_floor_step;                /* (4,120) */
    uint8_t *cm_is_gongb, *cm_not_gongb, *cm_atk_gongb; /* (4,120) bool */
    int16_t *hist_src, *hist_dst;      /* (32)   ring of the last 32 moves */
    int32_t *hist_count;               /* ()     moves recorded since reset */
    uint8_t *bel_code;                 /* (4,120) per-observer belief code */
    int16_t *remaining;                /* (4,4,12) per-observer enemy inventory */
    uint8_t *rem_tracked;              /* (4,4)  bool */
    int32_t rules;                     /* JQ_RULES_BATCHED or JQ_RULES_GAMESTATE */
    int32_t max_moves;                 /* episode cap in plies, 0: the rules' 4000 (see below) */
    const int8_t *pool;                /* (pool_size,120) setup lineups the resets of this batch
                                          draw from; NULL: the device-wide pool (jq_set_setup_pool) */
    int32_t pool_size;
} jq_batch;

/* jq_batch.max_moves: a game that reaches this many plies without a natural
 * result ends as a draw, checked after the victory and Q12 rules of the ply
 * (the reference's DeviceGameStateBatch max_num_moves, game_state.cu:1651-
 * 1655, like JunqiEnv's episode cap).  0 leaves only the rules' own draw at
 * move 4000 or 200 plies without combat (rules.py:444). */

/* Per-env step outputs (N each); any pointer may be NULL except valid. */
typedef struct jq_step_out {
    uint8_t *valid;
    int8_t *event;
    uint8_t *terminated;
    int8_t *winner;
    uint8_t *draw;
    uint8_t *flag_captured;
    float *reward;
    int32_t *world_action;   /* filled by jq_step_canonical */
    int64_t *zobrist;        /* post-step state hash, before any auto-reset
                                (replay self-check, junqi_core/replay.py:243-260) */
} jq_step_out;

#ifdef __cplusplus
extern "C" {
#endif

int jq_abi_version(void);
const char *jq_last_error(void);

/* Host-only dump of the board tables the kernels use, in flat cell space
 * (no device needed): on-board / rail / curve-id / flag bits per cell, rail
 * neighbours (289x4), straight rays (289x4x12), curve-chain rays (289x2x11),
 * compact->flat (129).  Mirrors the junqi_core tables of
 * _movegen_tables.py:130-470 and board.py:263-280 for parity tests. */
int jq_topology_dump(int32_t *on_board, int32_t *rail, int32_t *curve, int32_t *rail_adj,
                     int32_t *srays, int32_t *crays, int32_t *compact_to_flat, int32_t *flags);

/* Make `device` current and build the board topology tables in constant
 * memory.  Replaces init_tables / set_device (bindings.cpp:475-483,
 * tables.cu:397-524). */
int jq_init(int device);

/* Upload the ten Zobrist tables (host pointers; shapes as in
 * junqi_core/_zobrist.py:80-122).  Replaces upload_zobrist_tables
 * (bindings.cpp:485-517). */
int jq_upload_zobrist(const int64_t *piece /*120*14*289*/, const int64_t *turn /*4*/,
                      const int64_t *move_counter /*4096*/, const int64_t *mslc /*512*/,
                      const int64_t *winner /*3*/, int64_t terminated, int64_t draw,
                      const int64_t *seat_dead /*4*/, const int64_t *seat_flag /*4*/,
                      const int64_t *show_mode /*4*/);

/* Upload observation tables (host pointers): per-slot belief prior (30x12),
 * the uniform fallback vector (12) and the recency LUT (4 x 4097).
 * Replaces upload_belief_prior_table (bindings.cpp:1234-1242). */
int jq_upload_obs_tables(const float *prior /*30*12*/, const float *uniform12,
                         const float *recency /*4*4097*/);

/* Register the device-wide setup pool ((P,120) int8, piece type per pid,
 * 0 on camp slots): the pool of every batch whose own jq_batch.pool is
 * NULL.  The pointer is kept until the next call, so the caller keeps the
 * memory alive that long.  Replaces upload_setup_pool (bindings.cpp:1209-
 * 1222), whose pool is process-global as this one is; a caller with several
 * batches gives each its own jq_batch.pool instead. */
int jq_set_setup_pool(const int8_t *d_pool, int32_t pool_size);

/* Pool index used by every reset: splitmix64(seed, ply, env) mod P. */
int32_t jq_pool_index(uint64_t seed, uint64_t ply, int32_t env, int32_t pool_size);

/* Reset every env whose terminated flag is set (or all envs when `all`)
 * to GameState.new_game(pool[jq_pool_index(seed, ply, env)]) with fresh
 * beliefs, zeroed combat memory and empty move history.  Replaces
 * reset_terminated_envs + init_beliefs_for_reset_envs (bindings.cpp:1224-1262). */
int jq_reset(const jq_batch *b, uint64_t seed, uint64_t ply, int32_t all, int32_t show_mode,
             void *stream);

/* Reset env e to GameState.new_game(pool[d_rows[e]]) (as jq_reset) for every
 * e with 0 <= d_rows[e] < pool size; other envs are left as they are.  For
 * replaying recorded games from their own setups (junqi_core/replay.py:
 * 226-240 starts every replay from new_game(setups)). */
int jq_reset_rows(const jq_batch *b, const int32_t *d_rows, int32_t show_mode, void *stream);

/* Initial beliefs (BeliefTensor.initial for all four observers,
 * info_model.py:218-270) and an empty move history for every env, for
 * state written by the caller.  Replaces init_all_beliefs
 * (bindings.cpp:1262-1270). */
int jq_init_beliefs(const jq_batch *b, int32_t show_mode, void *stream);

/* Per-piece 80-slot legal mask of each env's seat (d_seats (N,) int8, or
 * NULL for the env's turn): d_slots is (N, 120, 80) uint8, 16-byte aligned,
 * 1 where piece pid can make the move of that slot -- slots 0..3 orthogonal
 * one-steps (+x, -x, +y, -y), 4..7 camp diagonals, 8..55 straight rail ray d
 * cell k at 8 + 12 d + k, 56..67 curve-rail cells off the source's row and
 * column in breadth-first order, and for engineers 8..79 the rail cells
 * reachable through empty rail in breadth-first order (orthogonal
 * neighbours excluded).  Replaces legal_action_mask_batch
 * (bindings.cpp:951-1000, game_state.cu:1985-2197). */
int jq_legal_slots(const jq_batch *b, const int8_t *d_seats, uint8_t *d_slots, void *stream);

/* Rebuild every env's Zobrist hash from its state, for state written by the
 * caller (a position built on the host).  Device counterpart of the
 * reference's host-side _recompute_zobrist (state.py:1761-1815), which
 * GameState.from_dict uses; bindings.cpp has no such entry point. */
int jq_rehash(const jq_batch *b, int32_t show_mode, void *stream);

/* One ply for every env: world action id src_flat*289+dst_flat per env.
 * BatchedGameState.step_batch semantics, plus combat memory, beliefs, move
 * history and terminal reward.  Replaces DeviceGameStateBatch.step_batch /
 * step_device (bindings.cpp:597-610, 1044-1074; game_state.cu:1307-1685). */
int jq_step(const jq_batch *b, const int32_t *d_world_actions, int32_t show_mode,
            const jq_step_out *out, void *stream);

/* As jq_step, taking compact canonical actions (cs*129+cd) in each env's
 * acting-seat frame; writes the world ids to out->world_action.
 * Replaces step_device's rotate_actions_kernel path (game_state.cu:2639-2797). */
int jq_step_canonical(const jq_batch *b, const int32_t *d_compact_actions,
                      const int8_t *d_seats, int32_t show_mode, const jq_step_out *out,
                      void *stream);

/* Compact canonical actions (cs*129+cd, in the frame of d_seats[e], or of
 * each env's turn when d_seats is NULL) to world flat ids src*289+dst; -1
 * for ids outside [0, 16641).  The rotation half of jq_step_canonical, for
 * callers that step through jq_ply (UNROTATE_LUT, action_lut.py:116-126;
 * rotate_actions_kernel, game_state.cu:2639-2685). */
int jq_canonical_to_world(const jq_batch *b, const int32_t *d_compact_actions, const int8_t *d_seats,
                          int32_t *d_world_actions, void *stream);

/* Fused ply: jq_step, then auto-reset of the envs it terminated (pool
 * index from (seed, ply, env)), then legal generation for the new turn
 * (see jq_legal).  d_world_actions may be NULL to skip the step.  When
 * d_stats is not NULL it accumulates int64[6] = {wins team 0, wins team 1,
 * draws, episodes, sum of episode lengths in plies, plies applied}: the
 * first five are the reference's per-rollout episode statistics, added at
 * each termination; the sixth counts steps with valid = 1. */
int jq_ply(const jq_batch *b, const int32_t *d_world_actions, int32_t show_mode,
           const jq_step_out *out, int32_t autoreset, uint64_t seed, uint64_t ply,
           int32_t *d_counts, int32_t *d_ids, int32_t cap, uint8_t *d_mask,
           int64_t *d_stats, void *stream);

/* Compact rollout history (replaces DeviceRolloutHistory, junqi_cuda.h:186-277,
 * bindings.cpp:728-800).  The caller owns a 16-byte aligned device buffer of
 * num_steps x N records of jq_history_record_bytes() bytes each; a record
 * holds what the observation and the legal mask of one seat read: the
 * board and piece state, that observer's combat-memory row, belief codes and
 * inventories, and the two opponents' views of its own pieces. */
int32_t jq_history_record_bytes(void);

/* Record every env of b (observer d_seats[e], NULL: its turn) as step `step`
 * of the history: record step * N + e. */
int jq_history_snapshot(const jq_batch *b, const int8_t *d_seats, void *d_history, int64_t step,
                        int64_t num_steps, void *stream);

/* Restore records d_indices[0 .. scratch->n) (flat step * N + env; out of
 * range: an empty, terminated env) into the envs of `scratch`, writing each
 * record's observer to d_observers.  jq_legal(scratch, d_observers, ...) and
 * jq_observe(scratch, d_observers, 1, ...) then rebuild the recorded seat's
 * legal actions, canonical mask and observation exactly as they were. */
int jq_history_restore(const void *d_history, int64_t num_records, const int64_t *d_indices,
                       const jq_batch *scratch, int8_t *d_observers, void *stream);

/* Per-cell float beliefs of the reference's GPU rollout (belief.cu), kept
 * by the caller in d_beliefs, a 16-byte aligned (N, 4, 12, 289) float32
 * array [env][observer][type][world flat cell] -- the input
 * jq_observe_beliefs reads.  These follow the reference GPU kernels' own
 * rules; the beliefs the step maintains itself (jq_batch.bel_code) follow
 * the CPU BeliefTensor.
 *
 * jq_cell_beliefs_init: clear the envs with d_env_mask[e] != 0 (NULL: all)
 * and seed every alive on-board piece: one-hot for its owner, the row of
 * its slot in d_prior (30 x 12 float32, device) for the other observers.
 * Replaces init_all_beliefs / init_beliefs_for_reset_envs
 * (bindings.cpp:1252-1270, belief.cu:172-248, 599-643). */
int jq_cell_beliefs_init(const jq_batch *b, const uint8_t *d_env_mask, const float *d_prior, float *d_beliefs,
                         void *stream);

/* seat_dead (N x 4) and terminated (N) as they are now, into caller buffers
 * (either may be NULL).  Replaces snapshot_pre_step_flags
 * (bindings.cpp:1272-1278, belief.cu:570-584, 645-671). */
int jq_cell_beliefs_snapshot(const jq_batch *b, uint8_t *d_prev_dead, uint8_t *d_prev_terminated, void *stream);

/* Update after a step, on the batch's post-step state: the step's event,
 * flag_captured and world action per env (jq_step_out fields), the
 * seat_dead snapshot d_prev_dead, and d_strongholds (4 x 2 int16, device:
 * each seat's two stronghold flat cells).  Envs now terminated, or whose
 * event is 0, are left as they are.  Rules R5/R7, R1, R6, R4 and the I5
 * sweep.  Replaces update_beliefs_after_step (bindings.cpp:1280-1300,
 * belief.cu:255-565, 673-706). */
int jq_cell_beliefs_update(const jq_batch *b, const int8_t *d_event, const uint8_t *d_flag_captured,
                           const int32_t *d_world_actions, const uint8_t *d_prev_dead, const int16_t *d_strongholds,
                           float *d_beliefs, void *stream);

/* Legal actions for `d_seats` (NULL: each env's turn), ascending and
 * de-duplicated per env (BatchedGameState.legal_action_ids_batch,
 * batched_state.py:370-409).  Writes d_counts (N) and d_ids (N x cap);
 * when d_mask is not NULL also the (N,16641) bool canonical mask in the
 * seat's frame (game_state.cu:2291-2508, action_lut.py:174-212).
 * Replaces legal_action_ids_batch / legal_mask_canonical_batch(_from_device). */
int jq_legal(const jq_batch *b, const int8_t *d_seats, int32_t *d_counts, int32_t *d_ids,
             int32_t cap, uint8_t *d_mask, void *stream);

/* CSR from jq_legal's output: d_offsets (N+1) and d_values (sum counts).
 * d_block_scratch must hold jq_csr_scratch_ints(N) int32.
 * Replaces legal_action_ids_batch_csr (bindings.cpp:892-950). */
int32_t jq_csr_scratch_ints(int32_t n);
int jq_csr(int32_t n, const int32_t *d_counts, const int32_t *d_ids, int32_t cap,
           int32_t *d_offsets, int32_t *d_values, int32_t *d_block_scratch, void *stream);

/* Allocation-free variant of jq_csr for callers that cannot allocate device
 * memory (a process whose CUDA allocator already owns the HBM budget, or a
 * thin FFI host holding only the buffers it was given).  No counterpart in
 * the reference.  The block-sum scratch is a 4 KiB file-scope device array
 * shared by every call on a GPU, so n is limited to JQ_NOALLOC_MAX_ENVS
 * (larger n returns JQ_ERR_CAPACITY) and calls that overlap on the GPU
 * (different streams without ordering) race on it.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.
 * Calls no cudaMalloc / cudaFree or allocating library routine. */
#define JQ_NOALLOC_MAX_ENVS (1 << 20)
int jq_csr_noalloc(int32_t n, const int32_t *d_counts, const int32_t *d_ids, int32_t cap,
                   int32_t *d_offsets, int32_t *d_values, void *stream);

/* 317-channel observation for `seats_per_env` observers per env:
 * d_observers is (N, seats_per_env) int8 (NULL with seats_per_env==1 means
 * each env's turn; NULL with 4 means seats 0..3).  Writes d_spatial
 * (N*seats, 317, 17, 17) float32 and d_global (N*seats, 28) float32.
 * ObservationBuilder._fill_into semantics (observation.py:598-858).
 * Replaces build_observation_batch(_resident) / build_observation_single_seat
 * (bindings.cpp:803-829, 1091-1182).  Units are scheduled through one of 256
 * device-side tickets per GPU, taken in call order: at most 256 calls may be
 * in flight on one GPU at a time (across all streams). */
int jq_observe(const jq_batch *b, const int8_t *d_observers, int32_t seats_per_env,
               int32_t show_mode, float *d_spatial, float *d_global, void *stream);

/* As jq_observe, with the belief input given by the caller instead of the
 * library's own per-piece beliefs: d_beliefs is (N, 4, 12, 289) float32,
 * [env][observer seat][tracked type][world flat cell] -- the reference's
 * d_belief layout.  The observer's slice is written at each alive
 * teammate / left / right piece's cell in channels 12-23 / 27-38 / 39-50
 * where it is > 0, and global[0:12] / [12:24] are its float32 sums over the
 * left / right enemy pieces' cells, added in ascending pid order (the
 * reference adds them with atomics in no fixed order).  Everything else is
 * jq_observe.  Replaces build_observation_batch with a beliefs argument
 * (bindings.cpp:1091-1134; observation.cu:246-253, 330-370, 417-424,
 * 533-544), e.g. beliefs refreshed by a belief network. */
int jq_observe_beliefs(const jq_batch *b, const int8_t *d_observers, int32_t seats_per_env,
                       int32_t show_mode, const float *d_beliefs, float *d_spatial, float *d_global,
                       void *stream);

/* Uniform-random legal action per env from jq_legal's output, counter-based
 * (seed, ply, env); -1 when an env has no legal action. */
int jq_sample_uniform(int32_t n, const int32_t *d_counts, const int32_t *d_ids, int32_t cap,
                      uint64_t seed, uint64_t ply, int32_t *d_actions, void *stream);

/* Masked-softmax sample over seeded N(0,1) logits on the compact canonical
 * action space (Gumbel-max over the legal set).  Writes the compact
 * canonical action (or -1) and its world id. */
int jq_sample_softmax(const jq_batch *b, const int32_t *d_counts, const int32_t *d_ids,
                      int32_t cap, uint64_t seed, uint64_t ply, int32_t *d_compact_actions,
                      int32_t *d_world_actions, void *stream);

/* Per-CTA timestamps of the last obs_kernel (kernel 0) or rules_kernel
 * (kernel 1) launch: `ctas` rows of 8 uint64 (globaltimer ns at fixed points
 * of the kernel; see junqi_b200/csrc/jq_trace.cuh), copied to host memory.
 * Available only in the tracing build of the library (libjq_trace.so, `make
 * trace`); the normal build returns JQ_ERR_NOT_READY.  A profiling aid with no
 * counterpart in the reference. */
int jq_trace_read(int32_t kernel, uint64_t *host, int32_t ctas);

#ifdef __cplusplus
}
#endif
#endif
