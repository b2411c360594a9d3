// jq_trace.cuh -- optional per-CTA timestamps of the hot kernels.
//
// Built only into the tracing variant of the library (`make trace`, which
// defines JQ_TRACE and writes libjq_trace.so); in the normal build every
// JQ_TRACE_AT is empty and the kernels are unchanged.  With tracing, one
// thread per CTA stores the %globaltimer value (ns) of a few points of the
// kernel into g_trace[kernel][cta][point]; jq_trace_read copies the table of
// the last launch of each kernel to the host (junqi_b200/trace.py turns it
// into a timeline).
#pragma once
#include <stdint.h>

namespace jq {

constexpr int TRACE_KERNELS = 2;   // 0: obs_kernel, 1: rules_kernel
constexpr int TRACE_CTAS = 1024;   // CTAs recorded per launch (grid beyond this is not traced)
constexpr int TRACE_POINTS = 20;

// obs_kernel points
enum : int { TO_ENTRY = 0, TO_WAITED = 1, TO_FIRST_STAGED = 2, TO_FIRST_STREAM = 3, TO_LAST_STREAMED = 4,
             TO_EXIT = 5, TO_UNITS = 6, TO_LAST_TICKET = 7, TO_LAST_STAGED = 8,
             // the CTA's units 0..2: streaming warp 0 passed the staged-buffer barrier (9 + 2k) and
             // finished streaming (10 + 2k); staging finished (15 + k); staging of units 2, 3 began
             // after the free-buffer barrier (18, 19)
             TO_UNIT_STREAM0 = 9, TO_UNIT_STAGED0 = 15, TO_UNIT_STAGE_START2 = 18 };
// rules_kernel points (the phases of warp 0's first env, then the CTA's exit)
enum : int { TR_ENTRY = 0, TR_WAITED = 1, TR_LOADED = 2, TR_STEPPED = 3, TR_RESET = 4, TR_IDS = 5, TR_MASKED = 6,
             TR_EXIT = 7,
             // inside the step of the same env
             TR_SCALAR = 8, TR_COMBAT = 9, TR_Q12 = 10, TR_COMMIT = 11,
             // counts: the env's event (0: no step), Q12 full destination scans
             TR_EVENT = 12, TR_Q12_SCANS = 13,
             // inside legal generation: destination sets done, ranking and scan done
             TR_DSTS = 14, TR_RANKED = 15,
             // inside the step: the engineer path check done, its rounds (0: not run), the moving piece's type
             TR_PATH = 16, TR_PATH_ROUNDS = 17, TR_ATYPE = 18,
             // the legal set's shape: engineers, their largest destination count, any piece's largest, total
             TR_LEGAL_SHAPE = 19 };

#ifdef JQ_TRACE
__device__ uint64_t g_trace[TRACE_KERNELS][TRACE_CTAS][TRACE_POINTS];
__device__ __forceinline__ uint64_t trace_clock() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define JQ_TRACE_AT(kernel, point)                                                          \
    do {                                                                                    \
        if (blockIdx.x < TRACE_CTAS) g_trace[kernel][blockIdx.x][point] = trace_clock();     \
    } while (0)
#define JQ_TRACE_COUNT(kernel, point, value)                                                \
    do {                                                                                    \
        if (blockIdx.x < TRACE_CTAS) g_trace[kernel][blockIdx.x][point] = (uint64_t)(value); \
    } while (0)
#else
#define JQ_TRACE_AT(kernel, point) \
    do {                           \
    } while (0)
#define JQ_TRACE_COUNT(kernel, point, value) \
    do {                                     \
    } while (0)
#endif

}  // namespace jq
