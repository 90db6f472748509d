// Optional per-CTA timeline of the grouped GEMM (compile with -DMOE_TRACE).
//
// Each CTA writes %globaltimer stamps into its own 64-slot row of a device
// array; `moe_trace_read` copies the rows of the last launch to the host.
// Without MOE_TRACE the hooks compile to nothing.
#pragma once

#ifdef MOE_TRACE
#include <cstdint>
namespace moe {
constexpr int kTraceSlots = 64;
constexpr int kTraceCtas = 160;
// defined here: only grouped_gemm.cu includes this header
__device__ unsigned long long g_trace[kTraceCtas * kTraceSlots];
// per k-block stamps of the CTA's first 32 k-blocks: [0, 32) the producer
// issued the loads, [32, 64) the MMA issuer (or a pair's relay) saw them land
__device__ unsigned long long g_trace_kb[kTraceCtas * kTraceSlots];
}  // namespace moe
#define MOE_TRACE_AT(slot)                                                                  \
  do {                                                                                      \
    if (blockIdx.x < moe::kTraceCtas && (slot) < moe::kTraceSlots)                          \
      moe::g_trace[blockIdx.x * moe::kTraceSlots + (slot)] = moe::global_timer_ns();       \
  } while (0)
// per-tile event `ev` (0..6) of the CTA's `i`-th tile (first 8 tiles only)
#define MOE_TRACE_TILE(i, ev)                      \
  do {                                             \
    if ((i) < 8) MOE_TRACE_AT(3 + (i) * 7 + (ev)); \
  } while (0)
#define MOE_TRACE_KB(j, ev)                                                                \
  do {                                                                                     \
    if (blockIdx.x < moe::kTraceCtas && (j) < 32)                                          \
      moe::g_trace_kb[blockIdx.x * moe::kTraceSlots + (ev) * 32 + (j)] =                  \
          moe::global_timer_ns();                                                          \
  } while (0)
#else
#define MOE_TRACE_AT(slot) \
  do {                     \
  } while (0)
#define MOE_TRACE_TILE(i, ev) \
  do {                        \
  } while (0)
#define MOE_TRACE_KB(j, ev) \
  do {                      \
  } while (0)
#endif
