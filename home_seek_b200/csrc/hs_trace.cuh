// Phase timeline of the token-mode layer call (tracing builds only).
//
// Compiled with -DHS_TRACE (python -m home_seek_b200.build --trace, which
// writes libhs_ext_trace.so), the layer call's kernels store %globaltimer at
// their phase boundaries into a device array: [slot][kernel][CTA][event] u64,
// slot = (layer call) % kSlots. The route kernel's CTA 0 advances the call
// counter at its end; the later kernels of the call read it back, so their
// stamps land in the same slot. home_seek_b200/trace.py reads the array and
// prints each phase's time after the route kernel's start. Without HS_TRACE
// every macro below expands to nothing.
#pragma once

#include "hs_common.cuh"

namespace hs {
namespace trace {
constexpr int kSlots = 32;
constexpr int kKernels = 5;  // route, gate/up, down, gate/up tail events, expert-parallel combine
constexpr int kCtas = 296;
constexpr int kEvents = 8;
// kGateUpTail (gate/up CTAs): 0 last ticket wait over, 1 last accumulator
// ready, 2 epilogue done, 3 MMA warp done, 4 last copy issued, 5 the number of
// epilogue segments (a count, not a time), 6 partial rows stored, 7 ticket
// wait begins; kCombine event 6 (gate/up CTAs): the producer warp added the
// published segment's ticket
enum Kernel { kRoute = 0, kGateUp = 1, kDown = 2, kGateUpTail = 3, kCombine = 4 };
}  // namespace trace
}  // namespace hs

#ifdef HS_TRACE
namespace hs {
namespace trace {
// one translation unit (hs_moe.cu) includes this header
static __device__ unsigned long long g_stamp[kSlots * kKernels * kCtas * kEvents];
static __device__ unsigned int g_calls;
HS_DI unsigned int calls_now() { return *reinterpret_cast<volatile unsigned int*>(&g_calls); }
HS_DI void stamp(unsigned int slot, int k, int c, int e, unsigned long long t) {
  if (c < kCtas) g_stamp[((static_cast<int>(slot % kSlots) * kKernels + k) * kCtas + c) * kEvents + e] = t;
}
}  // namespace trace
}  // namespace hs
// the slot of the running call: the route kernel before it advances the
// counter (HS_TRACE_SLOT_ROUTE), every later kernel of the call after
#define HS_TRACE_SLOT_ROUTE(var) const unsigned int var = ::hs::trace::calls_now()
#define HS_TRACE_SLOT(var) const unsigned int var = ::hs::trace::calls_now() - 1u
#define HS_TRACE_T(var) const unsigned long long var = ::hs::globaltimer_ns()
#define HS_TRACE_VAR(var) unsigned long long var = 0ull
#define HS_TRACE_SET(var) (var = ::hs::globaltimer_ns())
#define HS_STAMP(slot, k, c, e) ::hs::trace::stamp((slot), (k), (c), (e), ::hs::globaltimer_ns())
#define HS_STAMP_AT(slot, k, c, e, t) ::hs::trace::stamp((slot), (k), (c), (e), (t))
#define HS_TRACE_NEXT_CALL() \
  do {                       \
    __threadfence();         \
    atomicAdd(&::hs::trace::g_calls, 1u); \
  } while (0)
#else
#define HS_TRACE_SLOT_ROUTE(var)
#define HS_TRACE_SLOT(var)
#define HS_TRACE_T(var)
#define HS_TRACE_VAR(var)
#define HS_TRACE_SET(var) ((void)0)
#define HS_STAMP(slot, k, c, e) ((void)0)
#define HS_STAMP_AT(slot, k, c, e, t) ((void)0)
#define HS_TRACE_NEXT_CALL() ((void)0)
#endif
