// vbsr_dev_instrument.cuh — development instrumentation of spmm_tc_kernel, compiled out of the
// product build. Two switches, both off unless given on the nvcc command line (VBSR_EXTRA_FLAGS of
// build.py):
//   -DVBSR_PROF        per-CTA cycle counters by role (feeder wait, split, MMA issue, epilogue ...),
//                      16 per CTA, accumulated into KernelParams::prof (vbsr_plan_cta_timing reads
//                      them back after the 2 * tasks start/end timestamps). Entry points that keep
//                      no counter buffer pass prof = nullptr and nothing is written.
//   -DVBSR_TRACE=<cta> per-stage and per-item clock64() timestamps of one CTA into g_trace /
//                      g_trace_items (vbsr_debug_trace copies them out).
#pragma once

#ifdef VBSR_PROF
#define VBSR_PROF_T0(v) const long long v = clock64()
#define VBSR_PROF_ADD(p, slot, t0)                                                          \
  do {                                                                                     \
    if ((p).prof && (threadIdx.x & 31) == 0)                                               \
      atomicAdd((p).prof + 16 * blockIdx.x + (slot),                                       \
                (unsigned long long)(clock64() - (t0)));                                   \
  } while (0)
#else
#define VBSR_PROF_T0(v)
#define VBSR_PROF_ADD(p, slot, t0) do { } while (0)
#endif

#ifdef VBSR_TRACE
__device__ long long g_trace[4096 * 8];
__device__ long long g_trace_items[1024 * 4];
#define VBSR_TRACE_ST(k, e)                                                                      \
  do {                                                                                           \
    if (blockIdx.x == VBSR_TRACE && (threadIdx.x & 31) == 0 && (k) < 4096)                       \
      g_trace[(k) * 8 + (e)] = clock64();                                                        \
  } while (0)
#define VBSR_TRACE_IT(j, e)                                                                      \
  do {                                                                                           \
    if (blockIdx.x == VBSR_TRACE && (threadIdx.x & 31) == 0 && (j) < 1024)                       \
      g_trace_items[(j) * 4 + (e)] = clock64();                                                  \
  } while (0)
#else
#define VBSR_TRACE_ST(k, e) do { } while (0)
#define VBSR_TRACE_IT(j, e) do { } while (0)
#endif
