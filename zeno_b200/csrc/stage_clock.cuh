// Stage profile of a step kernel (profiling worlds only).  The block's first thread
// accumulates clock64 deltas per stage (zb::Stage) in shared memory; with C = false every
// call compiles to nothing.  At the end of the block that thread adds its sums, spans and
// maxima into StepArgs::stage_clk (layout in zeno_types.h).
#pragma once
#include "zeno_types.h"

namespace zb {

template <bool C>
struct StageClock {
  __device__ __forceinline__ void start(unsigned long long*, bool) {}
  __device__ __forceinline__ void mark(uint32_t) {}
  __device__ __forceinline__ void publish(unsigned long long*) {}
};

template <>
struct StageClock<true> {
  unsigned long long* acc = nullptr;  // shared, kStageCount entries
  long long first = 0, last = 0, ns0 = 0;
  bool on = false;  // the block's first thread
  // acc: the block's shared accumulator (zeroed here by the first kStageCount threads;
  // the caller synchronises the block before the first mark)
  __device__ __forceinline__ void start(unsigned long long* s_acc, bool first_thread) {
    acc = s_acc;
    on = first_thread;
    if (threadIdx.x < kStageCount) acc[threadIdx.x] = 0;
    last = first = clock64();
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ns0));
  }
  __device__ __forceinline__ void mark(uint32_t k) {
    if (on) {
      const long long t = clock64();
      acc[k] += static_cast<unsigned long long>(t - last);
      last = t;
    }
  }
  // by the first thread, after its last mark
  __device__ __forceinline__ void publish(unsigned long long* out) {
    if (!on) return;
    long long ns1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ns1));
    for (uint32_t k = 0; k < kStageCount; ++k) {
      atomicAdd(out + k, acc[k]);
      atomicMax(out + kStageMax + k, acc[k]);
    }
    const auto span = static_cast<unsigned long long>(last - first);
    const auto span_ns = static_cast<unsigned long long>(ns1 - ns0);
    atomicAdd(out + kStageCount, span);
    atomicAdd(out + kStageCount + 1, span_ns);
    atomicAdd(out + kStageCount + 2, 1ull);
    atomicMax(out + kStageCount + 3, span);
    atomicMax(out + kStageCount + 4, span_ns);
  }
};

}  // namespace zb
