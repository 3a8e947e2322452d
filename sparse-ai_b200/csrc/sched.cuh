// Work distribution inside the persistent tcgen05 kernels.
//
// The producer warp's elected thread fetches work entries -- from the planner's queue with an
// atomic counter (dynamic, heaviest first), or round-robin over the items when no planner
// workspace was given -- and hands each one to the MMA thread and the elementwise warps
// through a small ring in shared memory guarded by mbarriers (FULL: count 1, EMPTY: one
// arrival per consumer thread).  A WorkEntry with item < 0 ends every role's loop.
#pragma once

#include "attn_plan.cuh"

namespace sa {

constexpr int kRing = 4;

struct SchedArgs {
  PlanHeader* header;       // null: static round-robin over `items`
  const WorkEntry* queue;
  int64_t items;
};

__device__ __forceinline__ WorkEntry no_work() { return WorkEntry{-1, 0, 0, -1}; }

// Producer side: the next entry for this CTA.  `weight(i)` gives an item's sub-tile count
// in the static mode.
template <typename WeightFn>
__device__ __forceinline__ WorkEntry sched_fetch(const SchedArgs& s, int n_entries, uint32_t w,
                                                 WeightFn&& weight) {
  if (s.header) {
    const int idx = atomicAdd(&s.header->counter, 1);
    return idx < n_entries ? s.queue[idx] : no_work();
  }
  const int64_t idx = (int64_t)blockIdx.x + (int64_t)w * gridDim.x;
  return idx < s.items ? WorkEntry{(int)idx, 0, weight(idx), -1} : no_work();
}

__device__ __forceinline__ bool ring_put(WorkEntry* ring, uint64_t* full, uint64_t* empty,
                                         uint32_t w, const WorkEntry& e, unsigned* st) {
  const uint32_t s = w % kRing, ph = (w / kRing) & 1;
  if (!mbar_wait(&empty[s], ph ^ 1, st)) return false;
  ring[s] = e;
  mbar_arrive(&full[s]);
  return true;
}

__device__ __forceinline__ bool ring_get(const WorkEntry* ring, uint64_t* full, uint64_t* empty,
                                         uint32_t w, WorkEntry& e, unsigned* st) {
  const uint32_t s = w % kRing, ph = (w / kRing) & 1;
  if (!mbar_wait(&full[s], ph, st)) return false;
  e = ring[s];
  mbar_arrive(&empty[s]);
  return true;
}

}  // namespace sa
