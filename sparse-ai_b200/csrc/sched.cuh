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

// Producer side: yields this CTA's entries in order.  Dynamic mode keeps the queue walk two
// entries ahead -- the atomic for entry w+2 and the queue load for entry w+1 are in flight
// while entry w is being produced -- so the fetch latency stays off the critical path.
// `weight(i)` gives an item's sub-tile count in the static round-robin mode.
struct WorkFetcher {
  const SchedArgs* s;
  int n_entries;
  int idx_next;      // queue index of the entry after `e_next`
  WorkEntry e_next;  // the entry next() returns
  uint32_t w;

  __device__ __forceinline__ WorkEntry load(int idx) const {
    return idx < n_entries ? s->queue[idx] : no_work();
  }

  template <typename WeightFn>
  __device__ __forceinline__ WorkEntry statik(uint32_t k, WeightFn&& weight) const {
    const int64_t idx = (int64_t)blockIdx.x + (int64_t)k * gridDim.x;
    return idx < s->items ? WorkEntry{(int)idx, 0, weight(idx), -1} : no_work();
  }

  template <typename WeightFn>
  __device__ __forceinline__ void init(const SchedArgs* args, WeightFn&& weight) {
    s = args;
    w = 0;
    if (s->header) {
      n_entries = s->header->n_entries;
      const int i0 = atomicAdd(&s->header->counter, 1);
      idx_next = atomicAdd(&s->header->counter, 1);
      e_next = load(i0);
    } else {
      n_entries = 0;
      idx_next = 0;
      e_next = statik(0, weight);
    }
  }

  template <typename WeightFn>
  __device__ __forceinline__ WorkEntry next(WeightFn&& weight) {
    const WorkEntry e = e_next;
    ++w;
    if (e.item >= 0) {
      if (s->header) {
        e_next = load(idx_next);  // consumed at the next call
        idx_next = atomicAdd(&s->header->counter, 1);
      } else {
        e_next = statik(w, weight);
      }
    }
    return e;
  }
};

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
