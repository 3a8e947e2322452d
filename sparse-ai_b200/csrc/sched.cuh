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
  int first_static;         // 1: each CTA's first entry is item blockIdx.x (not in the queue),
                            // taken before waiting for the planner (a PDL prerequisite)
};

__device__ __forceinline__ WorkEntry no_work() { return WorkEntry{-1, 0, 0, -1}; }

// Producer side: yields this CTA's entries in order.  An entry is reserved (dynamic mode:
// atomic on the queue counter, then the queue load) only when the producer issues the last
// tile of the current entry -- late enough that a CTA never sits on queued work while other
// CTAs go idle, early enough (the producer runs a few stages ahead of the MMA) to hide the
// fetch latency.  `weight(i)` gives an item's sub-tile count in the static round-robin mode.
struct WorkFetcher {
  const SchedArgs* s;
  WorkEntry e_next;
  uint32_t w;
  bool reserved;
  bool waited;

  template <typename WeightFn>
  __device__ __forceinline__ void reserve(WeightFn&& weight) {
    if (reserved) return;
    reserved = true;
    if (s->header && s->first_static && w == 0) {
      // first wave: item = CTA index, while the planner (this grid's programmatic
      // prerequisite) still orders the rest
      e_next = (int64_t)blockIdx.x < s->items ? WorkEntry{(int)blockIdx.x, 0, weight(blockIdx.x), -1}
                                              : no_work();
    } else if (s->header) {
      if (s->first_static && !waited) {
        pdl_wait();  // the planner's queue and header are complete from here on
        waited = true;
      }
      const int idx = atomicAdd(&s->header->counter, 1);
      if (idx >= s->header->n_entries) {
        e_next = no_work();
      } else if (s->header->natural) {  // the planner found the index order heaviest-first
        const int64_t item = (s->first_static ? (int64_t)gridDim.x : 0) + idx;
        e_next = WorkEntry{(int)item, 0, weight(item), -1};
      } else {
        e_next = s->queue[idx];
      }
    } else {
      const int64_t idx = (int64_t)blockIdx.x + (int64_t)w * gridDim.x;
      e_next = idx < s->items ? WorkEntry{(int)idx, 0, weight(idx), -1} : no_work();
    }
  }

  template <typename WeightFn>
  __device__ __forceinline__ void init(const SchedArgs* args, WeightFn&& weight) {
    s = args;
    w = 0;
    reserved = false;
    waited = false;
    reserve(weight);
  }

  // The reserved entry; the caller reserves the following one with reserve().
  template <typename WeightFn>
  __device__ __forceinline__ WorkEntry next(WeightFn&& weight) {
    reserve(weight);
    reserved = false;
    ++w;
    return e_next;
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

// ring_get for a whole warp (every lane reads the entry); the result is warp-uniform.
__device__ __forceinline__ bool ring_get_warp(const WorkEntry* ring, uint64_t* full, uint64_t* empty,
                                              uint32_t w, WorkEntry& e, unsigned* st) {
  const uint32_t s = w % kRing, ph = (w / kRing) & 1;
  if (!mbar_wait_warp(&full[s], ph, st)) return false;
  e = ring[s];
  mbar_arrive(&empty[s]);
  return true;
}

}  // namespace sa
