// Work planning for the persistent tcgen05 attention kernels.
//
// A work item is a (query tile, z, h) for the forward and dQ kernels, a (key tile, z, KV head)
// for the dK/dV kernel.  Item weights (tiles of MMA work) vary by orders of magnitude with the
// lists (the sink column of a causal+sink layout is listed by every query block), so a static
// round-robin over items leaves most SMs idle while a few finish the heavy items.  The planner
// (one CTA) computes every item's weight, optionally splits heavy dK/dV items into chunks, and
// writes a queue of entries ordered heaviest-first; the kernels' producer warps pop entries
// with an atomic counter.  Split dK/dV chunks write fp32 partial tiles into their own slots and
// a reduce kernel sums them in chunk order (deterministic).
#pragma once

#include "attn_params.cuh"

namespace sa {

enum PlanKind : int { kPlanFwd = 0, kPlanDq = 1, kPlanDkdv = 2 };

struct WorkEntry {
  int item;   // item index in the kernel's item space (-1 = no more work)
  int begin;  // first sub-tile of the item handled by this entry
  int end;    // one past the last sub-tile
  int slot;   // partial slot of a split dK/dV chunk, or -1 (write the result directly)
};

struct SplitItem {
  int item;
  int slot_base;
  int chunks;
  int pad;
};

struct PlanHeader {
  int counter;    // next entry to hand out (atomic)
  int n_entries;
  int n_split;
  int natural;    // 0: the queue holds the entries; 1 + w: no queue was written, entry k is
                  // item skip + k, and every such item weighs w
};

// Bytes of planner workspace for `items` items and `ctas` persistent CTAs.  Split chunks need
// at most 4 * ctas partial slots of 128 x (2 * D) floats.
int64_t plan_workspace_bytes(int kind, int64_t items, int ctas, int64_t D);

struct PlanPtrs {
  PlanHeader* header;
  WorkEntry* queue;
  SplitItem* splits;
  float* partials;
};

PlanPtrs plan_carve(void* ws, int kind, int64_t items, int ctas, int64_t D);

// Launch the planner for `kind` over the items of `p` (sizes and lists as in the kernels).
int launch_plan(int kind, const AttnParams& p, int64_t items, int ctas, const PlanPtrs& plan,
                cudaStream_t stream, int skip = 0);

// Sum the split dK/dV partials and store bf16/fp16 dK, dV rows of the split items.
int launch_dkdv_reduce(const AttnParams& p, const PlanPtrs& plan, int ctas, cudaStream_t stream);

}  // namespace sa
