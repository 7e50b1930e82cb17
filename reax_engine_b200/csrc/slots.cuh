// slots.cuh -- canonical slot assignment of one routing segment (shared by the permute kernels and the
// expert-parallel dispatch).
#pragma once

#include "common.cuh"

namespace reaxmoe {

// Executed by ONE warp for the segment of nt <= kSegTokens rows starting at row t0 of ids [*, k]. On entry
// run[g] holds the first slot of group g for this segment (group offset + the slots of g in earlier segments) and
// mask[g] == 0 for every group g < G. For a chunk of 32 rows (one per lane) each lane sets its bit in a per-group
// shared mask for each of its k groups; the slot of (row, j) is run[g] + popc(mask[g] & lanes_below), so slots are
// row-major inside a group and no data-dependent atomics order them. Ids outside [0, G) get slot -1 (negative ids
// mark unused pairs; the count kernel flags ids >= G). Writes the segment-local pos_s / grp_s [nt * k] and, when
// c_map is not null, the global c_map [rows, k]. run[] ends holding the end of each group's range.
__device__ __forceinline__ void segment_slots(const int* __restrict__ ids, int64_t t0, int nt, int k, int G,
                                              int* run, uint32_t* mask, int* pos_s, short* grp_s, int* c_map) {
  const int lane = threadIdx.x & 31;
  const uint32_t below = (1u << lane) - 1u;
  for (int c0 = 0; c0 < nt; c0 += 32) {
    const int tl = c0 + lane;
    const bool active = tl < nt;
    int ej[kMaxTopk];
#pragma unroll
    for (int j = 0; j < kMaxTopk; ++j) {
      ej[j] = -1;
      if (j < k && active) {
        const int e = ids[(t0 + tl) * k + j];
        if ((unsigned)e < (unsigned)G) {
          ej[j] = e;
          atomicOr(&mask[e], 1u << lane);
        }
      }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kMaxTopk; ++j) {
      if (j < k && active) {
        int pos = -1;
        if (ej[j] >= 0) pos = run[ej[j]] + __popc(mask[ej[j]] & below);
        pos_s[tl * k + j] = pos;
        grp_s[tl * k + j] = (short)ej[j];
        if (c_map != nullptr) c_map[(t0 + tl) * k + j] = pos;
      }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kMaxTopk; ++j) {
      if (j < k && ej[j] >= 0) {
        const uint32_t mk = mask[ej[j]];
        if ((mk & below) == 0u) run[ej[j]] += __popc(mk);
      }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kMaxTopk; ++j)
      if (j < k && ej[j] >= 0) mask[ej[j]] = 0u;
    __syncwarp();
  }
}

}  // namespace reaxmoe
