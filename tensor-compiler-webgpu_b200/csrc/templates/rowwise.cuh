// tcb/rowwise.cuh -- helpers of the fused rowwise template (class 3 of the
// fusion pass; the reference's WGSL form is src/fusion/codegen-fused.js:271-354).
//
// A row of C elements belongs to a group of TPR threads (a warp, or TPR/32
// warps); a CTA holds GROUPS such groups.  The generated kernel loads each
// element-tier operand of its row ONCE into registers (one HBM pass over the
// row), then runs every reduction phase (max, sum, ...) over those registers
// with warp shuffles plus one shared-memory exchange between the group's
// warps, and writes the row.  Every thread of the CTA reaches every barrier,
// including threads whose row is past the end (they load nothing and store
// nothing).
#pragma once

namespace tcb {

// Reduce v over the TPR threads of this thread's group; every thread of the
// group gets the result.  `red` holds GROUPS * (TPR / 32) floats.  Combining
// order is fixed (lanes by xor tree, warps 0..NW-1 in order), so the result
// is deterministic.
template <int TPR, int GROUPS, bool IS_MAX>
__device__ __forceinline__ float group_reduce(float v, float* red) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  if constexpr (TPR <= 32) {
    return v;
  } else {
    constexpr int NW = TPR / 32;
    const int g = threadIdx.x / TPR;
    const int w = (threadIdx.x % TPR) >> 5;
    if ((threadIdx.x & 31) == 0) red[g * NW + w] = v;
    __syncthreads();
    float r = red[g * NW];
#pragma unroll
    for (int k = 1; k < NW; ++k) r = IS_MAX ? op_max(r, red[g * NW + k]) : op_add(r, red[g * NW + k]);
    __syncthreads();
    return r;
  }
}

}  // namespace tcb
