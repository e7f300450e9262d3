// tcb/rowsum.cuh -- an elementwise body fused with the sum over the last axis of its result.
//
// The reference's fusion pass leaves a sum over the last axis whose operand has other readers (the
// layer-norm and attention backward: sum(dy * g), sum(dy * g * xhat)) as a plain launch that reads back
// the tensor its producer just wrote (src/fusion/fuse.js:43-45 fuses only the rowwise patterns).  Here
// the producer's elementwise body and the row sums run in one pass: a warp per row, each lane computing
// the body for 4 consecutive values at a time (1 when the row length is not a multiple of 4), writing
// them when the value is needed elsewhere (TCB_WRITE), and adding them into its running sum in the
// order tcb_reduce_rows adds the stored values, then the same shuffle tree -- so the sums are bitwise
// those of the unfused pair of launches.
//
// The generated part defines, before including this file, struct Body (the elementwise template's load
// plan and compute, tcb/elementwise.cuh), TCB_WRITE, and the plain row sum's geometry (tcb/reduce.cuh):
// TCB_OUTER (rows), TCB_N (row length), TCB_INNER 1, TCB_SPLIT 1, TCB_IS_MAX 0.  The sums go to p[14]
// when the body's value is written to a.out, else to a.out.
#pragma once

#include "tcb/reduce.cuh"

extern "C" __global__ void __launch_bounds__(256) tcb_ew_rowsum(const tcb::Args a) {
  tcb::grid_dependency_sync();
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
  float* __restrict__ sums = TCB_WRITE ? reinterpret_cast<float*>(a.p[14]) : out;
  const u64 warp = ((u64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const u64 warps = ((u64)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int W = TCB_N % 4 == 0 ? 4 : 1;
  for (u64 o = warp; o < (u64)TCB_OUTER; o += warps) {
    const u64 row = o * (u64)TCB_N;
    float acc = tcb::red_init();
    for (u64 k = lane; k < (u64)TCB_N / W; k += 32) {
      typename Body::template Regs<W> r;
      Body::template load<W>(a, row + k * W, r);
      float v[W];
      Body::template compute<W>(r, v);
      if constexpr (TCB_WRITE) tcb::store<W>(out + row + k * W, v);
#pragma unroll
      for (int l = 0; l < W; ++l) acc = tcb::red_comb(acc, v[l]);
    }
    acc = tcb::warp_sum(acc);
    if (lane == 0) sums[o] = acc;
  }
}
