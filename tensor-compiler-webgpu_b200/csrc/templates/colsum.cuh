// tcb/colsum.cuh -- an elementwise body fused with the sum over axis 0 of its result.
//
// The reference's fusion pass leaves a column reduction (a bias gradient: sum over axis 0) as a plain
// launch that reads back the tensor its producer just wrote (src/fusion/fuse.js:43-45).  Here the
// producer's elementwise body and the column partial sums run in one pass over [R, C]: each thread owns
// W consecutive columns and walks its chunk of rows, computing the body, writing it when the value is
// needed elsewhere (TCB_WRITE), and adding it into W running column sums.
//
// The generated part defines, before including this file, struct Body (the elementwise template's
// load plan and compute, tcb/elementwise.cuh) and
//   TCB_W      columns per thread (4: 128-bit loads and stores; 1 when C is not a multiple of 4)
//   TCB_WRITE  1: also store the body's value to a.out
//   TCB_OUTER 1, TCB_N (= R), TCB_INNER (= C), TCB_SPLIT, TCB_IS_MAX 0 -- the plain column sum's
//              geometry (tcb/reduce.cuh), whose tcb_reduce_finish combines the partials.
// Chunk s of the rows is summed first to last into partial s, exactly as tcb_reduce_cols sums the
// materialised tensor, so the result is bitwise that of the unfused pair of launches.  Partials go to
// a.scratch ([SPLIT, C] floats) when TCB_SPLIT > 1, else straight to the sum's output: p[14] when the
// body's value is written to a.out, a.out otherwise.
#pragma once

#include "tcb/reduce.cuh"

extern "C" __global__ void __launch_bounds__(256) tcb_ew_colsum(const tcb::Args a) {
  tcb::grid_dependency_sync();
  constexpr int W = TCB_W;
  constexpr u64 R = (u64)TCB_N, C = (u64)TCB_INNER, groups = C / W;
  constexpr u64 chunk = (R + TCB_SPLIT - 1) / TCB_SPLIT;
  const u64 s = blockIdx.y;
  const u64 k0 = s * chunk;
  const u64 k1 = k0 + chunk < R ? k0 + chunk : R;
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
  float* __restrict__ dst = TCB_SPLIT > 1 ? reinterpret_cast<float*>(a.scratch)
                                          : (TCB_WRITE ? reinterpret_cast<float*>(a.p[14]) : out);
  for (u64 g = (u64)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += (u64)gridDim.x * blockDim.x) {
    float acc[W];
#pragma unroll
    for (int l = 0; l < W; ++l) acc[l] = 0.0f;
    u64 k = k0;
    for (; k + 4 <= k1; k += 4) {  // four rows' loads in flight, then computed and summed in row order
      typename Body::template Regs<W> r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) Body::template load<W>(a, (k + u) * C + g * W, r[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float o[W];
        Body::template compute<W>(r[u], o);
        if constexpr (TCB_WRITE) tcb::store<W>(out + (k + u) * C + g * W, o);
#pragma unroll
        for (int l = 0; l < W; ++l) acc[l] = tcb::op_add(acc[l], o[l]);
      }
    }
    for (; k < k1; ++k) {
      typename Body::template Regs<W> r;
      Body::template load<W>(a, k * C + g * W, r);
      float o[W];
      Body::template compute<W>(r, o);
      if constexpr (TCB_WRITE) tcb::store<W>(out + k * C + g * W, o);
#pragma unroll
      for (int l = 0; l < W; ++l) acc[l] = tcb::op_add(acc[l], o[l]);
    }
#pragma unroll
    for (int l = 0; l < W; ++l) dst[s * C + g * W + l] = acc[l];
  }
}
