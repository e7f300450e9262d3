// tcb/elementwise_mo.cuh -- an elementwise body with several outputs in one pass.
//
// The reference's fusion pass stores a value that more than one node reads and leaves each reader its
// own launch (src/fusion/fuse.js:54-169): the reader then loads the stored value back.  When a reader
// is itself elementwise over the same index space and its other operands already exist, the producer's
// launch computes it too, from the value still in registers, and stores both.  Each output is computed
// by the same operations as in its own launch, so the values are bitwise the separate launches'.
//
// The generated part defines, before including this file:
//   TCB_W      lanes per thread step (4: 128-bit loads and stores)
//   TCB_NOUT   outputs (2..4): output 0 at a.out, output k at the address in p[k]
//   struct Body { Regs<W>; load(a, i0, r); compute(r, float (&o)[TCB_NOUT][W]) }
// p[0] = element count.  Grid-stride over W-wide chunks, a scalar tail (tcb/elementwise.cuh's loop).
#pragma once

#ifndef TCB_UNROLL
#define TCB_UNROLL 2
#endif

extern "C" __global__ void __launch_bounds__(256) tcb_elementwise_mo(const tcb::Args a) {
  tcb::grid_dependency_sync();
  const u64 n = (u64)a.p[0];
  constexpr int W = TCB_W, U = TCB_UNROLL, NO = TCB_NOUT;
  float* outs[NO];
  outs[0] = reinterpret_cast<float*>(a.out);
#pragma unroll
  for (int k = 1; k < NO; ++k) outs[k] = reinterpret_cast<float*>(a.p[k]);
  const u64 chunks = n / W;
  const u64 t = (u64)blockIdx.x * blockDim.x + threadIdx.x;
  const u64 stride = (u64)gridDim.x * blockDim.x;
  u64 c = t;
  for (; c + (U - 1) * stride < chunks; c += U * stride) {
    typename Body::template Regs<W> r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) Body::template load<W>(a, (c + u * stride) * W, r[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float o[NO][W];
      Body::template compute<W>(r[u], o);
#pragma unroll
      for (int k = 0; k < NO; ++k) tcb::store<W>(outs[k] + (c + u * stride) * W, o[k]);
    }
  }
  for (; c < chunks; c += stride) {
    typename Body::template Regs<W> r;
    Body::template load<W>(a, c * W, r);
    float o[NO][W];
    Body::template compute<W>(r, o);
#pragma unroll
    for (int k = 0; k < NO; ++k) tcb::store<W>(outs[k] + c * W, o[k]);
  }
  if constexpr (W > 1) {
    for (u64 i = chunks * W + t; i < n; i += stride) {
      typename Body::template Regs<1> r;
      Body::template load<1>(a, i, r);
      float o[NO][1];
      Body::template compute<1>(r, o);
#pragma unroll
      for (int k = 0; k < NO; ++k) outs[k][i] = o[k][0];
    }
  }
}
