// tcb/elementwise.cuh -- fused elementwise template (class 1 of the fusion
// pass; the reference's WGSL form is src/fusion/codegen-fused.js:154-172).
//
// The generated part defines, before including this file:
//   TCB_W        lanes per thread step (4: 128-bit loads and stores; 1 otherwise)
//   TCB_UNROLL   independent steps whose loads are all issued before any compute
//   struct Body { struct Regs; template<int W> static void load(const tcb::Args&, u64 i0, Regs&);
//                 template<int W> static void compute(const Regs&, float (&o)[W]); }
//   (Regs is a template over W: Body::Regs<W>.)
// p[0] = element count.  Grid-stride over W-wide chunks, a scalar tail.
#pragma once

#ifndef TCB_UNROLL
#define TCB_UNROLL 2
#endif

namespace tcb {
__device__ __forceinline__ void elementwise_run(const tcb::Args& a) {
  const u64 n = (u64)a.p[0];
  constexpr int W = TCB_W;
  constexpr int U = TCB_UNROLL;
  const u64 chunks = n / W;
  const u64 t = (u64)blockIdx.x * blockDim.x + threadIdx.x;
  const u64 stride = (u64)gridDim.x * blockDim.x;
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
  u64 c = t;
  for (; c + (U - 1) * stride < chunks; c += U * stride) {
    typename Body::template Regs<W> r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) Body::template load<W>(a, (c + u * stride) * W, r[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float o[W];
      Body::template compute<W>(r[u], o);
      tcb::store<W>(out + (c + u * stride) * W, o);
    }
  }
  for (; c < chunks; c += stride) {
    typename Body::template Regs<W> r;
    Body::template load<W>(a, c * W, r);
    float o[W];
    Body::template compute<W>(r, o);
    tcb::store<W>(out + c * W, o);
  }
  if constexpr (W > 1) {
    for (u64 i = chunks * W + t; i < n; i += stride) {
      typename Body::template Regs<1> r;
      Body::template load<1>(a, i, r);
      float o[1];
      Body::template compute<1>(r, o);
      out[i] = o[0];
    }
  }
}
}  // namespace tcb

extern "C" __global__ void __launch_bounds__(256) tcb_elementwise(const tcb::Args a) { tcb::grid_dependency_sync(); tcb::elementwise_run(a); }

// Several launches of this same body over different buffers in one launch (a resident program batches
// small independent ones): a.scratch holds a device table of argument blocks, blockIdx.y picks one.
extern "C" __global__ void __launch_bounds__(256) tcb_elementwise_multi(const tcb::Args a) {
  tcb::grid_dependency_sync();
  tcb::elementwise_run(reinterpret_cast<const tcb::Args*>(a.scratch)[blockIdx.y]);
}
