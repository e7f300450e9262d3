// tcb/reduce.cuh -- the unfused sum/max along one axis (the reference's WGSL
// form is src/gpu/codegen.js:92-116: one thread per output, serial over n).
//
// The input is viewed as [outer, n, inner].  The generated part defines
// TCB_OUTER, TCB_N, TCB_INNER, TCB_SPLIT (chunks of n), TCB_IS_MAX and then
// includes this file.
//  - inner == 1 (last axis): tcb_reduce_rows, a warp per output, coalesced
//    loads along the row, shuffle tree.
//  - inner > 1: tcb_reduce_cols, a thread per output column (coalesced across
//    the warp), serial over its chunk of n.  With TCB_SPLIT > 1 each chunk
//    writes a partial to scratch ([SPLIT, outer*inner] floats) and
//    tcb_reduce_finish combines the partials in chunk order.
#pragma once

namespace tcb {
__device__ __forceinline__ float red_init() { return TCB_IS_MAX ? -__int_as_float(0x7f800000) : 0.0f; }
__device__ __forceinline__ float red_comb(float acc, float v) { return TCB_IS_MAX ? op_max(acc, v) : op_add(acc, v); }
}  // namespace tcb

extern "C" __global__ void __launch_bounds__(256) tcb_reduce_rows(const tcb::Args a) {
  tcb::grid_dependency_sync();
  const float* __restrict__ x = reinterpret_cast<const float*>(a.in[0]);
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
  const u64 warp = ((u64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const u64 warps = ((u64)gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  if constexpr ((u64)TCB_OUTER <= 8 && TCB_N >= 1024) {
    // at most 8 long rows (a loss summed over every token): the launch is one CTA, and its 8 warps share
    // each row -- thread t takes 4 consecutive values (1 when the row length is not a multiple of 4)
    // every 256, its warp sums, then warp 0 combines the 8 warp sums in warp order
    __shared__ float part[8];
    constexpr int W = TCB_N % 4 == 0 ? 4 : 1;
    for (u64 o = 0; o < (u64)TCB_OUTER; ++o) {
      const float* row = x + o * (u64)TCB_N;
      float acc = tcb::red_init();
      for (u64 k = threadIdx.x; k < (u64)TCB_N / W; k += blockDim.x) {
        if constexpr (W == 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(row) + k);
          acc = tcb::red_comb(acc, v.x); acc = tcb::red_comb(acc, v.y);
          acc = tcb::red_comb(acc, v.z); acc = tcb::red_comb(acc, v.w);
        } else {
          acc = tcb::red_comb(acc, __ldg(row + k));
        }
      }
      acc = TCB_IS_MAX ? tcb::warp_max(acc) : tcb::warp_sum(acc);
      if (lane == 0) part[threadIdx.x >> 5] = acc;
      __syncthreads();
      if (threadIdx.x == 0) {
        float s = part[0];
        for (unsigned w = 1; w < blockDim.x / 32; ++w) s = tcb::red_comb(s, part[w]);
        out[o] = s;
      }
      __syncthreads();
    }
    return;
  }
  for (u64 o = warp; o < (u64)TCB_OUTER; o += warps) {
    const float* row = x + o * (u64)TCB_N;
    float acc = tcb::red_init();
    if constexpr (TCB_N % 4 == 0) {
      // rows of a multiple of 4 floats start 16-byte aligned: 128-bit loads, 4 consecutive values per lane
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (u64 k = lane; k < (u64)TCB_N / 4; k += 32) {
        const float4 v = __ldg(r4 + k);
        acc = tcb::red_comb(acc, v.x); acc = tcb::red_comb(acc, v.y);
        acc = tcb::red_comb(acc, v.z); acc = tcb::red_comb(acc, v.w);
      }
    } else {
      for (u64 k = lane; k < (u64)TCB_N; k += 32) acc = tcb::red_comb(acc, __ldg(row + k));
    }
    acc = TCB_IS_MAX ? tcb::warp_max(acc) : tcb::warp_sum(acc);
    if (lane == 0) out[o] = acc;
  }
}

extern "C" __global__ void __launch_bounds__(256) tcb_reduce_cols(const tcb::Args a) {
  tcb::grid_dependency_sync();
  const float* __restrict__ x = reinterpret_cast<const float*>(a.in[0]);
  float* __restrict__ dst = TCB_SPLIT > 1 ? reinterpret_cast<float*>(a.scratch) : reinterpret_cast<float*>(a.out);
  constexpr u64 outs = (u64)TCB_OUTER * (u64)TCB_INNER;
  constexpr u64 chunk = ((u64)TCB_N + TCB_SPLIT - 1) / TCB_SPLIT;
  const u64 s = blockIdx.y;
  const u64 k0 = s * chunk;
  const u64 k1 = k0 + chunk < (u64)TCB_N ? k0 + chunk : (u64)TCB_N;
  for (u64 i = (u64)blockIdx.x * blockDim.x + threadIdx.x; i < outs; i += (u64)gridDim.x * blockDim.x) {
    const u64 o = i / (u64)TCB_INNER, j = i % (u64)TCB_INNER;
    const float* p = x + (o * (u64)TCB_N) * (u64)TCB_INNER + j;
    float acc = tcb::red_init();
    u64 k = k0;
    for (; k + 8 <= k1; k += 8) {  // eight independent loads in flight, combined in row order
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(p + (k + u) * (u64)TCB_INNER);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = tcb::red_comb(acc, v[u]);
    }
    for (; k < k1; ++k) acc = tcb::red_comb(acc, __ldg(p + k * (u64)TCB_INNER));
    dst[s * outs + i] = acc;
  }
}

// Combines the partials: a block takes 32 consecutive outputs (one per lane, so every load is a
// coalesced 128-byte row); its 8 warps take the chunks s = w, w + 8, ... in order, and the 8 warp
// results are combined in warp order -- a fixed order for every output, whatever the launch.
extern "C" __global__ void __launch_bounds__(256) tcb_reduce_finish(const tcb::Args a) {
  tcb::grid_dependency_sync();
  const float* __restrict__ part = reinterpret_cast<const float*>(a.scratch);
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
  constexpr u64 outs = (u64)TCB_OUTER * (u64)TCB_INNER;
  __shared__ float acc_w[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (u64 base = (u64)blockIdx.x * 32; base < outs; base += (u64)gridDim.x * 32) {
    const u64 i = base + lane;
    float acc = tcb::red_init();
    if (i < outs) {
      int s = w;
      for (; s + 56 < TCB_SPLIT; s += 64) {  // eight independent loads in flight, combined in chunk order
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = part[(u64)(s + 8 * u) * outs + i];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc = tcb::red_comb(acc, v[u]);
      }
      for (; s < TCB_SPLIT; s += 8) acc = tcb::red_comb(acc, part[(u64)s * outs + i]);
    }
    acc_w[w][lane] = acc;
    __syncthreads();
    if (w == 0 && i < outs) {
      float r = acc_w[0][lane];
#pragma unroll
      for (int k = 1; k < 8; ++k) r = tcb::red_comb(r, acc_w[k][lane]);
      out[i] = r;
    }
    __syncthreads();
  }
}
