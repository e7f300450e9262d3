// tcb/matmul.cuh -- float32 CUDA-core matmul with a fused epilogue (class 2 of
// the fusion pass on its exact-fp32 path; the reference's WGSL forms are
// src/gpu/codegen.js:119-193 and src/fusion/codegen-fused.js:176-265).
//
// OUT[b, i, j] = Epi::apply(sum_k A[b,i,k] * B[b,k,j], ...), k ascending with
// one fma per term, so every output sees interp.js's summation order.  Used
// for the `naive` variant and for contractions too short for the 3xTF32
// tensor-core path to stay inside the float32 budget.
//
// The generated part defines TCB_M, TCB_N, TCB_K, TCB_BATCH, TCB_IA, TCB_IB
// (operand slots of A and B) and struct Epi { static float apply(const
// tcb::Args&, float acc, u64 i, u64 row, u64 col, u64 b); }.
// Tile 128x128x8, 256 threads, an 8x8 register block per thread, the next
// k-slice prefetched into registers while the current one is consumed.
#pragma once

namespace tcb {
constexpr int MM_BM = 128, MM_BN = 128, MM_BK = 8;
}

extern "C" __global__ void __launch_bounds__(256) tcb_matmul(const tcb::Args a) {
  using namespace tcb;
  grid_dependency_sync();
  __shared__ __align__(16) float As[2][MM_BK][MM_BM];
  __shared__ __align__(16) float Bs[2][MM_BK][MM_BN];
  constexpr u64 M = TCB_M, N = TCB_N, K = TCB_K;
  const u64 b = blockIdx.z;
  const float* __restrict__ A = reinterpret_cast<const float*>(a.in[TCB_IA]) + b * M * K;
  const float* __restrict__ B = reinterpret_cast<const float*>(a.in[TCB_IB]) + b * K * N;
  const int tid = threadIdx.x;
  const u64 row0 = (u64)blockIdx.y * MM_BM, col0 = (u64)blockIdx.x * MM_BN;
  // loader coordinates
  const int a_r = tid >> 1, a_k = (tid & 1) * 4;
  const int b_k = tid >> 5, b_c = (tid & 31) * 4;
  // compute coordinates
  const int tx = tid & 15, ty = tid >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  float ra[4], rb[4];
  auto fetch = [&](u64 k0) {
    const u64 r = row0 + a_r;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const u64 k = k0 + a_k + q;
      ra[q] = (r < M && k < K) ? __ldg(A + r * K + k) : 0.0f;
    }
    const u64 kb = k0 + b_k;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const u64 c = col0 + b_c + q;
      rb[q] = (kb < K && c < N) ? __ldg(B + kb * N + c) : 0.0f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int q = 0; q < 4; ++q) As[buf][a_k + q][a_r] = ra[q];
    *reinterpret_cast<float4*>(&Bs[buf][b_k][b_c]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
  };

  const u64 tiles = (K + MM_BK - 1) / MM_BK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (u64 t = 0; t < tiles; ++t) {
    const int cur = t & 1;
    if (t + 1 < tiles) fetch((t + 1) * MM_BK);
#pragma unroll
    for (int k = 0; k < MM_BK; ++k) {
      float av[8], bv[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][64 + tx * 4]);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w; av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w; bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (t + 1 < tiles) {
      stash(cur ^ 1);
      __syncthreads();
    }
  }
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const u64 r = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const u64 c = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (c >= N) continue;
      const u64 idx = b * M * N + r * N + c;
      out[idx] = Epi::apply(a, acc[i][j], idx, r, c, b);
    }
  }
}
