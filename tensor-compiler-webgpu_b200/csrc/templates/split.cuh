// tcb/split.cuh -- the 3xTF32 operand split of many GEMM operands in one launch.
//
// A resident program splits every GEMM operand that is an input of the program (the weight
// matrices of a training step) once, at the start of each run, with this kernel, instead of one
// split pass inside each GEMM launch.  Each job is the split tcb_split_a / tcb_split_b would do:
// hi = rna_tf32(x), lo = rna_tf32(x - hi), written K-major as [batch, R, Kp] with zeros beyond C,
// from a source that is [batch, R, C] (rows) or [batch, C, R] (cols: transposed on the way).
// a.scratch holds the job table; blockIdx.y picks the job; each job is walked grid-stride.
#pragma once

namespace tcb {
struct SplitJob {
  u64 src, hi, lo;
  u64 batch, R, C, Kp;
  u64 cols;  // 1: the source is [batch, C, R]
};

__device__ __forceinline__ float split_rna(float x) {
  u32 r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
}  // namespace tcb

extern "C" __global__ void __launch_bounds__(256) tcb_split_multi(const tcb::Args a) {
  using namespace tcb;
  grid_dependency_sync();
  const SplitJob j = reinterpret_cast<const SplitJob*>(a.scratch)[blockIdx.y];
  const float* __restrict__ src = reinterpret_cast<const float*>(j.src);
  float* __restrict__ hi = reinterpret_cast<float*>(j.hi);
  float* __restrict__ lo = reinterpret_cast<float*>(j.lo);
  if (!j.cols) {
    const u64 n = j.batch * j.R * j.Kp;
    for (u64 i = (u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (u64)gridDim.x * blockDim.x) {
      const u64 k = i % j.Kp, row = i / j.Kp;
      const float x = k < j.C ? __ldg(src + row * j.C + k) : 0.0f;
      const float h = split_rna(x);
      hi[i] = h;
      lo[i] = split_rna(x - h);
    }
    return;
  }
  // transposing: 32 x 32 tiles through shared memory, tiles walked grid-stride
  __shared__ float t[32][33];
  const u64 tk = j.Kp / 32, tr = (j.R + 31) / 32, tiles = tk * tr * j.batch;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (u64 tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const u64 b = tile / (tk * tr), rest = tile % (tk * tr);
    const u64 k0 = (rest % tk) * 32, r0 = (rest / tk) * 32;
    __syncthreads();
    for (int q = ty; q < 32; q += 8) {
      const u64 k = k0 + q, r = r0 + tx;
      t[q][tx] = (k < j.C && r < j.R) ? __ldg(src + (b * j.C + k) * j.R + r) : 0.0f;
    }
    __syncthreads();
    for (int q = ty; q < 32; q += 8) {
      const u64 r = r0 + q, k = k0 + tx;
      if (r < j.R && k < j.Kp) {
        const float x = t[tx][q];
        const float h = split_rna(x);
        const u64 o = (b * j.R + r) * j.Kp + k;
        hi[o] = h;
        lo[o] = split_rna(x - h);
      }
    }
  }
}
