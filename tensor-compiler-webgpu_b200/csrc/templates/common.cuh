// tcb/common.cuh -- shared by every sm_100a template of libtcb200.
//
// Instantiated through NVRTC with the generated body of one fused node.  The
// op helpers give each IR op exactly one float32 rounding (the _rn intrinsics
// stop the compiler from contracting a*b+c into one fma), so a fused body
// computes what the unfused launches compute, value for value.  exp, log and
// tanh are CUDA's own expf/logf/tanhf (no fast-math); division and sqrt are
// the correctly rounded forms.
#pragma once

typedef unsigned long long u64;
typedef long long i64;
typedef unsigned int u32;

namespace tcb {

// The argument block every kernel takes by value (tc_args in include/tcb200.h).
struct Args {
  u64 in[8];
  u64 out;
  u64 scratch;
  i64 p[16];
};

__device__ __forceinline__ float op_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float op_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float op_mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float op_div(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float op_neg(float x) { return -x; }
__device__ __forceinline__ float op_exp(float x) { return expf(x); }
__device__ __forceinline__ float op_log(float x) { return logf(x); }
// interp.js: x > 0 ? x : 0 (so NaN and -0 give +0)
__device__ __forceinline__ float op_relu(float x) { return x > 0.0f ? x : 0.0f; }
__device__ __forceinline__ float op_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ float op_sqrt(float x) { return __fsqrt_rn(x); }
__device__ __forceinline__ float op_step(float x) { return x > 0.0f ? 1.0f : 0.0f; }
__device__ __forceinline__ float op_copy(float x) { return x; }
// max as interp.js folds it: v > acc ? v : acc (NaN never wins)
__device__ __forceinline__ float op_max(float acc, float v) { return v > acc ? v : acc; }

__device__ __forceinline__ float bits(u32 b) { return __uint_as_float(b); }

// Programmatic dependent launch.  A kernel replayed from a plan may be scheduled while the kernel before
// it is still draining (the launch carries the programmatic-serialization attribute); it waits here,
// before it touches any memory, until that kernel has completed and its writes are visible, then lets
// the kernel after it be scheduled in turn.  Launched without the attribute, both are no-ops.  Every
// kernel of the library's templates calls this first.
__device__ __forceinline__ void grid_dependency_sync() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Read-only loads (ld.global.nc); W consecutive floats from a 4W-byte aligned address.
template <int W>
__device__ __forceinline__ void load(float (&r)[W], const float* p) {
  if constexpr (W == 4) {
    float4 v = __ldg(reinterpret_cast<const float4*>(p));
    r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
  } else if constexpr (W == 2) {
    float2 v = __ldg(reinterpret_cast<const float2*>(p));
    r[0] = v.x; r[1] = v.y;
  } else {
#pragma unroll
    for (int l = 0; l < W; ++l) r[l] = __ldg(p + l);
  }
}

template <int W>
__device__ __forceinline__ void store(float* p, const float (&r)[W]) {
  if constexpr (W == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
  } else if constexpr (W == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
  } else {
#pragma unroll
    for (int l = 0; l < W; ++l) p[l] = r[l];
  }
}

__device__ __forceinline__ float ld1(const float* p) { return __ldg(p); }

// Warp reductions (all 32 lanes take part).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op_max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace tcb
