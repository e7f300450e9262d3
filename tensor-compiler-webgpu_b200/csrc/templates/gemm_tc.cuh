// tcb/gemm_tc.cuh -- the matmul epilogue on the 5th-generation tensor cores
// (class 2 of the fusion pass on its tensor-core path; the reference's WGSL
// forms are src/gpu/codegen.js:152-193 and src/fusion/codegen-fused.js:176-265).
//
// float32 accuracy from TF32 units by the 3xTF32 split of every operand value x
// into hi and lo, accumulated in float32 in tensor memory:
//   A.B ~= A_lo.B_hi + A_hi.B_lo + A_hi.B_hi     (A_lo.B_lo dropped)
// An operand is split either by a pass into scratch (tcb_split_a / tcb_split_b:
// hi = rna_tf32(x), lo = rna_tf32(x - hi), K-major, zero padded to Kp, a
// multiple of 32) or, when few output tiles load it (TCB_FS_A / TCB_FS_B), in
// the kernel: its raw tile arrives by TMA (K-major, or MN-major in the 128-byte
// swizzle of 32-byte chunks) and serves as hi -- the tensor core reads an fp32
// operand as tf32 by dropping 13 mantissa bits -- and lo = rna_tf32(x -
// trunc(x)) is written beside it in shared memory.
//
// tcb_gemm_tc is persistent: TCB_GRID CTAs (one per SM) walk work units --
// 128 x BN output tiles in grouped raster order, the last wave's tiles (or all
// tiles, when fewer than the SMs) cut into K ranges whose partial tiles the
// last-arriving warp sums in range order -- with warps specialised:
//   warp 0     TMA producer: the stage's operand tiles into a STAGES-deep ring;
//   warp 1     allocates 2 x BN TMEM columns (two accumulators) and one lane
//              issues tcgen05.mma.cta_group::1.kind::tf32 (M=128, N=BN, K=8),
//              three per K step, committing each stage back to the producer;
//   warps 2-5  epilogue: tcgen05.ld of one accumulator while the MMA warp fills
//              the other, the fused body (bias, activation, residual ...) on
//              each value, 32 x 32 blocks staged in swizzled shared memory and
//              written by TMA stores (split-K: the partial sums);
//   warps 6-9  (in-kernel split only) the lo tiles of each stage.
// No TMA multicast.  Every wait is bounded by the global timer; a wait that
// runs out sets the launch's error word (p[15]) and the kernel unwinds,
// freeing its TMEM.
//
// The generated part defines TCB_M, TCB_N, TCB_K, TCB_KP, TCB_BATCH, TCB_IA,
// TCB_IB, TCB_BN, TCB_BK, TCB_STAGES, TCB_SPLITK, TCB_GRID, TCB_TAIL_SPLIT,
// TCB_FS_A, TCB_FS_B, TCB_TMA_STORE, the scratch offsets and struct Epi (as for
// tcb/matmul.cuh).
#pragma once

namespace tcb {

struct alignas(64) TmaDesc { u64 v[16]; };
struct GemmParams {
  TmaDesc maps[5];  // A_hi / raw A, A_lo, B_hi / raw B, B_lo (3-D: {cols, rows, batch}); [4] the output
  Args a;
};

#ifndef TCB_BK
#define TCB_BK 32
#endif
#ifndef TCB_CROSS_BA
#define TCB_CROSS_BA 0  // 1: issue A_hi.B_lo before A_lo.B_hi (a GEMM computing (X.Y)^T as Y^T.X^T)
#endif
// K-block: 32 fp32 (128-byte rows, 128-byte swizzle) or 16 fp32 (64-byte rows, 64-byte swizzle).
constexpr int GB_M = 128, GB_K = TCB_BK;
static_assert(GB_K == 32 || GB_K == 16, "K-block of 16 or 32 floats");
#ifndef TCB_WAIT_NS
#define TCB_WAIT_NS 2000000000u  // 2 s: far above any legitimate wait
#endif
constexpr u32 WAIT_NS = TCB_WAIT_NS;

__device__ __forceinline__ u32 smem_u32(const void* p) { return (u32)__cvta_generic_to_shared(p); }
__device__ __forceinline__ u64 now_ns() { u64 t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }

__device__ __forceinline__ void mbar_init(u32 bar, u32 count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(u32 bar, u32 bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(u32 bar, u32 parity) {
  u32 ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: false (and the error word set) if the barrier phase never completes.
__device__ __forceinline__ bool mbar_wait(u32 bar, u32 parity, u32* err, u32 code) {
  if (mbar_try(bar, parity)) return true;
  const u64 t0 = now_ns();
  for (u32 it = 0;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 255) == 0 && (now_ns() - t0 > WAIT_NS || (err && *(volatile u32*)err))) {
      if (err) atomicCAS(err, 0u, code);
      return false;
    }
  }
}

// Shared -> global tensor store of one box (rows outside the tensor are not written); completion is
// tracked per thread in bulk groups.
__device__ __forceinline__ void tma_store_3d(const TmaDesc* map, u32 src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               :: "l"(reinterpret_cast<u64>(map)), "r"(src), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most one committed group still has to read its shared-memory source
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tma_load_3d(u32 dst, const TmaDesc* map, u32 bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      :: "r"(dst), "l"(reinterpret_cast<u64>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar) : "memory");
}

// tcgen05 shared-memory matrix descriptor, K-major: rows of GB_K floats, 8-row swizzle atoms
// (1024 B apart with the 128-byte swizzle, 512 B with the 64-byte one).
__device__ __forceinline__ u64 sw128_desc(u32 saddr) {
  u64 d = 0;
  d |= (u64)((saddr >> 4) & 0x3FFF);                    // start address
  d |= (u64)1 << 16;                                     // leading byte offset (unused for swizzled K-major)
  d |= (u64)((8 * GB_K * 4) >> 4) << 32;                 // stride byte offset: 8 rows
  d |= (u64)1 << 46;                                     // descriptor version for sm_100
  d |= (u64)(GB_K == 32 ? 2 : 4) << 61;                  // 128-byte or 64-byte swizzle
  return d;
}

// MN-major tf32 operand tile (the M or N index contiguous): rows of 32 floats (128 bytes) along M/N,
// one row per K index, in the 128-byte swizzle of 32-byte chunks (period 4 rows: the only MN-major
// shared-memory layout the tensor cores take for 32-bit operands); 4-row groups 512 bytes apart, and
// one such column of rows per 32 M (or N) indices, `lbo` bytes apart.
__device__ __forceinline__ u64 mn_desc(u32 saddr, u32 lbo) {
  u64 d = 0;
  d |= (u64)((saddr >> 4) & 0x3FFF);                    // start address
  d |= (u64)((lbo >> 4) & 0x3FFF) << 16;                 // leading byte offset: next 32 M/N indices
  d |= (u64)(512 >> 4) << 32;                            // stride byte offset: next 4 K rows
  d |= (u64)1 << 46;                                     // descriptor version for sm_100
  d |= (u64)1 << 61;                                     // 128-byte swizzle, 32-byte atoms
  return d;
}

// Instruction descriptor: D f32, A/B tf32, M = 128, N = n; a_mn / b_mn: that operand is MN-major.
__host__ __device__ constexpr u32 idesc_tf32(u32 n, u32 a_mn = 0, u32 b_mn = 0) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) |
         ((u32)(GB_M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(u32 tmem, u64 a, u64 b, u32 idesc, u32 accumulate) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}"
               :: "r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void mma_commit(u32 bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(u32 taddr, float (&r)[16]) {
  u32 v[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) r[j] = __uint_as_float(v[j]);
}

// The low part of x for the in-kernel split: the tensor core reads an fp32 operand as tf32 by
// dropping its 13 low mantissa bits, so the raw value serves as hi and lo = rna_tf32(x - trunc(x)).
__device__ __forceinline__ float tf32_lo(float x) {
  const float t = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  u32 r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(__fsub_rn(x, t)));
  return __uint_as_float(r);
}

__device__ __forceinline__ float tf32_rna(float x) {
  u32 r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

}  // namespace tcb

#ifndef TCB_SPLITK
#define TCB_SPLITK 1
#endif

#ifndef TCB_A_T
#define TCB_A_T 0   // 1: operand A arrives as its transpose X [batch, K, M] (a folded transposeLast2)
#endif
#ifndef TCB_B_T
#define TCB_B_T 0   // 1: operand B arrives as its transpose Y [batch, N, K]
#endif
#ifndef TCB_PART_OFFSET
#define TCB_PART_OFFSET 0ull
#endif
#ifndef TCB_FS_A
#define TCB_FS_A 0   // 1: the GEMM reads raw A and makes its lo in shared memory (no split pass for A)
#endif
#ifndef TCB_FS_B
#define TCB_FS_B 0   // the same for B
#endif
#ifndef TCB_SPLIT_B_OFFSET  // where split_b's B_hi, B_lo start in scratch (after A_hi, A_lo when A is split)
#define TCB_SPLIT_B_OFFSET (2ull * TCB_BATCH * TCB_M * TCB_KP * 4)
#endif
#ifndef TCB_TMA_STORE
#define TCB_TMA_STORE 0   // 1: the epilogue stages 32 x 32 output blocks in shared memory for TMA stores (map 4)
#endif
#ifndef TCB_GRID
#define TCB_GRID 148
#endif
#ifndef TCB_TAIL_SPLIT
#define TCB_TAIL_SPLIT 1
#endif
#ifndef TCB_TAIL_OFFSET
#define TCB_TAIL_OFFSET 0ull
#endif

namespace tcb {
// Work units of the persistent GEMM (TCB_GRID CTAs, unit u on CTA u % GRID).  Units below U_FULL are
// whole output tiles (of one K split).  When the last wave would hold only REM <= GRID/2 tiles, each
// of those tiles becomes TAIL units over equal K ranges instead, so the last wave fills the SMs; their
// partial tiles meet in scratch and the warp that finishes a tile's quarter last reduces it, adding the
// partials in unit order (so the result does not depend on which CTA came last).
struct GemmShape {
  static constexpr u32 KB_ALL = TCB_KP / GB_K;
  static constexpr u32 TILES_M = (TCB_M + GB_M - 1) / GB_M, TILES_N = (TCB_N + TCB_BN - 1) / TCB_BN;
  static constexpr u32 TILES_PER = TILES_M * TILES_N;
  static constexpr u32 TILES = TILES_PER * TCB_BATCH * TCB_SPLITK;
  static constexpr u32 GRID = TCB_GRID;
  static constexpr u32 TAIL = TCB_TAIL_SPLIT;
  static constexpr u32 REM = TAIL > 1 ? TILES % GRID : 0;
  static constexpr u32 U_FULL = TILES - REM;
  static constexpr u32 UNITS = U_FULL + REM * TAIL;
};
static_assert(TCB_TAIL_SPLIT == 1 || TCB_SPLITK == 1, "tail split and split-K are exclusive");
// The launch's control block at p[15]: the error word (16 bytes), then 4 arrival counters per split tile.
__device__ __forceinline__ u32* tail_counters(const Args& a) { return reinterpret_cast<u32*>(a.p[15]) + 4; }
__device__ __forceinline__ void clear_ctrl(const Args& a) {
  u32* w = reinterpret_cast<u32*>(a.p[15]);
  for (u32 i = threadIdx.x; i < 4 + 4 * GemmShape::REM; i += blockDim.x) w[i] = 0u;
}
static_assert(TCB_TAIL_SPLIT <= GemmShape::KB_ALL, "every tail unit has at least one k-block");

// Row-major src [batch, R, C] -> hi, lo [batch, R, Kp] with Kp >= C (zero beyond C), 4 elements per step.
__device__ __forceinline__ void split_rows(const float* __restrict__ src, float* __restrict__ hi, float* __restrict__ lo,
                                           u64 rows, u64 C, u64 Kp) {
  const u64 n4 = rows * Kp / 4;
  for (u64 v = (u64)blockIdx.x * blockDim.x + threadIdx.x; v < n4; v += (u64)gridDim.x * blockDim.x) {
    const u64 i = v * 4;
    const u64 k = i % Kp, row = i / Kp;
    float x[4];
    if ((C % 4) == 0 && k + 4 <= C) {
      const float4 q = __ldg(reinterpret_cast<const float4*>(src + row * C + k));
      x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = (k + j < C) ? __ldg(src + row * C + k + j) : 0.0f;
    }
    float h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) { h[j] = tf32_rna(x[j]); l[j] = tf32_rna(x[j] - h[j]); }
    *reinterpret_cast<float4*>(hi + i) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + i) = make_float4(l[0], l[1], l[2], l[3]);
  }
}
// Row-major src [batch, C, R] -> hi, lo [batch, R, Kp] (transposed), 32x32 tiles through shared memory.
// grid (Kp/32, ceil(R/32), batch), 256 threads.
__device__ __forceinline__ void split_cols(const float* __restrict__ src, float* __restrict__ hi, float* __restrict__ lo,
                                           u64 R, u64 C, u64 Kp) {
  __shared__ float t[32][33];
  const u64 b = blockIdx.z;
  const u64 k0 = (u64)blockIdx.x * 32, r0 = (u64)blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int q = ty; q < 32; q += 8) {
    const u64 k = k0 + q, r = r0 + tx;
    t[q][tx] = (k < C && r < R) ? __ldg(src + (b * C + k) * R + r) : 0.0f;
  }
  __syncthreads();
  for (int q = ty; q < 32; q += 8) {
    const u64 r = r0 + q, k = k0 + tx;
    if (r < R && k < Kp) {
      const float x = t[tx][q];
      const float h = tf32_rna(x);
      const u64 o = (b * R + r) * Kp + k;
      hi[o] = h;
      lo[o] = tf32_rna(x - h);
    }
  }
}
}  // namespace tcb

// A -> A_hi, A_lo [batch, M, Kp] (scratch), zero beyond K.  It runs first in every tensor-core
// launch, so it also clears that launch's error word (p[15]) in the reused scratch.
extern "C" __global__ void __launch_bounds__(256) tcb_split_a(const tcb::Args a) {
  tcb::grid_dependency_sync();
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && a.p[15]) tcb::clear_ctrl(a);
  float* hi = reinterpret_cast<float*>(a.scratch);
  float* lo = hi + (u64)TCB_BATCH * TCB_M * TCB_KP;
  const float* src = reinterpret_cast<const float*>(a.in[TCB_IA]);
#if TCB_A_T
  tcb::split_cols(src, hi, lo, TCB_M, TCB_K, TCB_KP);
#else
  tcb::split_rows(src, hi, lo, (u64)TCB_BATCH * TCB_M, TCB_K, TCB_KP);
#endif
}

// B [batch, K, N] -> B_hi^T, B_lo^T [batch, N, Kp] so both operands are K-major.
extern "C" __global__ void __launch_bounds__(256) tcb_split_b(const tcb::Args a) {
  tcb::grid_dependency_sync();
  float* hi = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(a.scratch) + TCB_SPLIT_B_OFFSET);
  float* lo = hi + (u64)TCB_BATCH * TCB_N * TCB_KP;
  const float* src = reinterpret_cast<const float*>(a.in[TCB_IB]);
#if TCB_B_T
  tcb::split_rows(src, hi, lo, (u64)TCB_BATCH * TCB_N, TCB_K, TCB_KP);
#else
  tcb::split_cols(src, hi, lo, TCB_N, TCB_K, TCB_KP);
#endif
}

// With A split in the kernel there is no tcb_split_a: this one-block launch, first in the tensor-core
// launch, clears its error word (p[15]) and the tail units' arrival counters instead.
extern "C" __global__ void __launch_bounds__(128) tcb_gemm_prep(const tcb::Args a) {
  tcb::grid_dependency_sync();
  if (a.p[15]) tcb::clear_ctrl(a);
}

// Persistent: TCB_GRID CTAs (one per SM) walk the work units (grouped raster for L2 reuse); TMEM holds
// two BN-column accumulators so the epilogue of unit j overlaps the mainloop of unit j+1.
// An operand split in the kernel (TCB_FS_A / TCB_FS_B) arrives in the ring as its raw tile (K-major,
// or MN-major when it arrives transposed: TCB_A_T for A, !TCB_B_T for B) and four more warps (6-9)
// write the stage's lo tile beside it; the MMA reads the raw tile as hi.  An operand that is loaded by
// many tiles keeps its split pass instead, so its conversion is not repeated per tile.
extern "C" __global__ void __launch_bounds__((TCB_FS_A || TCB_FS_B) ? 320 : 192, 1)
    tcb_gemm_tc(const __grid_constant__ tcb::GemmParams P) {
  using namespace tcb;
  using S = GemmShape;
  constexpr int BN = TCB_BN, STAGES = TCB_STAGES;
  constexpr bool FA = TCB_FS_A != 0, FB = TCB_FS_B != 0, FS = FA || FB;
  constexpr bool A_MN = FA && TCB_A_T, B_MN = FB && !TCB_B_T;
  constexpr u32 A_BYTES = GB_M * GB_K * 4, B_BYTES = BN * GB_K * 4;
  constexpr u32 STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  constexpr u32 KB_PER = (S::KB_ALL + TCB_SPLITK - 1) / TCB_SPLITK;  // k-blocks per split
  constexpr u32 GROUP = 8;
  constexpr u64 CHUNK = (u64)GB_M * 16;                    // floats of one 16-column slice of a partial tile
  extern __shared__ unsigned char smem_raw[];
  u32* err = reinterpret_cast<u32*>(P.a.p[15]);  // global error word (may be null)
  if (gridDim.x != S::GRID) {                     // the unit schedule assumes exactly GRID CTAs
    grid_dependency_sync();
    if (threadIdx.x == 0 && err) atomicCAS(err, 0u, 9u);
    return;
  }
  const u32 raw = smem_u32(smem_raw);
  const u32 base = (raw + 1023u) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  const u32 bars = base + STAGES * STAGE_BYTES;  // full[S], empty[S], accf[2], acce[2], conv[S]
  // output staging (TCB_TMA_STORE): two 32 x 32 float blocks per epilogue warp, after a 1 KB barrier area
  const u32 staging = bars + 1024;
  static_assert((3 * STAGES + 4) * 8 + 16 <= 1024, "barrier area");
  u32* tmem_slot = reinterpret_cast<u32*>(gbase + STAGES * STAGE_BYTES + (3 * STAGES + 4) * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (STAGES + s); };
  auto accf = [&](u32 b) { return bars + 8u * (2 * STAGES + b); };
  auto acce = [&](u32 b) { return bars + 8u * (2 * STAGES + 2 + b); };
  auto conv = [&](int s) { return bars + 8u * (2 * STAGES + 4 + s); };
  struct Tile { int m0, n0, bz; u32 kb0, kb; int tail; u32 piece; };
  auto decode = [&](u32 u) {
    Tile T;
    u32 t = u;
    T.tail = -1;
    T.piece = 0;
    if (u >= S::U_FULL) {  // a K range of a last-wave tile
      const u32 v = u - S::U_FULL;
      T.tail = (int)(v / S::TAIL);
      T.piece = v % S::TAIL;
      t = S::U_FULL + v / S::TAIL;
    }
    const u32 bs = t / S::TILES_PER, r = t % S::TILES_PER;
    T.bz = (int)(bs / TCB_SPLITK);
    const u32 split = bs % TCB_SPLITK;
    const u32 group = r / (GROUP * S::TILES_N), first = group * GROUP;
    const u32 gsz = S::TILES_M - first < GROUP ? S::TILES_M - first : GROUP;
    const u32 w = r % (GROUP * S::TILES_N);
    T.m0 = (int)((first + w % gsz) * GB_M);
    T.n0 = (int)((w / gsz) * BN);
    if (T.tail >= 0) {
      T.kb0 = T.piece * S::KB_ALL / S::TAIL;
      T.kb = (T.piece + 1) * S::KB_ALL / S::TAIL - T.kb0;
    } else {
      T.kb0 = split * KB_PER;
      const u32 kb1 = T.kb0 + KB_PER < S::KB_ALL ? T.kb0 + KB_PER : S::KB_ALL;
      T.kb = kb1 > T.kb0 ? kb1 - T.kb0 : 0;
    }
    return T;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(full(s), 1); mbar_init(empty(s), 1); }
    for (u32 b = 0; b < 2; ++b) { mbar_init(accf(b), 1); mbar_init(acce(b), 4); }
    if (FS) for (int s = 0; s < STAGES; ++s) mbar_init(conv(s), 128);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(smem_u32(tmem_slot)),
                 "r"((u32)(2 * BN)) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const u32 tmem = *tmem_slot;
  // the set-up above touches only this CTA's shared and tensor memory, so it may overlap the previous
  // kernel's tail (programmatic dependent launch); every global access comes after this wait
  grid_dependency_sync();

  if (warp == 0) {
    if (lane == 0) {
      u32 it = 0;
      bool ok = true;
      for (u32 t = blockIdx.x; ok && t < S::UNITS; t += S::GRID) {
        const Tile T = decode(t);
        for (u32 kb = 0; kb < T.kb; ++kb, ++it) {
          const int s = it % STAGES;
          if (it >= (u32)STAGES && !mbar_wait(empty(s), ((it / STAGES) - 1) & 1, err, 1)) { ok = false; break; }
          const u32 st = base + s * STAGE_BYTES;
          const int kc = (int)((T.kb0 + kb) * GB_K);
          // maps: [0] A_hi or raw A, [1] A_lo, [2] B_hi or raw B, [3] B_lo; an MN-major raw tile is GB_K
          // rows of 32 floats per 32 M (N) indices (128-byte swizzle of 32-byte chunks)
          mbar_expect_tx(full(s), (FA ? A_BYTES : 2 * A_BYTES) + (FB ? B_BYTES : 2 * B_BYTES));
          if (A_MN) {
#pragma unroll
            for (int q = 0; q < GB_M / 32; ++q)
              tma_load_3d(st + q * GB_K * 128, &P.maps[0], full(s), T.m0 + 32 * q, kc, T.bz);
          } else {
            tma_load_3d(st, &P.maps[0], full(s), kc, T.m0, T.bz);
          }
          if (!FA) tma_load_3d(st + A_BYTES, &P.maps[1], full(s), kc, T.m0, T.bz);
          if (B_MN) {
#pragma unroll
            for (int q = 0; q < BN / 32; ++q)
              tma_load_3d(st + 2 * A_BYTES + q * GB_K * 128, &P.maps[2], full(s), T.n0 + 32 * q, kc, T.bz);
          } else {
            tma_load_3d(st + 2 * A_BYTES, &P.maps[2], full(s), kc, T.n0, T.bz);
          }
          if (!FB) tma_load_3d(st + 2 * A_BYTES + B_BYTES, &P.maps[3], full(s), kc, T.n0, T.bz);
        }
      }
      // drain: wait (bounded) for the copies still in flight before this CTA may exit
      for (u32 i = it > (u32)STAGES ? it - STAGES : 0; i < it; ++i) mbar_wait(full(i % STAGES), (i / STAGES) & 1, err, 2);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr u32 ID = idesc_tf32(BN, A_MN ? 1u : 0u, B_MN ? 1u : 0u);
      // operand descriptors of K step k (8 K indices) in a tile at `t`
      auto da = [&](u32 t, int k) { return A_MN ? mn_desc(t + 1024 * k, GB_K * 128) : sw128_desc(t + 32 * k); };
      auto db = [&](u32 t, int k) { return B_MN ? mn_desc(t + 1024 * k, GB_K * 128) : sw128_desc(t + 32 * k); };
      u32 it = 0, j = 0;
      bool ok = true;
      for (u32 t = blockIdx.x; ok && t < S::UNITS; t += S::GRID, ++j) {
        const Tile T = decode(t);
        const u32 buf = j & 1;
        if (j >= 2 && !mbar_wait(acce(buf), ((j >> 1) - 1) & 1, err, 5)) break;
        tc_fence_after();
        const u32 acc = tmem + buf * BN;
        for (u32 kb = 0; kb < T.kb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(full(s), (it / STAGES) & 1, err, 3)) { ok = false; break; }
          if (FS && !mbar_wait(conv(s), (it / STAGES) & 1, err, 7)) { ok = false; break; }
          tc_fence_after();
          const u32 st = base + s * STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < GB_K / 8; ++k) {
            const u64 ah = da(st, k), al = da(st + A_BYTES, k);
            const u64 bh = db(st + 2 * A_BYTES, k), bl = db(st + 2 * A_BYTES + B_BYTES, k);
            if (TCB_CROSS_BA) {  // a transposed product: the mixed terms in the order of the untransposed one
              mma_tf32(acc, ah, bl, ID, (kb | k) != 0);
              mma_tf32(acc, al, bh, ID, 1);
            } else {
              mma_tf32(acc, al, bh, ID, (kb | k) != 0);
              mma_tf32(acc, ah, bl, ID, 1);
            }
            mma_tf32(acc, ah, bh, ID, 1);
          }
          mma_commit(empty(s));
        }
        mma_commit(accf(buf));  // with no k-block in this split the accumulator is never enabled: see the epilogue
      }
    }
  } else if (FS && warp >= 6) {
    // in-kernel split: lo of every raw value of the stage, written beside it (same swizzled position)
    const int tid = threadIdx.x - 192;
    u32 it = 0;
    bool ok = true;
    for (u32 t = blockIdx.x; ok && t < S::UNITS; t += S::GRID) {
      const Tile T = decode(t);
      for (u32 kb = 0; kb < T.kb; ++kb, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(full(s), (it / STAGES) & 1, err, 6)) { ok = false; break; }
        unsigned char* st = gbase + s * STAGE_BYTES;
        if (FA) {
          const float4* ra = reinterpret_cast<const float4*>(st);
          float4* la = reinterpret_cast<float4*>(st + A_BYTES);
#pragma unroll
          for (u32 v = tid; v < A_BYTES / 16; v += 128) {
            const float4 x = ra[v];
            la[v] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
          }
        }
        if (FB) {
          const float4* rb = reinterpret_cast<const float4*>(st + 2 * A_BYTES);
          float4* lb = reinterpret_cast<float4*>(st + 2 * A_BYTES + B_BYTES);
#pragma unroll
          for (u32 v = tid; v < B_BYTES / 16; v += 128) {
            const float4 x = rb[v];
            lb[v] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
          }
        }
        // make these generic-proxy writes visible to the tensor core, then release the stage to the MMA
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(conv(s)) : "memory");
      }
    }
  } else {
    // epilogue: warps 2..5 -> TMEM lane quarter (warp % 4)
    const int q = warp & 3;
    float* __restrict__ out = reinterpret_cast<float*>(P.a.out);
    unsigned char* scr = reinterpret_cast<unsigned char*>(P.a.scratch);
    // the fused body on 16 accumulator values of one row, stored to the output
    auto finish16 = [&](const Tile& T, u64 row, int c0, float (&v)[16]) {
      if (row >= (u64)TCB_M || (u64)(T.n0 + c0) >= (u64)TCB_N) return;
      const u64 base_i = (u64)T.bz * TCB_M * TCB_N + row * TCB_N + (u64)(T.n0 + c0);
      float o[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const u64 col = (u64)(T.n0 + c0 + jj);
        o[jj] = col < (u64)TCB_N ? Epi::apply(P.a, v[jj], base_i + jj, row, col, (u64)T.bz) : 0.0f;
      }
      if ((TCB_N % 4) == 0 && (u64)(T.n0 + c0 + 16) <= (u64)TCB_N) {
#pragma unroll
        for (int jj = 0; jj < 16; jj += 4)
          *reinterpret_cast<float4*>(out + base_i + jj) = make_float4(o[jj], o[jj + 1], o[jj + 2], o[jj + 3]);
      } else {
        for (int jj = 0; jj < 16; ++jj) if ((u64)(T.n0 + c0 + jj) < (u64)TCB_N) out[base_i + jj] = o[jj];
      }
    };
    u32 j = 0, nstore = 0;
    for (u32 t = blockIdx.x; t < S::UNITS; t += S::GRID, ++j) {
      const Tile T = decode(t);
      const u32 buf = j & 1;
      if (!mbar_wait(accf(buf), (j >> 1) & 1, err, 4)) break;
      tc_fence_after();
      const u64 row = (u64)T.m0 + 32 * q + lane;
      if (S::TAIL > 1 && T.tail >= 0) {
        // partial tiles in scratch: [tail tile][piece][BN/16 slices][128 rows][16], one 64-byte run per row
        float* tp = reinterpret_cast<float*>(scr + TCB_TAIL_OFFSET) + (u64)T.tail * S::TAIL * (BN / 16) * CHUNK +
                    (u64)(32 * q + lane) * 16;
        float* mine = tp + (u64)T.piece * (BN / 16) * CHUNK;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(tmem + buf * BN + ((u32)(32 * q) << 16) + (u32)c0, v);
          float4* d = reinterpret_cast<float4*>(mine + (u64)(c0 / 16) * CHUNK);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) d[jj] = make_float4(v[4 * jj], v[4 * jj + 1], v[4 * jj + 2], v[4 * jj + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(acce(buf)) : "memory");
        // publish this warp's rows, then count the arrival; the last of the TAIL pieces reduces them
        __threadfence();
        __syncwarp();
        u32 old = 0;
        if (lane == 0)
          old = atomicAdd(tail_counters(P.a) + 4 * (u32)T.tail + (u32)q, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == S::TAIL - 1) {
          __threadfence();
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            const float* src = tp + (u64)(c0 / 16) * CHUNK;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const float4 x = __ldcg(reinterpret_cast<const float4*>(src) + jj);
              v[4 * jj] = x.x; v[4 * jj + 1] = x.y; v[4 * jj + 2] = x.z; v[4 * jj + 3] = x.w;
            }
#pragma unroll 1
            for (u32 pc = 1; pc < S::TAIL; ++pc) {
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                const float4 x = __ldcg(reinterpret_cast<const float4*>(src + (u64)pc * (BN / 16) * CHUNK) + jj);
                v[4 * jj] = op_add(v[4 * jj], x.x);
                v[4 * jj + 1] = op_add(v[4 * jj + 1], x.y);
                v[4 * jj + 2] = op_add(v[4 * jj + 2], x.z);
                v[4 * jj + 3] = op_add(v[4 * jj + 3], x.w);
              }
            }
            finish16(T, row, c0, v);
          }
          // every piece has arrived: leave the counter at zero for the next launch
          if (lane == 0) tail_counters(P.a)[4 * (u32)T.tail + (u32)q] = 0u;
        }
        continue;
      }
      if (TCB_TMA_STORE) {
        // 32 columns at a time: this row's 32 accumulator values (split-K: the raw partial sums) written
        // into a 128-byte-swizzled 32 x 32 staging block (conflict-free: 16-byte chunk c of row r at
        // r * 128 + (c ^ (r & 7)) * 16), then one TMA store of the block -- to the output, or with
        // split-K to this split's slice of the partial sums [SPLITK * batch, M, N]; two blocks per warp
        // alternate.  The fused body runs on the staged block row by row, lane l on column c0 + l, so
        // the operands it loads (a residual, another [M, N] value) are read 32 consecutive floats per
        // warp instruction -- one 128-byte line -- where a thread per row would touch 32 lines.  Each
        // element goes through the same operations as before: the values are unchanged.
        const int zc = TCB_SPLITK > 1 ? (int)(((t / S::TILES_PER) % TCB_SPLITK) * TCB_BATCH) + T.bz : T.bz;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32, ++nstore) {
          float v[32];
          tmem_ld16(tmem + buf * BN + ((u32)(32 * q) << 16) + (u32)c0, *reinterpret_cast<float(*)[16]>(&v[0]));
          tmem_ld16(tmem + buf * BN + ((u32)(32 * q) << 16) + (u32)(c0 + 16), *reinterpret_cast<float(*)[16]>(&v[16]));
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) v[jj] = T.kb == 0 ? 0.0f : v[jj];
          const u32 blk = staging + (u32)((q * 2 + (nstore & 1)) * 4096);
          if (lane == 0 && nstore >= 2) bulk_wait_read1();
          __syncwarp();
          float4* sp = reinterpret_cast<float4*>(gbase + (blk - base));
#pragma unroll
          for (int c = 0; c < 8; ++c)
            sp[lane * 8 + (c ^ (lane & 7))] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
          if (TCB_SPLITK == 1) {
            // all 32 rows into registers before any result is written back: no store stands between the
            // operand loads, so they are all in flight at once
            __syncwarp();
            float* sf = reinterpret_cast<float*>(sp);
            const u64 col = (u64)(T.n0 + c0 + lane);
            float o[32];
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) {
              const u64 grow = (u64)T.m0 + 32 * q + rr;
              const float acc = sf[rr * 32 + (((lane >> 2) ^ (rr & 7)) << 2) + (lane & 3)];
              o[rr] = (grow < (u64)TCB_M && col < (u64)TCB_N)
                          ? Epi::apply(P.a, acc, (u64)T.bz * TCB_M * TCB_N + grow * TCB_N + col, grow, col, (u64)T.bz)
                          : 0.0f;
            }
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) sf[rr * 32 + (((lane >> 2) ^ (rr & 7)) << 2) + (lane & 3)] = o[rr];
            __syncwarp();
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&P.maps[4], blk, T.n0 + c0, T.m0 + 32 * q, zc);
            bulk_commit();
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(acce(buf)) : "memory");
        continue;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + buf * BN + ((u32)(32 * q) << 16) + (u32)c0, v);
        if (T.kb == 0) {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) v[jj] = 0.0f;
        }
        if (TCB_SPLITK > 1) {
          // partial sums of this split: [SPLITK][batch][M][N] floats after the split operands in scratch
          if (row < (u64)TCB_M) {
            const u64 split = (t / S::TILES_PER) % TCB_SPLITK;
            float* part = reinterpret_cast<float*>(P.a.scratch) + TCB_PART_OFFSET / 4 +
                          ((split * TCB_BATCH + (u64)T.bz) * TCB_M + row) * TCB_N;
            for (int jj = 0; jj < 16; ++jj)
              if ((u64)(T.n0 + c0 + jj) < (u64)TCB_N) part[T.n0 + c0 + jj] = v[jj];
          }
          continue;
        }
        finish16(T, row, c0, v);
      }
      // this warp's reads of the accumulator are complete: hand the buffer back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(acce(buf)) : "memory");
    }
    if (TCB_TMA_STORE && lane == 0) bulk_wait_all();  // the staged stores are done before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"((u32)(2 * BN)) : "memory");
  }
}

// Split-K: out = Epi(sum over splits s = 0.. of partial[s]), in split order (deterministic).
extern "C" __global__ void __launch_bounds__(256) tcb_splitk_finish(const tcb::Args a) {
  tcb::grid_dependency_sync();
#if TCB_SPLITK > 1
  const float* __restrict__ part = reinterpret_cast<const float*>(a.scratch) + TCB_PART_OFFSET / 4;
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
  constexpr u64 n = (u64)TCB_BATCH * TCB_M * TCB_N;
  for (u64 i = (u64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (u64)gridDim.x * blockDim.x) {
    float acc = part[i];
    for (int s = 1; s < TCB_SPLITK; ++s) acc = tcb::op_add(acc, part[(u64)s * n + i]);
    const u64 col = i % TCB_N, row = (i / TCB_N) % TCB_M, b = i / ((u64)TCB_M * TCB_N);
    out[i] = Epi::apply(a, acc, i, row, col, b);
  }
#endif
}
