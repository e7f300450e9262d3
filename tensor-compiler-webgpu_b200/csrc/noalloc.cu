// tc_colsum_f32_static: the column-sum reduction (sum over axis 0) with its
// scratch in a fixed device array instead of memory the caller or the library
// allocates.
//
// Why it exists: some callers cannot allocate device memory at the point
// where they need this reduction -- code running while a stream is being
// captured into a CUDA graph (an allocation there is illegal or breaks the
// capture), hosts whose device memory belongs to another allocator with a
// fixed budget (a framework's caching pool), and latency-critical paths that
// cannot afford cudaMalloc's implicit device-wide synchronisation.  Those
// callers pass only the input and the output; the partial sums live in
// `tcb_colsum_scratch` below.
//
// Limits and behaviour (also stated beside the declaration in include/tcb200.h):
//  - the scratch holds TC_COLSUM_STATIC_MAX_FLOATS floats (16 MiB); every GPU
//    that loads this library keeps that much device memory until the process
//    exits;
//  - cols above TC_COLSUM_STATIC_MAX_FLOATS is rejected with TC_ERR_INVALID;
//  - all calls share the one array and it keeps the previous call's partials:
//    nothing in it needs to start at zero, because every partial is written
//    before it is read; calls whose executions overlap on the GPU (different
//    streams, or different host threads) race on it and must be serialised by
//    the caller;
//  - the first call on a device looks up the array's device address (with
//    that device current) and caches it; make that first call before any
//    stream capture begins;
//  - the current device must be the one `in` and `out` live on (checked:
//    TC_ERR_INVALID otherwise), and `stream` must belong to it;
//  - the sums are bitwise those of the regular `sum` over axis 0 launch
//    (tcb_reduce_cols + tcb_reduce_finish) for the same matrix when cols > 1;
//    a single column is reduced there as a row (tcb_reduce_rows), in another
//    order.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/tcb200.h"

namespace tcb_detail {
int fail_msg(int status, const std::string& msg);
}

#define TC_COLSUM_STATIC_MAX_FLOATS (1u << 22)

static __device__ __align__(256) float tcb_colsum_scratch[TC_COLSUM_STATIC_MAX_FLOATS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_addr[kMaxDevices] = {nullptr};

// The per-column arithmetic of the NVRTC template tcb/reduce.cuh (tcb_reduce_cols +
// tcb_reduce_finish), operation for operation, so that both entry points give bitwise the
// same sums: chunk s of the rows is summed first to last (four loads in flight), then the
// chunk partials are combined by 8 warps -- warp w takes chunks w, w + 8, w + 16, ... in
// order -- and the 8 warp results are added in warp order.  With one chunk the column sums
// go straight to `out`, as the template's do.
__global__ void __launch_bounds__(256) colsum_partial(const float* __restrict__ x, float* __restrict__ dst,
                                                      uint64_t rows, uint64_t cols, uint64_t chunk) {
  const uint64_t s = blockIdx.y;
  const uint64_t k0 = s * chunk;
  const uint64_t k1 = k0 + chunk < rows ? k0 + chunk : rows;
  for (uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; j < cols; j += (uint64_t)gridDim.x * blockDim.x) {
    const float* p = x + j;
    float acc = 0.0f;
    uint64_t k = k0;
    for (; k + 4 <= k1; k += 4) {
      float v0 = __ldg(p + (k + 0) * cols), v1 = __ldg(p + (k + 1) * cols);
      float v2 = __ldg(p + (k + 2) * cols), v3 = __ldg(p + (k + 3) * cols);
      acc = __fadd_rn(acc, v0); acc = __fadd_rn(acc, v1);
      acc = __fadd_rn(acc, v2); acc = __fadd_rn(acc, v3);
    }
    for (; k < k1; ++k) acc = __fadd_rn(acc, __ldg(p + k * cols));
    dst[s * cols + j] = acc;
  }
}

__global__ void __launch_bounds__(256) colsum_finish(const float* __restrict__ part, float* __restrict__ out,
                                                     uint64_t cols, uint64_t split) {
  __shared__ float acc_w[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (uint64_t base = (uint64_t)blockIdx.x * 32; base < cols; base += (uint64_t)gridDim.x * 32) {
    const uint64_t j = base + lane;
    float acc = 0.0f;
    if (j < cols) {
      uint64_t s = w;
      for (; s + 24 < split; s += 32) {
        const float v0 = part[s * cols + j], v1 = part[(s + 8) * cols + j];
        const float v2 = part[(s + 16) * cols + j], v3 = part[(s + 24) * cols + j];
        acc = __fadd_rn(acc, v0); acc = __fadd_rn(acc, v1);
        acc = __fadd_rn(acc, v2); acc = __fadd_rn(acc, v3);
      }
      for (; s < split; s += 8) acc = __fadd_rn(acc, part[s * cols + j]);
    }
    acc_w[w][lane] = acc;
    __syncthreads();
    if (w == 0 && j < cols) {
      float r = acc_w[0][lane];
#pragma unroll
      for (int k = 1; k < 8; ++k) r = __fadd_rn(r, acc_w[k][lane]);
      out[j] = r;
    }
    __syncthreads();
  }
}

// The device a pointer's memory lives on, or -1 when it is not device (or managed) memory.
int device_of(uint64_t ptr) {
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, reinterpret_cast<const void*>(ptr));
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // not a pointer the runtime knows: clear the error it recorded
    return -1;
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) return -1;
  return attr.device;
}

int scratch_for_current_device(uint64_t in, uint64_t out, float** scratch) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return tcb_detail::fail_msg(TC_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return tcb_detail::fail_msg(TC_ERR_INVALID, "device ordinal out of range");
  // the scratch address belongs to the current device: the operands must live there too
  const int din = device_of(in), dout = device_of(out);
  if (din != dev || dout != dev)
    return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_colsum_f32_static: input on device " + std::to_string(din) +
                                                    ", output on device " + std::to_string(dout) +
                                                    ", current device " + std::to_string(dev) +
                                                    " (-1: not device memory); make the operands' device current");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, tcb_colsum_scratch);
    if (e != cudaSuccess)
      return tcb_detail::fail_msg(TC_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_addr[dev] = static_cast<float*>(p);
  }
  *scratch = g_addr[dev];
  return TC_OK;
}

}  // namespace

extern "C" int tc_colsum_f32_static(uint64_t in, uint64_t out, uint64_t rows, uint64_t cols, uint64_t stream) {
  if (!in || !out) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_colsum_f32_static: null input or output");
  if (rows == 0 || cols == 0) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_colsum_f32_static: empty matrix");
  if (cols > TC_COLSUM_STATIC_MAX_FLOATS)
    return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_colsum_f32_static: " + std::to_string(cols) +
                                                    " columns is above the static scratch maximum of " +
                                                    std::to_string(TC_COLSUM_STATIC_MAX_FLOATS));
  float* scratch = nullptr;
  if (int s = scratch_for_current_device(in, out, &scratch)) return s;
  // the split policy of the NVRTC path (codegen._reduce_source: at most 65535 chunks, the grid's y
  // limit), capped by the array's capacity -- a cap the policy never reaches, since it keeps
  // split x cols near 148 x 2048
  const uint64_t sm = 148;
  uint64_t split = 1;
  if (cols < 2 * sm * 256 && rows >= 64) {
    uint64_t a = (rows + 31) / 32, b = (sm * 2048 + cols - 1) / cols;
    split = a < b ? a : b;
    if (split > 65535) split = 65535;
    if (split < 1) split = 1;
  }
  const uint64_t cap = TC_COLSUM_STATIC_MAX_FLOATS / cols;
  if (split > cap) split = cap;
  const uint64_t chunk = (rows + split - 1) / split;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const uint64_t gx = (cols + 255) / 256 < sm * 8 ? (cols + 255) / 256 : sm * 8;
  float* dst = split > 1 ? scratch : reinterpret_cast<float*>(out);
  colsum_partial<<<dim3((unsigned)gx, (unsigned)split, 1), 256, 0, st>>>(reinterpret_cast<const float*>(in), dst,
                                                                          rows, cols, chunk);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return tcb_detail::fail_msg(TC_ERR_CUDA, std::string("tc_colsum_f32_static: partial sums launch: ") +
                                                 cudaGetErrorString(e));
  if (split > 1) {
    const uint64_t fx = (cols + 31) / 32 < sm * 8 ? (cols + 31) / 32 : sm * 8;
    colsum_finish<<<dim3((unsigned)fx, 1, 1), 256, 0, st>>>(scratch, reinterpret_cast<float*>(out), cols, split);
    e = cudaGetLastError();
    if (e != cudaSuccess)
      return tcb_detail::fail_msg(TC_ERR_CUDA, std::string("tc_colsum_f32_static: finishing launch: ") +
                                                   cudaGetErrorString(e));
  }
  return TC_OK;
}
