// libtcb200: the C-ABI runtime of the B200 backend (declared in include/tcb200.h).
//
// CUDA driver API on the device's primary context (so pointers and streams
// interoperate with any runtime-API user of the same device), NVRTC for the
// per-fused-node kernels, NCCL loaded with dlopen for the data-parallel
// allreduce.  No call blocks without a bound; every failure is a status plus
// a thread-local message.
#include <cuda.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include "cuapi.h"

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/tcb200.h"
#include "tcb_templates.inc"  // generated: kTemplates[] = {name, text}

namespace {

thread_local std::string g_err;

int fail(int status, const char* fmt, ...) {
  char buf[2048];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return status;
}

const char* cu_name(CUresult r) {
  const char* s = nullptr;
  CU(cuGetErrorName)(r, &s);
  return s ? s : "CUDA_ERROR_UNKNOWN";
}

#define CU_TRY(call)                                                                 \
  do {                                                                               \
    CUresult _r = (call);                                                            \
    if (_r != CUDA_SUCCESS) {                                                        \
      if (_r == CUDA_ERROR_OUT_OF_MEMORY) return fail(TC_ERR_OOM, "%s: %s", #call, cu_name(_r)); \
      return fail(TC_ERR_CUDA, "%s: %s", #call, cu_name(_r));                       \
    }                                                                                \
  } while (0)

uint64_t fnv1a(const char* s, size_t n) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; i++) { h ^= (unsigned char)s[i]; h *= 1099511628211ull; }
  return h;
}

}  // namespace

struct tc_module {
  tc_ctx* ctx = nullptr;
  CUmodule mod = nullptr;
  std::map<std::string, CUfunction> fns;
  int refs = 1;
};

struct tc_ctx {
  int ordinal = 0;
  CUdevice dev = 0;
  CUcontext cu = nullptr;
  CUstream own_stream = nullptr;
  CUstream stream = nullptr;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  std::map<uint64_t, tc_module*> cache;  // source hash -> module
  std::map<uint64_t, std::string> cache_src;
};

struct tc_buf {
  tc_ctx* ctx = nullptr;
  CUdeviceptr ptr = 0;
  uint64_t bytes = 0;
  uint64_t canary = 0;
};

static const uint32_t kCanary = 0xdeadbeefu;

static int bind(tc_ctx* ctx) {
  if (!ctx) return fail(TC_ERR_INVALID, "null context");
  CU_TRY(CU(cuCtxSetCurrent)(ctx->cu));
  return TC_OK;
}

extern "C" {

const char* tc_last_error(void) { return g_err.c_str(); }

uint64_t tc_templates_hash(void) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < sizeof(kTemplates) / sizeof(kTemplates[0]); i++) {
    h ^= fnv1a(kTemplates[i].name, strlen(kTemplates[i].name));
    h *= 1099511628211ull;
    h ^= fnv1a(kTemplates[i].text, strlen(kTemplates[i].text));
    h *= 1099511628211ull;
  }
  return h;
}
int tc_version(void) { return 1; }

int tc_open(int device_ordinal, tc_ctx** out) {
  if (!out) return fail(TC_ERR_INVALID, "null out");
  *out = nullptr;
  if (!tcb_cu().ok) return fail(TC_ERR_UNAVAILABLE, "no CUDA driver: libcuda.so.1 could not be loaded");
  CU_TRY(CU(cuInit)(0));
  int n = 0;
  CU_TRY(CU(cuDeviceGetCount)(&n));
  if (device_ordinal < 0 || device_ordinal >= n)
    return fail(TC_ERR_INVALID, "device %d not present (%d devices)", device_ordinal, n);
  auto ctx = std::make_unique<tc_ctx>();
  ctx->ordinal = device_ordinal;
  CU_TRY(CU(cuDeviceGet)(&ctx->dev, device_ordinal));
  CU_TRY(CU(cuDevicePrimaryCtxRetain)(&ctx->cu, ctx->dev));
  CU_TRY(CU(cuCtxSetCurrent)(ctx->cu));
  CU_TRY(CU(cuDeviceGetAttribute)(&ctx->sm_count, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, ctx->dev));
  CU_TRY(CU(cuDeviceGetAttribute)(&ctx->cc_major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, ctx->dev));
  CU_TRY(CU(cuDeviceGetAttribute)(&ctx->cc_minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, ctx->dev));
  if (ctx->cc_major != 10 || ctx->cc_minor != 0) {
    CU(cuDevicePrimaryCtxRelease)(ctx->dev);
    return fail(TC_ERR_UNAVAILABLE, "device %d is sm_%d%d; this library is built for sm_100a only", device_ordinal,
                ctx->cc_major, ctx->cc_minor);
  }
  CU_TRY(CU(cuStreamCreate)(&ctx->own_stream, CU_STREAM_NON_BLOCKING));
  ctx->stream = ctx->own_stream;
  *out = ctx.release();
  return TC_OK;
}

int tc_close(tc_ctx* ctx) {
  if (!ctx) return TC_OK;
  CU(cuCtxSetCurrent)(ctx->cu);
  CU(cuStreamSynchronize)(ctx->stream);
  for (auto& kv : ctx->cache) {
    if (kv.second->mod) CU(cuModuleUnload)(kv.second->mod);
    delete kv.second;
  }
  if (ctx->own_stream) CU(cuStreamDestroy)(ctx->own_stream);
  CU(cuDevicePrimaryCtxRelease)(ctx->dev);
  delete ctx;
  return TC_OK;
}

int tc_info(tc_ctx* ctx, char* json, size_t cap) {
  if (int s = bind(ctx)) return s;
  char name[256] = {0};
  CU_TRY(CU(cuDeviceGetName)(name, sizeof name, ctx->dev));
  size_t mem = 0;
  CU_TRY(CU(cuDeviceTotalMem)(&mem, ctx->dev));
  int drv = 0;
  CU_TRY(CU(cuDriverGetVersion)(&drv));
  int smem_optin = 0, clock = 0, l2 = 0;
  CU(cuDeviceGetAttribute)(&smem_optin, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, ctx->dev);
  CU(cuDeviceGetAttribute)(&l2, CU_DEVICE_ATTRIBUTE_L2_CACHE_SIZE, ctx->dev);
  int nvrtc_major = 0, nvrtc_minor = 0;
  nvrtcVersion(&nvrtc_major, &nvrtc_minor);
  int n = snprintf(json, cap,
                   "{\"device\": \"%s\", \"ordinal\": %d, \"sm\": \"sm_%d%d\", \"sm_count\": %d, "
                   "\"memory_bytes\": %zu, \"l2_bytes\": %d, \"smem_optin_bytes\": %d, \"driver\": %d, "
                   "\"nvrtc\": \"%d.%d\", \"kernels_cached\": %zu}",
                   name, ctx->ordinal, ctx->cc_major, ctx->cc_minor, ctx->sm_count, mem, l2, smem_optin, drv,
                   nvrtc_major, nvrtc_minor, ctx->cache.size());
  (void)clock;
  if (n < 0 || (size_t)n >= cap) return fail(TC_ERR_INVALID, "info buffer too small");
  return TC_OK;
}

int tc_get_stream(tc_ctx* ctx, uint64_t* stream) {
  if (!ctx || !stream) return fail(TC_ERR_INVALID, "null argument");
  *stream = (uint64_t)(uintptr_t)ctx->stream;
  return TC_OK;
}

int tc_set_stream(tc_ctx* ctx, uint64_t stream) {
  if (!ctx) return fail(TC_ERR_INVALID, "null context");
  ctx->stream = stream ? (CUstream)(uintptr_t)stream : ctx->own_stream;
  return TC_OK;
}

// ---------------------------------------------------------------- buffers
int tc_alloc(tc_ctx* ctx, uint64_t bytes, uint64_t canary_bytes, tc_buf** out) {
  if (!out) return fail(TC_ERR_INVALID, "null out");
  *out = nullptr;
  if (int s = bind(ctx)) return s;
  canary_bytes = (canary_bytes + 3) / 4 * 4;
  uint64_t total = std::max<uint64_t>(4, (bytes + 3) / 4 * 4 + canary_bytes);
  auto b = std::make_unique<tc_buf>();
  b->ctx = ctx;
  b->bytes = bytes;
  b->canary = canary_bytes;
  CU_TRY(CU(cuMemAlloc)(&b->ptr, total));
  if (canary_bytes) {
    uint64_t off = (bytes + 3) / 4 * 4;
    CUresult r = CU(cuMemsetD32Async)(b->ptr + off, kCanary, canary_bytes / 4, ctx->stream);
    if (r != CUDA_SUCCESS) { CU(cuMemFree)(b->ptr); return fail(TC_ERR_CUDA, "canary fill: %s", cu_name(r)); }
    // the bytes between `bytes` and the 4-byte boundary keep the pattern too
    if (bytes % 4) {
      uint32_t w = kCanary;
      r = CU(cuMemcpyHtoDAsync)(b->ptr + bytes / 4 * 4, &w, 4, ctx->stream);
      if (r == CUDA_SUCCESS) r = CU(cuStreamSynchronize)(ctx->stream);
      if (r != CUDA_SUCCESS) { CU(cuMemFree)(b->ptr); return fail(TC_ERR_CUDA, "canary fill: %s", cu_name(r)); }
    }
  }
  *out = b.release();
  return TC_OK;
}

int tc_free(tc_buf* buf) {
  if (!buf) return TC_OK;
  CU(cuCtxSetCurrent)(buf->ctx->cu);
  CUresult r = CU(cuMemFree)(buf->ptr);
  delete buf;
  if (r != CUDA_SUCCESS) return fail(TC_ERR_CUDA, "cuMemFree: %s", cu_name(r));
  return TC_OK;
}

int tc_buf_ptr(tc_buf* buf, uint64_t* dptr) {
  if (!buf || !dptr) return fail(TC_ERR_INVALID, "null argument");
  *dptr = (uint64_t)buf->ptr;
  return TC_OK;
}

int tc_upload(tc_buf* buf, const void* host, uint64_t bytes, uint64_t offset) {
  if (!buf || (!host && bytes)) return fail(TC_ERR_INVALID, "null argument");
  if (offset + bytes > buf->bytes) return fail(TC_ERR_INVALID, "upload of %llu bytes at %llu past a %llu-byte buffer",
                                               (unsigned long long)bytes, (unsigned long long)offset,
                                               (unsigned long long)buf->bytes);
  if (int s = bind(buf->ctx)) return s;
  CU_TRY(CU(cuMemcpyHtoDAsync)(buf->ptr + offset, host, bytes, buf->ctx->stream));
  CU_TRY(CU(cuStreamSynchronize)(buf->ctx->stream));
  return TC_OK;
}

int tc_download(tc_buf* buf, void* host, uint64_t bytes, uint64_t offset) {
  if (!buf || (!host && bytes)) return fail(TC_ERR_INVALID, "null argument");
  if (offset + bytes > buf->bytes + buf->canary)
    return fail(TC_ERR_INVALID, "download past the end of the buffer");
  if (int s = bind(buf->ctx)) return s;
  CU_TRY(CU(cuMemcpyDtoHAsync)(host, buf->ptr + offset, bytes, buf->ctx->stream));
  CU_TRY(CU(cuStreamSynchronize)(buf->ctx->stream));
  return TC_OK;
}

int tc_check_canary(tc_buf* buf, int* intact) {
  if (!buf || !intact) return fail(TC_ERR_INVALID, "null argument");
  *intact = 1;
  if (!buf->canary && buf->bytes % 4 == 0) return TC_OK;
  if (int s = bind(buf->ctx)) return s;
  uint64_t start = buf->bytes / 4 * 4;
  uint64_t words = ((buf->bytes + 3) / 4 * 4 + buf->canary - start) / 4;
  std::vector<uint32_t> h(words);
  CU_TRY(CU(cuMemcpyDtoHAsync)(h.data(), buf->ptr + start, words * 4, buf->ctx->stream));
  CU_TRY(CU(cuStreamSynchronize)(buf->ctx->stream));
  for (uint64_t i = (buf->bytes % 4) ? 1 : 0; i < words; i++)
    if (h[i] != kCanary) { *intact = 0; break; }
  if (buf->bytes % 4) {  // the partial word: only its tail bytes are padding
    const unsigned char* p = (const unsigned char*)h.data();
    const unsigned char* c = (const unsigned char*)&kCanary;
    for (uint64_t k = buf->bytes % 4; k < 4; k++) if (p[k] != c[k]) *intact = 0;
  }
  return TC_OK;
}

int tc_memcpy_htod(tc_ctx* ctx, uint64_t dst, const void* host, uint64_t bytes) {
  if (int s = bind(ctx)) return s;
  if (bytes) CU_TRY(CU(cuMemcpyHtoDAsync)((CUdeviceptr)dst, host, bytes, ctx->stream));
  return TC_OK;
}

int tc_memcpy_dtoh(tc_ctx* ctx, void* host, uint64_t src, uint64_t bytes) {
  if (int s = bind(ctx)) return s;
  if (bytes) CU_TRY(CU(cuMemcpyDtoHAsync)(host, (CUdeviceptr)src, bytes, ctx->stream));
  return TC_OK;
}

int tc_memcpy_dtod(tc_ctx* ctx, uint64_t dst, uint64_t src, uint64_t bytes) {
  if (int s = bind(ctx)) return s;
  if (bytes) CU_TRY(CU(cuMemcpyDtoDAsync)((CUdeviceptr)dst, (CUdeviceptr)src, bytes, ctx->stream));
  return TC_OK;
}

int tc_memset32(tc_ctx* ctx, uint64_t dst, uint32_t value, uint64_t count) {
  if (int s = bind(ctx)) return s;
  if (count) CU_TRY(CU(cuMemsetD32Async)((CUdeviceptr)dst, value, count, ctx->stream));
  return TC_OK;
}

int tc_host_alloc(uint64_t bytes, void** out) {
  if (!out) return fail(TC_ERR_INVALID, "null out");
  CU_TRY(CU(cuInit)(0));
  CUcontext cur = nullptr;
  CU(cuCtxGetCurrent)(&cur);
  if (!cur) return fail(TC_ERR_INVALID, "tc_host_alloc needs an open context on this thread");
  CU_TRY(CU(cuMemHostAlloc)(out, std::max<uint64_t>(bytes, 1), CU_MEMHOSTALLOC_PORTABLE));
  return TC_OK;
}

int tc_host_free(void* p) {
  if (p) CU_TRY(CU(cuMemFreeHost)(p));
  return TC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- kernels
namespace {

struct TmaBlock {
  alignas(64) CUtensorMap maps[5];
  tc_args args;
};

int get_fn(tc_module* mod, const char* name, CUfunction* fn) {
  auto it = mod->fns.find(name);
  if (it != mod->fns.end()) { *fn = it->second; return TC_OK; }
  CUresult r = CU(cuModuleGetFunction)(fn, mod->mod, name);
  if (r != CUDA_SUCCESS) return fail(TC_ERR_INVALID, "kernel '%s' not in module: %s", name, cu_name(r));
  mod->fns[name] = *fn;
  return TC_OK;
}

int check_geometry(tc_ctx* ctx, const uint32_t grid[3], const uint32_t block[3], uint32_t smem) {
  (void)ctx;
  if (!grid || !block) return fail(TC_ERR_INVALID, "null grid or block");
  uint64_t threads = (uint64_t)block[0] * block[1] * block[2];
  if (threads == 0 || threads > 1024) return fail(TC_ERR_INVALID, "block of %llu threads", (unsigned long long)threads);
  if (grid[0] == 0 || grid[1] == 0 || grid[2] == 0) return fail(TC_ERR_INVALID, "empty grid");
  if (grid[1] > 65535 || grid[2] > 65535) return fail(TC_ERR_INVALID, "grid y/z above 65535");
  if (smem > 232448) return fail(TC_ERR_INVALID, "%u bytes of shared memory requested", smem);
  return TC_OK;
}

int prepare_smem(CUfunction fn, uint32_t smem) {
  if (smem > 48 * 1024) {
    CU_TRY(CU(cuFuncSetAttribute)(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem));
  }
  return TC_OK;
}

int encode_maps(int n_maps, const uint64_t* d, TmaBlock* blk) {
  if (n_maps < 0 || n_maps > 5) return fail(TC_ERR_INVALID, "%d tensor maps (at most 5)", n_maps);
  for (int m = 0; m < n_maps; m++) {
    const uint64_t* v = d + 8 * m;
    uint64_t addr = v[0], cols = v[1], rows = v[2], batches = v[3], rs = v[4], bs = v[5], bc = v[6] & 0xFFFFFFFFull,
             br = v[7];
    const bool atom32 = (v[6] >> 32) & 1;  // 128-byte swizzle of 32-byte chunks (MN-major tf32 tiles)
    if (atom32 && bc * 4 != 128) return fail(TC_ERR_INVALID, "tensor map %d: 32-byte-atom swizzle needs 128-byte rows", m);
    if (addr % 16) return fail(TC_ERR_INVALID, "tensor map %d: address not 16-byte aligned", m);
    if (rs % 16 || bs % 16) return fail(TC_ERR_INVALID, "tensor map %d: strides must be multiples of 16 bytes", m);
    if ((bc * 4 != 128 && bc * 4 != 64 && bc * 4 != 32) || br == 0 || br > 256)
      return fail(TC_ERR_INVALID, "tensor map %d: box of %llu x %llu floats", m, (unsigned long long)bc,
                  (unsigned long long)br);
    if (cols == 0 || rows == 0 || batches == 0) return fail(TC_ERR_INVALID, "tensor map %d: empty", m);
    cuuint64_t dims[3] = {cols, rows, batches};
    cuuint64_t strides[2] = {rs, bs};
    cuuint32_t box[3] = {(cuuint32_t)bc, (cuuint32_t)br, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    // the swizzle spans one box row: 128, 64 or 32 bytes
    CUtensorMapSwizzle sw = atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                            : bc * 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                            : bc * 4 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
    CUresult r = CU(cuTensorMapEncodeTiled)(&blk->maps[m], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)addr, dims, strides,
                                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TC_ERR_INVALID, "cuTensorMapEncodeTiled (map %d): %s", m, cu_name(r));
  }
  return TC_OK;
}

}  // namespace

extern "C" {

static int nvrtc_build(const char* src, char* log, size_t log_cap, std::vector<char>* cubin) {
  if (log && log_cap) log[0] = 0;
  std::vector<const char*> hdr_text, hdr_name;
  for (size_t i = 0; i < sizeof(kTemplates) / sizeof(kTemplates[0]); i++) {
    hdr_name.push_back(kTemplates[i].name);
    hdr_text.push_back(kTemplates[i].text);
  }
  nvrtcProgram prog;
  nvrtcResult nr = nvrtcCreateProgram(&prog, src, "tcb_kernel.cu", (int)hdr_text.size(), hdr_text.data(), hdr_name.data());
  if (nr != NVRTC_SUCCESS) return fail(TC_ERR_COMPILE, "nvrtcCreateProgram: %s", nvrtcGetErrorString(nr));
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-lineinfo", "--device-as-default-execution-space",
                        "-DTCB_NVRTC=1"};
  nr = nvrtcCompileProgram(prog, (int)(sizeof opts / sizeof opts[0]), opts);
  size_t log_size = 0;
  nvrtcGetProgramLogSize(prog, &log_size);
  std::string plog(log_size, '\0');
  if (log_size) nvrtcGetProgramLog(prog, &plog[0]);
  if (log && log_cap) {
    size_t n = std::min(log_cap - 1, plog.size());
    memcpy(log, plog.data(), n);
    log[n] = 0;
  }
  if (nr != NVRTC_SUCCESS) {
    nvrtcDestroyProgram(&prog);
    return fail(TC_ERR_COMPILE, "NVRTC: %s\n%s", nvrtcGetErrorString(nr), plog.c_str());
  }
  size_t cubin_size = 0;
  nvrtcGetCUBINSize(prog, &cubin_size);
  cubin->resize(cubin_size);
  nvrtcGetCUBIN(prog, cubin->data());
  nvrtcDestroyProgram(&prog);
  return TC_OK;
}

int tc_compile_check(const char* src, char* log, size_t log_cap, uint64_t* cubin_bytes) {
  if (!src) return fail(TC_ERR_INVALID, "null source");
  std::vector<char> cubin;
  if (int s = nvrtc_build(src, log, log_cap, &cubin)) return s;
  if (cubin_bytes) *cubin_bytes = cubin.size();
  return TC_OK;
}

int tc_compile_cubin(const char* src, void* out, uint64_t cap, uint64_t* cubin_bytes, char* log, size_t log_cap) {
  if (!src || !cubin_bytes) return fail(TC_ERR_INVALID, "null argument");
  std::vector<char> cubin;
  if (int s = nvrtc_build(src, log, log_cap, &cubin)) return s;
  *cubin_bytes = cubin.size();
  if (out) {
    if (cap < cubin.size()) return fail(TC_ERR_INVALID, "cubin buffer of %llu bytes, need %zu", (unsigned long long)cap,
                                        cubin.size());
    memcpy(out, cubin.data(), cubin.size());
  }
  return TC_OK;
}

int tc_module_load(tc_ctx* ctx, const void* cubin, uint64_t bytes, tc_module** out) {
  if (!cubin || !out || !bytes) return fail(TC_ERR_INVALID, "null argument");
  *out = nullptr;
  if (int s = bind(ctx)) return s;
  uint64_t h = fnv1a((const char*)cubin, (size_t)bytes) ^ 0x9e3779b97f4a7c15ull;
  auto it = ctx->cache.find(h);
  if (it != ctx->cache.end()) {
    it->second->refs++;
    *out = it->second;
    return TC_OK;
  }
  auto mod = std::make_unique<tc_module>();
  mod->ctx = ctx;
  CU_TRY(CU(cuModuleLoadData)(&mod->mod, cubin));
  mod->refs = 2;
  ctx->cache[h] = mod.get();
  ctx->cache_src[h] = std::string();
  *out = mod.release();
  return TC_OK;
}

int tc_compile(tc_ctx* ctx, const char* src, tc_module** out, char* log, size_t log_cap) {
  if (!out || !src) return fail(TC_ERR_INVALID, "null argument");
  *out = nullptr;
  if (int s = bind(ctx)) return s;
  size_t len = strlen(src);
  uint64_t h = fnv1a(src, len);
  auto it = ctx->cache.find(h);
  if (it != ctx->cache.end() && !ctx->cache_src[h].empty() && ctx->cache_src[h] == src) {
    it->second->refs++;
    *out = it->second;
    return TC_OK;
  }
  std::vector<char> cubin;
  if (int s = nvrtc_build(src, log, log_cap, &cubin)) return s;
  auto mod = std::make_unique<tc_module>();
  mod->ctx = ctx;
  CUresult r = CU(cuModuleLoadData)(&mod->mod, cubin.data());
  if (r != CUDA_SUCCESS) return fail(TC_ERR_CUDA, "cuModuleLoadData: %s", cu_name(r));
  mod->refs = 2;  // the cache's reference and the caller's
  ctx->cache[h] = mod.get();
  ctx->cache_src[h] = src;
  *out = mod.release();
  return TC_OK;
}

int tc_module_free(tc_module* mod) {
  if (!mod) return TC_OK;
  mod->refs--;  // the context's cache keeps the module until tc_close
  return TC_OK;
}

int tc_launch(tc_module* mod, const char* kernel, const uint32_t grid[3], const uint32_t block[3], uint32_t smem,
              const tc_args* args) {
  if (!mod || !kernel || !args) return fail(TC_ERR_INVALID, "null argument");
  if (int s = bind(mod->ctx)) return s;
  if (int s = check_geometry(mod->ctx, grid, block, smem)) return s;
  CUfunction fn;
  if (int s = get_fn(mod, kernel, &fn)) return s;
  if (int s = prepare_smem(fn, smem)) return s;
  tc_args a = *args;
  void* params[] = {&a};
  CU_TRY(CU(cuLaunchKernel)(fn, grid[0], grid[1], grid[2], block[0], block[1], block[2], smem, mod->ctx->stream, params,
                        nullptr));
  return TC_OK;
}

int tc_launch_tma(tc_module* mod, const char* kernel, const uint32_t grid[3], const uint32_t block[3], uint32_t smem,
                  int n_maps, const uint64_t* map_desc, const tc_args* args) {
  if (!mod || !kernel || !args || (n_maps && !map_desc)) return fail(TC_ERR_INVALID, "null argument");
  if (int s = bind(mod->ctx)) return s;
  if (int s = check_geometry(mod->ctx, grid, block, smem)) return s;
  CUfunction fn;
  if (int s = get_fn(mod, kernel, &fn)) return s;
  if (int s = prepare_smem(fn, smem)) return s;
  TmaBlock blk;
  memset(&blk, 0, sizeof blk);
  if (int s = encode_maps(n_maps, map_desc, &blk)) return s;
  blk.args = *args;
  void* params[] = {&blk};
  CU_TRY(CU(cuLaunchKernel)(fn, grid[0], grid[1], grid[2], block[0], block[1], block[2], smem, mod->ctx->stream, params,
                        nullptr));
  return TC_OK;
}

// ---------------------------------------------------------------- sync, events
int tc_sync(tc_ctx* ctx, int timeout_ms) {
  if (int s = bind(ctx)) return s;
  CUevent ev;
  CU_TRY(CU(cuEventCreate)(&ev, CU_EVENT_DISABLE_TIMING));
  CUresult r = CU(cuEventRecord)(ev, ctx->stream);
  if (r != CUDA_SUCCESS) { CU(cuEventDestroy)(ev); return fail(TC_ERR_CUDA, "cuEventRecord: %s", cu_name(r)); }
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    r = CU(cuEventQuery)(ev);
    if (r == CUDA_SUCCESS) break;
    if (r != CUDA_ERROR_NOT_READY) { CU(cuEventDestroy)(ev); return fail(TC_ERR_CUDA, "stream: %s", cu_name(r)); }
    double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) {
      CU(cuEventDestroy)(ev);
      return fail(TC_ERR_TIMEOUT, "stream not done after %d ms", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(ms < 5 ? 10 : 200));
  }
  CU(cuEventDestroy)(ev);
  return TC_OK;
}

int tc_stream_create(tc_ctx* ctx, uint64_t* stream) {
  if (!stream) return fail(TC_ERR_INVALID, "null out");
  if (int s = bind(ctx)) return s;
  CUstream st;
  CU_TRY(CU(cuStreamCreate)(&st, CU_STREAM_NON_BLOCKING));
  *stream = (uint64_t)(uintptr_t)st;
  return TC_OK;
}

int tc_stream_destroy(tc_ctx* ctx, uint64_t stream) {
  if (int s = bind(ctx)) return s;
  if (stream) CU_TRY(CU(cuStreamDestroy)((CUstream)(uintptr_t)stream));
  return TC_OK;
}

int tc_memcpy_htod_on(tc_ctx* ctx, uint64_t dst, const void* host, uint64_t bytes, uint64_t stream) {
  if (int s = bind(ctx)) return s;
  if (bytes) CU_TRY(CU(cuMemcpyHtoDAsync)((CUdeviceptr)dst, host, bytes, (CUstream)(uintptr_t)stream));
  return TC_OK;
}

int tc_memcpy_dtoh_on(tc_ctx* ctx, void* host, uint64_t src, uint64_t bytes, uint64_t stream) {
  if (int s = bind(ctx)) return s;
  if (bytes) CU_TRY(CU(cuMemcpyDtoHAsync)(host, (CUdeviceptr)src, bytes, (CUstream)(uintptr_t)stream));
  return TC_OK;
}

int tc_event_record_on(tc_ctx* ctx, uint64_t ev, uint64_t stream) {
  if (int s = bind(ctx)) return s;
  CU_TRY(CU(cuEventRecord)((CUevent)(uintptr_t)ev, (CUstream)(uintptr_t)stream));
  return TC_OK;
}

int tc_stream_wait_event(tc_ctx* ctx, uint64_t stream, uint64_t ev) {
  if (int s = bind(ctx)) return s;
  CU_TRY(CU(cuStreamWaitEvent)((CUstream)(uintptr_t)stream, (CUevent)(uintptr_t)ev, 0));
  return TC_OK;
}

int tc_event_sync(uint64_t ev, int timeout_ms) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    CUresult r = CU(cuEventQuery)((CUevent)(uintptr_t)ev);
    if (r == CUDA_SUCCESS) return TC_OK;
    if (r != CUDA_ERROR_NOT_READY) return fail(TC_ERR_CUDA, "event: %s", cu_name(r));
    double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) return fail(TC_ERR_TIMEOUT, "event not reached after %d ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(ms < 5 ? 10 : 200));
  }
}

int tc_event_create(tc_ctx* ctx, uint64_t* ev) {
  if (!ev) return fail(TC_ERR_INVALID, "null out");
  if (int s = bind(ctx)) return s;
  CUevent e;
  CU_TRY(CU(cuEventCreate)(&e, CU_EVENT_DEFAULT));
  *ev = (uint64_t)(uintptr_t)e;
  return TC_OK;
}

int tc_event_record(tc_ctx* ctx, uint64_t ev) {
  if (int s = bind(ctx)) return s;
  CU_TRY(CU(cuEventRecord)((CUevent)(uintptr_t)ev, ctx->stream));
  return TC_OK;
}

int tc_event_elapsed_ms(uint64_t start, uint64_t end, float* ms) {
  if (!ms) return fail(TC_ERR_INVALID, "null out");
  CU_TRY(CU(cuEventSynchronize)((CUevent)(uintptr_t)end));
  CU_TRY(CU(cuEventElapsedTime)(ms, (CUevent)(uintptr_t)start, (CUevent)(uintptr_t)end));
  return TC_OK;
}

int tc_event_destroy(uint64_t ev) {
  if (ev) CU_TRY(CU(cuEventDestroy)((CUevent)(uintptr_t)ev));
  return TC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- plans
struct tc_plan {
  tc_ctx* ctx = nullptr;
  struct Entry {
    int kind = 0;  // 0 launch, 1 launch with tensor maps, 2 copy, 3 sum-allreduce on the collective stream
    CUfunction fn = nullptr;
    uint32_t grid[3] = {1, 1, 1}, block[3] = {1, 1, 1}, smem = 0;
    tc_args args = {};
    std::shared_ptr<TmaBlock> tma;
    uint64_t dst = 0, src = 0, bytes = 0;   // a copy; an allreduce: dst = buffer, bytes = float count
    bool waits = false;   // a template kernel: it waits for its predecessor itself (grid_dependency_sync)
    tc_comm* comm = nullptr;
    float scale = 1.0f;
    CUevent ready = nullptr;  // an allreduce: recorded on the plan's stream, waited for by the collective stream
  };
  std::vector<Entry> entries;
  // Programmatic dependent launch between consecutive template kernels: $TCB_PDL=0 never, 1 always, 2 where
  // both grids fit in one wave (at most one CTA per SM), unset (the default, 3) where the kernel being
  // launched fits in one wave.  Measured on the B200: a chain of one-wave kernels (the C1 step) gains 9 %;
  // the transformer step, whose elementwise kernels fill the GPU, loses 6 % with every edge programmatic,
  // and gains 0.8 % at 64 sequences when its one-wave GEMMs start their set-up under the previous tail.
  int pdl = 3;
  // Captured form: one graph per segment between allreduce entries (a collective is never captured; it is
  // enqueued between the segments' graph launches).  Empty segments have none.
  bool captured = false;
  std::vector<CUgraph> graphs;
  std::vector<CUgraphExec> execs;
  // The collective stream (highest priority, created with the first allreduce entry) and the event the
  // plan's stream waits for at the plan's end, after its last collective.
  CUstream coll = nullptr;
  CUevent joined = nullptr;
};

extern "C" {

int tc_plan_create(tc_ctx* ctx, tc_plan** out) {
  if (!ctx || !out) return fail(TC_ERR_INVALID, "null argument");
  *out = new tc_plan();
  (*out)->ctx = ctx;
  const char* e = getenv("TCB_PDL");
  (*out)->pdl = e && e[0] == '0' ? 0 : e && e[0] == '1' ? 1 : e && e[0] == '2' ? 2 : 3;
  return TC_OK;
}

static int plan_add(tc_plan* plan, tc_module* mod, const char* kernel, const uint32_t grid[3], const uint32_t block[3],
                    uint32_t smem, int n_maps, const uint64_t* map_desc, const tc_args* args, bool tma) {
  if (!plan || !mod || !kernel || !args) return fail(TC_ERR_INVALID, "null argument");
  if (plan->captured) return fail(TC_ERR_INVALID, "plan already captured");
  if (int s = bind(plan->ctx)) return s;
  if (int s = check_geometry(plan->ctx, grid, block, smem)) return s;
  tc_plan::Entry e;
  if (int s = get_fn(mod, kernel, &e.fn)) return s;
  if (int s = prepare_smem(e.fn, smem)) return s;
  e.kind = tma ? 1 : 0;
  e.waits = strncmp(kernel, "tcb_", 4) == 0;
  for (int i = 0; i < 3; i++) { e.grid[i] = grid[i]; e.block[i] = block[i]; }
  e.smem = smem;
  e.args = *args;
  if (tma) {
    e.tma = std::make_shared<TmaBlock>();
    memset(e.tma.get(), 0, sizeof(TmaBlock));
    if (int s = encode_maps(n_maps, map_desc, e.tma.get())) return s;
    e.tma->args = *args;
  }
  plan->entries.push_back(e);
  return TC_OK;
}

int tc_plan_add_launch(tc_plan* plan, tc_module* mod, const char* kernel, const uint32_t grid[3],
                       const uint32_t block[3], uint32_t smem, const tc_args* args) {
  return plan_add(plan, mod, kernel, grid, block, smem, 0, nullptr, args, false);
}

int tc_plan_add_launch_tma(tc_plan* plan, tc_module* mod, const char* kernel, const uint32_t grid[3],
                           const uint32_t block[3], uint32_t smem, int n_maps, const uint64_t* map_desc,
                           const tc_args* args) {
  return plan_add(plan, mod, kernel, grid, block, smem, n_maps, map_desc, args, true);
}

int tc_plan_add_copy(tc_plan* plan, uint64_t dst, uint64_t src, uint64_t bytes) {
  if (!plan) return fail(TC_ERR_INVALID, "null plan");
  if (plan->captured) return fail(TC_ERR_INVALID, "plan already captured");
  tc_plan::Entry e;
  e.kind = 2;
  e.dst = dst; e.src = src; e.bytes = bytes;
  plan->entries.push_back(e);
  return TC_OK;
}

int tc_plan_add_allreduce(tc_plan* plan, tc_comm* comm, uint64_t buf, uint64_t count, float scale) {
  if (!plan || !comm) return fail(TC_ERR_INVALID, "null argument");
  if (plan->captured) return fail(TC_ERR_INVALID, "plan already captured");
  if (int s = bind(plan->ctx)) return s;
  if (!plan->coll) {
    int least = 0, greatest = 0;
    CU_TRY(CU(cuCtxGetStreamPriorityRange)(&least, &greatest));
    CU_TRY(CU(cuStreamCreateWithPriority)(&plan->coll, CU_STREAM_NON_BLOCKING, greatest));
    CU_TRY(CU(cuEventCreate)(&plan->joined, CU_EVENT_DISABLE_TIMING));
  }
  tc_plan::Entry e;
  e.kind = 3;
  e.comm = comm;
  e.dst = buf;
  e.bytes = count;
  e.scale = scale;
  CU_TRY(CU(cuEventCreate)(&e.ready, CU_EVENT_DISABLE_TIMING));
  plan->entries.push_back(e);
  return TC_OK;
}

// Entries [b, end) of one segment (kernels and copies) on `st`.  A template kernel that follows another
// kernel of the segment is launched with programmatic stream serialization (where the plan's policy
// allows it for the two grids): it may be scheduled while its predecessor drains, and waits for it
// (complete, writes visible) before touching memory.  A copy, a kernel that is not a template's, or the
// segment's first entry keeps the full ordering.
static int plan_issue(tc_plan* plan, size_t b, size_t end, CUstream st) {
  bool prev_kernel = false;
  uint64_t prev_ctas = 0;
  const uint64_t wave = (uint64_t)plan->ctx->sm_count;
  for (size_t i = b; i < end; i++) {
    auto& e = plan->entries[i];
    if (e.kind == 2) {
      if (e.bytes) CU_TRY(CU(cuMemcpyDtoDAsync)((CUdeviceptr)e.dst, (CUdeviceptr)e.src, e.bytes, st));
      prev_kernel = false;
      continue;
    }
    const uint64_t ctas = (uint64_t)e.grid[0] * e.grid[1] * e.grid[2];
    const bool pdl = plan->pdl == 1 || (plan->pdl == 2 && ctas <= wave && prev_ctas <= wave) ||
                     (plan->pdl == 3 && ctas <= wave);
    prev_ctas = ctas;
    void* params[1];
    tc_args a = e.args;
    if (e.kind == 1) params[0] = e.tma.get();
    else params[0] = &a;
    if (pdl && e.waits && prev_kernel) {
      CUlaunchAttribute attr[1];
      memset(attr, 0, sizeof attr);
      attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
      attr[0].value.programmaticStreamSerializationAllowed = 1;
      CUlaunchConfig cfg;
      memset(&cfg, 0, sizeof cfg);
      cfg.gridDimX = e.grid[0]; cfg.gridDimY = e.grid[1]; cfg.gridDimZ = e.grid[2];
      cfg.blockDimX = e.block[0]; cfg.blockDimY = e.block[1]; cfg.blockDimZ = e.block[2];
      cfg.sharedMemBytes = e.smem;
      cfg.hStream = st;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      CU_TRY(CU(cuLaunchKernelEx)(&cfg, e.fn, params, nullptr));
    } else {
      CU_TRY(CU(cuLaunchKernel)(e.fn, e.grid[0], e.grid[1], e.grid[2], e.block[0], e.block[1], e.block[2], e.smem, st,
                            params, nullptr));
    }
    prev_kernel = true;
  }
  return TC_OK;
}

// The segments of a plan: the runs of entries between its allreduce entries (possibly empty).
static std::vector<std::pair<size_t, size_t>> plan_segments(const tc_plan* plan) {
  std::vector<std::pair<size_t, size_t>> segs;
  size_t b = 0;
  for (size_t i = 0; i < plan->entries.size(); i++)
    if (plan->entries[i].kind == 3) { segs.push_back({b, i}); b = i + 1; }
  segs.push_back({b, plan->entries.size()});
  return segs;
}

// Segment by segment on the plan's stream; after segment k, allreduce entry k is enqueued on the
// collective stream behind an event of the plan's stream, so it runs while segment k+1 computes.  The
// plan's stream waits for the collective stream at the end: the next work on it sees every sum.
static int plan_run(tc_plan* plan) {
  CUstream st = plan->ctx->stream;
  auto segs = plan_segments(plan);
  for (size_t k = 0; k < segs.size(); k++) {
    if (plan->captured) {
      if (plan->execs[k]) CU_TRY(CU(cuGraphLaunch)(plan->execs[k], st));
    } else if (int s = plan_issue(plan, segs[k].first, segs[k].second, st)) {
      return s;
    }
    if (k + 1 == segs.size()) break;
    auto& c = plan->entries[segs[k].second];
    CU_TRY(CU(cuEventRecord)(c.ready, st));
    CU_TRY(CU(cuStreamWaitEvent)(plan->coll, c.ready, 0));
    if (int s = tc_allreduce_f32_on(c.comm, c.dst, c.bytes, c.scale, (uint64_t)(uintptr_t)plan->coll)) return s;
  }
  if (segs.size() > 1) {
    CU_TRY(CU(cuEventRecord)(plan->joined, plan->coll));
    CU_TRY(CU(cuStreamWaitEvent)(st, plan->joined, 0));
  }
  return TC_OK;
}

int tc_plan_run(tc_plan* plan) {
  if (!plan) return fail(TC_ERR_INVALID, "null plan");
  if (int s = bind(plan->ctx)) return s;
  return plan_run(plan);  // a captured plan's graphs replay on any stream of the context
}

int tc_plan_run_on(tc_plan* plan, uint64_t stream) {
  if (!plan) return fail(TC_ERR_INVALID, "null plan");
  CUstream saved = plan->ctx->stream;
  plan->ctx->stream = stream ? (CUstream)(uintptr_t)stream : plan->ctx->own_stream;
  int s = tc_plan_run(plan);
  plan->ctx->stream = saved;
  return s;
}

static void plan_drop_graphs(tc_plan* plan) {
  for (auto x : plan->execs) if (x) CU(cuGraphExecDestroy)(x);
  for (auto g : plan->graphs) if (g) CU(cuGraphDestroy)(g);
  plan->execs.clear();
  plan->graphs.clear();
}

int tc_plan_capture(tc_plan* plan) {
  if (!plan) return fail(TC_ERR_INVALID, "null plan");
  if (int s = bind(plan->ctx)) return s;
  if (plan->captured) return TC_OK;
  CUstream st = plan->ctx->stream;
  for (auto& seg : plan_segments(plan)) {
    CUgraph g = nullptr;
    CUgraphExec x = nullptr;
    if (seg.second > seg.first) {
      CU_TRY(CU(cuStreamBeginCapture)(st, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL));
      int s = plan_issue(plan, seg.first, seg.second, st);
      CUresult r = CU(cuStreamEndCapture)(st, &g);
      if (s) { if (g) CU(cuGraphDestroy)(g); plan_drop_graphs(plan); return s; }
      if (r != CUDA_SUCCESS) { plan_drop_graphs(plan); return fail(TC_ERR_CUDA, "cuStreamEndCapture: %s", cu_name(r)); }
      r = CU(cuGraphInstantiate)(&x, g, 0);
      if (r != CUDA_SUCCESS) {
        CU(cuGraphDestroy)(g);
        plan_drop_graphs(plan);
        return fail(TC_ERR_CUDA, "cuGraphInstantiate: %s", cu_name(r));
      }
    }
    plan->graphs.push_back(g);
    plan->execs.push_back(x);
  }
  plan->captured = true;
  return TC_OK;
}

int tc_plan_launch_count(tc_plan* plan, int* n) {
  if (!plan || !n) return fail(TC_ERR_INVALID, "null argument");
  int k = 0;
  for (auto& e : plan->entries) if (e.kind < 2) k++;
  *n = k;
  return TC_OK;
}

int tc_plan_free(tc_plan* plan) {
  if (!plan) return TC_OK;
  CU(cuCtxSetCurrent)(plan->ctx->cu);
  plan_drop_graphs(plan);
  for (auto& e : plan->entries) if (e.ready) CU(cuEventDestroy)(e.ready);
  if (plan->joined) CU(cuEventDestroy)(plan->joined);
  if (plan->coll) CU(cuStreamDestroy)(plan->coll);
  delete plan;
  return TC_OK;
}

// ---------------------------------------------------------------- arena planning
int tc_plan_memory(int n, const uint64_t* bytes, const int32_t* first_use, const int32_t* last_use, uint64_t* offsets,
                   uint64_t* total) {
  if (n < 0 || (n && (!bytes || !first_use || !last_use || !offsets)) || !total)
    return fail(TC_ERR_INVALID, "null argument");
  std::vector<int> order(n);
  for (int i = 0; i < n; i++) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return bytes[a] > bytes[b]; });
  struct Placed { uint64_t off, end; int first, last; };
  std::vector<Placed> placed;
  placed.reserve(n);
  uint64_t top = 0;
  for (int idx : order) {
    uint64_t sz = (std::max<uint64_t>(bytes[idx], 1) + 255) / 256 * 256;
    // candidate offsets: 0 and the end of every placed block whose lifetime overlaps
    std::vector<std::pair<uint64_t, uint64_t>> busy;
    for (auto& p : placed)
      if (!(p.last < first_use[idx] || last_use[idx] < p.first)) busy.push_back({p.off, p.end});
    std::sort(busy.begin(), busy.end());
    uint64_t best = UINT64_MAX, best_gap = UINT64_MAX, cur = 0;
    for (auto& b : busy) {
      if (b.first > cur && b.first - cur >= sz && b.first - cur < best_gap) { best = cur; best_gap = b.first - cur; }
      cur = std::max(cur, b.second);
    }
    if (best == UINT64_MAX) best = cur;
    offsets[idx] = best;
    placed.push_back({best, best + sz, first_use[idx], last_use[idx]});
    top = std::max(top, best + sz);
  }
  *total = top;
  return TC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- internal accessors for comm.cpp
namespace tcb_detail {
int fail_msg(int status, const std::string& msg) { g_err = msg; return status; }
CUcontext ctx_of(tc_ctx* ctx) { return ctx->cu; }
CUstream stream_of(tc_ctx* ctx) { return ctx->stream; }
}  // namespace tcb_detail
