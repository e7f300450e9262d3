// Data-parallel collectives for libtcb200 (declared in include/tcb200.h).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2: the copy the host
// framework already loaded if any, else the system one), so the library
// links and loads without it.  Communicators are non-blocking
// (ncclConfig_t.blocking = 0): every wait is a poll of
// ncclCommGetAsyncError with a deadline, and a deadline that passes aborts
// the communicator and returns TC_ERR_TIMEOUT instead of hanging.
#include <cuda.h>
#include <dlfcn.h>
#include <nccl.h>

#include "cuapi.h"

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>

#include "../../include/tcb200.h"

namespace tcb_detail {
int fail_msg(int status, const std::string& msg);
CUcontext ctx_of(tc_ctx* ctx);
CUstream stream_of(tc_ctx* ctx);
}  // namespace tcb_detail

namespace {

struct Nccl {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*RedOpCreatePreMulSum)(ncclRedOp_t*, void*, ncclDataType_t, ncclScalarResidence_t, ncclComm_t) = nullptr;
  ncclResult_t (*RedOpDestroy)(ncclRedOp_t, ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

Nccl* nccl() {
  static Nccl n;
  static bool tried = false;
  if (tried) return n.h ? &n : nullptr;
  tried = true;
  const char* env = getenv("TCB_NCCL_LIBRARY");
  n.h = dlopen(env && *env ? env : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!n.h) return nullptr;
#define LOAD(field, sym) n.field = reinterpret_cast<decltype(n.field)>(dlsym(n.h, sym))
  LOAD(GetUniqueId, "ncclGetUniqueId");
  LOAD(CommInitRankConfig, "ncclCommInitRankConfig");
  LOAD(CommGetAsyncError, "ncclCommGetAsyncError");
  LOAD(AllReduce, "ncclAllReduce");
  LOAD(RedOpCreatePreMulSum, "ncclRedOpCreatePreMulSum");
  LOAD(RedOpDestroy, "ncclRedOpDestroy");
  LOAD(CommAbort, "ncclCommAbort");
  LOAD(CommDestroy, "ncclCommDestroy");
  LOAD(CommFinalize, "ncclCommFinalize");
  LOAD(GetErrorString, "ncclGetErrorString");
#undef LOAD
  if (!n.GetUniqueId || !n.CommInitRankConfig || !n.CommGetAsyncError || !n.AllReduce || !n.CommAbort ||
      !n.CommDestroy || !n.GetErrorString) {
    dlclose(n.h);
    n.h = nullptr;
    return nullptr;
  }
  return &n;
}

int fail(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  return tcb_detail::fail_msg(status, buf);
}

}  // namespace

struct tc_comm {
  tc_ctx* ctx = nullptr;
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  bool aborted = false;
};

static int wait_ready(tc_comm* c, int timeout_ms, const char* what) {
  Nccl* n = nccl();
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = n->CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return fail(TC_ERR_NCCL, "%s: ncclCommGetAsyncError: %s", what, n->GetErrorString(r));
    if (st == ncclSuccess) return TC_OK;
    if (st != ncclInProgress) {
      n->CommAbort(c->comm);
      c->aborted = true;
      return fail(TC_ERR_NCCL, "%s: %s", what, n->GetErrorString(st));
    }
    double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) {
      n->CommAbort(c->comm);
      c->aborted = true;
      return fail(TC_ERR_TIMEOUT, "%s: not complete after %d ms; communicator aborted", what, timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

extern "C" {

int tc_comm_unique_id(char id[128]) {
  Nccl* n = nccl();
  if (!n) return fail(TC_ERR_UNAVAILABLE, "NCCL could not be loaded (libnccl.so.2)");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId uid;
  ncclResult_t r = n->GetUniqueId(&uid);
  if (r != ncclSuccess) return fail(TC_ERR_NCCL, "ncclGetUniqueId: %s", n->GetErrorString(r));
  memcpy(id, &uid, 128);
  return TC_OK;
}

int tc_comm_init(tc_ctx* ctx, int rank, int world, const char id[128], int timeout_ms, tc_comm** out) {
  if (!ctx || !id || !out) return fail(TC_ERR_INVALID, "null argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return fail(TC_ERR_INVALID, "rank %d of world %d", rank, world);
  Nccl* n = nccl();
  if (!n) return fail(TC_ERR_UNAVAILABLE, "NCCL could not be loaded (libnccl.so.2)");
  if (CU(cuCtxSetCurrent)(tcb_detail::ctx_of(ctx)) != CUDA_SUCCESS) return fail(TC_ERR_CUDA, "cuCtxSetCurrent");
  auto* c = new tc_comm();
  c->ctx = ctx;
  c->rank = rank;
  c->world = world;
  ncclUniqueId uid;
  memcpy(&uid, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = n->CommInitRankConfig(&c->comm, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return fail(TC_ERR_NCCL, "ncclCommInitRankConfig: %s", n->GetErrorString(r));
  }
  if (int s = wait_ready(c, timeout_ms, "communicator init")) {
    if (c->comm) n->CommDestroy(c->comm);
    delete c;
    return s;
  }
  *out = c;
  return TC_OK;
}

int tc_allreduce_f32_on(tc_comm* c, uint64_t buf, uint64_t count, float scale, uint64_t stream) {
  if (!c) return fail(TC_ERR_INVALID, "null communicator");
  if (c->aborted) return fail(TC_ERR_NCCL, "communicator was aborted");
  Nccl* n = nccl();
  if (CU(cuCtxSetCurrent)(tcb_detail::ctx_of(c->ctx)) != CUDA_SUCCESS) return fail(TC_ERR_CUDA, "cuCtxSetCurrent");
  cudaStream_t st = stream ? (cudaStream_t)(uintptr_t)stream : (cudaStream_t)tcb_detail::stream_of(c->ctx);
  ncclRedOp_t op = ncclSum;
  bool custom = false;
  if (scale != 1.0f) {
    if (!n->RedOpCreatePreMulSum) return fail(TC_ERR_UNAVAILABLE, "ncclRedOpCreatePreMulSum missing");
    ncclResult_t r = n->RedOpCreatePreMulSum(&op, &scale, ncclFloat32, ncclScalarHostImmediate, c->comm);
    if (r == ncclInProgress) { if (int s = wait_ready(c, 60000, "op create")) return s; r = ncclSuccess; }
    if (r != ncclSuccess) return fail(TC_ERR_NCCL, "ncclRedOpCreatePreMulSum: %s", n->GetErrorString(r));
    custom = true;
  }
  ncclResult_t r = n->AllReduce((const void*)buf, (void*)buf, count, ncclFloat32, op, c->comm, st);
  if (r == ncclInProgress) { if (int s = wait_ready(c, 60000, "allreduce enqueue")) return s; r = ncclSuccess; }
  if (custom && n->RedOpDestroy) n->RedOpDestroy(op, c->comm);
  if (r != ncclSuccess) return fail(TC_ERR_NCCL, "ncclAllReduce: %s", n->GetErrorString(r));
  return TC_OK;
}

int tc_allreduce_f32(tc_comm* c, uint64_t buf, uint64_t count, float scale) {
  return tc_allreduce_f32_on(c, buf, count, scale, 0);
}

int tc_comm_wait(tc_comm* c, int timeout_ms) {
  if (!c) return fail(TC_ERR_INVALID, "null communicator");
  Nccl* n = nccl();
  if (CU(cuCtxSetCurrent)(tcb_detail::ctx_of(c->ctx)) != CUDA_SUCCESS) return fail(TC_ERR_CUDA, "cuCtxSetCurrent");
  CUevent ev;
  if (CU(cuEventCreate)(&ev, CU_EVENT_DISABLE_TIMING) != CUDA_SUCCESS) return fail(TC_ERR_CUDA, "cuEventCreate");
  CU(cuEventRecord)(ev, tcb_detail::stream_of(c->ctx));
  auto t0 = std::chrono::steady_clock::now();
  int status = TC_OK;
  for (;;) {
    CUresult q = CU(cuEventQuery)(ev);
    if (q == CUDA_SUCCESS) break;
    if (q != CUDA_ERROR_NOT_READY) { status = fail(TC_ERR_CUDA, "stream error while waiting for a collective"); break; }
    ncclResult_t st = ncclSuccess;
    n->CommGetAsyncError(c->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      n->CommAbort(c->comm);
      c->aborted = true;
      status = fail(TC_ERR_NCCL, "collective failed: %s", n->GetErrorString(st));
      break;
    }
    double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) {
      n->CommAbort(c->comm);
      c->aborted = true;
      status = fail(TC_ERR_TIMEOUT, "collective not complete after %d ms; communicator aborted", timeout_ms);
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  CU(cuEventDestroy)(ev);
  return status;
}

int tc_comm_abort(tc_comm* c) {
  if (!c) return TC_OK;
  Nccl* n = nccl();
  if (!c->aborted && n) n->CommAbort(c->comm);
  c->aborted = true;
  return TC_OK;
}

int tc_comm_destroy(tc_comm* c) {
  if (!c) return TC_OK;
  Nccl* n = nccl();
  if (n && c->comm) {
    if (c->aborted) { /* an aborted communicator is already released */ }
    else {
      if (n->CommFinalize) {
        ncclResult_t r = n->CommFinalize(c->comm);
        if (r == ncclInProgress || r == ncclSuccess) wait_ready(c, 30000, "finalize");
      }
      if (!c->aborted) n->CommDestroy(c->comm);
    }
  }
  delete c;
  return TC_OK;
}

}  // extern "C"
