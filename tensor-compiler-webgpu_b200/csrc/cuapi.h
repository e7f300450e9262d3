// The CUDA driver API, resolved at run time (dlopen of libcuda.so.1).
//
// libtcb200 links no driver library, so it loads on a machine without a GPU
// driver (where tc_compile_check still works: NVRTC needs no device) and
// tc_open reports TC_ERR_UNAVAILABLE there instead of the loader failing.
// Each entry is looked up under the versioned name cuda.h maps it to.
#pragma once
#include <cuda.h>
#include <dlfcn.h>

#define TCB_CU_FUNCS(X)                                                                                   \
  X(cuCtxGetCurrent) X(cuCtxSetCurrent) X(cuDeviceGet) X(cuDeviceGetAttribute) X(cuDeviceGetCount)        \
  X(cuDeviceGetName) X(cuDevicePrimaryCtxRelease) X(cuDevicePrimaryCtxRetain) X(cuDeviceTotalMem)         \
  X(cuDriverGetVersion) X(cuEventCreate) X(cuEventDestroy) X(cuEventElapsedTime) X(cuEventQuery)          \
  X(cuEventRecord) X(cuEventSynchronize) X(cuFuncSetAttribute) X(cuGetErrorName) X(cuGraphDestroy)        \
  X(cuGraphExecDestroy) X(cuGraphInstantiate) X(cuGraphLaunch) X(cuInit) X(cuLaunchKernel) X(cuLaunchKernelEx) X(cuMemAlloc) \
  X(cuMemFree) X(cuMemFreeHost) X(cuMemHostAlloc) X(cuMemcpyDtoDAsync) X(cuMemcpyDtoHAsync)              \
  X(cuMemcpyHtoDAsync) X(cuMemsetD32Async) X(cuModuleGetFunction) X(cuModuleLoadData) X(cuModuleUnload)  \
  X(cuStreamBeginCapture) X(cuStreamCreate) X(cuStreamDestroy) X(cuStreamEndCapture)                      \
  X(cuStreamSynchronize) X(cuTensorMapEncodeTiled) X(cuStreamWaitEvent) X(cuStreamCreateWithPriority)     \
  X(cuCtxGetStreamPriorityRange)

#define TCB_STR2(x) #x
#define TCB_STR(x) TCB_STR2(x)

struct TcbCuApi {
#define TCB_DECL(fn) decltype(&fn) p_##fn = nullptr;
  TCB_CU_FUNCS(TCB_DECL)
#undef TCB_DECL
  bool ok = false;
};

inline TcbCuApi& tcb_cu() {
  static TcbCuApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      bool all = true;
#define TCB_LOAD(fn)                                                            \
  api.p_##fn = reinterpret_cast<decltype(api.p_##fn)>(dlsym(h, TCB_STR(fn)));   \
  if (!api.p_##fn) all = false;
      TCB_CU_FUNCS(TCB_LOAD)
#undef TCB_LOAD
      api.ok = all;
    }
  }
  return api;
}

// A driver that is missing reads as CUDA_ERROR_NOT_INITIALIZED from every call.
template <class F, class... A>
inline CUresult tcb_cu_call(F f, A... a) {
  return f ? f(a...) : CUDA_ERROR_NOT_INITIALIZED;
}
#define CU(fn) [&](auto... a_) { return tcb_cu_call(tcb_cu().p_##fn, a_...); }
