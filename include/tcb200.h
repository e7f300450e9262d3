/*
 * tcb200.h -- the C ABI of the B200 backend for the compiler's fused-kernel hot path.
 *
 * This is the whole boundary between a host (the reference's JavaScript via a
 * koffi/N-API binding, or this repository's Python/ctypes host) and the GPU.
 * It replaces what the reference's src/gpu layer does through WebGPU: device
 * creation, buffers, shader compilation, dispatch, readback and the
 * persistent training loop.  Plain C types only: pointers, sizes, handles.
 *
 * Conventions
 *  - Every call returns a tc_status; on failure tc_last_error() gives a
 *    thread-local message (the reference throws exceptions carrying it:
 *    src/gpu/runtime.js:61,114-115).
 *  - A context owns one device's primary CUDA context and one stream.  Calls
 *    on one context are not thread-safe; use one context per thread.
 *  - Device addresses are uint64_t; stream handles are uint64_t (a CUstream).
 *  - Kernels are CUDA C++ source text instantiated from the library's own
 *    sm_100a templates (the library registers them with NVRTC as headers
 *    "tcb/elementwise.cuh", "tcb/rowwise.cuh", "tcb/reduce.cuh",
 *    "tcb/matmul.cuh", "tcb/common.cuh").
 */
#ifndef TCB200_H
#define TCB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tc_status {
  TC_OK = 0,
  TC_ERR_INVALID = 1,      /* bad argument or launch geometry, found on the host */
  TC_ERR_CUDA = 2,         /* a CUDA driver call failed */
  TC_ERR_COMPILE = 3,      /* NVRTC rejected the source; the log is returned */
  TC_ERR_OOM = 4,          /* device allocation failed */
  TC_ERR_TIMEOUT = 5,      /* a bounded wait ran out */
  TC_ERR_NCCL = 6,         /* a collective failed or was aborted */
  TC_ERR_UNAVAILABLE = 7   /* a dependency (NCCL) could not be loaded */
} tc_status;

typedef struct tc_ctx tc_ctx;
typedef struct tc_buf tc_buf;
typedef struct tc_module tc_module;
typedef struct tc_plan tc_plan;
typedef struct tc_comm tc_comm;

/* Kernel argument block shared by every template: operand pointers, the
 * output, scratch, and up to 16 integer parameters.  Passed by value. */
#define TC_MAX_OPERANDS 8
#define TC_MAX_PARAMS 16
typedef struct tc_args {
  uint64_t in[TC_MAX_OPERANDS];
  uint64_t out;
  uint64_t scratch;
  int64_t p[TC_MAX_PARAMS];
} tc_args;

/* ---- errors, version ---- */
const char* tc_last_error(void);
int tc_version(void);

/* ---- device / context: GpuRunner.create() and .info()
 *      (src/gpu/runtime.js:17-25, :33-41) ---- */
int tc_open(int device_ordinal, tc_ctx** out);
int tc_close(tc_ctx* ctx);
int tc_info(tc_ctx* ctx, char* json, size_t cap);
int tc_get_stream(tc_ctx* ctx, uint64_t* stream);
/* Launch on an external stream (e.g. the host framework's current stream); 0 restores the context's own. */
int tc_set_stream(tc_ctx* ctx, uint64_t stream);

/* ---- buffers: createBuffer / writeBuffer / mapAsync readback and the
 *      canary padding of GpuRunner.run (src/gpu/runtime.js:12,64-83,116-125) ---- */
int tc_alloc(tc_ctx* ctx, uint64_t bytes, uint64_t canary_bytes, tc_buf** out);
int tc_free(tc_buf* buf);
int tc_buf_ptr(tc_buf* buf, uint64_t* dptr);
int tc_upload(tc_buf* buf, const void* host, uint64_t bytes, uint64_t offset);
int tc_download(tc_buf* buf, void* host, uint64_t bytes, uint64_t offset);
int tc_check_canary(tc_buf* buf, int* intact);
/* Raw device-address forms (async on the context's stream; host memory should be pinned for overlap). */
int tc_memcpy_htod(tc_ctx* ctx, uint64_t dst, const void* host, uint64_t bytes);
int tc_memcpy_dtoh(tc_ctx* ctx, void* host, uint64_t src, uint64_t bytes);
int tc_memcpy_dtod(tc_ctx* ctx, uint64_t dst, uint64_t src, uint64_t bytes);
int tc_memset32(tc_ctx* ctx, uint64_t dst, uint32_t value, uint64_t count);
int tc_host_alloc(uint64_t bytes, void** out);   /* page-locked host memory */
int tc_host_free(void* p);

/* ---- kernels: GpuRunner.pipeline(code), cached by source text
 *      (src/gpu/runtime.js:44-52) -- here NVRTC for sm_100a, cached by a hash of the source ---- */
int tc_compile(tc_ctx* ctx, const char* cuda_src, tc_module** out, char* log, size_t log_cap);
/* Compile only (no device needed): NVRTC for sm_100a; *cubin_bytes gets the image size. */
int tc_compile_check(const char* cuda_src, char* log, size_t log_cap, uint64_t* cubin_bytes);
/* Compile to a cubin image in caller memory (no device needed); with out == NULL only the size is returned. */
int tc_compile_cubin(const char* cuda_src, void* out, uint64_t cap, uint64_t* cubin_bytes, char* log, size_t log_cap);
/* A hash of the sm_100a templates compiled into this library: part of any on-disk kernel cache key, so
 * a cubin built against other template text is never reused. */
uint64_t tc_templates_hash(void);
/* Load a cubin made by tc_compile_cubin (e.g. from an on-disk kernel cache). */
int tc_module_load(tc_ctx* ctx, const void* cubin, uint64_t bytes, tc_module** out);
int tc_module_free(tc_module* mod);
/* One dispatch (runtime.js:86-101's setPipeline/setBindGroup/dispatchWorkgroups). */
int tc_launch(tc_module* mod, const char* kernel, const uint32_t grid[3], const uint32_t block[3],
              uint32_t smem_bytes, const tc_args* args);
/* A dispatch of a TMA-fed kernel: up to 5 fp32 tensor maps (zero fill out
 * of bounds) are built from 8 values each -- (address, cols, rows, batches,
 * row_stride_bytes, batch_stride_bytes, box_cols, box_rows) -- and passed,
 * 64-byte aligned, in five map slots before the tc_args block.  The address must be 16-byte
 * aligned, the strides multiples of 16 bytes, box_cols * 4 one of 128, 64 or
 * 32 bytes (the swizzle width: 128B, 64B or 32B), box_rows at most 256.
 * Bit 32 of box_cols (with 32 floats in its low bits) asks for the 128-byte
 * swizzle of 32-byte chunks instead: the shared-memory layout the tensor cores
 * read an MN-major tf32 operand tile in. */
int tc_launch_tma(tc_module* mod, const char* kernel, const uint32_t grid[3], const uint32_t block[3],
                  uint32_t smem_bytes, int n_maps, const uint64_t* map_desc /* 8 per map */,
                  const tc_args* args);

/* ---- extra streams (pipelining copies against compute): handles are CUstreams ---- */
int tc_stream_create(tc_ctx* ctx, uint64_t* stream);
int tc_stream_destroy(tc_ctx* ctx, uint64_t stream);
int tc_memcpy_htod_on(tc_ctx* ctx, uint64_t dst, const void* host, uint64_t bytes, uint64_t stream);
int tc_memcpy_dtoh_on(tc_ctx* ctx, void* host, uint64_t src, uint64_t bytes, uint64_t stream);
int tc_event_record_on(tc_ctx* ctx, uint64_t ev, uint64_t stream);
int tc_stream_wait_event(tc_ctx* ctx, uint64_t stream, uint64_t ev);
int tc_event_sync(uint64_t ev, int timeout_ms);    /* bounded wait for an event; TC_ERR_TIMEOUT when it runs out */

/* ---- synchronisation and timing ---- */
int tc_sync(tc_ctx* ctx, int timeout_ms);          /* TC_ERR_TIMEOUT when the wait runs out */
int tc_event_create(tc_ctx* ctx, uint64_t* ev);
int tc_event_record(tc_ctx* ctx, uint64_t ev);
int tc_event_elapsed_ms(uint64_t start, uint64_t end, float* ms);
int tc_event_destroy(uint64_t ev);

/* ---- plans: the persistent step of GpuTrainer / FusedTrainer
 *      (src/gpu/trainer.js:33-73, src/fusion/trainer-fused.js:148-185): a launch
 *      list with resolved addresses, replayed without host work, optionally
 *      as one CUDA graph ---- */
int tc_plan_create(tc_ctx* ctx, tc_plan** out);
int tc_plan_add_launch(tc_plan* plan, tc_module* mod, const char* kernel, const uint32_t grid[3],
                       const uint32_t block[3], uint32_t smem_bytes, const tc_args* args);
int tc_plan_add_launch_tma(tc_plan* plan, tc_module* mod, const char* kernel, const uint32_t grid[3],
                           const uint32_t block[3], uint32_t smem_bytes, int n_maps, const uint64_t* map_desc,
                           const tc_args* args);
int tc_plan_add_copy(tc_plan* plan, uint64_t dst, uint64_t src, uint64_t bytes);
/* A sum-allreduce of `count` floats at `buf` (scaled by `scale`) over `comm`, ordered after every entry
 * before it but run on the plan's own high-priority collective stream, so the entries after it compute
 * while it runs: the data-parallel step's gradient buckets, each reduced as soon as the backward has
 * written it.  The reference has no collective; this replaces the one allreduce that otherwise runs
 * between the gradient and Adam programs.  The plan's end waits for every collective it issued. */
int tc_plan_add_allreduce(tc_plan* plan, tc_comm* comm, uint64_t buf, uint64_t count, float scale);
int tc_plan_run(tc_plan* plan);                    /* every entry, in order, on the context's stream */
int tc_plan_run_on(tc_plan* plan, uint64_t stream);  /* the same on another stream of the context */
int tc_plan_capture(tc_plan* plan);                /* later runs replay one CUDA graph per segment between
                                                      allreduce entries; the collectives stay outside them */
int tc_plan_launch_count(tc_plan* plan, int* n);
int tc_plan_free(tc_plan* plan);

/* ---- memory planning for a step's arena: interval best-fit over
 *      (bytes, first_use, last_use) lifetimes; offsets are 256-byte aligned ---- */
int tc_plan_memory(int n, const uint64_t* bytes, const int32_t* first_use, const int32_t* last_use,
                   uint64_t* offsets, uint64_t* total);

/* ---- lowering from a graph, with no host language in between: lower() (src/gpu/lower.js:68-114),
 *      lowerFused() (src/fusion/lower-fused.js:32-45) and fusedKernel()
 *      (src/fusion/codegen-fused.js:357-362).  `graph_json` is the reference's Graph.toJSON form
 *      ({"nodes": [{op, inputs, attrs, shape}]}, src/ir/graph.js:48-50); with "fused" true it may hold
 *      the fusion pass's fused nodes (attrs {kind, pattern, body, output}, src/fusion/fuse.js:278-279).
 *      `opts_json` (NULL = defaults): {"fused": true (lowerFused; false: lower), "matmul": "naive" |
 *      "tiled" (the tcgen05 3xTF32 GEMM where K >= 32), "sabotage": one of the reference's
 *      FUSED_SABOTAGE names or null, "fold": false (transposes read only as GEMM operands get no launch,
 *      and a GEMM read only by a transpose computes the transposed product in its place),
 *      "colfuse": false (sums over axis 0, and over the last axis of at least 1184 rows, run inside
 *      their elementwise producer), "mofuse": false (an
 *      elementwise reader whose other operands already exist is computed in its elementwise producer's
 *      pass, both stored), "keep": [node ids that must exist after the launches]}.  No device is needed.  Each launch's CUDA source, kernel calls
 *      (grid, block, shared memory, parameters, tensor maps, error word) and scratch are those the
 *      repository's Python host makes, character for character. ---- */
typedef struct tc_lowered tc_lowered;
int tc_lower_json(const char* graph_json, const char* opts_json, tc_lowered** out);
int tc_lowered_count(tc_lowered* l, int* n);
/* The launch records as JSON ({"launches": [{node, nodes?, op, kind, pattern, inputs, code, scratch_bytes,
 * bytes, calls: [{name, grid, block, smem, params, err_offset, out_node, ptr_params, tma}], info}],
 * "folded": [...], "transposed": [[transpose id, matmul id], ...]}, the reference's {node, op, kind,
 * pattern, inputs, params, grid, code} record,
 * src/gpu/lower.js:108-111) into `json` (cap bytes); *needed = its size with the NUL.  json may be NULL. */
int tc_lowered_json(tc_lowered* l, char* json, uint64_t cap, uint64_t* needed);
int tc_lowered_free(tc_lowered* l);

/* GpuRunner.run (src/gpu/runtime.js:60-129) of a lowering: a buffer per node (canary-padded when
 * `canary`), the inputs and constants uploaded, every launch in order, every requested node read back.
 * inputs[i]: float32 host data of input node i (other entries ignored); values[i]: where node i's value
 * goes (NULL = not read; values itself may be NULL); canary_intact[i] (optional): 1 when node i's padding
 * is intact.  Arrays are indexed by node id.  Kernels come from the on-disk cache beside the library
 * ($TCB_KERNEL_CACHE overrides), compiled by NVRTC on a miss. */
int tc_lowered_run(tc_ctx* ctx, tc_lowered* l, const float* const* inputs, float* const* values, int canary,
                   int* canary_intact);

/* The resident program of GpuTrainer / FusedTrainer (src/gpu/trainer.js:13-104,
 * src/fusion/trainer-fused.js:135-213): inputs, constants, `keep` values and both ends of each
 * `feedback` pair (from, to: after the launches `from` is copied into `to`) own buffers, every other
 * value lives in one lifetime-planned arena, a plain reshape shares its source's memory, a launch nothing
 * kept or fed back depends on is left out; the launches and copies replay from one native plan (one CUDA
 * graph with `capture`).  The lowering must outlive the program. */
typedef struct tc_program tc_program;
int tc_program_create(tc_ctx* ctx, tc_lowered* l, const int32_t* keep, int n_keep, const int32_t* feedback,
                      int n_feedback, int capture, tc_program** out);
int tc_program_write(tc_program* p, int node, const float* host, uint64_t count);   /* synchronous */
int tc_program_read(tc_program* p, int node, float* host, uint64_t count);          /* synchronous */
int tc_program_run(tc_program* p);                                                   /* asynchronous */
int tc_program_check(tc_program* p);     /* TC_ERR_TIMEOUT if a launch's bounded wait ran out (syncs) */
int tc_program_ptr(tc_program* p, int node, uint64_t* dptr);
int tc_program_launch_count(tc_program* p, int* n);
int tc_program_free(tc_program* p);

/* ---- allocation-free column sum.  No counterpart in the reference: it exists for
 *      callers that cannot allocate device memory where they need the reduction (inside
 *      a stream capture, under another allocator's fixed budget, or on a path that
 *      cannot take cudaMalloc's device-wide synchronisation).
 *      out[j] = sum over i of in[i * cols + j] (the sum over axis 0 of a row-major
 *      [rows, cols] float32 matrix), partial sums kept in a library-owned 16 MiB
 *      static device array (held by every GPU that loads the library until exit).
 *      cols above 4,194,304 is rejected with TC_ERR_INVALID.  The array is shared by
 *      all calls and needs no clearing (every partial is written before it is read);
 *      calls that overlap on the GPU race on it.  The first call on a device looks up
 *      the array's address with that device current: make it before any stream
 *      capture.  The current device must be the one `in` and `out` live on (else
 *      TC_ERR_INVALID), and `stream` (a CUstream / cudaStream_t handle, 0 = legacy
 *      default) must belong to it.  For cols > 1 the sums are bitwise those of the
 *      regular `sum` over axis 0 launch of the same matrix. ---- */
int tc_colsum_f32_static(uint64_t in, uint64_t out, uint64_t rows, uint64_t cols, uint64_t stream);

/* ---- data-parallel collectives (NCCL, loaded at run time) ---- */
int tc_comm_unique_id(char id[128]);
int tc_comm_init(tc_ctx* ctx, int rank, int world, const char id[128], int timeout_ms, tc_comm** out);
/* Sum-allreduce `count` floats in place, then scale by `scale` (fused into the same stream). */
int tc_allreduce_f32(tc_comm* comm, uint64_t buf, uint64_t count, float scale);
/* The same on `stream` (a CUstream of the communicator's context; 0 = the context's stream). */
int tc_allreduce_f32_on(tc_comm* comm, uint64_t buf, uint64_t count, float scale, uint64_t stream);
int tc_comm_wait(tc_comm* comm, int timeout_ms);   /* bounded; aborts the communicator on timeout */
int tc_comm_abort(tc_comm* comm);
int tc_comm_destroy(tc_comm* comm);

#ifdef __cplusplus
}
#endif
#endif /* TCB200_H */
