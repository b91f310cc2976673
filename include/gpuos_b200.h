/* gpuos_b200.h — C ABI of the B200 aggregated small-op executor.
 *
 * Plain C types only (no torch, no C++): a caller that cannot link C++ (cgo,
 * JNI, ctypes, N-API) binds these symbols directly.  Every entry point
 * returns a status (0 = success, negative = error; gpuos_last_error() gives
 * the message of the calling thread's last failure) instead of terminating
 * the process the way the reference does (pytorch_ext/gpuos_ext.cpp:32-58).
 *
 * Each declaration names the reference interface it replaces.  Reference
 * paths are relative to the Multi-V-VM/GPUOS repository.
 */
#ifndef GPUOS_B200_H
#define GPUOS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GPUOS_ABI_VERSION 1

/* status codes */
#define GPUOS_OK 0
#define GPUOS_EINVAL (-1)       /* bad argument (shape, dtype, slot, ...) */
#define GPUOS_ECUDA (-2)        /* CUDA runtime / driver error */
#define GPUOS_ETIMEOUT (-3)     /* a bounded wait expired */
#define GPUOS_ESTATE (-4)       /* executor not initialised / shut down */
#define GPUOS_EUNSUPPORTED (-5) /* feature not available (e.g. JIT without NVRTC) */
#define GPUOS_EDEVICE (-6)      /* a batch reported an error on the device */
#define GPUOS_ENVRTC (-7)       /* NVRTC compilation failed */

/* dtype codes: the reference's DType enum (src/common.h:14-20) */
#define GPUOS_F32 0
#define GPUOS_F16 1
#define GPUOS_BF16 2

/* execution modes */
#define GPUOS_MODE_PERSISTENT 0 /* resident worker grid fed through a mapped doorbell */
#define GPUOS_MODE_STREAM 1     /* one kernel per batch on the caller's CUDA stream */

/* builtin operator codes accepted by gpuos_submit_builtin: the op codes of the
 * reference's op_batch switch (src/persistent_kernel.cu:101-106) */
#define GPUOS_OP_ADD 0
#define GPUOS_OP_MUL 1
#define GPUOS_OP_SUB 2
#define GPUOS_OP_DIV 3 /* B == 0 gives 0, as op_batch does */

/* A strided tensor view: element strides, up to 8 dims.  Same layout as the
 * reference's TensorRef (src/common.h:25-31). */
typedef struct gpuos_tensor {
  void* data;
  int32_t dtype;
  int32_t ndim;
  int64_t sizes[8];
  int64_t strides[8];
} gpuos_tensor;

typedef struct gpuos_executor gpuos_executor;

typedef struct gpuos_options {
  int32_t capacity;          /* queue capacity in requests; sizes the staging arena
                                (reference: init(capacity), gpuos_ext.cpp:328-339) */
  int32_t threads_per_block; /* worker CTA size (reference default 256, gpuos_ext.cpp:863) */
  int32_t mode;              /* GPUOS_MODE_* */
  int32_t blocks_per_sm;     /* 0 = from the occupancy calculator */
  double idle_ms;            /* persistent worker exits after this long idle (0 = default) */
  double sync_timeout_s;     /* bound on every host wait (0 = default) */
  int32_t max_batch;         /* requests per batch (reference GPUOS_BATCH_SHARD, default 512) */
  int32_t wait_limit_us;     /* bound of every wait inside a kernel, in microseconds (a stage
                                barrier, an earlier batch); on expiry the batch completes with
                                an error.  0 = default: sync_timeout_s clamped to [1, 10] s.
                                (The reference's waits are unbounded.) */
  int32_t reserved[6];
} gpuos_options;

typedef struct gpuos_stats {
  uint64_t published;   /* batches published (reference: tail) */
  uint64_t staged;      /* batches staged on the device (reference: head) */
  uint64_t processed;   /* batches completed */
  uint64_t retired;     /* batches whose staging memory was reclaimed */
  uint64_t heartbeat;   /* idle polls of the worker's ingest CTA (reference g_heartbeat) */
  uint64_t requests;    /* requests submitted */
  uint64_t pending;     /* requests waiting for the next flush */
  uint64_t errors;      /* device-reported request errors */
  uint64_t relaunches;  /* persistent worker launches */
  uint64_t dev_ns;      /* device time of completed batches, ns: first CTA in -> last chunk
                           (persistent worker and lean batches) */
  uint64_t lean;        /* stream-mode batches run by the lean kernel (parameters only) */
  uint64_t chain;       /* stream-mode batches with stage barriers run on one cluster */
  int32_t capacity;
  int32_t max_batch;
  int32_t mode;
  int32_t worker_alive;
  int32_t quit;
  int32_t grid;
  int32_t block;
  int32_t device;
} gpuos_stats;

/* ABI version (reference: abi_version() -> 1, gpuos_ext.cpp:865). */
int32_t gpuos_abi_version(void);

/* Message of the calling thread's last failed call. */
const char* gpuos_last_error(void);

/* Create one executor on `device` (replaces init(): gpuos_ext.cpp:328-382 and
 * launch_init_builtin_ops / launch_persistent_worker, persistent_kernel.cu:203-213).
 * opt may be NULL for defaults. */
int32_t gpuos_executor_create(int32_t device, const gpuos_options* opt, gpuos_executor** out);

/* Drain every published batch, stop the worker, free everything
 * (replaces shutdown(): gpuos_ext.cpp:384-421). */
int32_t gpuos_executor_destroy(gpuos_executor* ex);

/* Queue out = a <op> b with op in GPUOS_OP_* (replaces submit_add / submit_mul /
 * submit_sub / submit_div: gpuos_ext.cpp:459-493).  Broadcasting follows
 * torch: right-aligned, size-1 dims repeat. */
int32_t gpuos_submit_builtin(gpuos_executor* ex, int32_t op, const gpuos_tensor* a,
                             const gpuos_tensor* b, const gpuos_tensor* out);

/* Queue a request through jump-table slot `slot` (replaces submit_unary /
 * submit_binary: gpuos_ext.cpp:695-707).  The slot is resolved when the
 * request is flushed, so a hot swap affects every request flushed after it. */
int32_t gpuos_submit_unary(gpuos_executor* ex, int32_t slot, const gpuos_tensor* a,
                           const gpuos_tensor* out);
int32_t gpuos_submit_binary(gpuos_executor* ex, int32_t slot, const gpuos_tensor* a,
                            const gpuos_tensor* b, const gpuos_tensor* out);

/* Queue a request of `nin` (1 to 4) inputs ins[0..nin-1] through slot `slot`:
 * out = expr(A, B, C, D).  No counterpart in the reference, whose requests
 * carry at most two inputs (src/common.h:34-46); it lets a chain of
 * elementwise ops composed into one expression (a fused chain of the
 * scheduler) run as one request.  The slot's arity must equal nin. */
int32_t gpuos_submit_nary(gpuos_executor* ex, int32_t slot, int32_t nin,
                          const gpuos_tensor* ins, const gpuos_tensor* out);

/* Register an fp32 expression over A (and B) and return its slot (replaces
 * register_elementwise: gpuos_ext.cpp:681-692).  The expressions the
 * reference scheduler emits map onto precompiled operators; any other
 * expression is compiled with NVRTC for sm_100a.  Arity 3 and 4 (operands C
 * and D, for gpuos_submit_nary) go beyond the reference's 1 and 2.  Custom
 * expressions may call gpuos_keep_f32 / gpuos_keep_f16 / gpuos_keep_bf16(x):
 * the value x has once stored in that dtype, with the rounding of a separate
 * operation (no contraction into the operation that consumes it). */
int32_t gpuos_register_elementwise(gpuos_executor* ex, const char* key, const char* expr,
                                   int32_t arity, int32_t* slot_out);

/* Register "sum" or "mean" and return its slot (replaces register_reduce:
 * gpuos_ext.cpp:814-825, 847-849). */
int32_t gpuos_register_reduce(gpuos_executor* ex, const char* key, const char* op_name,
                              int32_t* slot_out);

/* Queue a sum/mean of x over `axes` into out (replaces submit_reduce:
 * gpuos_ext.cpp:827-856). */
int32_t gpuos_submit_reduce(gpuos_executor* ex, int32_t slot, const gpuos_tensor* x,
                            const gpuos_tensor* out, const int32_t* axes, int32_t naxes,
                            int32_t keepdim);

/* Queue one request given in the reference's 496-byte Task layout
 * (src/common.h:34-46): op is a jump-table slot, in0/in1/out0 are TensorRefs
 * whose sizes/strides are already aligned to the output. */
int32_t gpuos_submit_task(gpuos_executor* ex, const void* task);

/* Publish every queued request as one or more batches.  `stream` is the
 * cudaStream_t the inputs were produced on (NULL: the legacy default stream,
 * as everywhere in CUDA).  In
 * stream mode the batches run on that stream; in persistent mode the host
 * waits for that stream before ringing the doorbell.  With sync != 0 the call
 * returns after the batches are done (replaces flush(sync):
 * gpuos_ext.cpp:496-622; the wait is bounded and polls mapped memory
 * instead of sleeping 5 ms between device reads). *ticket_out (optional)
 * receives a ticket for gpuos_wait. */
int32_t gpuos_flush(gpuos_executor* ex, int32_t sync, void* stream, uint64_t* ticket_out);

/* Wait until every batch published before `ticket` is done. */
int32_t gpuos_wait(gpuos_executor* ex, uint64_t ticket, double timeout_s);

/* Dual-slot hot swap: route logical slot to physical slot (replaces
 * gpu_set_alias_async, persistent_kernel.cu:224-226). */
int32_t gpuos_set_alias(gpuos_executor* ex, int32_t logical, int32_t physical);

/* Online hot swap: overwrite what a physical slot runs (replaces
 * gpu_set_op_table_async, persistent_kernel.cu:220-222; takes an operator
 * id instead of a raw device function pointer).  In persistent mode the
 * worker resolves a slot request from its device copy of the table when it
 * starts the request, so a swap reaches batches already published but not yet
 * started, as in the reference; in stream mode a request's slot is resolved
 * when it is flushed. */
int32_t gpuos_set_slot(gpuos_executor* ex, int32_t slot, int32_t variant, float p0, float p1);

/* The reference's hot-swap entry points under their own names, for programs
 * ported from its tests (gpu_set_op_table_async / gpu_set_alias_async,
 * src/persistent_kernel.cu:220-226).  They act on the executor most recently
 * created on the calling thread's current device.  `fn` is an operator id
 * (gpuos_variant_by_name, or the operator a registered slot holds, from
 * gpuos_get_slot) where the reference takes a device function pointer, as
 * gpuos_set_slot does.  The table is published before the call returns, so
 * `stream` is not used.  Return 0 (cudaSuccess), or 1 (cudaErrorInvalidValue)
 * with the message in gpuos_last_error(). */
int32_t gpu_set_op_table_async(int32_t index, uint64_t fn, void* stream);
int32_t gpu_set_alias_async(int32_t logical_id, int32_t physical_slot, void* stream);

/* Read a slot (variant id, parameters) and the alias of a logical slot. */
int32_t gpuos_get_slot(gpuos_executor* ex, int32_t slot, int32_t* variant, float* p0, float* p1,
                       int32_t* alias);

/* Operator id of a builtin by name ("add", "gelu", "sum", ...), or -1. */
int32_t gpuos_variant_by_name(const char* name);

/* Per-launch timing of the batch kernel in stream mode: with timing on, a
 * CUDA event pair brackets every launch; gpuos_take_timings waits for them,
 * writes up to `cap` durations in milliseconds and returns the count in
 * *n_out.  (No counterpart in the reference, which has no kernel timing.) */
int32_t gpuos_set_timing(gpuos_executor* ex, int32_t on);
int32_t gpuos_take_timings(gpuos_executor* ex, float* ms, uint64_t cap, uint64_t* n_out);

/* Fault injection for tests of the bounded waits (no counterpart in the
 * reference, whose waits are unbounded): the next batch published with stage
 * barriers gets one stage wait that no chunk can meet.  The kernel's bounded
 * wait runs out after wait_limit_us, the batch records a stage-timeout error
 * and completes, and the next synchronous flush or wait returns
 * GPUOS_EDEVICE.  The executor stays usable. */
int32_t gpuos_debug_stall_next_batch(gpuos_executor* ex);

/* Worker control (replaces gpu_set_yield_every_async / gpu_set_debug_level_async,
 * persistent_kernel.cu:232-238, and worker_alive(), gpuos_ext.cpp:128-135). */
int32_t gpuos_set_yield_every(gpuos_executor* ex, uint64_t every);
int32_t gpuos_set_debug_level(gpuos_executor* ex, int32_t level);
int32_t gpuos_worker_alive(gpuos_executor* ex);

/* How the executor lays out one request, without running it (no GPU
 * needed): the 128-byte request record (layout: gpuos_b200/csrc/gpuos_abi.h,
 * struct Req), its chunk count and scratch needs.  Planning is the host half
 * of build_binary_task / build_reduce_task (gpuos_ext.cpp:167-201, 827-845). */
typedef struct gpuos_plan {
  uint8_t record[128];
  uint32_t nchunk;
  uint32_t has_ext;
  uint64_t partials; /* floats of reduction scratch */
  uint64_t counters; /* combine counters */
} gpuos_plan;

int32_t gpuos_plan_elementwise(int32_t variant, float p0, float p1, const gpuos_tensor* a,
                               const gpuos_tensor* b, const gpuos_tensor* out, gpuos_plan* plan);
int32_t gpuos_plan_reduce(int32_t variant, const gpuos_tensor* x, const gpuos_tensor* out,
                          const int32_t* axes, int32_t naxes, int32_t keepdim, gpuos_plan* plan);

/* ---- multi-process sharing ------------------------------------------------
 * No counterpart in the reference, which gives every process its own
 * persistent kernel and executor (benchmarks/bench_mps.py:54-92).  One server
 * per GPU owns an executor and a device pool exported with CUDA IPC; client
 * processes place their tensors in the pool (each in its own region) and
 * write requests into their own ring in POSIX shared memory "/<name>".  The
 * server drains every ring into the one executor, so requests of different
 * processes share batches.  A client waits on its own flushes only.  A client
 * process must finish the GPU work that produced its inputs before it
 * flushes (the Python client synchronizes its current stream), and it may
 * read results after a synchronous flush returns.  device < 0 creates a
 * server in record mode: no GPU, no pool, requests are counted and every
 * flush completes at once (protocol tests without a GPU). */
typedef struct gpuos_ipc_server gpuos_ipc_server;
typedef struct gpuos_ipc_client gpuos_ipc_client;

int32_t gpuos_ipc_server_create(const char* name, int32_t device, uint64_t pool_bytes,
                                int32_t max_clients, int32_t ring_entries,
                                const gpuos_options* opt, gpuos_ipc_server** out);
/* Stops the server thread, drains and shuts down the executor, frees the pool
 * and removes the shared memory name; clients still connected see their waits
 * end with GPUOS_ESTATE and must not use their pool mappings any more. */
int32_t gpuos_ipc_server_destroy(gpuos_ipc_server* s);
int32_t gpuos_ipc_server_stats(gpuos_ipc_server* s, uint64_t* requests, uint64_t* client_flushes,
                               uint64_t* launch_flushes, int32_t* clients);

/* Take a free client slot of server `name`; map its pool on the server's
 * device.  Waits of this client give up after timeout_s (0: 60 s). */
int32_t gpuos_ipc_connect(const char* name, double timeout_s, gpuos_ipc_client** out);
/* Flush, wait for this client's requests, release the slot and the mapping. */
int32_t gpuos_ipc_disconnect(gpuos_ipc_client* c);
/* The pool as this process sees it, this client's region of it, the device. */
int32_t gpuos_ipc_pool(gpuos_ipc_client* c, void** base, uint64_t* bytes, uint64_t* region_off,
                       uint64_t* region_bytes, int32_t* device);
/* The submission calls of the executor, over tensors in the pool. */
int32_t gpuos_ipc_submit_builtin(gpuos_ipc_client* c, int32_t op, const gpuos_tensor* a,
                                 const gpuos_tensor* b, const gpuos_tensor* out);
int32_t gpuos_ipc_submit_slot(gpuos_ipc_client* c, int32_t slot, int32_t nin,
                              const gpuos_tensor* ins, const gpuos_tensor* out);
int32_t gpuos_ipc_submit_reduce(gpuos_ipc_client* c, int32_t slot, const gpuos_tensor* x,
                                const gpuos_tensor* out, const int32_t* axes, int32_t naxes,
                                int32_t keepdim);
/* Publish a flush marker; sync: wait for this client's requests before it and
 * raise the first error the server met in them. */
int32_t gpuos_ipc_flush(gpuos_ipc_client* c, int32_t sync);
/* kind 1: register_elementwise(key, expr, arity); kind 2: register_reduce(key,
 * op_name in expr), run by the server; the slot is the server executor's. */
int32_t gpuos_ipc_register(gpuos_ipc_client* c, int32_t kind, const char* key, const char* expr,
                           int32_t arity, int32_t* slot_out);

/* Compile a custom expression with NVRTC only, to check it (no GPU needed):
 * GPUOS_OK, GPUOS_ENVRTC with the compiler log in gpuos_last_error(), or
 * GPUOS_EUNSUPPORTED when NVRTC is not installed (replaces the compile step of
 * ensure_elementwise_registered: gpuos_ext.cpp:625-692). */
int32_t gpuos_jit_check(const char* expr, int32_t arity);

/* Which precompiled operator (and parameters) an expression string of the
 * reference scheduler maps to; *variant = -1 when it needs NVRTC. */
int32_t gpuos_match_expression(const char* expr, int32_t arity, int32_t* variant, float* p0,
                               float* p1);

/* Counters (replaces peek_queue(), gpuos_ext.cpp:435-456, and
 * gpu_get_processed_count_async / gpu_get_heartbeat_async,
 * persistent_kernel.cu:216-230). */
int32_t gpuos_get_stats(gpuos_executor* ex, gpuos_stats* out);

/* Sum (variant = the "sum" operator) or mean ("mean") over the last dimension
 * of the row-major tensor x[rows, cols] (row i at x + i * row_stride elements)
 * into out[rows], on `stream` (a cudaStream_t; NULL = the legacy stream), for
 * callers that cannot allocate device memory.  No counterpart in the
 * reference.  It allocates nothing: rows longer than 8192 columns are split
 * into segments whose partial sums use a 1 MiB static device array that every
 * GPU loading this library holds until exit, so a call may split at most
 * 65,536 rows into at most 196,608 (row, segment) pairs; larger calls return
 * GPUOS_EINVAL.  The first call on a device (the current one) looks the array
 * up once per device, so make it before any stream capture.  All calls share
 * the array: calls that overlap on the GPU race.  Results are those of
 * gpuos_submit_reduce on the same input. */
int32_t gpuos_reduce_rows_noalloc(int32_t variant, const void* x, int32_t x_dtype, int64_t rows,
                                  int64_t cols, int64_t row_stride, void* out, int32_t out_dtype,
                                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GPUOS_B200_H */
