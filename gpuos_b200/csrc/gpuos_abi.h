// Shared host/device layout of the aggregated small-op path.
//
// One *request* is one micro-op (an elementwise op or a sum/mean over the
// last dims) on tensors that already live in HBM.  Requests are gathered on
// the host into a *batch*: a header, an array of 128-byte request records,
// a prefix array of per-request chunk counts and (for general strided
// requests) extension records.  A batch is executed by warps that claim
// fixed-size chunks of work with one atomic each.
//
// This header is compiled by nvcc (device + host), by g++ (host runtime and
// oracle-free tests) and by NVRTC (the JIT executor).  It therefore uses no
// standard headers under NVRTC.
//
// Reference correspondence (Multi-V-VM/GPUOS):
//   Req          replaces the 496-byte Task of src/common.h:34-46 for the
//                work itself; the Task layout stays accepted at the C ABI.
//   DType codes  are the reference's (src/common.h:14-20).
//   Slot tables  replace g_op_table/g_op_alias (src/persistent_kernel.cu:10-11)
//                with variant ids instead of device function pointers.
#pragma once

#if defined(__CUDACC_RTC__)
typedef unsigned char      uint8_t;
typedef unsigned short     uint16_t;
typedef unsigned int       uint32_t;
typedef int                int32_t;
typedef long long          int64_t;
typedef unsigned long long uint64_t;
#else
#include <stdint.h>
#endif

namespace gpuos {

// dtype codes: same numbering as the reference DType enum (src/common.h:14-20)
enum DTypeCode : int { kF32 = 0, kF16 = 1, kBF16 = 2, kI32 = 3, kF64 = 4 };

// Builtin operator variants.  0..3 are the op codes that the reference's
// op_batch switch understands (persistent_kernel.cu:101-106); the rest are the
// expressions the reference scheduler compiles through NVRTC
// (pytorch_ext/scheduler.py:145-153, 192-205, 244-290).
enum Variant : int {
  V_ADD = 0, V_MUL = 1, V_SUB = 2, V_DIV0 = 3,   // op_batch codes; DIV0: B==0 -> 0
  V_DIV = 4, V_MAX = 5, V_MIN = 6, V_POW = 7,
  V_RELU = 8, V_SIGMOID = 9, V_TANH = 10, V_EXP = 11, V_LOG = 12, V_SQRT = 13,
  V_ABS = 14, V_HARDSIGMOID = 15, V_HARDSWISH = 16, V_GELU = 17, V_SIN = 18,
  V_COS = 19, V_LEAKY_RELU = 20, V_CLAMP = 21, V_ELU = 22, V_SOFTPLUS = 23,
  V_CLAMP_MIN = 24, V_CLAMP_MAX = 25, V_COPY = 26,
  V_NUM_EW = 27,
  V_SUM = 32, V_MEAN = 33,
  V_JIT_BASE = 64,        // custom expression k has variant V_JIT_BASE + k
  V_JIT_MAX = 64,         // at most 64 custom expressions per executor
  V_LIMIT = 128,
  V_NONE = -1
};

// request kinds
enum ReqKind : uint8_t { RK_EW = 0, RK_RED = 1 };

// elementwise layouts (chosen by the host after broadcasting + dim coalescing)
enum EwLayout : uint8_t {
  EL_CONTIG = 0,   // every operand contiguous over numel (or a scalar), out contiguous
  EL_ROW2D = 1,    // [rows, inner]; each operand: any row stride, inner stride 0 or 1
  EL_STRIDED = 2,  // general <= 8 dims through an extension record
  EL_TILE2D = 3,   // [rows, inner], output inner stride 1, operands with any row and inner
                   // strides (transposed views, [B,N] op [N] / [B,1] with N not a multiple
                   // of 4); a chunk is `chunk` columns of every row (rows in nseg)
};

// reduction layouts: input seen as [rows, cols], reduce over cols
enum RedLayout : uint8_t {
  RL_ROWS = 0,     // cols contiguous (stride 1), rows at a + r*row_stride
  RL_COLS = 1,     // rows adjacent (stride 1), cols at a + c*col_stride
  RL_GENERIC = 2,  // anything else, through an extension record
};

// request flags
enum ReqFlags : uint8_t {
  RF_HAS_B = 1,      // binary op
  RF_VEC = 2,        // 16-byte vector path legal (alignment + shape checked on host)
  RF_SLOT = 4,       // `op` is a jump-table slot resolved at execution time
  RF_A_SCALAR = 8,   // operand A is a single element broadcast everywhere
  RF_B_SCALAR = 16,  // operand B is a single element broadcast everywhere
  RF_BIG = 32,       // indices may exceed 2^31: use 64-bit index math
  RF_NARY = 64,      // operands C (and D) from the extension record: a custom
                     // expression of arity 3 or 4 (the general body only)
};

static constexpr int kMaxDims = 8;
static constexpr int kMaxSlots = 128;              // GPUOS_MAX_OPS (src/common.h:9-11)
static constexpr int kMaxReqPerBatch = 4096;       // chunk prefix fits 16 KB of smem
static constexpr int kWarpStep = 256;              // elements per warp step (8 per lane)

// 128-byte request record.
static constexpr uint16_t kOpNone = 0xffff;  // Req::op of a slot with no operator

struct alignas(16) Req {
  uint16_t op;           // variant id, or slot id if (flags & RF_SLOT); a published record
                         // always holds the variant (the host resolves the slot at flush),
                         // kOpNone when the slot names no operator
  uint8_t  kind;         // ReqKind
  uint8_t  layout;       // EwLayout or RedLayout
  uint8_t  dta, dtb, dto;
  uint8_t  flags;        // ReqFlags
  float    p0, p1;       // operator parameters (for RF_SLOT: taken from the slot at flush)
  // 16
  uint32_t chunk;        // EW: elements per chunk (a multiple of 4)
                         // RED: rows per chunk (nseg == 1) or columns per segment
  uint32_t nseg;         // RED: column segments per row group (1 = no combine)
  int64_t  numel;        // EW: output elements; RED: output rows
  // 32
  uint64_t a, b, o;      // device addresses
  // 56
  int64_t  inner;        // EW ROW2D: inner size N; RED: reduced length C
  // 64
  int64_t  sa_row, sb_row, so_row;   // row strides in elements
  // 88
  int64_t  sa_in, sb_in; // EW ROW2D: inner strides (0 or 1); RED: column stride in sa_in
  // 104
  uint32_t ext;          // byte offset of the extension record inside the batch
  uint32_t part;         // RED: float offset of this request's partials in batch scratch
  uint32_t cnt;          // RED: u32 offset of this request's counters in the counter pool
  uint32_t fdiv_m;       // fast division by `inner` (EW ROW2D) or by rows per group (RED)
  uint32_t fdiv_s;
  uint32_t rg;           // RED RL_COLS: rows per group (power of two <= 32)
};
static_assert(sizeof(Req) == 128, "Req must stay 128 bytes");

// Extension record for EL_STRIDED, RL_GENERIC and RF_NARY requests (placed
// after the records).
// EW: dims 0..ndim-1 of the output with per-operand element strides.
// RED: `ndim` outer (kept) dims followed by `rdim` reduced dims; sa holds the
//      input strides, so the output strides (output may be non-contiguous).
// RF_NARY: operands C and D (d == 0: none) with their strides in sc / sd:
//      EL_CONTIG sc[0] (0 or 1), EL_ROW2D sc[0] row and sc[1] inner stride,
//      EL_STRIDED sc[d] per dim.
struct alignas(16) ExtRec {
  int32_t ndim;
  int32_t rdim;
  int64_t sizes[kMaxDims];
  int64_t sa[kMaxDims];
  int64_t sb[kMaxDims];
  int64_t so[kMaxDims];
  union {
    int64_t rsizes[kMaxDims];
    int64_t sc[kMaxDims];
  };
  union {
    int64_t rstrides[kMaxDims];
    int64_t sd[kMaxDims];
  };
  uint64_t c, d;         // RF_NARY: device addresses of operands C and D
  int32_t dtc, dtd;      // and their dtypes
};
static_assert(sizeof(ExtRec) == 416, "ExtRec layout");

// Batch header at offset 0 of every batch payload.
struct alignas(16) BatchHdr {
  uint64_t seq;          // monotonically increasing batch sequence number
  uint32_t nreq;
  uint32_t nchunk;
  uint32_t rec_off;      // byte offset of Req[nreq]
  uint32_t cb_off;       // byte offset of uint32 chunk_base[nreq + 1]
  uint32_t bytes;        // payload bytes (header included)
  uint32_t flags;
  uint64_t scratch;      // device address of this batch's partials area (floats)
  uint64_t counters;     // device address of the counter pool (u32, self-cleaning)
  uint64_t wait_from;    // BF_AFTER_PREV: batches [wait_from, seq) must be done first
  uint32_t gtab_off;     // byte offset of uint32x2 gtab[ceil(nchunk / gran)]: the request
                         // that owns each granule's first chunk, and that request's
                         // first chunk
  uint32_t gran;         // chunks per granule (the unit a warp takes at a time)
};
static_assert(sizeof(BatchHdr) == 64, "BatchHdr must stay 64 bytes");

// Per-batch device-side counters: slot seq % kDoneRing of a device array,
// zero at first use; the last CTA to leave a batch zeroes them again.
struct alignas(16) BatchState {
  uint32_t claim;        // next granule to hand out (batches with stage barriers)
  uint32_t done;         // chunks finished
  uint32_t ctas_left;    // CTAs that left the batch
  uint32_t err;          // ErrBits
  uint64_t nt0;          // ~(%globaltimer) of the first CTA to enter (atomicMax of the
                         // complement: 0 means none yet)
  uint64_t pad;
};
static_assert(sizeof(BatchState) == 32, "BatchState must stay 32 bytes");

enum ErrBits : uint32_t {
  ERR_BAD_OP = 1,        // slot resolved to no variant (reference drops such tasks silently)
  ERR_BAD_KIND = 2,      // variant does not fit the request kind
  ERR_STAGE_TIMEOUT = 4, // a bounded wait for staging expired
  ERR_IDLE_EXIT = 8,
  ERR_CUDA = 32,         // host-side: CUDA reported an error for the batch's launch
};

// Jump table: logical slot -> alias -> physical slot -> (variant, params).
struct alignas(16) SlotEntry {
  int32_t variant;       // V_NONE when empty
  float   p0, p1;
  int32_t arity;
};

struct alignas(16) Tables {
  int32_t   alias[kMaxSlots];
  SlotEntry slot[kMaxSlots];
};

// Control block in mapped pinned host memory: written by the host and read by
// the persistent worker (doorbell), or the other way round (completion).
struct alignas(64) HostCtrl {
  // host -> device
  volatile uint64_t tail;          // batches published (doorbell)
  volatile uint32_t quit;          // 1: drain staged batches and exit
  volatile uint32_t pad0;
  volatile uint64_t yield_every;   // exit after every N completed batches (0 = never)
  volatile uint64_t idle_ns;       // exit after this long without work
  volatile uint32_t debug_level;
  volatile uint32_t pad1[5];
  // device -> host
  volatile uint64_t staged;        // batches staged into device memory
  volatile uint64_t processed;     // batches completed (any order)
  volatile uint64_t heartbeat;     // idle polls of the ingest CTA
  volatile uint64_t err;           // sticky ErrBits of the worker
  volatile uint32_t running;       // 1 while a worker grid is alive
  volatile uint32_t exit_reason;
  volatile uint64_t pad2[2];
};

// Ring of completion words (one per in-flight batch), in mapped host memory.
// done_ring[seq % kDoneRing] == seq + 1 once every chunk of batch `seq` is
// finished; retired_ring[...] == seq + 1 once no CTA reads its payload.
static constexpr int kDoneRing = 1024;

enum BatchFlags : uint32_t {
  BF_STAGED = 1,      // per-request stage waits follow the chunk prefix array
  BF_AFTER_PREV = 2,  // do not start before the previous batch is done
  BF_CLAIM = 4,       // warps claim granules one at a time (large batches, whose
                      // chunks differ in cost), and the batch ends through its counters
};

// Publication record of one batch (mapped host memory, ring of kDoneRing).
struct alignas(16) Pub {
  uint64_t seq;
  uint32_t off;      // byte offset of the payload in the arena / device ring
  uint32_t bytes;    // payload bytes (multiple of 16)
};

// Device-memory control block of the persistent worker.
struct alignas(64) DevCtrl {
  uint64_t ready;        // batches staged into the device ring (release/acquire)
  uint64_t stop_at;      // processors exit when they reach this batch
  uint64_t pad[6];
  uint64_t done_dev[kDoneRing];   // device copy of the completion words
  uint32_t ready_off[kDoneRing];
};

// ---- lean batches --------------------------------------------------------
// A stream-mode batch whose requests are all contiguous, 16-byte aligned fp32
// elementwise requests of a precompiled operator with tensor (not scalar)
// operands (the mixed-operator stream,
// the add/mul stream) travels entirely in the kernel's parameters: no staging
// copy, no granule table.  Warp g of W runs the chunks
// [g * nchunk / W, (g + 1) * nchunk / W), so the warps of one SM work on
// neighbouring chunks, which the host has grouped by operator.
static constexpr int kLeanThreads = 512;    // one CTA per SM, room for the next batch's
static constexpr int kLeanPar = 16;         // distinct (p0, p1) pairs per batch
static constexpr int kLeanMaxReq = 512;     // largest parameter block (about 22 KB)

enum LeanFlags : uint32_t {
  LEAN_WAIT_FIRST = 1,   // wait for the previous grid in the stream before touching memory
};

struct alignas(8) LeanRec {
  uint64_t a, b, o;      // device addresses (b unused without RF_HAS_B)
  uint32_t numel;        // output elements (< 2^31)
  uint32_t chunk;        // elements per chunk (a multiple of 4)
  uint8_t  op;           // precompiled elementwise variant
  uint8_t  flags;        // RF_HAS_B
  uint8_t  pidx;         // its (p0, p1) in LeanHdr::par
  uint8_t  pad[5];
};
static_assert(sizeof(LeanRec) == 40, "LeanRec must stay 40 bytes");

struct alignas(16) LeanHdr {
  uint64_t seq;
  uint64_t st;           // BatchState* of the batch (device)
  uint64_t done_ring;    // completion words (device view of mapped host memory)
  uint64_t dur_ring;     // device time of each batch, ns (same)
  uint32_t nreq, nchunk;
  uint32_t flags;        // LeanFlags
  uint32_t pad;
  float    par[kLeanPar][2];
};

template <int N>
struct LeanBatch {
  LeanHdr  h;
  uint32_t cb[N + 1];    // first chunk of every request; cb[nreq] = nchunk
  LeanRec  rec[N];
};

// A lean batch of up to 1024 requests of one shape (the same element count
// and chunk length, e.g. the add/mul stream): no chunk prefix, and 26 bytes
// per request, so twice as many requests fit the parameter space.
static constexpr int kLeanUniMax = 1024;
struct LeanUniBatch {
  LeanHdr  h;
  uint32_t numel;        // every request's elements (< 2^31)
  uint32_t chunk;        // elements per chunk (a multiple of 4)
  uint32_t kpr;          // chunks per request
  uint32_t pad;
  uint64_t a[kLeanUniMax], b[kLeanUniMax], o[kLeanUniMax];
  uint8_t  op[kLeanUniMax];
  uint8_t  pidx[kLeanUniMax];
};
static_assert(sizeof(LeanUniBatch) <= 32764, "kernel parameter space");

// Arguments of the persistent worker kernel.
struct WorkerArgs {
  uint8_t* ring;                 // device staging ring
  const uint8_t* arena;          // device view of the pinned host arena
  BatchState* states;            // device array of kDoneRing batch counters
  volatile HostCtrl* hctrl;      // device view of the host control block
  const volatile Pub* pub;       // device view of the publication ring
  DevCtrl* dctrl;                // device control block
  volatile uint64_t* done_ring;
  volatile uint64_t* retired_ring;
  volatile uint64_t* dur_ring;   // device time of each batch (first CTA in -> last chunk), ns
  const Tables* tab;             // device copy of the jump table (slot requests resolve here)
  uint64_t start_seq;
  uint64_t wait_limit_ns;        // bound of every wait inside a batch
  uint64_t idle_ns;              // ingest: stop after this long without a batch
};

}  // namespace gpuos
