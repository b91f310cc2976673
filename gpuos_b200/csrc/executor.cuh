// Batch executor building blocks: request records, jump-table resolution,
// and the per-warp chunk processors (vector, 2-D tile and strided
// elementwise bodies, reductions).  The loop that hands chunks to warps is
// in batch.cuh; the lean kernel for fp32 contiguous batches in lean.cuh.
//
// Replaces the reference's op_batch (src/persistent_kernel.cu:81-112), which
// walks the sub-tasks of a 512-task shard one after another inside a single
// CTA with int64 div/mod index math per element, and the NVRTC operators of
// pytorch_ext/gpuos_ext.cpp:625-679 (elementwise) and 726-806 (reduce), which
// run one request per CTA.  Here every request is split into chunks and the
// chunks of a batch are spread over every SM.
//
// Chunks that are not staged through shared memory (misaligned views,
// arbitrary strides up to 8 dims, reductions) run here, one warp per chunk.
// A request record is decoded from eight 16-byte loads straight into
// registers.
//
// Compiled by nvcc into the library and by NVRTC for custom expressions.
#pragma once
#include "gpuos_abi.h"
#include "ops.cuh"

namespace gpuos {

#define GPUOS_FULL 0xffffffffu

// The elementwise variants this kernel can run (GPUOS_APPLY_EW): the
// precompiled operators, and in the kernel linked with custom expressions
// those as well.
__device__ __forceinline__ bool ew_known(int v) {
#ifdef GPUOS_JIT_LINK
  if (v >= V_JIT_BASE && v < V_JIT_BASE + kJitOps) return true;
#endif
  return v >= 0 && v < V_NUM_EW;
}

// The variants with vector bodies in this kernel (GPUOS_ALL_EW).
__device__ __forceinline__ bool ew_vec_known(int v) {
#ifdef GPUOS_JIT_LINK
  return v >= V_JIT_BASE && v < V_JIT_BASE + kJitOps;
#else
  return v >= 0 && v < V_NUM_EW;
#endif
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int32_t ld_acquire_s32(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const volatile uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u64(volatile uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void st_release_gpu_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// n / d for n < 2^31 with a precomputed multiplier (Granlund & Montgomery,
// "Division by invariant integers using multiplication", PLDI 1994).
__device__ __forceinline__ uint32_t fdiv_u32(uint32_t n, uint32_t m, uint32_t s) {
  return (__umulhi(n, m) + n) >> s;
}

// A request record in registers (fields as in struct Req).
struct ReqView {
  uint64_t a, b, o;
  int64_t numel, inner, sa_row, sb_row, so_row, sa_in, sb_in;
  uint32_t chunk, nseg, ext, part, cnt, fdiv_m, fdiv_s, rg;
  int op, kind, layout, dta, dtb, dto, flags;
  float p0, p1;
};

__device__ __forceinline__ uint64_t u64of(uint32_t lo, uint32_t hi) {
  return ((uint64_t)hi << 32) | lo;
}

// Decode the 128-byte record (whole warp): lanes 0..7 read it as one
// coalesced 128-byte load through L2 (the staging ring is rewritten for later
// batches, so never from L1), and shuffles hand the words to every lane.
__device__ __forceinline__ uint4 load_req_words(const Req* g, int lane) {
  uint4 w = make_uint4(0u, 0u, 0u, 0u);
  if (lane < 8) w = __ldcg(reinterpret_cast<const uint4*>(g) + lane);
  return w;
}

// The record from the words lanes 0..7 hold (load_req_words).
__device__ __forceinline__ ReqView decode_req(uint4 w) {
  auto word = [&](int i) {
    uint4 r;
    r.x = __shfl_sync(GPUOS_FULL, w.x, i);
    r.y = __shfl_sync(GPUOS_FULL, w.y, i);
    r.z = __shfl_sync(GPUOS_FULL, w.z, i);
    r.w = __shfl_sync(GPUOS_FULL, w.w, i);
    return r;
  };
  const uint4 w0 = word(0), w1 = word(1), w2 = word(2), w3 = word(3);
  const uint4 w4 = word(4), w5 = word(5), w6 = word(6), w7 = word(7);
  ReqView q;
  q.op = (int)(w0.x & 0xffffu);
  q.kind = (int)((w0.x >> 16) & 0xffu);
  q.layout = (int)(w0.x >> 24);
  q.dta = (int)(w0.y & 0xffu);
  q.dtb = (int)((w0.y >> 8) & 0xffu);
  q.dto = (int)((w0.y >> 16) & 0xffu);
  q.flags = (int)(w0.y >> 24);
  q.p0 = __uint_as_float(w0.z);
  q.p1 = __uint_as_float(w0.w);
  q.chunk = w1.x;
  q.nseg = w1.y;
  q.numel = (int64_t)u64of(w1.z, w1.w);
  q.a = u64of(w2.x, w2.y);
  q.b = u64of(w2.z, w2.w);
  q.o = u64of(w3.x, w3.y);
  q.inner = (int64_t)u64of(w3.z, w3.w);
  q.sa_row = (int64_t)u64of(w4.x, w4.y);
  q.sb_row = (int64_t)u64of(w4.z, w4.w);
  q.so_row = (int64_t)u64of(w5.x, w5.y);
  q.sa_in = (int64_t)u64of(w5.z, w5.w);
  q.sb_in = (int64_t)u64of(w6.x, w6.y);
  q.ext = w6.z;
  q.part = w6.w;
  q.cnt = w7.x;
  q.fdiv_m = w7.y;
  q.fdiv_s = w7.z;
  q.rg = w7.w;
  return q;
}

__device__ __forceinline__ ReqView load_req(const Req* g, int lane) {
  return decode_req(load_req_words(g, lane));
}

__device__ __forceinline__ int64_t row_of(const ReqView& q, int64_t e) {
  if (q.flags & RF_BIG) return e / q.inner;
  return (int64_t)fdiv_u32((uint32_t)e, q.fdiv_m, q.fdiv_s);
}

// Execution context of one warp inside one batch.
struct Exec {
  const uint8_t* base;          // batch payload in device memory
  BatchState* st;
  const Req* recs;
  const uint32_t* gcb;          // chunk prefix: first chunk of every request
  const uint2* gtab;            // per granule: (request, that request's first chunk)
  const uint32_t* req_wait;     // per-request chunk count that must be done first (0: none)
  float* scratch;               // partial sums of split reductions
  uint32_t* counters;           // self-cleaning combine counters
  volatile uint64_t* done_ring; // completion words in mapped host memory
  uint64_t* done_dev;           // device copy of the completion words (worker only)
  volatile uint64_t* dur_ring;  // device time of each batch (mapped host memory), or null
  const Tables* tab;            // device jump table (persistent worker), or null: records
                                // then carry resolved operators
  uint64_t wait_limit_ns;
  uint64_t seq;                 // batch sequence number
  uint64_t wait_from;           // BF_AFTER_PREV: batches [wait_from, seq) first
  uint32_t nchunk;              // chunks in the batch
  uint32_t gran;                // chunks per granule
  uint32_t flags;               // BatchFlags
  int lane;
};

// A stream-mode batch without stage barriers or claimed granules has no
// end-of-batch protocol (the event recorded after its launch completes it),
// so an error is posted to the host at once: the completion word with the
// bits this warp knows; the host reads the batch's full error bits from `st`
// after the kernel.
__device__ __forceinline__ bool posts_own_errors(const Exec& ex) {
  return !ex.done_dev && !(ex.flags & (BF_STAGED | BF_CLAIM));
}

__device__ __forceinline__ void set_err(const Exec& ex, uint32_t bits) {
  atomicOr(&ex.st->err, bits);
  if (posts_own_errors(ex))
    ex.done_ring[ex.seq % kDoneRing] = (ex.seq + 1) | ((uint64_t)(bits & 0xffu) << 48);
}

// ---------------------------------------------------------------------------
// Elementwise generic path (one shared body): misaligned views, arbitrary
// inner strides, and general strided requests of up to 8 dims.  Each round a
// lane computes the offsets of K elements (lane, lane + 32, ...) and issues
// all their loads, raw, before converting or computing any, so that a chunk
// costs one memory round trip per 32 K elements: one element at a time would
// wait a full round trip each, since a store may alias the next load.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ew_generic(const ReqView& q, const ExtRec* x, int v, float p0,
                                           float p1, int64_t e0, int64_t e1, int lane) {
  constexpr int K = 4;
  const bool hasb = q.flags & RF_HAS_B;
  const int lay = q.layout;
  const int64_t N = q.inner;
#pragma unroll 1
  for (int64_t eb = e0 + lane; eb < e1; eb += 32 * K) {
    // the offsets and raw bits of this lane's K elements of the round
    uint32_t ra[K], rb[K];
    int64_t oo[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t e = eb + 32 * k;
      ra[k] = 0u;
      rb[k] = 0u;
      oo[k] = 0;
      if (e < e1) {
        int64_t oa, ob;
        if (lay == EL_CONTIG) {
          oa = (q.flags & RF_A_SCALAR) ? 0 : e;
          ob = (q.flags & RF_B_SCALAR) ? 0 : e;
          oo[k] = e;
        } else if (lay == EL_ROW2D) {
          const int64_t r = row_of(q, e), c = e - r * N;
          oa = r * q.sa_row + c * q.sa_in;
          ob = r * q.sb_row + c * q.sb_in;
          oo[k] = r * q.so_row + c;
        } else {
          int64_t rem = e, o = 0;
          oa = ob = 0;
          for (int d = x->ndim - 1; d >= 0; --d) {
            const int64_t sz = x->sizes[d];
            const int64_t i = rem % sz;
            rem /= sz;
            oa += i * x->sa[d];
            ob += i * x->sb[d];
            o += i * x->so[d];
          }
          oo[k] = o;
        }
        ra[k] = ld1_raw(q.a, q.dta, oa);
        if (hasb) rb[k] = ld1_raw(q.b, q.dtb, ob);
      }
    }
    // then one element at a time, from one copy of the operator switch: the
    // arrays shift down by one per step (their indices stay constant)
    const int nk = (int)min((int64_t)K, (e1 - eb + 31) / 32);
#pragma unroll 1
    for (int k = 0; k < nk; ++k) {
      float R = 0.f;
      ew_apply1(v, cvt1(ra[0], q.dta), hasb ? cvt1(rb[0], q.dtb) : 0.f, R, p0, p1);
      st1(q.o, q.dto, oo[0], R);
#pragma unroll
      for (int j = 0; j + 1 < K; ++j) {
        ra[j] = ra[j + 1];
        rb[j] = rb[j + 1];
        oo[j] = oo[j + 1];
      }
    }
  }
}

#ifdef GPUOS_JIT_LINK
// The general body for a custom expression of three or four operands
// (RF_NARY): A and B as in ew_generic, C and D from the extension record.
// The same rounds of K elements per lane, every load of a round issued
// before any element is computed.
__device__ __forceinline__ void ew_generic_nary(const ReqView& q, const ExtRec* x, int v,
                                                float p0, float p1, int64_t e0, int64_t e1,
                                                int lane) {
  constexpr int K = 4;
  const bool hasb = q.flags & RF_HAS_B;
  const bool hasd = x->d != 0;
  const int lay = q.layout;
  const int64_t N = q.inner;
#pragma unroll 1
  for (int64_t eb = e0 + lane; eb < e1; eb += 32 * K) {
    uint32_t ra[K], rb[K], rc[K], rd[K];
    int64_t oo[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t e = eb + 32 * k;
      ra[k] = rb[k] = rc[k] = rd[k] = 0u;
      oo[k] = 0;
      if (e < e1) {
        int64_t oa, ob, oc, od;
        if (lay == EL_CONTIG) {
          oa = (q.flags & RF_A_SCALAR) ? 0 : e;
          ob = (q.flags & RF_B_SCALAR) ? 0 : e;
          oc = e * x->sc[0];
          od = e * x->sd[0];
          oo[k] = e;
        } else if (lay == EL_ROW2D) {
          const int64_t r = row_of(q, e), c = e - r * N;
          oa = r * q.sa_row + c * q.sa_in;
          ob = r * q.sb_row + c * q.sb_in;
          oc = r * x->sc[0] + c * x->sc[1];
          od = r * x->sd[0] + c * x->sd[1];
          oo[k] = r * q.so_row + c;
        } else {
          int64_t rem = e, o = 0;
          oa = ob = oc = od = 0;
          for (int d = x->ndim - 1; d >= 0; --d) {
            const int64_t sz = x->sizes[d];
            const int64_t i = rem % sz;
            rem /= sz;
            oa += i * x->sa[d];
            ob += i * x->sb[d];
            oc += i * x->sc[d];
            od += i * x->sd[d];
            o += i * x->so[d];
          }
          oo[k] = o;
        }
        ra[k] = ld1_raw(q.a, q.dta, oa);
        if (hasb) rb[k] = ld1_raw(q.b, q.dtb, ob);
        rc[k] = ld1_raw(x->c, x->dtc, oc);
        if (hasd) rd[k] = ld1_raw(x->d, x->dtd, od);
      }
    }
    const int nk = (int)min((int64_t)K, (e1 - eb + 31) / 32);
#pragma unroll 1
    for (int k = 0; k < nk; ++k) {
      float R = 0.f;
      ew_apply4(v, cvt1(ra[0], q.dta), hasb ? cvt1(rb[0], q.dtb) : 0.f, cvt1(rc[0], x->dtc),
                hasd ? cvt1(rd[0], x->dtd) : 0.f, R, p0, p1);
      st1(q.o, q.dto, oo[0], R);
#pragma unroll
      for (int j = 0; j + 1 < K; ++j) {
        ra[j] = ra[j + 1];
        rb[j] = rb[j + 1];
        rc[j] = rc[j + 1];
        rd[j] = rd[j + 1];
        oo[j] = oo[j + 1];
      }
    }
  }
}
#endif

// ---------------------------------------------------------------------------
// 2-D elementwise tiles (EL_TILE2D): a chunk is a block of `chunk` columns of
// every one of the request's rows.  Lane l owns the kTileC columns
// c0 + l + 32 j (j < kTileC) of each group of 32 kTileC columns and walks
// down the rows kTileR at a time: kTileR x kTileC loads per operand in
// flight, issued raw before any is converted.  The output and row-contiguous
// operands move 32 adjacent columns per instruction; a transposed operand
// (row stride 1) is read by each lane along its own contiguous runs, which L1
// serves for the neighbouring rows.  Each column's operand pointers are set
// up once per tile and advanced by the row strides: no division and no index
// multiplication per element.  Whole blocks of rows of a tile whose columns
// are all in range run without per-element bounds checks.  The dtypes and
// the operator are template parameters for the broadcast configuration's
// combinations (-1: read at run time).
// ---------------------------------------------------------------------------
static constexpr int kTileC = 2;
static constexpr int kTileR = 4;

template <int DT>
__device__ __forceinline__ int t2_esz(int dt) {
  return (DT >= 0 ? DT : dt) == kF32 ? 4 : 2;
}

template <int DT>
__device__ __forceinline__ uint32_t t2_ld(const uint8_t* p, int dt) {
  if ((DT >= 0 ? DT : dt) == kF32) return *reinterpret_cast<const uint32_t*>(p);
  return *reinterpret_cast<const uint16_t*>(p);
}

template <int DT>
__device__ __forceinline__ float t2_cvt(uint32_t r, int dt) {
  return cvt1(r, DT >= 0 ? DT : dt);
}

template <int DT>
__device__ __forceinline__ void t2_st(uint8_t* p, int dt, float v) {
  st1(reinterpret_cast<uint64_t>(p), DT >= 0 ? DT : dt, 0, v);
}

template <int V>
__device__ __forceinline__ float t2_op(int v, float A, float B, float p0, float p1) {
  if constexpr (V >= 0) {
    return op1<V>(A, B, p0, p1);
  } else {
    float r = 0.f;
    ew_apply1(v, A, B, r, p0, p1);
    return r;
  }
}

// One block of kTileR rows of a lane's kTileC columns.  CHECK: the last
// block of a tile, or a tile whose columns run past the chunk: loads and
// stores are predicated on the row and column being in range.
template <int DA, int DB, int DO, int V, bool CHECK>
__device__ __forceinline__ void tile2d_rows(const ReqView& q, int v, float p0, float p1,
                                            const uint8_t* const* pa, const uint8_t* const* pb,
                                            uint8_t* const* po, const float* bc, const bool* ok,
                                            int64_t rows_left, bool hasb, bool b_col,
                                            int64_t ra_b, int64_t rb_b, int64_t ro_b) {
  uint32_t ra[kTileR][kTileC], rb[kTileR][kTileC];
#pragma unroll
  for (int u = 0; u < kTileR; ++u) {
#pragma unroll
    for (int j = 0; j < kTileC; ++j) {
      ra[u][j] = 0u;
      rb[u][j] = 0u;
      if (!CHECK || (ok[j] && u < rows_left)) {
        ra[u][j] = t2_ld<DA>(pa[j] + u * ra_b, q.dta);
        if (hasb && !b_col) rb[u][j] = t2_ld<DB>(pb[j] + u * rb_b, q.dtb);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < kTileR; ++u) {
#pragma unroll
    for (int j = 0; j < kTileC; ++j) {
      if (!CHECK || (ok[j] && u < rows_left)) {
        const float A = t2_cvt<DA>(ra[u][j], q.dta);
        const float B = hasb ? (b_col ? bc[j] : t2_cvt<DB>(rb[u][j], q.dtb)) : 0.f;
        t2_st<DO>(po[j] + u * ro_b, q.dto, t2_op<V>(v, A, B, p0, p1));
      }
    }
  }
}

template <int DA, int DB, int DO, int V>
__device__ __forceinline__ void ew_tile2d(const ReqView& q, int v, float p0, float p1, uint32_t k,
                                          int lane) {
  // the broadcast configuration's operators all take B
  constexpr bool kBin = V == V_ADD || V == V_SUB || V == V_MUL || V == V_DIV0 || V == V_MAX ||
                        V == V_MIN;
  const int64_t N = q.inner, R = q.nseg;
  const int64_t cb = (int64_t)k * q.chunk;
  const int64_t ce = min(N, cb + (int64_t)q.chunk);
  const bool hasb = kBin || (q.flags & RF_HAS_B);
  const bool a_sc = q.flags & RF_A_SCALAR, b_sc = q.flags & RF_B_SCALAR;
  const int ea = t2_esz<DA>(q.dta), eb = t2_esz<DB>(q.dtb), eo = t2_esz<DO>(q.dto);
  // byte strides down the rows (0 for a scalar operand)
  const int64_t ra_b = a_sc ? 0 : q.sa_row * ea, rb_b = b_sc ? 0 : q.sb_row * eb;
  const int64_t ro_b = q.so_row * eo;
  // B that does not vary down the rows ([N]) or at all: one value per column
  const bool b_col = hasb && (b_sc || q.sb_row == 0);
  const int64_t rfull = R - R % kTileR;  // rows in whole blocks
#pragma unroll 1
  for (int64_t c0 = cb + lane; c0 < ce; c0 += 32 * kTileC) {
    const uint8_t* pa[kTileC];
    const uint8_t* pb[kTileC];
    uint8_t* po[kTileC];
    float bc[kTileC];
    bool ok[kTileC];
#pragma unroll
    for (int j = 0; j < kTileC; ++j) {
      const int64_t c = c0 + 32 * j;
      ok[j] = c < ce;
      const int64_t cc = ok[j] ? c : c0;  // an in-range column keeps the pointers valid
      pa[j] = reinterpret_cast<const uint8_t*>(q.a) + (a_sc ? 0 : cc * q.sa_in * ea);
      pb[j] = reinterpret_cast<const uint8_t*>(q.b) + (b_sc ? 0 : cc * q.sb_in * eb);
      po[j] = reinterpret_cast<uint8_t*>(q.o) + cc * eo;
      bc[j] = b_col ? t2_cvt<DB>(t2_ld<DB>(pb[j], q.dtb), q.dtb) : 0.f;
    }
    const bool all_cols = ok[kTileC - 1];  // columns are in range up to the first that is not
    int64_t i0 = 0;
    if (all_cols) {
#pragma unroll 1
      for (; i0 < rfull; i0 += kTileR) {
        tile2d_rows<DA, DB, DO, V, false>(q, v, p0, p1, pa, pb, po, bc, ok, kTileR, hasb, b_col,
                                          ra_b, rb_b, ro_b);
#pragma unroll
        for (int j = 0; j < kTileC; ++j) {
          pa[j] += kTileR * ra_b;
          pb[j] += kTileR * rb_b;
          po[j] += kTileR * ro_b;
        }
      }
    }
#pragma unroll 1
    for (; i0 < R; i0 += kTileR) {
      tile2d_rows<DA, DB, DO, V, true>(q, v, p0, p1, pa, pb, po, bc, ok, R - i0, hasb, b_col,
                                       ra_b, rb_b, ro_b);
#pragma unroll
      for (int j = 0; j < kTileC; ++j) {
        pa[j] += kTileR * ra_b;
        pb[j] += kTileR * rb_b;
        po[j] += kTileR * ro_b;
      }
    }
  }
}

#ifndef GPUOS_JIT_LINK
// The dtype triples of the broadcast configuration (fp32+fp32, fp16+fp32,
// bf16+bf16, fp16+fp16) with its six operators get their own bodies; any
// other request runs the body with run-time dtypes and operator.
template <int DA, int DB, int DO>
__device__ __forceinline__ void tile2d_ops(const ReqView& q, int v, float p0, float p1, uint32_t k,
                                           int lane) {
  switch (v) {
    case V_ADD: ew_tile2d<DA, DB, DO, V_ADD>(q, v, p0, p1, k, lane); return;
    case V_SUB: ew_tile2d<DA, DB, DO, V_SUB>(q, v, p0, p1, k, lane); return;
    case V_MUL: ew_tile2d<DA, DB, DO, V_MUL>(q, v, p0, p1, k, lane); return;
    case V_DIV0: ew_tile2d<DA, DB, DO, V_DIV0>(q, v, p0, p1, k, lane); return;
    case V_MAX: ew_tile2d<DA, DB, DO, V_MAX>(q, v, p0, p1, k, lane); return;
    case V_MIN: ew_tile2d<DA, DB, DO, V_MIN>(q, v, p0, p1, k, lane); return;
    default: ew_tile2d<DA, DB, DO, -1>(q, v, p0, p1, k, lane); return;
  }
}
#endif

__device__ __forceinline__ void tile2d_dispatch(const ReqView& q, int v, float p0, float p1,
                                                uint32_t k, int lane) {
#ifndef GPUOS_JIT_LINK
  const bool hasb = q.flags & RF_HAS_B;
  if (hasb) {
    if (q.dta == kF32 && q.dtb == kF32 && q.dto == kF32) return tile2d_ops<kF32, kF32, kF32>(q, v, p0, p1, k, lane);
    if (q.dta == kF16 && q.dtb == kF32 && q.dto == kF32) return tile2d_ops<kF16, kF32, kF32>(q, v, p0, p1, k, lane);
    if (q.dta == kBF16 && q.dtb == kBF16 && q.dto == kBF16) return tile2d_ops<kBF16, kBF16, kBF16>(q, v, p0, p1, k, lane);
    if (q.dta == kF16 && q.dtb == kF16 && q.dto == kF16) return tile2d_ops<kF16, kF16, kF16>(q, v, p0, p1, k, lane);
  }
#endif
  ew_tile2d<-1, -1, -1, -1>(q, v, p0, p1, k, lane);
}

// ---------------------------------------------------------------------------
// Elementwise vector path: contiguous or row-strided requests whose pointers,
// strides and row length are multiples of 4 elements (RF_VEC).  Each lane
// handles groups of 4 adjacent elements; vec_groups<V>() groups per lane are
// loaded (128-bit for fp32, 64-bit for fp16/bf16) before any is computed or
// stored, so that a warp keeps 32 x groups x 16 bytes per operand in flight:
// 8 groups for the light operators (4 with per-row operands, whose offsets
// take registers), 2 for the transcendental ones: their code is long, and a
// batch that mixes operators runs many of them on one SM, so fewer unrolled
// copies keep the instruction cache warm.
// ---------------------------------------------------------------------------
template <int V>
__device__ __forceinline__ constexpr int vec_groups() {
  return op_unroll<V>() == 2 ? 8 : 2;
}

enum OperandMode : int32_t { OM_LINEAR = 1, OM_ROW = 2, OM_ROWSPLAT = 3, OM_SCALAR = 4 };

struct VecView {
  uint64_t a, b, o;
  int64_t numel, inner, sa_row, sb_row, so_row;
  uint32_t chunk;
  int ma, mb, dta, dtb, dto, flags;
  bool rows, mo;
  float As, Bs;
  uint32_t fdiv_m, fdiv_s;
};

__device__ __forceinline__ VecView vec_view(const ReqView& q) {
  VecView u;
  const bool row2d = q.layout == EL_ROW2D;
  auto mode = [&](bool scalar, int64_t srow, int64_t sin) -> int {
    if (scalar) return OM_SCALAR;
    if (!row2d) return OM_LINEAR;
    if (sin == 0) return OM_ROWSPLAT;
    return srow == q.inner ? OM_LINEAR : OM_ROW;
  };
  u.a = q.a; u.b = q.b; u.o = q.o;
  u.numel = q.numel; u.chunk = q.chunk;
  u.inner = q.inner; u.sa_row = q.sa_row; u.sb_row = q.sb_row; u.so_row = q.so_row;
  u.ma = mode(q.flags & RF_A_SCALAR, q.sa_row, q.sa_in);
  u.mb = (q.flags & RF_HAS_B) ? mode(q.flags & RF_B_SCALAR, q.sb_row, q.sb_in) : OM_SCALAR;
  u.mo = row2d && q.so_row != q.inner;
  u.rows = u.ma == OM_ROW || u.ma == OM_ROWSPLAT || u.mb == OM_ROW || u.mb == OM_ROWSPLAT || u.mo;
  u.dta = q.dta; u.dtb = q.dtb; u.dto = q.dto; u.flags = q.flags;
  u.fdiv_m = q.fdiv_m; u.fdiv_s = q.fdiv_s;
  u.As = u.ma == OM_SCALAR ? ld1(q.a, q.dta, 0) : 0.f;
  u.Bs = (u.mb == OM_SCALAR && (q.flags & RF_HAS_B)) ? ld1(q.b, q.dtb, 0) : 0.f;
  return u;
}

__device__ __forceinline__ int64_t vec_row(const VecView& u, int64_t e) {
  if (u.flags & RF_BIG) return e / u.inner;
  return (int64_t)fdiv_u32((uint32_t)e, u.fdiv_m, u.fdiv_s);
}

__device__ __forceinline__ void vec_opnd4(int mode, uint64_t p, int dt, float sc, int64_t e,
                                          int64_t rowoff, int64_t c, float* v) {
  if (mode == OM_LINEAR) {
    ld4(p, dt, e, v);
  } else if (mode == OM_ROW) {
    ld4(p, dt, rowoff + c, v);
  } else if (mode == OM_ROWSPLAT) {
    const float x = ld1(p, dt, rowoff);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = x;
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = sc;
  }
}

__device__ __forceinline__ float vec_opnd1(int mode, uint64_t p, int dt, float sc, int64_t e,
                                           int64_t rowoff, int64_t c) {
  if (mode == OM_LINEAR) return ld1(p, dt, e);
  if (mode == OM_ROW) return ld1(p, dt, rowoff + c);
  if (mode == OM_ROWSPLAT) return ld1(p, dt, rowoff);
  return sc;
}

// elements [e0, e0 + n) of a request whose operands are all linear or scalar.
// The chunk is walked in whole groups of 4 elements, group q on lane q % 32:
// each round loads up to kG groups per lane, each under its own bound, before
// any is computed, so a chunk of any length costs one memory round trip per
// kG x 128 elements; the last n % 4 elements (the ragged end of a request) go
// one per lane.  Every group's registers are defined on every path (a load
// under a predicate alone would keep them live across the loop's back edge).
template <int V>
__device__ __forceinline__ void ew_vec_flat(const VecView& u, float p0, float p1, int64_t e0,
                                            int64_t n, int lane) {
  constexpr int kG = vec_groups<V>();
  const bool as = u.ma == OM_SCALAR, bs = u.mb == OM_SCALAR;
  const int64_t nq = n >> 2;
#pragma unroll 1
  for (int64_t q0 = lane; q0 < nq; q0 += 32 * kG) {
    const int64_t eb = e0 + 4 * q0;   // this lane's first element of the round
    const int left = (int)(nq - q0);  // groups from there to the chunk's end
    float A[kG][4], B[kG][4];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        A[g][k] = u.As;
        B[g][k] = u.Bs;
      }
      if (32 * g < left) {
        if (!as) ld4(u.a, u.dta, eb + 128 * g, A[g]);
        if (!bs) ld4(u.b, u.dtb, eb + 128 * g, B[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (32 * g < left) {
        float R[4];
        op4<V>(A[g], B[g], R, p0, p1);
        st4(u.o, u.dto, eb + 128 * g, R);
      }
    }
  }
  if (lane < (int)(n & 3)) {
    const int64_t e = e0 + 4 * nq + lane;
    const float A = vec_opnd1(u.ma, u.a, u.dta, u.As, e, 0, 0);
    const float B = vec_opnd1(u.mb, u.b, u.dtb, u.Bs, e, 0, 0);
    st1(u.o, u.dto, e, op1<V>(A, B, p0, p1));
  }
}

// elements [e0, e0 + n) of a request with a per-row operand or output
// (rows of u.inner elements, a multiple of 4, so a group of 4 never straddles
// two rows); walked in predicated groups as ew_vec_flat.
template <int V>
__device__ __forceinline__ void ew_vec_rows(const VecView& u, float p0, float p1, int64_t e0,
                                            int64_t n, int lane) {
  constexpr int kG = op_unroll<V>() == 2 ? 4 : 2;
  const int64_t nq = n >> 2;
#pragma unroll 1
  for (int64_t q0 = lane; q0 < nq; q0 += 32 * kG) {
    const int64_t eb = e0 + 4 * q0;
    const int left = (int)(nq - q0);
    float A[kG][4], B[kG][4];
    int64_t oo[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const int64_t e = eb + 128 * g;
      const int64_t r = vec_row(u, e), c = e - r * u.inner;
      oo[g] = u.mo ? r * u.so_row + c : e;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        A[g][k] = u.As;
        B[g][k] = u.Bs;
      }
      if (32 * g < left) {
        vec_opnd4(u.ma, u.a, u.dta, u.As, e, r * u.sa_row, c, A[g]);
        vec_opnd4(u.mb, u.b, u.dtb, u.Bs, e, r * u.sb_row, c, B[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (32 * g < left) {
        float R[4];
        op4<V>(A[g], B[g], R, p0, p1);
        st4(u.o, u.dto, oo[g], R);
      }
    }
  }
  if (lane < (int)(n & 3)) {
    const int64_t ek = e0 + 4 * nq + lane;
    const int64_t r = vec_row(u, ek), c = ek - r * u.inner;
    const float A = vec_opnd1(u.ma, u.a, u.dta, u.As, ek, r * u.sa_row, c);
    const float B = vec_opnd1(u.mb, u.b, u.dtb, u.Bs, ek, r * u.sb_row, c);
    st1(u.o, u.dto, u.mo ? r * u.so_row + c : ek, op1<V>(A, B, p0, p1));
  }
}

// All-fp32 flat requests (the common case) run a body with no dtype
// branches: its code is a fraction of the general one's, which keeps the
// instruction cache warm when a batch mixes operators.  Same walk in
// predicated groups as ew_vec_flat.
template <int V>
__device__ __forceinline__ void ew_vec_f32(const VecView& u, float p0, float p1, int64_t e0,
                                           int64_t n, int lane) {
  constexpr int kG = vec_groups<V>();
  const bool as = u.ma == OM_SCALAR, bs = u.mb == OM_SCALAR;
  const int64_t nq = n >> 2;
#pragma unroll 1
  for (int64_t q0 = lane; q0 < nq; q0 += 32 * kG) {
    const int64_t eb = e0 + 4 * q0;
    const int left = (int)(nq - q0);
    const float4* A = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(u.a) + eb);
    const float4* B = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(u.b) + eb);
    float4* O = reinterpret_cast<float4*>(reinterpret_cast<float*>(u.o) + eb);
    // every group is defined on every path (a load under a predicate alone
    // would keep the registers live across the loop's back edge)
    float4 a[kG], b[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      a[g] = make_float4(u.As, u.As, u.As, u.As);
      b[g] = make_float4(u.Bs, u.Bs, u.Bs, u.Bs);
      if (32 * g < left) {
        if (!as) a[g] = A[32 * g];
        if (!bs) b[g] = B[32 * g];
      }
    }
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (32 * g < left) {
        float4 r;
        r.x = op1<V>(a[g].x, b[g].x, p0, p1);
        r.y = op1<V>(a[g].y, b[g].y, p0, p1);
        r.z = op1<V>(a[g].z, b[g].z, p0, p1);
        r.w = op1<V>(a[g].w, b[g].w, p0, p1);
        O[32 * g] = r;
      }
    }
  }
  if (lane < (int)(n & 3)) {
    const int64_t e = e0 + 4 * nq + lane;
    const float* A = reinterpret_cast<const float*>(u.a);
    const float* B = reinterpret_cast<const float*>(u.b);
    const float x = as ? u.As : A[e];
    const float y = bs ? u.Bs : (u.mb == OM_LINEAR ? B[e] : 0.f);
    reinterpret_cast<float*>(u.o)[e] = op1<V>(x, y, p0, p1);
  }
}

template <int V>
__device__ __forceinline__ void ew_vec(const VecView& u, float p0, float p1, int64_t e0, int64_t n,
                                       int lane) {
  if (u.rows) ew_vec_rows<V>(u, p0, p1, e0, n, lane);
  else if (u.dta == kF32 && u.dtb == kF32 && u.dto == kF32) ew_vec_f32<V>(u, p0, p1, e0, n, lane);
  else ew_vec_flat<V>(u, p0, p1, e0, n, lane);
}

#define GPUOS_VEC_CASE(V) case V: ew_vec<V>(u, p0, p1, e0, n, lane); return true;

__device__ __forceinline__ bool ew_vec_dispatch(int v, const VecView& u, float p0, float p1,
                                                int64_t e0, int64_t n, int lane) {
  switch (v) {
    GPUOS_ALL_EW(GPUOS_VEC_CASE)
    default: return false;
  }
}

// ---------------------------------------------------------------------------
// Reductions (sum / mean over the reduced columns), fp32 accumulation.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float red_finish(float s, bool mean, int64_t C) {
  return mean ? s / (float)C : s;
}

// Combine the partial sums of one output (or a group of outputs) once every
// segment is in.  The warp that brings the counter to nseg sums the partials
// in segment order, so the result does not depend on which warp came last.
__device__ __forceinline__ bool combine_arrive(const Exec& ex, uint32_t* cnt, uint32_t nseg) {
  __threadfence();  // every lane releases its partial-sum store
  __syncwarp();
  uint32_t last = 0;
  if (ex.lane == 0) last = (atomicAdd(cnt, 1u) == nseg - 1) ? 1u : 0u;
  last = __shfl_sync(GPUOS_FULL, last, 0);
  if (last) __threadfence();
  return last != 0;
}

// Rows contiguous: a lane group of q.rg lanes sums one row (nseg == 1), or the
// whole warp sums one segment of a long row (nseg > 1).  A row (or segment)
// is read in aligned 16-byte blocks, 4 fp32 or 8 fp16 / bf16 elements,
// whatever the alignment of its first element: the blocks that cover the
// span are loaded whole, and the elements of the first and last block that
// lie outside the span are zeroed before they are added.  (A 16-byte block
// that holds an element of the tensor lies in the same memory page, so the
// whole-block load is always in bounds.)  Lane i of a group takes blocks i,
// i + G, ..., kRedVU of them in flight, converted and added after all are
// issued.
static constexpr int kRedVU = 8;

template <int DT>
__device__ __forceinline__ void add16_t(uint4 w, float& acc0, float& acc1) {
  if constexpr (DT == kF32) {
    acc0 += __uint_as_float(w.x) + __uint_as_float(w.z);
    acc1 += __uint_as_float(w.y) + __uint_as_float(w.w);
  } else {
    float v[8];
    if constexpr (DT == kF16) {
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
      }
    } else {
      bf2_to_f(w.x, v[0], v[1]);
      bf2_to_f(w.y, v[2], v[3]);
      bf2_to_f(w.z, v[4], v[5]);
      bf2_to_f(w.w, v[6], v[7]);
    }
    acc0 += (v[0] + v[2]) + (v[4] + v[6]);
    acc1 += (v[1] + v[3]) + (v[5] + v[7]);
  }
}

// Zero the elements of the block at byte address `blk` that lie outside [s, e).
template <int DT>
__device__ __forceinline__ uint4 mask16_t(uint4 w, uint64_t blk, uint64_t s, uint64_t e) {
  uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint64_t a = blk + 4 * j;
    if constexpr (DT == kF32) {
      if (a < s || a >= e) v[j] = 0u;
    } else {
      uint32_t m = 0u;
      if (a >= s && a < e) m |= 0x0000ffffu;
      if (a + 2 >= s && a + 2 < e) m |= 0xffff0000u;
      v[j] &= m;
    }
  }
  return make_uint4(v[0], v[1], v[2], v[3]);
}

// Sum of the elements at byte addresses [s, e) of one span: lane li of G.
template <int DT>
__device__ __forceinline__ void red_span_t(uint64_t s, uint64_t e, int li, int G, float& acc0,
                                           float& acc1) {
  if (e <= s) return;
  const uint64_t b0 = s & ~15ull;
  const uint32_t nb = (uint32_t)((((e + 15) & ~15ull) - b0) >> 4);
  const uint32_t step = (uint32_t)G;
#pragma unroll 1
  for (uint32_t i = (uint32_t)li; i < nb; i += step * kRedVU) {
    uint4 w[kRedVU];
#pragma unroll
    for (int u = 0; u < kRedVU; ++u) {
      const uint32_t bi = i + step * u;
      w[u] = make_uint4(0u, 0u, 0u, 0u);
      if (bi < nb) w[u] = *reinterpret_cast<const uint4*>(b0 + 16ull * bi);
    }
#pragma unroll
    for (int u = 0; u < kRedVU; ++u) {
      const uint32_t bi = i + step * u;
      if (bi < nb) {
        uint4 x = w[u];
        if (bi == 0 || bi == nb - 1) x = mask16_t<DT>(x, b0 + 16ull * bi, s, e);
        add16_t<DT>(x, acc0, acc1);
      }
    }
  }
}

template <int DT>
__device__ __forceinline__ void red_rows_t(const Exec& ex, const ReqView& q, bool mean,
                                           uint32_t k) {
  constexpr int ES = DT == kF32 ? 4 : 2;
  const int lane = ex.lane;
  const int64_t C = q.inner;
  if (q.nseg == 1) {
    const int G = (int)q.rg;                   // lanes per row (power of two)
    const int per = 32 / G;                    // rows per warp step
    const int sub = lane / G, li = lane % G;
    const int64_t r0 = (int64_t)k * q.chunk;
    int64_t r1 = r0 + q.chunk;
    if (r1 > q.numel) r1 = q.numel;
    for (int64_t rb = r0; rb < r1; rb += per) {
      const int64_t r = rb + sub;
      const bool valid = r < r1;
      float acc0 = 0.f, acc1 = 0.f;
      if (valid) {
        const uint64_t s = q.a + (uint64_t)(r * q.sa_row * ES);
        red_span_t<DT>(s, s + (uint64_t)(C * ES), li, G, acc0, acc1);
      }
      float acc = acc0 + acc1;
      for (int off = G >> 1; off > 0; off >>= 1) acc += __shfl_xor_sync(GPUOS_FULL, acc, off);
      if (valid && li == 0) st1(q.o, q.dto, r * q.so_row, red_finish(acc, mean, C));
    }
    return;
  }
  // long rows: one warp per (row, segment)
  const uint32_t nseg = q.nseg;
  const int64_t r = k / nseg;
  const uint32_t seg = k % nseg;
  const int64_t c0 = (int64_t)seg * q.chunk;
  int64_t c1 = c0 + q.chunk;
  if (c1 > C) c1 = C;
  const uint64_t rowp = q.a + (uint64_t)(r * q.sa_row * ES);
  float acc0 = 0.f, acc1 = 0.f;
  red_span_t<DT>(rowp + (uint64_t)(c0 * ES), rowp + (uint64_t)(c1 * ES), lane, 32, acc0, acc1);
  float acc = acc0 + acc1;
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(GPUOS_FULL, acc, off);
  float* part = ex.scratch + q.part + r * nseg;
  if (lane == 0) part[seg] = acc;
  uint32_t* cnt = ex.counters + q.cnt + r;
  if (combine_arrive(ex, cnt, nseg)) {
    float s = 0.f;
    for (uint32_t i = lane; i < nseg; i += 32) s += __ldcg(part + i);
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(GPUOS_FULL, s, off);
    if (lane == 0) {
      st1(q.o, q.dto, r * q.so_row, red_finish(s, mean, C));
      *cnt = 0u;  // leave the counter clean for the next batch
    }
  }
}

__device__ __forceinline__ void red_rows(const Exec& ex, const ReqView& q, bool mean, uint32_t k) {
  if (q.dta == kF32) red_rows_t<kF32>(ex, q, mean, k);
  else if (q.dta == kF16) red_rows_t<kF16>(ex, q, mean, k);
  else red_rows_t<kBF16>(ex, q, mean, k);
}

// Rows adjacent in memory (a transposed view): lanes own rows, so every step
// of the column loop reads rg adjacent rows of cl columns; kColU columns per
// lane are in flight (raw loads, converted after all are issued), whole
// rounds without bounds checks and one guarded round for the rest.
static constexpr int kColU = 16;

template <int DT>
__device__ __forceinline__ uint32_t ldraw_t(const uint8_t* p) {
  if constexpr (DT == kF32) return *reinterpret_cast<const uint32_t*>(p);
  else return *reinterpret_cast<const uint16_t*>(p);
}

template <int DT>
__device__ __forceinline__ float cvraw_t(uint32_t w) {
  if constexpr (DT == kF32) return __uint_as_float(w);
  else if constexpr (DT == kF16) return __half2float(__ushort_as_half((unsigned short)w));
  else return __uint_as_float(w << 16);
}

template <int DT>
__device__ __forceinline__ void red_cols_t(const Exec& ex, const ReqView& q, bool mean,
                                           uint32_t k) {
  constexpr int ES = DT == kF32 ? 4 : 2;
  const int lane = ex.lane;
  const int64_t C = q.inner, R = q.numel;
  const int rg = (int)q.rg, cl = 32 / rg;
  const int rl = lane % rg, ci = lane / rg;
  const uint32_t nseg = q.nseg;
  const int64_t gi = k / nseg;
  const uint32_t seg = k % nseg;
  const int64_t r = gi * rg + rl;
  const bool valid = r < R;
  const int64_t c0 = (int64_t)seg * q.chunk;
  int64_t c1 = c0 + q.chunk;
  if (c1 > C) c1 = C;
  float acc0 = 0.f, acc1 = 0.f;
  if (valid) {
    const int64_t ls = q.sa_in * ES * cl;      // bytes between a lane's columns
    int64_t c = c0 + ci;
    const uint8_t* pc = reinterpret_cast<const uint8_t*>(q.a) + (r * q.sa_row + c * q.sa_in) * ES;
#pragma unroll 1
    for (; c + (int64_t)cl * (kColU - 1) < c1; c += (int64_t)cl * kColU) {
      uint32_t w[kColU];
#pragma unroll
      for (int u = 0; u < kColU; ++u) w[u] = ldraw_t<DT>(pc + u * ls);
      pc += ls * kColU;
#pragma unroll
      for (int u = 0; u < kColU; ++u) (u & 1 ? acc1 : acc0) += cvraw_t<DT>(w[u]);
    }
    if (c < c1) {
      uint32_t w[kColU];
#pragma unroll
      for (int u = 0; u < kColU; ++u) {
        w[u] = 0u;
        if (c + (int64_t)cl * u < c1) w[u] = ldraw_t<DT>(pc + u * ls);
      }
#pragma unroll
      for (int u = 0; u < kColU; ++u)
        if (c + (int64_t)cl * u < c1) (u & 1 ? acc1 : acc0) += cvraw_t<DT>(w[u]);
    }
  }
  float acc = acc0 + acc1;
  for (int off = rg; off < 32; off <<= 1) acc += __shfl_xor_sync(GPUOS_FULL, acc, off);
  if (nseg == 1) {
    if (valid && ci == 0) st1(q.o, q.dto, r * q.so_row, red_finish(acc, mean, C));
    return;
  }
  float* part = ex.scratch + q.part + (gi * nseg) * rg;
  if (ci == 0) part[seg * rg + rl] = acc;
  uint32_t* cnt = ex.counters + q.cnt + gi;
  if (combine_arrive(ex, cnt, nseg)) {
    if (ci == 0) {
      float s = 0.f;
      for (uint32_t i = 0; i < nseg; ++i) s += __ldcg(part + i * rg + rl);
      if (valid) st1(q.o, q.dto, r * q.so_row, red_finish(s, mean, C));
    }
    if (lane == 0) *cnt = 0u;
  }
}

__device__ __forceinline__ void red_cols(const Exec& ex, const ReqView& q, bool mean, uint32_t k) {
  if (q.dta == kF32) red_cols_t<kF32>(ex, q, mean, k);
  else if (q.dta == kF16) red_cols_t<kF16>(ex, q, mean, k);
  else red_cols_t<kBF16>(ex, q, mean, k);
}

// Rows adjacent in memory, vector form (RF_VEC on an RL_COLS request: the row
// count times the element size is a multiple of 16 bytes and the base is
// 16-byte aligned): lane l of row group gi owns the GE adjacent rows
// gi * 32 GE + GE l .. + GE - 1 and reads them as one 16-byte load per
// column, kRedVU columns in flight; q.rg = 32 GE rows per group.
__device__ __forceinline__ void red_cols_vec(const Exec& ex, const ReqView& q, bool mean,
                                             uint32_t k) {
  const int lane = ex.lane;
  const int64_t C = q.inner, R = q.numel;
  const int GE = q.dta == kF32 ? 4 : 8;
  const int es = q.dta == kF32 ? 4 : 2;
  const uint32_t nseg = q.nseg;
  const int64_t gi = k / nseg;
  const uint32_t seg = k % nseg;
  const int64_t r0 = gi * q.rg + (int64_t)GE * lane;
  const bool valid = r0 < R;  // R is a multiple of GE, so the whole group is in range
  const int64_t c0 = (int64_t)seg * q.chunk;
  const int64_t c1 = min(C, c0 + (int64_t)q.chunk);
  const int64_t sc = q.sa_in;
  const uint8_t* p = reinterpret_cast<const uint8_t*>(q.a);
  float acc[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) acc[t] = 0.f;
  if (valid) {
#pragma unroll 1
    for (int64_t c = c0; c < c1; c += kRedVU) {
      uint4 w[kRedVU];
#pragma unroll
      for (int u = 0; u < kRedVU; ++u) {
        w[u] = make_uint4(0u, 0u, 0u, 0u);
        if (c + u < c1) w[u] = *reinterpret_cast<const uint4*>(p + (r0 + (c + u) * sc) * es);
      }
#pragma unroll
      for (int u = 0; u < kRedVU; ++u) {
        if (c + u < c1) {
          if (q.dta == kF32) {
            acc[0] += __uint_as_float(w[u].x);
            acc[1] += __uint_as_float(w[u].y);
            acc[2] += __uint_as_float(w[u].z);
            acc[3] += __uint_as_float(w[u].w);
          } else {
            float v[8];
            if (q.dta == kF16) {
              const uint32_t uu[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&uu[t]));
                v[2 * t] = f.x;
                v[2 * t + 1] = f.y;
              }
            } else {
              bf2_to_f(w[u].x, v[0], v[1]);
              bf2_to_f(w[u].y, v[2], v[3]);
              bf2_to_f(w[u].z, v[4], v[5]);
              bf2_to_f(w[u].w, v[6], v[7]);
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t] += v[t];
          }
        }
      }
    }
  }
  if (nseg == 1) {
    if (valid)
      for (int t = 0; t < GE; ++t) st1(q.o, q.dto, (r0 + t) * q.so_row, red_finish(acc[t], mean, C));
    return;
  }
  // partial sums of this segment: part[(gi * nseg + seg) * rg + row in group]
  float* part = ex.scratch + q.part + ((int64_t)gi * nseg) * q.rg;
  if (valid)
    for (int t = 0; t < GE; ++t) part[(int64_t)seg * q.rg + GE * lane + t] = acc[t];
  uint32_t* cnt = ex.counters + q.cnt + gi;
  if (combine_arrive(ex, cnt, nseg)) {
    if (valid) {
      for (int t = 0; t < GE; ++t) {
        float s = 0.f;
        for (uint32_t i = 0; i < nseg; ++i) s += __ldcg(part + (int64_t)i * q.rg + GE * lane + t);
        st1(q.o, q.dto, (r0 + t) * q.so_row, red_finish(s, mean, C));
      }
    }
    if (lane == 0) *cnt = 0u;
  }
}

// Anything else: one lane per output element, serial over the reduced
// elements with the first reduced axis varying fastest (the order of the
// reference's generic path, pytorch_ext/gpuos_ext.cpp:794-798).
__device__ __forceinline__ void red_generic(const Exec& ex, const ReqView& q, const ExtRec* x,
                                            bool mean, uint32_t k) {
  const int64_t o0 = (int64_t)k * q.chunk;
  int64_t o1 = o0 + q.chunk;
  if (o1 > q.numel) o1 = q.numel;
  const int nd = x->ndim, rd = x->rdim;
  for (int64_t oi = o0 + ex.lane; oi < o1; oi += 32) {
    int64_t rem = oi, ib = 0, ob = 0;
    for (int d = nd - 1; d >= 0; --d) {
      const int64_t sz = x->sizes[d];
      const int64_t i = rem % sz;
      rem /= sz;
      ib += i * x->sa[d];
      ob += i * x->so[d];
    }
    float acc = 0.f;
    for (int64_t rv = 0; rv < q.inner; ++rv) {
      int64_t t = rv, off = 0;
      for (int j = 0; j < rd; ++j) {
        const int64_t sz = x->rsizes[j];
        off += (t % sz) * x->rstrides[j];
        t /= sz;
      }
      acc += ld1(q.a, q.dta, ib + off);
    }
    st1(q.o, q.dto, ob, red_finish(acc, mean, q.inner));
  }
}

// Anything else with at least 64 reduced elements per output (q.rg == 1): a
// segmented reduction, one warp per output: the lanes split the reduced
// index space, with the last reduced axis (normally the one of smallest
// stride) varying fastest so that neighbouring lanes read neighbouring
// elements; four raw loads in flight per lane, then a shuffle tree.
__device__ __forceinline__ void red_generic_warp(const Exec& ex, const ReqView& q, const ExtRec* x,
                                                 bool mean, uint32_t k) {
  const int lane = ex.lane;
  const int64_t o0 = (int64_t)k * q.chunk;
  const int64_t o1 = min(q.numel, o0 + (int64_t)q.chunk);
  const int nd = x->ndim, rd = x->rdim;
  const int64_t inner = q.inner;
  constexpr int U = 4;
  for (int64_t oi = o0; oi < o1; ++oi) {
    int64_t rem = oi, ib = 0, ob = 0;
    for (int d = nd - 1; d >= 0; --d) {
      const int64_t sz = x->sizes[d];
      const int64_t i = rem % sz;
      rem /= sz;
      ib += i * x->sa[d];
      ob += i * x->so[d];
    }
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
    for (int64_t rv = lane; rv < inner; rv += 32 * U) {
      uint32_t w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        w[u] = 0u;
        const int64_t r = rv + 32 * u;
        if (r < inner) {
          int64_t t = r, off = 0;
          for (int j = rd - 1; j >= 0; --j) {
            const int64_t sz = x->rsizes[j];
            off += (t % sz) * x->rstrides[j];
            t /= sz;
          }
          w[u] = ld1_raw(q.a, q.dta, ib + off);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (rv + 32 * u < inner) (u & 1 ? acc1 : acc0) += cvt1(w[u], q.dta);
    }
    float acc = acc0 + acc1;
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(GPUOS_FULL, acc, off);
    if (lane == 0) st1(q.o, q.dto, ob, red_finish(acc, mean, inner));
  }
}

// ---------------------------------------------------------------------------
// One chunk of one request.
// ---------------------------------------------------------------------------
// The bodies a kernel carries: a batch of only elementwise or only reduction
// requests runs a kernel with just those bodies (less code to fetch, fewer
// registers, more resident warps); mixed batches and the persistent worker
// carry both.
enum Bodies : int { BODY_EW = 1, BODY_RED = 2, BODY_ALL = 3 };

// `x` is the request's ExtRec, copied to shared memory (strided layouts only).
template <int BODIES>
__device__ __forceinline__ void process_chunk(const Exec& ex, const ReqView& q, int v, float p0,
                                              float p1, uint32_t k, const ExtRec* x) {
  if (q.kind == RK_EW) {
    if constexpr (!(BODIES & BODY_EW)) {
      if (ex.lane == 0) set_err(ex, ERR_BAD_KIND);
      return;
    }
    if (!ew_known(v)) {
      if (ex.lane == 0) set_err(ex, ERR_BAD_OP);
      return;
    }
    if (q.layout == EL_TILE2D) {
      tile2d_dispatch(q, v, p0, p1, k, ex.lane);
      return;
    }
    const int64_t e0 = (int64_t)k * q.chunk;
    int64_t e1 = e0 + q.chunk;
    if (e1 > q.numel) e1 = q.numel;
#ifdef GPUOS_JIT_LINK
    if (q.flags & RF_NARY) {
      ew_generic_nary(q, x, v, p0, p1, e0, e1, ex.lane);
      return;
    }
#else
    if (q.flags & RF_NARY) {  // only custom expressions take more than two operands
      if (ex.lane == 0) set_err(ex, ERR_BAD_KIND);
      return;
    }
#endif
    ew_generic(q, x, v, p0, p1, e0, e1, ex.lane);
    return;
  }
  if constexpr (!(BODIES & BODY_RED)) {
    if (ex.lane == 0) set_err(ex, ERR_BAD_KIND);
    return;
  }
  if (v != V_SUM && v != V_MEAN) {
    if (ex.lane == 0) set_err(ex, v < 0 ? ERR_BAD_OP : ERR_BAD_KIND);
    return;
  }
  const bool mean = (v == V_MEAN);
  if (q.layout == RL_ROWS) red_rows(ex, q, mean, k);
  else if (q.layout == RL_COLS) {
    if (q.flags & RF_VEC) red_cols_vec(ex, q, mean, k);
    else red_cols(ex, q, mean, k);
  }
  else if (q.rg == 1) red_generic_warp(ex, q, x, mean, k);
  else red_generic(ex, q, x, mean, k);
}

// Called by the thread that counted the last chunk of the batch.  The
// completion word is seq + 1 with the batch's error bits in bits 48..55.  The
// persistent worker publishes it to the device ring (for batches that wait on
// this one) and, with system scope, to the host.  A stream-mode batch is
// complete when the event recorded after its launch is; the kernel writes the
// word to the host only when the batch has an error (the host reads it after
// that event, which makes the kernel's writes visible), so that a clean batch
// ends without a write over PCIe.
__device__ __forceinline__ void finish_batch(const Exec& ex) {
  __threadfence();
  const uint64_t seq = ex.seq;
  const uint32_t err = atomicOr(&ex.st->err, 0u);
  const uint64_t word = (seq + 1) | ((uint64_t)(err & 0xffu) << 48);
  if (ex.dur_ring) {
    // device time of the batch: first CTA in -> this last chunk
    const uint64_t nt0 = atomicAdd(reinterpret_cast<unsigned long long*>(&ex.st->nt0), 0ull);
    ex.dur_ring[seq % kDoneRing] = nt0 ? globaltimer() - ~nt0 : 0ull;
  }
  if (ex.done_dev) {
    st_release_gpu_u64(&ex.done_dev[seq % kDoneRing], word);
    st_release_sys_u64(&ex.done_ring[seq % kDoneRing], word);
  } else if (err) {
    ex.done_ring[seq % kDoneRing] = word;
  }
}

// Bind the execution context of one batch: its payload in the device staging
// ring, a copy of its header (a kernel parameter, or shared memory in the
// worker) and its device-side counters.
__device__ __forceinline__ Exec bind_batch(const uint8_t* payload, const BatchHdr& h,
                                           BatchState* st, volatile uint64_t* done_ring,
                                           uint64_t* done_dev, uint64_t wait_limit_ns,
                                           volatile uint64_t* dur_ring = nullptr,
                                           const Tables* tab = nullptr) {
  Exec ex;
  ex.base = payload;
  ex.st = st;
  ex.recs = reinterpret_cast<const Req*>(payload + h.rec_off);
  ex.gcb = reinterpret_cast<const uint32_t*>(payload + h.cb_off);
  ex.gtab = reinterpret_cast<const uint2*>(payload + h.gtab_off);
  ex.nchunk = h.nchunk;
  ex.gran = h.gran;
  ex.flags = h.flags;
  const uint32_t ngran = h.gran ? (h.nchunk + h.gran - 1) / h.gran : 0u;
  ex.req_wait = (h.flags & BF_STAGED) ? reinterpret_cast<const uint32_t*>(ex.gtab + ngran) : nullptr;
  ex.scratch = reinterpret_cast<float*>(h.scratch);
  ex.counters = reinterpret_cast<uint32_t*>(h.counters);
  ex.seq = h.seq;
  ex.wait_from = h.wait_from;
  ex.done_ring = done_ring;
  ex.done_dev = done_dev;
  ex.dur_ring = dur_ring;
  ex.tab = tab;
  ex.wait_limit_ns = wait_limit_ns;
  ex.lane = threadIdx.x & 31;
  return ex;
}

}  // namespace gpuos
